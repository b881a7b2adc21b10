"""Fused peer-to-peer all-reduce: one-GPU emulation of several ranks, and two real ranks."""
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.parametrize("world", [2, 4, 8])
def test_p2p_allreduce_emulated(world):
    from xnn_b200.parallel.p2p_allreduce import P2PAllReduce
    n = 64 * world * 37
    ar = P2PAllReduce(n, torch.float32, torch.device("cuda:0"), emulate_world=world, nblocks=8)
    try:
        for it in range(3):   # the per-CTA epochs advance across calls
            data = [torch.randn(n, device="cuda") for _ in range(world)]
            for b, d in zip(ar.buffers, data):
                b.copy_(d)
            want = torch.stack(data).mean(0)
            ar.all_reduce_mean_()
            torch.cuda.synchronize()
            assert ar.status() == 0
            for b in ar.buffers:
                torch.testing.assert_close(b, want, rtol=1e-6, atol=1e-6)
    finally:
        ar.close()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_p2p_allreduce_two_ranks(tmp_path):
    script = tmp_path / "ar.py"
    script.write_text(
        "import os, sys, torch\n"
        f"sys.path.insert(0, {ROOT!r})\n"
        "from xnn_b200.parallel import distributed as D\n"
        "from xnn_b200.parallel.p2p_allreduce import P2PAllReduce\n"
        "dev = D.init_process_group('cuda', timeout_s=60)\n"
        "r, w = D.rank(), D.world_size()\n"
        "n = 64 * w * 1000\n"
        "ar = P2PAllReduce(n, torch.float32, dev)\n"
        "for it in range(5):\n"
        "    g = torch.Generator(device='cpu').manual_seed(100 * it + r)\n"
        "    ar.buffer.copy_(torch.randn(n, generator=g).to(dev))\n"
        "    ar.all_reduce_mean_()\n"
        "    torch.cuda.synchronize()\n"
        "    ar.check()\n"
        "    want = sum(torch.randn(n, generator=torch.Generator().manual_seed(100 * it + k)) for k in range(w)) / w\n"
        "    assert torch.allclose(ar.buffer.cpu(), want, atol=1e-5), 'mismatch'\n"
        "ar.close()\n"
        "D.destroy_process_group()\n"
        "print('ok')\n")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "10", "120", sys.executable, "-m", "torch.distributed.run", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", "29517", str(script)]
    out = subprocess.run(cmd, capture_output=True, text=True, env=env)
    assert out.returncode == 0, out.stdout + out.stderr


def test_p2p_allreduce_bucket_ranges_emulated():
    """Bucket-by-bucket reduction (sub-ranges of the buffer, several per step, the per-CTA epochs
    advancing across launches) gives the mean of every range."""
    from xnn_b200.parallel.p2p_allreduce import P2PAllReduce
    world = 4
    sizes = [64 * world * 3, 64 * world * 40, 64 * world]
    n = sum(sizes)
    ar = P2PAllReduce(n, torch.float32, torch.device("cuda:0"), emulate_world=world, nblocks=8)
    try:
        for it in range(2):
            data = [torch.randn(n, device="cuda") for _ in range(world)]
            for b, d in zip(ar.buffers, data):
                b.copy_(d)
            want = torch.stack(data).mean(0)
            off = 0
            for sz in reversed(sizes):           # any fixed order, the same on every rank
                start = n - off - sz
                ar.all_reduce_mean_(offset=start, numel=sz)
                off += sz
            torch.cuda.synchronize()
            assert ar.status() == 0
            for b in ar.buffers:
                torch.testing.assert_close(b, want, rtol=1e-6, atol=1e-6)
    finally:
        ar.close()


def test_p2p_allreduce_timeout_reports_status():
    """A peer that never gets as far: rank 0's target epoch is moved out of reach, so its bounded
    wait gives up; the kernel records the peer in the host-mapped status word and returns, and
    ``check`` raises (the GPU stays usable)."""
    from xnn_b200.parallel.p2p_allreduce import P2PAllReduce
    world = 2
    n = 64 * world * 8
    ar = P2PAllReduce(n, torch.float32, torch.device("cuda:0"), emulate_world=world, nblocks=2,
                      spin_limit=200_000)
    try:
        ar.epochs[0:64] += 5                     # rank 0 now waits for an epoch nobody will write
        ar.all_reduce_mean_()
        torch.cuda.synchronize()
        assert ar.status() != 0
        with pytest.raises(RuntimeError, match="waited in vain for rank"):
            ar.check()
        # the device is still usable
        assert float(torch.ones(4, device="cuda").sum()) == 4.0
    finally:
        ar.close()
