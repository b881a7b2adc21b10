"""The hand-written MACE training step against autograd: loss, forces and every parameter gradient.

On the CPU in float64 both run the PyTorch formulas, so they must agree to rounding; on a GPU the
step runs on the package's kernels and is compared in float32 (and float64) with the autograd
step of the same model."""
import pytest
import torch

from xnn_b200.data import collate, structure_to_graph, synthetic
from xnn_b200.models import ForceStressOutput
from xnn_b200.models.mace import MACE
from xnn_b200.train import mace_step
from xnn_b200.train.losses import weighted_loss


def _setup(dtype, device, channels=8, seed=0, n_struct=3, max_ell=3, correlation=3):
    torch.manual_seed(seed)
    model = MACE(species=[1, 6, 7, 8, 9, 16, 17], cutoff=4.5, num_channels=channels, n_rbf=8, num_interactions=2,
                 max_ell=max_ell, correlation=correlation, avg_num_neighbors=9.0).to(device=device, dtype=dtype)
    # non-trivial readouts, self-connections and reference energies
    with torch.no_grad():
        for p in model.parameters():
            p.add_(0.05 * torch.randn_like(p))
        model.atom_ref.weight.normal_()
    mols = synthetic.organic_molecules(n_struct, seed=seed + 11, n_min=8, n_max=20)
    b = collate([structure_to_graph(s, 4.5) for s in mols]).to(device)
    b.pos = b.pos.to(dtype)
    b.weight = torch.linspace(0.5, 1.5, b.num_graphs, dtype=torch.float64, device=device)
    pot = ForceStressOutput(model).train()
    return pot, b


def _autograd(pot, b, we, wf):
    params = [p for p in pot.parameters() if p.requires_grad]
    for p in params:
        p.grad = None
    out = pot(b.clone())
    loss, logs = weighted_loss(out, b, we, wf)
    loss.backward()
    return loss.detach(), out["forces"].detach(), {n: p.grad.clone() for n, p in pot.named_parameters()
                                                    if p.grad is not None}


def _engine(pot, b, we, wf):
    for p in pot.parameters():
        p.grad = None
    step = mace_step.MACEStep(pot, we, wf)
    loss, logs, out = step(b.clone())
    return loss.detach(), out["forces"], {n: p.grad.clone() for n, p in pot.named_parameters() if p.grad is not None}


class _Optim:
    stress_weight = dipole_weight = polarizability_weight = charge_weight = property_weight = 0.0
    huber_delta = 0.0
    huber_delta_energy = huber_delta_forces = None
    reaction_weight = 0.0


def test_supports_bench_architecture():
    pot, _ = _setup(torch.float64, "cpu")
    ok, why = mace_step.supports(pot, _Optim())
    assert ok, why


@pytest.mark.parametrize("we,wf", [(1.0, 10.0), (0.0, 1.0), (1.0, 0.0)])
def test_step_matches_autograd_cpu_float64(we, wf):
    pot, b = _setup(torch.float64, "cpu")
    pot.model.set_use_fast(True)          # the fused-path mathematics on the CPU (PyTorch formulas)
    l0, f0, g0 = _autograd(pot, b, we, wf)
    l1, f1, g1 = _engine(pot, b, we, wf)
    torch.testing.assert_close(l1, l0, rtol=1e-10, atol=1e-12)
    torch.testing.assert_close(f1, f0, rtol=1e-9, atol=1e-10)
    assert set(g1) == set(g0)
    for name in g0:
        scale = g0[name].abs().max().clamp_min(1e-12)
        err = (g1[name] - g0[name]).abs().max() / scale
        assert err < 1e-8, (name, float(err))


def _gpu_compare(dtype, channels, tol):
    pot, b = _setup(dtype, "cuda", channels=channels, seed=2, n_struct=6)
    pot.model.set_use_fast(True)
    l0, f0, g0 = _autograd(pot, b, 1.0, 10.0)
    l1, f1, g1 = _engine(pot, b, 1.0, 10.0)
    torch.cuda.synchronize()
    assert abs(float(l1) - float(l0)) <= tol * abs(float(l0))
    assert float((f1 - f0).abs().max() / f0.abs().max()) < tol
    for name in g0:
        err = float((g1[name] - g0[name]).abs().max() / g0[name].abs().max().clamp_min(1e-12))
        assert err < tol, (name, err)


@pytest.mark.gpu
def test_step_matches_autograd_gpu_float64():
    _gpu_compare(torch.float64, 16, 1e-8)


@pytest.mark.gpu
def test_step_matches_autograd_gpu_float32_bench_width():
    # the benchmarked width (96 channels, l <= 3, correlation 3): fp32 parity at 1e-3 relative
    _gpu_compare(torch.float32, 96, 1e-3)


@pytest.mark.parametrize("max_ell,correlation", [(2, 2), (1, 3)])
def test_step_matches_autograd_other_degrees(max_ell, correlation):
    pot, b = _setup(torch.float64, "cpu", max_ell=max_ell, correlation=correlation)
    pot.model.set_use_fast(True)
    l0, f0, g0 = _autograd(pot, b, 1.0, 10.0)
    l1, f1, g1 = _engine(pot, b, 1.0, 10.0)
    torch.testing.assert_close(l1, l0, rtol=1e-10, atol=1e-12)
    for name in g0:
        err = (g1[name] - g0[name]).abs().max() / g0[name].abs().max().clamp_min(1e-12)
        assert err < 1e-8, (name, float(err))


@pytest.mark.gpu
def test_fused_loss_kernel_matches_formulas(monkeypatch):
    """The one-kernel loss (both terms, sums, cotangents) against the PyTorch formulas, on a padded
    batch (structure masks and per-atom force weights)."""
    import xnn_b200.ops.mace_ops as K
    from xnn_b200.train.graphed import pad_graph
    pot, b = _setup(torch.float32, "cuda", channels=8, n_struct=5)
    b = pad_graph(b, b.num_nodes + 12, b.num_edges + 40, b.num_graphs + 2, 4.5)
    b.weight = torch.linspace(0.5, 1.5, b.num_graphs, dtype=torch.float64, device="cuda")
    step = mace_step.MACEStep(pot, 1.0, 10.0)
    g0 = torch.Generator(device="cuda").manual_seed(3)
    energy = torch.randn(b.num_graphs, device="cuda", generator=g0)
    forces = torch.randn(b.num_nodes, 3, device="cuda", dtype=torch.float64, generator=g0)
    assert hasattr(K._C(), "mace_loss")
    l1, logs1, a1, f1 = step._loss(b, energy, forces)
    monkeypatch.setattr(K, "_C", lambda: object())        # no kernel: the PyTorch formulas
    l0, logs0, a0, f0 = step._loss(b, energy, forces)
    torch.testing.assert_close(l1, l0, rtol=1e-12, atol=1e-14)
    torch.testing.assert_close(a1.to(a0.dtype), a0, rtol=1e-10, atol=1e-14)
    torch.testing.assert_close(f1, f0, rtol=1e-10, atol=1e-14)
    for k in logs0:
        torch.testing.assert_close(logs1[k], logs0[k], rtol=1e-12, atol=1e-14)


@pytest.mark.gpu
def test_grouped_species_linear_matches_all_blocks():
    from xnn_b200.models.mace_fast import species_linear
    from xnn_b200.ops import node_gemm as NG
    torch.manual_seed(0)
    N, n_el, C = 1000, 5, 96
    z = torch.randint(0, n_el, (N,), device="cuda")
    z[z == 3] = 2                                            # one element absent
    Wz = torch.randn(n_el, C, C, device="cuda") / C ** 0.5
    for lead in ((), (7,)):
        h = torch.randn(*lead, N, C, device="cuda", requires_grad=True)
        ref = species_linear(h, z, Wz)
        got = NG.species_linear(h, z, Wz)
        torch.testing.assert_close(got, ref, rtol=2e-5, atol=2e-5)
        g = torch.randn_like(ref)
        (dr,) = torch.autograd.grad(ref, h, g)
        (dg,) = torch.autograd.grad(got, h, g)
        torch.testing.assert_close(dg, dr, rtol=2e-5, atol=2e-5)


@pytest.mark.gpu
def test_grouped_species_linear_blocks():
    from xnn_b200.models.mace_fast import species_linear
    from xnn_b200.ops import node_gemm as NG
    torch.manual_seed(1)
    N, n_el, C = 777, 4, 96
    z = torch.randint(0, n_el, (N,), device="cuda")
    sizes = [1, 3, 5, 7]
    Ws = [torch.randn(n_el, C, C, device="cuda") / C ** 0.5 for _ in sizes]
    h = torch.randn(16, N, C, device="cuda", requires_grad=True)
    ref = torch.cat([species_linear(b, z, W) for b, W in zip(h.split(sizes, 0), Ws)], 0)
    got = NG.species_linear_blocks(h, z, Ws, sizes)
    torch.testing.assert_close(got, ref, rtol=2e-5, atol=2e-5)
    g = torch.randn_like(ref)
    torch.testing.assert_close(torch.autograd.grad(got, h, g)[0], torch.autograd.grad(ref, h, g)[0],
                               rtol=2e-5, atol=2e-5)
    # the library sort path of large systems gives the same grouping as the kernel
    zz = torch.randint(0, n_el, (100_000,), device="cuda")
    p, s = NG.species_sort(zz, n_el)
    assert torch.equal(zz[p.long()], torch.sort(zz, stable=True).values) and int(s[-1]) == 100_000
