"""Micro-benchmarks of the hot CUDA kernels on a config-4-shaped water box.

Each op is timed with CUDA events on the current stream after warm-up; between timed launches a
buffer larger than L2 is overwritten so every launch reads its operands from HBM. The printed
line gives the duration, the algorithmic bytes moved (the operands each kernel must read and the
results it must write, once) and the achieved fraction of a reference bandwidth.

    python -m xnn_b200.utils.kernel_bench --atoms 20000 --ops conv_gather,gemm_reduce

The same command with ``--iters 1 --warmup 1`` is a small case for a profiler capture.
"""
from __future__ import annotations

import argparse
import json
import os
from typing import Callable, Dict, List

import torch

from .. import _ext
from ..data import synthetic
from ..data.neighborlist import build_neighbor_list
from ..ops import gemm
from ..ops import mace_ops as K

L2_FLUSH_BYTES = 256 << 20


def peaks() -> Dict[str, float]:
    """Measured HBM bandwidth (GB/s) from MEASURED_PEAKS.json at the repository root, else 6650."""
    path = os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))),
                        "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return {"hbm_gbs": float(d["hbm_gbs"]), "source": "measured"}
    except (OSError, KeyError, ValueError):
        return {"hbm_gbs": 6650.0, "source": "fallback"}


def time_op(fn: Callable[[], object], iters: int, warmup: int) -> float:
    """Median milliseconds of ``fn`` over ``iters`` launches, L2 flushed before each."""
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device="cuda")
    for _ in range(warmup):
        fn()
    times: List[float] = []
    for _ in range(iters):
        flush.fill_(1.0)
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        times.append(a.elapsed_time(b))
    times.sort()
    return times[len(times) // 2]


def water_case(n_atoms: int, cutoff: float = 4.5, C: int = 96, P: int = 4, seed: int = 0):
    s = synthetic.water_box(n_atoms, seed=seed)
    dev = torch.device("cuda")
    pos, cell = s["pos"].to(dev), s["cell"].to(dev)
    ei, shifts = build_neighbor_list(pos, cutoff, cell, s["pbc"], engine="native")
    order = torch.argsort(ei[1], stable=True)
    ei, shifts = ei[:, order], shifts[order]
    vec = (pos[ei[1]] - pos[ei[0]] + shifts.to(pos.dtype) @ cell).float()
    N, E = pos.shape[0], ei.shape[1]
    g = torch.Generator(device=dev).manual_seed(seed)
    return {
        "pos": pos, "cell": cell, "pbc": s["pbc"], "cutoff": cutoff, "ei": ei, "vec": vec, "N": N, "E": E,
        "plan": K.EdgePlan.build(ei, N, assume_dst_sorted=True),
        "x": torch.randn(N, C, device=dev, generator=g),
        "R": torch.randn(E, P, C, device=dev, generator=g),
        "Y": torch.randn(E, P * P, device=dev, generator=g),
        "G": torch.randn(P * P, N, C, device=dev, generator=g),
        "C": C, "P": P,
    }


def build_ops(case) -> Dict[str, tuple]:
    """name -> (callable, algorithmic bytes)."""
    C, P, N, E = case["C"], case["P"], case["N"], case["E"]
    plan, x, R, Y, G = case["plan"], case["x"], case["R"], case["Y"], case["G"]
    ops = _ext.ops()
    f = 4
    T1 = torch.randn(E, P, C, device="cuda")
    out: Dict[str, tuple] = {}
    out["conv_gather"] = (lambda: ops.conv_gather(N, C, P, plan.dst_ptr, plan.src32, plan.dst_perm, [x], [R], [Y]),
                          f * (E * P * C + E * P * P + N * C + P * P * N * C))
    out["conv_edge"] = (lambda: ops.conv_edge(N, C, P, E, plan.dst_ptr, plan.src32, plan.dst_perm, G, [Y], [x],
                                              [True], True, [], []),
                        f * (P * P * N * C + E * P * P + N * C + 2 * E * P * C))
    out["conv_scatter"] = (lambda: ops.conv_scatter(N, C, P, plan.src_ptr, plan.src_perm, [R], [T1]),
                           f * (2 * E * P * C + N * C))
    Rd = torch.randn(E, P, C, device="cuda")
    # force pass (MD): reads R, Rd, Y, x[src], G once per receiver; writes g_r, gY, the (E, C) sender terms
    out["conv_force"] = (lambda: ops.conv_force(N, C, P, E, plan.dst_ptr, plan.src32, G, Y, x, R, Rd),
                         f * (2 * E * P * C + E * P * P + E * C + P * P * N * C + E + E * P * P + E * C))
    out["conv_edge_force"] = (lambda: ops.conv_edge(N, C, P, E, plan.dst_ptr, plan.src32, None, G, [Y], [x], [False],
                                                    True, [x], [R], Rd, R),
                              f * (2 * E * P * C + E * P * P + E * C + P * P * N * C + E + E * P * P + E * C))
    gxe = torch.randn(E, C, device="cuda")
    out["conv_sender_sum"] = (lambda: ops.conv_sender_sum(N, plan.src_ptr, plan.src_perm, gxe),
                              f * (E * C + N * C) + 8 * E)
    H = 64
    Hr = torch.randn(2 * E, H, device="cuda")
    W2 = torch.randn(H, P * C, device="cuda")
    out["gemm_rows_64x384"] = (lambda: gemm.mm_raw(Hr[:E], W2), f * (E * H + E * P * C + H * P * C))
    Wh = torch.randn(H, H, device="cuda")
    out["gemm_rows_64x64"] = (lambda: gemm.mm_raw(Hr, Wh), f * (2 * E * H * 2 + H * H))
    D = torch.randn(E, P * C, device="cuda")
    out["gemm_reduce_64x384"] = (lambda: gemm.mm_t_raw(Hr[:E], D), f * (E * H + E * P * C))
    Dh = torch.randn(2 * E, H, device="cuda")
    out["gemm_reduce_64x64"] = (lambda: gemm.mm_t_raw(Hr, Dh), f * (2 * E * H * 2))
    vec = case["vec"]
    freqs = torch.pi * torch.arange(1, 9, dtype=torch.float32, device="cuda")
    out["edge_geometry"] = (lambda: K.edge_geometry(vec, 3, freqs, (2 / 4.5) ** 0.5, 4.5, 5),
                            f * (3 * E + 16 * E + 8 * E))
    D16 = 16
    A = 0.5 * torch.randn(D16, N, C, device="cuda")
    Ws = torch.randn(2, K.num_invariants(3, 3), C, device="cuda")
    z = torch.randint(0, 2, (N,), device="cuda")
    out["symcon_fwd"] = (lambda: K.symmetric_contraction(A, Ws, z, 3, 3), f * (D16 * N * C + N * C))
    pos, cell, pbc, rc = case["pos"], case["cell"], case["pbc"], case["cutoff"]
    out["neighbor_list"] = (lambda: build_neighbor_list(pos, rc, cell, pbc, engine="native"),
                            8 * 3 * N + E * (2 * 8 + 3 * 8))
    out.update(pme_ops(N))
    out.update(dispersion_ops(case))
    return out


def dispersion_ops(case) -> Dict[str, tuple]:
    """The D4 three-body kernel on the water box (triple cutoff 6 A, 23 Casimir-Polder frequencies;
    the byte figure is the edges' rows once: the kernel is bound by the pair walk, see ``pairs``)
    and the EEQ Coulomb product of a 20,000-atom molecule (one right-hand side pair)."""
    pos, cell, pbc = case["pos"], case["cell"], case["pbc"]
    N = pos.shape[0]
    n = min(N, 4000)
    ei, sh = build_neighbor_list(pos[:n], 6.0, cell, pbc, engine="native")
    order = torch.argsort(ei[1], stable=True)
    ei, sh = ei[:, order], sh[order]
    vec = ((pos[ei[0]] - pos[ei[1]] + sh.to(pos.dtype) @ cell) / 0.529177210903).double().contiguous()
    ptr = torch.zeros(n + 1, dtype=torch.long, device="cuda")
    ptr[1:] = torch.cumsum(torch.bincount(ei[1], minlength=n), 0)
    z = torch.where(torch.arange(n, device="cuda") % 3 == 0, 8, 1).long()
    g = torch.Generator(device="cuda").manual_seed(0)
    fa = 1.0 + torch.rand(n, 23, device="cuda", dtype=torch.float64, generator=g)
    fb = fa.clone()
    c6e = (fa[ei[1]] * fb[ei[0]]).sum(-1).contiguous()
    r0 = 4.0 + torch.rand(104, 104, device="cuda", dtype=torch.float64, generator=g)
    r0 = (0.5 * (r0 + r0.t())).contiguous()
    ops = _ext.ops()
    go = torch.ones(n, device="cuda", dtype=torch.float64)
    E = ei.shape[1]
    deg = torch.bincount(ei[1], minlength=n).double()
    pairs = float((deg * (deg - 1)).sum())
    out = {"d4_atm_energy": (lambda: ops.atm(ptr, ei[0].contiguous(), vec, z, fa, fb, c6e, r0, 1.0, 16.0 / 3.0,
                                             6.0 / 0.529177210903, 0.0, None), 8 * (4 * E + 23 * 2 * n)),
           "d4_atm_grad": (lambda: ops.atm(ptr, ei[0].contiguous(), vec, z, fa, fb, c6e, r0, 1.0, 16.0 / 3.0,
                                           6.0 / 0.529177210903, 0.0, go), 8 * (8 * E + 23 * 2 * n))}
    print(json.dumps({"op": "d4_atm", "atoms": n, "edges": E, "ordered_edge_pairs_per_call": pairs}))
    m = 20000
    pm = (torch.rand(m, 3, device="cuda", dtype=torch.float64, generator=g) * 60.0).contiguous()
    rad = (1.0 + torch.rand(m, device="cuda", dtype=torch.float64, generator=g)).contiguous()
    v = torch.randn(m, 2, device="cuda", dtype=torch.float64, generator=g).contiguous()
    out["eeq_coulomb_matvec"] = (lambda: ops.coulomb_matvec(pm, rad, v), 8 * (4 * m + 4 * m))
    return out



def pme_ops(n_atoms: int) -> Dict[str, tuple]:
    """The multipole PME kernels on a water box of ``n_atoms``: order-5 spreading of charges,
    dipoles and quadrupoles onto a float32 128^3 mesh, the gather of fields and forces, and the
    float64 real-space pair kernel (7 A, Thole-damped)."""
    from ..ffnn import multipoles as MP
    from ..ffnn.water import multipole_water
    w = multipole_water(n_atoms, seed=0, device=torch.device("cuda"))
    mesh, p = [128, 128, 128], 5
    K = torch.tensor(mesh, dtype=torch.float64, device="cuda")
    G = (torch.linalg.inv(w["cell"].double()) * K[None, :]).contiguous()
    args = (w["pos"].contiguous(), G, mesh, p, 0, mesh[2], w["q"].contiguous(), w["d"].contiguous(),
            w["Q"].reshape(-1, 9).contiguous())
    ops = _ext.ops()
    phi = torch.randn(mesh, dtype=torch.float32, device="cuda")
    n, m = w["pos"].shape[0], 128 ** 3
    site = 8 * (3 + 1 + 3 + 9)
    out = {"pme_spread": (lambda: ops.pme_spread(*args), n * site + 4 * m),
           "pme_gather": (lambda: ops.pme_gather(*args, phi, True, True), n * site + 4 * m + 2 * 3 * 8 * n)}
    i, j, shift, excl = MP.multipole_pairs(w["pos"], w["cell"], 7.0, w["molecule"])
    pol = w["pol"].contiguous()
    q, d, Q = w["q"].contiguous(), w["d"].contiguous(), w["Q"].reshape(-1, 9).contiguous()
    out["mp_real"] = (lambda: ops.mp_real(w["pos"], w["cell"], q, d, Q, pol, i, j, shift, excl, 0.4, 0.39, True,
                                          True),
                      i.shape[0] * (8 + 8 + 24 + 1) + n * site)
    # one induction iteration's pieces: the dipole field product over receiver-ordered pair entries
    # (int32 partner, 3 + 2 float64 per entry, each pair twice) and the dipole-only spread / gather
    mod = MP.PolarizableMultipoles(MP.EwaldSetup(alpha=0.4, cutoff=7.0, mesh=(128, 128, 128), order=5))
    T = MP.DipoleOperator(mod, w["pos"], w["cell"], (i, j, shift, excl), pol)
    rows = T._csr()
    out["dipole_csr_matvec"] = (lambda: T.real(d), 2 * i.shape[0] * (4 + 5 * 8) + n * 8 * (3 + 3) + 8 * (n + 1))
    dargs = args[:6] + (None, d, None)
    out["pme_spread_dipoles"] = (lambda: ops.pme_spread(*dargs), n * (8 * 6) + 4 * m)
    out["pme_gather_dipoles"] = (lambda: ops.pme_gather(*dargs, phi, True, False), n * (8 * 6 + 8 * 3) + 4 * m)
    del rows
    return out


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--atoms", type=int, default=20000)
    ap.add_argument("--ops", default="all")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    args = ap.parse_args(argv)
    if not _ext.cuda_available():
        raise SystemExit(f"native extension not loaded: {_ext.error()}")
    case = water_case(args.atoms)
    ops = build_ops(case)
    names = list(ops) if args.ops == "all" else args.ops.split(",")
    pk = peaks()
    with torch.no_grad():
        for name in names:
            fn, nbytes = ops[name]
            ms = time_op(fn, args.iters, args.warmup)
            gbs = nbytes / (ms * 1e-3) / 1e9
            print(json.dumps({"op": name, "atoms": case["N"], "edges": case["E"], "ms": round(ms, 4),
                              "alg_bytes": int(nbytes), "gb_s": round(gbs, 1),
                              f"frac_hbm_{pk['source']}": round(gbs / pk["hbm_gbs"], 3)}), flush=True)


if __name__ == "__main__":
    main()
