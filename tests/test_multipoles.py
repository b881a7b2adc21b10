"""Polarizable multipole Ewald: closed-form pair terms, alpha independence, PME accuracy,
induction and forces (CPU, float64)."""
import math

import pytest
import torch

from xnn_b200.ffnn import multipoles as M


@pytest.fixture(autouse=True)
def _f64():
    old = torch.get_default_dtype()
    torch.set_default_dtype(torch.float64)
    yield
    torch.set_default_dtype(old)


def _traceless(A):
    A = 0.5 * (A + A.transpose(-1, -2))
    return A - torch.eye(3) * A.diagonal(dim1=-2, dim2=-1).sum(-1)[..., None, None] / 3.0


def _system(n=24, L=11.0, seed=0, charge_scale=0.3):
    g = torch.Generator().manual_seed(seed)
    pos = torch.rand(n, 3, generator=g) * L
    cell = torch.tensor([[L, 0.0, 0.0], [0.6, L * 1.05, 0.0], [-0.4, 0.5, L * 0.95]])
    pos = pos @ torch.linalg.inv(torch.diag(torch.tensor([L, L, L]))) @ cell
    q = charge_scale * torch.randn(n, generator=g)
    d = 0.3 * torch.randn(n, 3, generator=g)
    Q = _traceless(0.3 * torch.randn(n, 3, 3, generator=g))
    return pos, cell, q, d, Q


def _operator_energy(v, qi, di, Qi, qj, dj, Qj, g):
    """L_i L_j g(|r_j - r_i|) by automatic differentiation (reference for the closed form)."""
    ri = torch.zeros(3, requires_grad=True)
    rj = v.clone().requires_grad_(True)

    def kern(a, b):
        return g(torch.linalg.norm(b - a))

    def apply_L(f, r, q, d, Q):
        val = f()
        (gr,) = torch.autograd.grad(val, r, create_graph=True)
        out = q * val + (d * gr).sum()
        for a in range(3):
            (h,) = torch.autograd.grad(gr[a], r, create_graph=True)
            out = out + (Q[a] * h).sum() / 3.0
        return out

    inner = lambda: apply_L(lambda: kern(ri, rj), rj, qj, dj, Qj)  # noqa: E731
    return apply_L(inner, ri, qi, di, Qi)


def test_pair_energy_closed_form_matches_operator():
    g = torch.Generator().manual_seed(1)
    alpha = 0.45
    for _ in range(4):
        v = torch.randn(3, generator=g) * 2.0
        qi, qj = torch.randn(2, generator=g)
        di, dj = torch.randn(2, 3, generator=g)
        Qi, Qj = _traceless(torch.randn(2, 3, 3, generator=g))
        r = torch.linalg.norm(v)
        for kind, fn in (("erfc", lambda x: torch.erfc(alpha * x) / x),
                         ("neg_erf", lambda x: -torch.erf(alpha * x) / x)):
            B = M._bn(r.reshape(1), alpha, kind)
            e = M.pair_energy(v[None], qi, di[None], Qi[None], qj, dj[None], Qj[None], B)
            ref = _operator_energy(v, qi, di, Qi, qj, dj, Qj, fn)
            torch.testing.assert_close(e[0], ref, rtol=1e-10, atol=1e-12)


def _energy(pos, cell, q, d, Q, alpha, mesh, order, cutoff, molecule=None):
    mod = M.PolarizableMultipoles(M.EwaldSetup(alpha=alpha, cutoff=cutoff, mesh=mesh, order=order,
                                               fft_dtype=torch.float64))
    pairs = M.multipole_pairs(pos, cell, cutoff, molecule)
    return mod.electrostatic(pos, cell, pairs, q, d, Q)


@pytest.mark.parametrize("with_molecules", [False, True])
def test_ewald_energy_independent_of_alpha(with_molecules):
    pos, cell, q, d, Q = _system()
    mol = torch.arange(pos.shape[0]) // 3 if with_molecules else None
    if with_molecules:                       # put each triple within 1.5 A of its first site
        g = torch.Generator().manual_seed(7)
        pos = pos.clone()
        pos[1::3] = pos[0::3] + 0.9 * torch.nn.functional.normalize(torch.randn(8, 3, generator=g), dim=-1)
        pos[2::3] = pos[0::3] + 1.0 * torch.nn.functional.normalize(torch.randn(8, 3, generator=g), dim=-1)
    e1 = _energy(pos, cell, q, d, Q, 0.75, (64, 64, 64), 8, 5.2, mol)
    e2 = _energy(pos, cell, q, d, Q, 0.95, (96, 96, 96), 10, 5.2, mol)
    assert abs(float(e1 - e2)) < 2e-6 * max(1.0, abs(float(e1))), (float(e1), float(e2))


def test_forces_match_finite_differences_and_induction_converges():
    pos, cell, q, d, Q = _system(n=18, seed=3)
    mol = torch.arange(18) // 3
    pol = torch.full((18,), 0.9)
    mod = M.PolarizableMultipoles(M.EwaldSetup(alpha=0.5, cutoff=5.2, mesh=(32, 32, 32), order=6,
                                               fft_dtype=torch.float64), tol_debye=1e-9, max_iter=200)
    out = mod(pos, cell, q, d, Q, pol, mol)
    assert float(out["residual_debye"]) < 1e-9
    # induced dipoles solve mu = alpha (F_perm + T mu)
    pairs = M.multipole_pairs(pos, cell, 5.2, mol)
    F = mod.field(pos, cell, pairs, q, d + out["induced_dipoles"], Q, pol=pol) / M.KE
    torch.testing.assert_close(out["induced_dipoles"], pol[:, None] * F, rtol=1e-7, atol=1e-9)
    eps = 1e-5
    for k in (0, 5, 11):
        for a in range(3):
            pp, pm = pos.clone(), pos.clone()
            pp[k, a] += eps
            pm[k, a] -= eps
            ep = mod(pp, cell, q, d, Q, pol, mol, compute_forces=False)["energy"]
            em = mod(pm, cell, q, d, Q, pol, mol, compute_forces=False)["energy"]
            fd = -(ep - em) / (2 * eps)
            assert abs(float(fd - out["forces"][k, a])) < 1e-6 * max(1.0, abs(float(fd))), (k, a, float(fd),
                                                                                          float(out["forces"][k, a]))


def _slab_rank(rank, world, mesh):
    import torch as T
    T.set_default_dtype(T.float64)
    from xnn_b200.ffnn import multipoles as MM
    from xnn_b200.ffnn.slab_fft import SlabFFT
    pos, cell, q, d, Q = _system(n=18, seed=3)
    mol = T.arange(18) // 3
    pol = T.full((18,), 0.9)
    setup = MM.EwaldSetup(alpha=0.5, cutoff=5.2, mesh=mesh, order=6, fft_dtype=T.float64)
    mod = MM.PolarizableMultipoles(setup, tol_debye=1e-9, max_iter=200, mesh_backend=SlabFFT(list(mesh)))
    out = mod(pos, cell, q, d, Q, pol, mol)
    return {"energy": out["energy"], "forces": out["forces"], "mu": out["induced_dipoles"]}


@pytest.mark.parametrize("world", [1, 2, 3])
def test_slab_decomposed_mesh_matches_single_process(world):
    from dist_util import run_ranks
    mesh = (32, 30, 28)
    pos, cell, q, d, Q = _system(n=18, seed=3)
    mol = torch.arange(18) // 3
    pol = torch.full((18,), 0.9)
    ref = M.PolarizableMultipoles(M.EwaldSetup(alpha=0.5, cutoff=5.2, mesh=mesh, order=6, fft_dtype=torch.float64),
                                  tol_debye=1e-9, max_iter=200)(pos, cell, q, d, Q, pol, mol)
    outs = run_ranks(_slab_rank, world, mesh)
    for o in outs:
        torch.testing.assert_close(o["energy"], ref["energy"], rtol=1e-9, atol=1e-9)
        torch.testing.assert_close(o["forces"], ref["forces"], rtol=1e-7, atol=1e-8)
        torch.testing.assert_close(o["mu"], ref["induced_dipoles"], rtol=1e-7, atol=1e-9)


@pytest.mark.parametrize("damped", [True, False])
def test_dipole_operator_matches_energy_gradient(damped):
    """The direct dipole operator of the induction solve against ``-dE/d(mu)`` of the energy
    with dipoles only (Thole-damped and undamped)."""
    pos, cell, q, d, Q = _system(n=21, seed=4)
    mol = torch.arange(21) // 3
    pol = 0.6 + 0.6 * torch.rand(21, generator=torch.Generator().manual_seed(5))
    mod = M.PolarizableMultipoles(M.EwaldSetup(alpha=0.45, cutoff=5.0, mesh=(24, 24, 24), order=5,
                                               fft_dtype=torch.float64))
    pairs = mod.pairs(pos, cell, mol)
    damp = pol if damped else None
    v = 0.2 * torch.randn(21, 3, generator=torch.Generator().manual_seed(6))
    ref = mod.dipole_field(pos, cell, pairs, v, pol=damp) / M.KE      # eV / (e A) -> Coulomb units
    got = M.DipoleOperator(mod, pos, cell, pairs, damp)(v)
    torch.testing.assert_close(got, ref, rtol=1e-10, atol=1e-12)


@pytest.mark.gpu
def test_dipole_operator_kernels_match_cpu():
    pos, cell, q, d, Q = _system(n=300, L=20.0, seed=7)
    mol = torch.arange(300) // 3
    pol = 0.6 + 0.6 * torch.rand(300, generator=torch.Generator().manual_seed(8))
    v = 0.2 * torch.randn(300, 3, generator=torch.Generator().manual_seed(9))
    setup = M.EwaldSetup(alpha=0.4, cutoff=7.0, mesh=(32, 32, 32), order=5, fft_dtype=torch.float64)
    mod = M.PolarizableMultipoles(setup)
    pairs = mod.pairs(pos, cell, mol)
    ref = M.DipoleOperator(mod, pos, cell, pairs, pol)(v)
    dev = torch.device("cuda")
    modg = M.PolarizableMultipoles(setup)
    pg = tuple(t.to(dev) for t in pairs)
    op = M.DipoleOperator(modg, pos.to(dev), cell.to(dev), pg, pol.to(dev))
    assert op.kernel, "the dipole pair kernels did not load"
    got = op(v.to(dev)).cpu()
    torch.testing.assert_close(got, ref, rtol=1e-9, atol=1e-11)


@pytest.mark.gpu
def test_direct_reciprocal_field_matches_energy_gradient():
    """The reciprocal dipole field by spread / FFT / gather (no graph) against the gradient of the
    reciprocal energy on the same float32 mesh."""
    dev = torch.device("cuda")
    pos, cell, q, d, Q = _system(n=500, L=22.0, seed=11)
    pos, cell = pos.to(dev), cell.to(dev)
    v = (0.2 * torch.randn(500, 3, generator=torch.Generator().manual_seed(12), dtype=torch.float64)).to(dev)
    mod = M.PolarizableMultipoles(M.EwaldSetup(alpha=0.4, cutoff=7.0, mesh=(40, 40, 40), order=5,
                                               fft_dtype=torch.float32))
    pairs = mod.pairs(pos, cell, None)
    op = M.DipoleOperator(mod, pos, cell, pairs, None)
    assert op._direct_setup()
    got = op.recip(v)
    vv = v.clone().requires_grad_(True)
    e = mod.recip(pos, cell, v.new_zeros(500), vv, v.new_zeros(500, 3, 3))
    (g,) = torch.autograd.grad(e, vv)
    torch.testing.assert_close(got, -g, rtol=1e-4, atol=1e-6 * float(g.abs().max()))


def test_pairs_split_over_receiver_ranges():
    """Receiver-range searches give disjoint pair sets whose union is the full set, and each
    range holds a share close to its atoms' share."""
    pos, cell, q, d, Q = _system(n=60, L=12.0, seed=9)
    mol = torch.arange(60) // 3
    full = M.multipole_pairs(pos, cell, 5.0, mol)

    def keyset(pairs):
        i, j, s, ex = pairs
        out = set()
        for a, b, sh, e in zip(i.tolist(), j.tolist(), s.tolist(), ex.tolist()):
            if (a, b) > (b, a) or (a == b and tuple(sh) < (0, 0, 0)):
                a, b, sh = b, a, [-x for x in sh]
            out.add((min(a, b), max(a, b), tuple(sh) if a <= b else tuple(-x for x in sh), e))
        return out

    ref = keyset(full)
    parts = [M.multipole_pairs(pos, cell, 5.0, mol, receivers=r) for r in ((0, 20), (20, 41), (41, 60))]
    sets = [keyset(p) for p in parts]
    assert sum(len(x) for x in sets) == len(ref)
    assert set().union(*sets) == ref
    for x in sets:
        assert 0.2 * len(ref) < len(x) < 0.5 * len(ref)
