"""PM3 on the NDDO machinery against the reference implementation (run on the CPU with the synthetic
parameter file ``tests/data/nddo_test_params.txt``; values in ``tests/data/pm3_gold.json``)."""
import json
import math
from pathlib import Path

import pytest
import torch

from xnn_b200.data import collate as batch_graphs
from xnn_b200.data.dataset import structure_to_graph
from xnn_b200.sqm import PM3, load_parameters, save_parameters
from xnn_b200.sqm import integrals as I

DATA = Path(__file__).parent / "data"
PARAMS = DATA / "nddo_test_params.txt"
GOLD = json.loads((DATA / "pm3_gold.json").read_text())


def _graph(rec, name, dtype=torch.float64, device="cpu"):
    d = structure_to_graph({"pos": torch.tensor(rec["pos"], dtype=dtype), "atomic_numbers": torch.tensor(rec["z"])},
                           cutoff=5.0)
    if name == "hydronium":
        d.total_charge = torch.tensor([1.0])
    if name == "methyl":
        d.spin_multiplicity = torch.tensor([2])
    return d.to(device) if device != "cpu" else d


@pytest.mark.parametrize("name", sorted(GOLD))
def test_pm3_matches_reference(name):
    rec = GOLD[name]
    model = PM3(PARAMS)
    d = _graph(rec, name)
    d.pos.requires_grad_(True)
    out = model(d)
    forces = -torch.autograd.grad(out["energy"].sum(), d.pos)[0]
    assert out["heat_of_formation"].item() == pytest.approx(rec["heat_of_formation"][0], abs=2e-6)
    assert out["electronic_energy"].item() == pytest.approx(rec["electronic_energy"][0], abs=1e-6)
    assert out["core_core_energy"].item() == pytest.approx(rec["core_core_energy"][0], abs=1e-9)
    torch.testing.assert_close(forces, torch.tensor(rec["forces"], dtype=torch.float64), atol=1e-6, rtol=0)
    torch.testing.assert_close(out["charges"], torch.tensor(rec["charges"], dtype=torch.float64), atol=1e-7, rtol=0)
    torch.testing.assert_close(out["dipole"].reshape(-1), torch.tensor(rec["dipole"], dtype=torch.float64), atol=1e-7, rtol=0)


def test_batch_equals_single():
    names = ["water", "methyl", "nmf", "hydronium", "h2s"]
    model = PM3(PARAMS)
    graphs = [_graph(GOLD[n], n) for n in names]
    out = model(batch_graphs(graphs))
    ref = torch.tensor([GOLD[n]["heat_of_formation"][0] for n in names], dtype=torch.float64)
    torch.testing.assert_close(out["heat_of_formation"], ref, atol=2e-6, rtol=0)


def test_forces_finite_difference():
    rec = GOLD["formaldehyde"]
    model = PM3(PARAMS)
    d = _graph(rec, "formaldehyde")
    d.pos.requires_grad_(True)
    e = model(d)["energy"].sum()
    g = torch.autograd.grad(e, d.pos)[0]
    h = 1e-5
    for atom, axis in ((0, 2), (2, 1), (1, 0)):
        p = d.pos.detach().clone()
        p[atom, axis] += h
        ep = model(_with_pos(d, p))["energy"].item()
        p[atom, axis] -= 2 * h
        em = model(_with_pos(d, p))["energy"].item()
        assert (ep - em) / (2 * h) == pytest.approx(g[atom, axis].item(), abs=1e-6)


def _with_pos(d, p):
    e = d.clone() if hasattr(d, "clone") else d
    e.pos = p
    return e


def test_parameter_gradient_of_energy():
    rec = GOLD["water"]
    model = PM3(PARAMS, trainable=("BETAP", "GSS"))
    e = model(_graph(rec, "water"))["energy"].sum()
    gb, gg = torch.autograd.grad(e, [model.p_BETAP, model.p_GSS])
    h = 1e-6
    for tab, grad, z in ((model.p_BETAP, gb, 8), (model.p_GSS, gg, 1)):
        with torch.no_grad():
            tab[z] += h
        ep = model(_graph(rec, "water"))["energy"].item()
        with torch.no_grad():
            tab[z] -= 2 * h
        em = model(_graph(rec, "water"))["energy"].item()
        with torch.no_grad():
            tab[z] += h
        assert (ep - em) / (2 * h) == pytest.approx(grad[z].item(), rel=1e-5, abs=1e-8)


def test_parameter_file_round_trip(tmp_path):
    p = load_parameters(PARAMS)
    q = load_parameters(save_parameters(p, tmp_path / "x.txt", comment="round trip"))
    assert q.elements == p.elements and q.pairs == p.pairs
    model = PM3(PARAMS)
    r = load_parameters(save_parameters(model.parameter_set(), tmp_path / "y.txt"))
    assert r.elements[8]["BETAP"] == p.elements[8]["BETAP"]
    with pytest.raises(FileNotFoundError):
        load_parameters("pm3-not-there")


def test_sto_overlap_closed_forms():
    r = torch.tensor([0.7, 1.4, 3.0], dtype=torch.float64)
    z = torch.full_like(r, 1.2)
    rho = z * r
    s = I.sto_overlap(1, 0, z, 1, 0, z, r)
    torch.testing.assert_close(s, torch.exp(-rho) * (1 + rho + rho ** 2 / 3), atol=1e-13, rtol=0)
    # 2p-pi with equal exponents: exp(-rho) (1 + rho + 2 rho^2 / 5 + rho^3 / 15)
    s = I.sto_overlap(2, 1, z, 2, 1, z, r, pi=True)
    ref = torch.exp(-rho) * (1 + rho + 2 * rho ** 2 / 5 + rho ** 3 / 15)
    torch.testing.assert_close(s, ref, atol=1e-13, rtol=0)
    # unequal exponents cross the series / recursion switch of the B integrals
    za, zb = torch.full_like(r, 2.5), torch.full_like(r, 0.9)
    s1 = I.sto_overlap(2, 0, za, 1, 0, zb, r * 3.0)
    s2 = I.sto_overlap(1, 0, zb, 2, 0, za, r * 3.0)
    torch.testing.assert_close(s1, s2, atol=1e-13, rtol=0)


def test_one_center_limit_of_multipoles():
    """At zero separation the point-charge model reproduces Gss, Hsp and (p_z p_x | p_z p_x) = (Gpp - Gp2) / 2."""
    model = PM3(PARAMS)
    el = model._elements([6], torch.device("cpu"), torch.float64)
    d = I._separations(el["dd"], el["qq"])
    rho = I._slot_rho(el["rho"])
    W = I.local_repulsion(torch.tensor([1e-9], dtype=torch.float64), d, rho, d, rho)[0]
    tab = el["table"]
    assert W[0, 0, 0, 0].item() == pytest.approx(tab["GSS"].item(), rel=1e-9)
    assert W[0, 3, 0, 3].item() == pytest.approx(tab["HSP"].item(), rel=1e-9)
    assert W[3, 1, 3, 1].item() == pytest.approx(0.5 * (tab["GPP"] - tab["GP2"]).item(), rel=1e-9)


@pytest.mark.gpu
def test_pm3_cuda_matches_cpu():
    names = ["water", "methanol_dimer", "methyl", "nmf"]
    model = PM3(PARAMS)
    cpu = model(batch_graphs([_graph(GOLD[n], n) for n in names]))
    gpu_model = PM3(PARAMS).cuda()
    d = batch_graphs([_graph(GOLD[n], n) for n in names]).to("cuda")
    d.pos.requires_grad_(True)
    out = gpu_model(d)
    f = -torch.autograd.grad(out["energy"].sum(), d.pos)[0]
    torch.testing.assert_close(out["heat_of_formation"].cpu(), cpu["heat_of_formation"], atol=1e-6, rtol=0)
    ref_f = torch.cat([torch.tensor(GOLD[n]["forces"], dtype=torch.float64) for n in names])
    torch.testing.assert_close(f.cpu(), ref_f, atol=1e-6, rtol=0)
