"""Fast-path switch: mode validation, the auto policy, set_use_fast on wrappers, and the formulas
and kernels agreeing per model."""
import warnings

import pytest
import torch

from xnn_b200.models import fast
from xnn_b200.models.fast import AutoPolicy, FastPathPrecisionWarning, choose, resolve_use_fast, set_use_fast


def test_resolve_modes():
    assert resolve_use_fast(True) is True and resolve_use_fast(False) is False
    assert resolve_use_fast("AUTO") == "auto"
    with pytest.raises(ValueError):
        resolve_use_fast("fast")
    with pytest.raises(TypeError):
        resolve_use_fast(1)


def test_policy_cpu_and_bounds(monkeypatch):
    cpu = torch.device("cpu")
    assert not AutoPolicy().decide(cpu, torch.float32, 10 ** 6)
    assert AutoPolicy(cpu_min_edges=100).decide(cpu, torch.float32, 100)
    assert not AutoPolicy(cpu_min_edges=100).decide(cpu, torch.float32, 99)
    monkeypatch.setattr(torch.cuda, "get_device_name", lambda d=None: "NVIDIA B200")
    gpu = torch.device("cuda", 0)
    p = AutoPolicy(min_edges={"B200": 500, "H100": 50}, min_edges_float64={"B200": 5000}, default_min_edges=7,
                   max_edges={"b200": 10 ** 5})
    assert p.threshold(gpu) == 500 and p.threshold(gpu, torch.float64) == 5000
    assert not p.decide(gpu, torch.float32, 499) and p.decide(gpu, torch.float32, 500)
    assert not p.decide(gpu, torch.float32, 10 ** 5)
    monkeypatch.setattr(torch.cuda, "get_device_name", lambda d=None: "Other GPU")
    assert p.threshold(gpu) == 7 and p.decide(gpu, torch.float32, 10 ** 6)


def test_choose_and_warning(monkeypatch):
    cpu = torch.device("cpu")
    assert not choose(True, False, None, cpu, torch.float32, 10)
    assert not choose(False, True, None, cpu, torch.float32, 10)
    assert not choose("auto", True, AutoPolicy(), cpu, torch.float64, 10)
    monkeypatch.setitem(fast._WARNED, "float32", False)
    with pytest.warns(FastPathPrecisionWarning):
        assert choose(True, True, None, cpu, torch.float32, 10)
    with warnings.catch_warnings():
        warnings.simplefilter("error")
        assert choose(True, True, None, cpu, torch.float32, 10)     # once only
        assert choose(True, True, None, cpu, torch.float64, 10)


def test_set_use_fast_reaches_wrapped_models():
    from xnn_b200.models import build_model
    from xnn_b200.config import from_dict
    inner = build_model(from_dict({"model": {"name": "schnet", "n_features": 16, "n_interactions": 1,
                                             "n_rbf": 8, "cutoff": 4.0}}).model)
    outer = torch.nn.ModuleDict({"a": inner})
    set_use_fast(outer, False)
    assert inner.use_fast is False
    set_use_fast(outer, "auto")
    assert inner.use_fast == "auto"
    with pytest.raises(ValueError):
        set_use_fast(outer, "yes")


@pytest.mark.gpu
def test_tensornet_formulas_and_kernels_agree():
    from xnn_b200.data import collate, structure_to_graph, synthetic
    from xnn_b200.models import ForceStressOutput
    from xnn_b200.models.tensornet import TensorNet
    torch.manual_seed(0)
    m = TensorNet(n_features=32, n_interactions=2, n_rbf=8, cutoff=5.0, n_elements=90).double().cuda()
    crys = synthetic.triclinic_crystals(2, seed=4, n_min=8, n_max=14, labels=False)
    g = collate([structure_to_graph(s, 5.0) for s in crys]).to("cuda")
    g.pos, g.cell = g.pos.double(), g.cell.double()
    o_fast = ForceStressOutput(m.set_use_fast(True), compute_stress=True)(g.clone())
    o_ref = ForceStressOutput(m.set_use_fast(False), compute_stress=True)(g.clone())
    for k in ("energy", "forces", "stress"):
        torch.testing.assert_close(o_fast[k], o_ref[k], rtol=1e-9, atol=1e-10)


def test_tensornet_kernel_switch_records_mode():
    """With use_fast=False the ops never reach the kernels, forward or backward."""
    from xnn_b200.ops import tensornet_ops as T
    seen = []
    real = T._kernels
    try:
        T._kernels = lambda t: seen.append(T._allowed()) or real(t)
        a = torch.randn(4, 3, 3, 2, dtype=torch.float64, requires_grad=True)
        with T.kernels_enabled(False):
            y = T.matmul3(a, a)
        y.sum().backward()
        assert seen and not any(seen)
    finally:
        T._kernels = real
