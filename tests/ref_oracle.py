"""The reference framework (installed under ``baseline/_ref``) as an oracle: load its module, copy
a batch into its graph type and compare energies / forces / stress of the same state dict."""
import importlib
import os
import sys
import warnings

import pytest
import torch

from xnn_b200.data import collate, structure_to_graph, synthetic
from xnn_b200.models import ForceStressOutput

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "baseline", "_ref")


def _stub_e3nn():
    """The reference's equivariant models import ``e3nn`` (absent here). It is stood in for by this
    framework's own ``xnn_b200.o3`` (the same conventions: irreps, real spherical harmonics, Wigner
    3j, path-normalised linear and tensor-product layers, normalised MLPs), so the reference's
    models run as oracles for the model logic; names this framework does not provide become
    placeholder types that refuse to be used."""
    import importlib.util
    import types
    if "e3nn" in sys.modules or importlib.util.find_spec("e3nn") is not None:
        return
    import xnn_b200.o3 as mine

    class _Absent:
        def __init__(self, *args, **kwargs):
            raise ImportError("e3nn is not installed")

    def _attr(name):
        if name.startswith("__"):        # module dunders (__file__, __path__, ...) stay absent
            raise AttributeError(name)
        return type(name, (_Absent,), {})

    class _Entry:
        # the entry points e3nn's subclasses call
        def _compiled_main_left_right(self, x, y, w):
            return mine.TensorProduct.forward(self, x, y, w)

        def _get_weights(self, w):
            return self.weight if w is None else w

    class TensorProduct(_Entry, mine.TensorProduct):
        pass

    class FullyConnectedTensorProduct(_Entry, mine.FullyConnectedTensorProduct):
        pass

    class Linear(mine.Linear):
        def _compiled_main(self, x, w=None, b=None):
            return mine.Linear.forward(self, x, w, b)

    provided = {"o3": {k: getattr(mine, k) for k in dir(mine) if not k.startswith("_")},
                "nn": {"FullyConnectedNet": mine.FullyConnectedNet},
                "math": {"normalize2mom": mine.normalize2mom}}
    provided["o3"]["TensorProduct"] = TensorProduct
    provided["o3"]["Linear"] = Linear
    provided["o3"]["FullyConnectedTensorProduct"] = FullyConnectedTensorProduct
    pkg = types.ModuleType("e3nn")
    _opt = {"jit_script_fx": True, "specialized_code": True, "optimize_einsums": True}
    pkg.get_optimization_defaults = lambda: dict(_opt)
    pkg.set_optimization_defaults = lambda **kw: _opt.update(kw)
    for sub in ("o3", "nn", "math"):
        mod = types.ModuleType("e3nn." + sub)
        for k, v in provided[sub].items():
            setattr(mod, k, v)
        mod.__getattr__ = _attr
        setattr(pkg, sub, mod)
        sys.modules["e3nn." + sub] = mod
    sys.modules["e3nn"] = pkg


def ref_module(name):
    if not os.path.isdir(os.path.join(REF, "xnn")):
        pytest.skip("reference framework not installed under baseline/_ref")
    if REF not in sys.path:
        sys.path.insert(0, REF)
    _stub_e3nn()
    with warnings.catch_warnings():
        warnings.simplefilter("ignore")
        return importlib.import_module(name)


def batch(periodic=False, cutoff=5.0, n=3, species=None, seed=2):
    if periodic:
        ss = synthetic.triclinic_crystals(2, seed=5, labels=False)
        for s in ss:
            s["atomic_numbers"] = torch.full_like(s["atomic_numbers"], 8)
    else:
        ss = synthetic.organic_molecules(n, seed=seed, labels=False)
    if species is not None:
        for s in ss:
            z = s["atomic_numbers"]
            s["atomic_numbers"] = torch.as_tensor(species)[torch.arange(len(z)) % len(species)]
    return collate([structure_to_graph(s, cutoff) for s in ss])


def ref_graph(b, **extra):
    ad = ref_module("xnn.common.data")
    return ad.AtomicGraph(pos=b.pos.clone(), atomic_numbers=b.atomic_numbers, edge_index=b.edge_index,
                          cell_shifts=b.cell_shifts, batch=b.batch, n_atoms=b.n_atoms, cell=b.cell, pbc=b.pbc,
                          **extra)


def load_same_weights(mine, ref):
    missing, unexpected = mine.load_state_dict(ref.state_dict(), strict=False)
    assert not missing and not unexpected, (missing, unexpected)


def compare(mine, ref, b, periodic=False, rtol=1e-10, atol=1e-11, keys=(), **extra):
    outs = ref_module("xnn.common.models.outputs")
    o_ref = outs.ForceStressOutput(ref, compute_stress=periodic)(ref_graph(b, **extra))
    g = b.clone()
    for k, v in extra.items():
        setattr(g, k, v)
    o = ForceStressOutput(mine, compute_stress=periodic)(g)
    torch.testing.assert_close(o["energy"], o_ref["energy"], rtol=rtol, atol=atol)
    torch.testing.assert_close(o["forces"], o_ref["forces"], rtol=rtol, atol=atol)
    if periodic:
        torch.testing.assert_close(o["stress"], o_ref["stress"], rtol=rtol, atol=atol)
    for k in keys:
        torch.testing.assert_close(o[k], o_ref[k], rtol=rtol, atol=atol)
    return o, o_ref
