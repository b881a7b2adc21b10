"""Loader of the compiled extension ``xnn_b200/_C*.so`` (sm_100a CUDA kernels + C++/OpenMP twins).

The extension is built in-tree by :func:`xnn_b200.build.build` (or ``__graft_entry__.build``).
On a machine with a CUDA device the extension is mandatory for the fused paths: every
op asks for it through :func:`ops` and fails loudly when it is missing instead of
silently running PyTorch code. CPU-only use works without it (PyTorch reference paths).
"""
from __future__ import annotations

import glob
import importlib.util
import os
import sys
import threading

_LOCK = threading.Lock()
_MOD = None
_ERR: str | None = None
_HERE = os.path.dirname(os.path.abspath(__file__))


def _find() -> str | None:
    cands = sorted(glob.glob(os.path.join(_HERE, "_C*.so")))
    return cands[0] if cands else None


def _load():
    global _MOD, _ERR
    with _LOCK:
        if _MOD is not None or _ERR is not None:
            return _MOD
        path = _find()
        if path is None or os.environ.get("XNN_B200_DISABLE_EXT") == "1":
            _ERR = "xnn_b200 native extension not built (run xnn_b200.build.build())"
            return None
        try:
            import torch  # noqa: F401  (the extension links against libtorch)
            spec = importlib.util.spec_from_file_location("xnn_b200._C", path)
            mod = importlib.util.module_from_spec(spec)
            spec.loader.exec_module(mod)
            sys.modules["xnn_b200._C"] = mod
            _MOD = mod
        except Exception as exc:  # pragma: no cover - depends on the build
            _ERR = f"failed to load {path}: {exc}"
        return _MOD


def available() -> bool:
    return _load() is not None


def cuda_available() -> bool:
    m = _load()
    return m is not None and bool(getattr(m, "HAS_CUDA", False))


def ops():
    """The extension module; raises when it is not built or failed to load."""
    m = _load()
    if m is None:
        raise RuntimeError(_ERR or "xnn_b200 native extension unavailable")
    return m


def error() -> str | None:
    _load()
    return _ERR
