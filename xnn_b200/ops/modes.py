"""Which derivatives the fused ops may skip, scoped to one pass of autograd.

A force-loss training step differentiates twice. In the force pass
(``autograd.grad(E, pos)``) no parameter gradient is used, and in the parameter pass
(``loss.backward(inputs=params)``) no cotangent of a purely geometric input (the edge
vectors and their features) is used. The fused ops read these flags and skip that work;
a caller that needs full derivatives (Hessians, vibrations) simply does not set them.

The flags are process-wide, not thread-local: PyTorch runs the backward functions of CUDA
tensors on its own autograd worker thread, which would not see a thread-local value set by
the caller. A flag is only set around a synchronous autograd call, so within a process the
backward that reads it is the one its caller started.
"""
from __future__ import annotations

import contextlib


class _Modes:
    def __init__(self):
        self.force_pass = False
        self.params_only = False


MODES = _Modes()


@contextlib.contextmanager
def force_pass(enabled: bool = True):
    """Within: parameter gradients of the fused ops are not formed."""
    prev = MODES.force_pass
    MODES.force_pass = enabled
    try:
        yield
    finally:
        MODES.force_pass = prev


@contextlib.contextmanager
def params_only(enabled: bool = True):
    """Within: cotangents of geometric inputs (edge vectors, their features) are not formed."""
    prev = MODES.params_only
    MODES.params_only = enabled
    try:
        yield
    finally:
        MODES.params_only = prev
