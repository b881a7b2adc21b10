"""Matrix products of the hot paths on the sm_100a tensor cores (``csrc/gemm_tc.cu``).

:func:`matmul` computes ``X @ W`` (optionally times a per-column scale) for float32 CUDA
operands with a tcgen05 kernel accumulating in TMEM, using the 3xTF32 split so the result
keeps float32 accuracy; it is differentiable (the backward products run through it as well).
Other dtypes, devices or shapes fall back to ``torch.mm``. ``XNN_B200_TC_GEMM=0`` disables
the tensor-core path.
"""
from __future__ import annotations

import os
from typing import Dict, Optional

import torch
from torch import Tensor

from .. import _ext

SPIN_LIMIT = 50_000_000
_STATUS: Dict[torch.device, Tensor] = {}


def _status(dev: torch.device) -> Tensor:
    t = _STATUS.get(dev)
    if t is None:
        t = torch.zeros(1, dtype=torch.int32, device=dev)
        _STATUS[dev] = t
    return t


def tc_status(dev: torch.device) -> int:
    """Non-zero when a tensor-core GEMM on ``dev`` gave up waiting for its MMAs (read syncs)."""
    t = _STATUS.get(dev)
    return 0 if t is None else int(t.item())


def enabled() -> bool:
    return os.environ.get("XNN_B200_TC_GEMM", "1") != "0"


def supported(X: Tensor, W: Tensor) -> bool:
    if not (enabled() and X.is_cuda and X.dtype == torch.float32 and W.dtype == torch.float32):
        return False
    if X.dim() != 2 or W.dim() != 2 or X.stride(1) != 1 or X.stride(0) % 4 or X.data_ptr() % 16:
        return False
    N = W.shape[1]
    if N < 16 or N > 512 or N % 16:
        return False
    parts = (N + 255) // 256
    return (N // parts) % 16 == 0 and (N // parts) * parts == N and _ext.cuda_available()


def mm_raw(X: Tensor, W: Tensor, col_scale: Optional[Tensor] = None) -> Tensor:
    """``X @ W`` (times ``col_scale``) without autograd."""
    if supported(X, W):
        return _ext.ops().gemm_tf32x3(X, W, col_scale, _status(X.device), SPIN_LIMIT)
    Y = X @ W
    return Y * col_scale if col_scale is not None else Y


def reduce_supported(X: Tensor, D: Tensor) -> bool:
    if not (enabled() and X.is_cuda and X.dtype == torch.float32 and D.dtype == torch.float32):
        return False
    if X.dim() != 2 or D.dim() != 2 or X.stride(1) != 1 or D.stride(1) != 1:
        return False
    K1, N = X.shape[1], D.shape[1]
    if K1 < 1 or K1 > 128 or N < 16 or N > 512 or N % 16:
        return False
    parts = (N + 255) // 256
    return (N // parts) % 16 == 0 and (N // parts) * parts == N and _ext.cuda_available()


def rows_per_cta(M: int, target_ctas: int = 296) -> int:
    r = -(-M // target_ctas)
    r = max(256, -(-r // 32) * 32)
    return r


def mm_t_raw(X: Tensor, D: Tensor) -> Tensor:
    """``X^T @ D`` summed over the rows, without autograd (tensor cores, deterministic split-K)."""
    if reduce_supported(X, D):
        return _ext.ops().gemm_reduce_tf32x3(X, D, rows_per_cta(X.shape[0]), 1.0, _status(X.device), SPIN_LIMIT)
    return X.t() @ D
