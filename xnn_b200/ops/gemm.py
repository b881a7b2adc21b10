"""Matrix products of the hot paths on the sm_100a tensor cores (``csrc/gemm_tc.cu``).

:func:`matmul` computes ``X @ W`` for float32 CUDA operands with a tcgen05 kernel accumulating
in TMEM, using the 3xTF32 split so the result keeps float32 accuracy; it is differentiable to
any order (its backward products run through :func:`matmul` / :func:`matmul_t` again).
:func:`mm_raw` / :func:`mm_t_raw` are the same products without autograd (with an optional
per-column scale).
Other dtypes, devices or shapes fall back to ``torch.mm``. ``XNN_B200_TC_GEMM=0`` disables
the tensor-core path.
"""
from __future__ import annotations

import os
from typing import Dict, Optional

import torch
from torch import Tensor
from torch.autograd import Function

from .. import _ext
from .modes import MODES

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


def mm_act(X: Tensor, W: Tensor, mode: int, c: float) -> Optional[Tensor]:
    """``X @ W`` with the activation fused into the tensor-core epilogue: ``mode`` 1 gives
    ``c silu(XW)``; ``mode`` 2 treats the output columns as ``[a | a']`` and gives
    ``[c silu(a) | c silu'(a) a']`` (``W`` block-diagonal over the two halves). ``None`` when the
    kernel does not take the operands (the caller evaluates the stages separately)."""
    if not supported(X, W):
        return None
    return _ext.ops().gemm_tf32x3(X, W, None, _status(X.device), SPIN_LIMIT, int(mode), float(c))


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
    """``X^T @ D`` summed over the rows, without autograd (tensor cores, deterministic split-K;
    ``(D^T X)^T`` when only the swapped operands fit the kernel)."""
    if reduce_supported(X, D):
        return _ext.ops().gemm_reduce_tf32x3(X, D, rows_per_cta(X.shape[0]), 1.0, _status(X.device), SPIN_LIMIT)
    if reduce_supported(D, X):
        return _ext.ops().gemm_reduce_tf32x3(D, X, rows_per_cta(D.shape[0]), 1.0, _status(D.device), SPIN_LIMIT).t()
    return X.t() @ D


# --------------------------------------------------------------------------- differentiable products
class _MM(Function):
    """``X @ W`` on the tensor cores; its derivatives are products of the same two kinds, so it
    differentiates to any order (force training takes second derivatives through node linears)."""

    @staticmethod
    def forward(ctx, X: Tensor, W: Tensor) -> Tensor:
        ctx.save_for_backward(X, W)
        return mm_raw(X.contiguous(), W)

    @staticmethod
    def backward(ctx, G: Tensor):
        X, W = ctx.saved_tensors
        gX = matmul(G, W.t()) if ctx.needs_input_grad[0] else None
        # a force pass differentiates only towards the positions: no weight gradient is used
        gW = matmul_t(X, G) if ctx.needs_input_grad[1] and not MODES.force_pass else None
        return gX, gW


class _MMT(Function):
    """``X^T @ D`` (a reduction over the rows) on the tensor cores."""

    @staticmethod
    def forward(ctx, X: Tensor, D: Tensor) -> Tensor:
        ctx.save_for_backward(X, D)
        return mm_t_raw(X.contiguous(), D.contiguous())

    @staticmethod
    def backward(ctx, G: Tensor):
        X, D = ctx.saved_tensors
        gX = matmul(D, G.t()) if ctx.needs_input_grad[0] else None
        gD = matmul(X, G) if ctx.needs_input_grad[1] else None
        return gX, gD


def _column_block(N: int) -> int:
    """Largest multiple of 16 up to 256 dividing ``N`` (0: none)."""
    for c in range(256, 15, -16):
        if N % c == 0:
            return c
    return 0


#: below this many rows the library GEMM wins: a 128-row tile per CTA leaves most SMs idle
MIN_ROWS = int(os.environ.get("XNN_B200_TC_MIN_ROWS", "16384"))


def _tc_ok(X: Tensor, W: Tensor) -> bool:
    rows = X.numel() // max(X.shape[-1], 1) if X.dim() else 0
    return (enabled() and X.is_cuda and X.dtype == torch.float32 and W.dtype == torch.float32
            and rows >= MIN_ROWS and _ext.cuda_available())


def matmul(X: Tensor, W: Tensor) -> Tensor:
    """``X @ W`` for ``X (..., K)``, ``W (K, N)``: tensor cores for float32 CUDA operands
    (columns in blocks when ``N > 512``), ``torch.matmul`` otherwise."""
    if not _tc_ok(X, W) or X.shape[-1] == 0:
        return X @ W
    lead = X.shape[:-1]
    X2 = X.reshape(-1, X.shape[-1])
    N = W.shape[1]
    if 16 <= N <= 512 and N % 16 == 0:
        Y = _MM.apply(X2, W)
    else:
        c = _column_block(N)
        if c == 0:
            return X @ W
        Y = torch.cat([_MM.apply(X2, W[:, j:j + c]) for j in range(0, N, c)], dim=1)
    return Y.reshape(*lead, N)


def matmul_t(X: Tensor, D: Tensor) -> Tensor:
    """``X^T @ D`` summed over the rows of ``X (M, K1)`` and ``D (M, N)``."""
    if not _tc_ok(X, D):
        return X.t() @ D
    Xc, Dc = X.contiguous(), D.contiguous()
    if reduce_supported(Xc, Dc):
        return _MMT.apply(X, D)
    if reduce_supported(Dc, Xc):
        return _MMT.apply(D, X).t()
    return X.t() @ D
