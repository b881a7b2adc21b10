"""Allocation-free C entry point of the tensor-core reduction GEMM, called through its exported
symbol with ctypes and checked against the allocating entry point and an fp64 reference.

The file name sorts last so that it also runs after every other test module."""
import ctypes

import pytest
import torch

from xnn_b200 import _ext

pytestmark = pytest.mark.gpu

ERR_SCRATCH = -1
ERR_SHAPE = -2
SCRATCH_FLOATS = 2 * 1024 * 1024


def _lib():
    if not _ext.cuda_available():
        pytest.fail(f"native extension not loaded: {_ext.error()}")
    lib = ctypes.CDLL(_ext.ops().__file__)
    f = lib.xnn_gemm_reduce_tf32x3_noalloc
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p,
                  ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_void_p, ctypes.c_void_p]
    lib.xnn_gemm_reduce_noalloc_setup.restype = ctypes.c_int
    lib.xnn_gemm_reduce_noalloc_status.restype = ctypes.c_int
    lib.xnn_gemm_reduce_noalloc_status.argtypes = [ctypes.POINTER(ctypes.c_int)]
    lib.xnn_gemm_reduce_noalloc_error_string.restype = ctypes.c_char_p
    lib.xnn_gemm_reduce_noalloc_error_string.argtypes = [ctypes.c_int]
    return lib


def _auto_rows(M, K1, N):
    ctas = min(296, SCRATCH_FLOATS // (K1 * N))
    r = -(-M // ctas)
    return max(256, -(-r // 32) * 32)


def _call(lib, X, D, rows_per_cta, scale):
    M, K1 = X.shape
    N = D.shape[1]
    out = torch.empty(K1, N, device=X.device, dtype=torch.float32)
    stream = torch.cuda.current_stream(X.device).cuda_stream
    rc = lib.xnn_gemm_reduce_tf32x3_noalloc(M, K1, N, X.data_ptr(), X.stride(0), D.data_ptr(), D.stride(0),
                                            rows_per_cta, scale, out.data_ptr(), stream)
    assert rc == 0, lib.xnn_gemm_reduce_noalloc_error_string(rc).decode()
    return out


def _existing(X, D, rows_per_cta, scale):
    status = torch.zeros(1, dtype=torch.int32, device=X.device)
    out = _ext.ops().gemm_reduce_tf32x3(X, D, rows_per_cta, scale, status, 50_000_000)
    assert int(status.item()) == 0
    return out


def _rel_err(out, X, D, scale):
    ref = scale * (X.double().t() @ D.double())
    return ((out.double() - ref).abs().max() / ref.abs().max().clamp_min(1e-30)).item()


def test_noalloc_matches_existing_entry_point_twice_in_a_row():
    lib = _lib()
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    assert lib.xnn_gemm_reduce_noalloc_setup() == 0
    g = torch.Generator(device=dev).manual_seed(7)
    cases = [
        # (M, K1, N, rows_per_cta passed to the C entry point, scale)
        (68000, 64, 64, 256, 1.0),
        (70000, 64, 384, 0, 0.5),  # automatic rows per CTA (the scratch limit picks 832)
    ]
    for M, K1, N, rows, scale in cases:
        X = torch.randn(M, K1, device=dev, generator=g)
        D = torch.randn(M, N, device=dev, generator=g)
        out = _call(lib, X, D, rows, scale)
        used = rows if rows else _auto_rows(M, K1, N)
        want = _existing(X, D, used, scale)
        torch.cuda.synchronize()
        assert torch.allclose(out, want, rtol=1e-6, atol=1e-6), (out - want).abs().max().item()
        assert _rel_err(out, X, D, scale) < 1e-5
    status = ctypes.c_int(-1)
    assert lib.xnn_gemm_reduce_noalloc_status(ctypes.byref(status)) == 0
    assert status.value == 0


def test_noalloc_rejects_oversized_scratch():
    lib = _lib()
    dev = torch.device("cuda:0")
    X = torch.zeros(70000, 128, device=dev)
    D = torch.zeros(70000, 512, device=dev)
    out = torch.full((128, 512), 3.0, device=dev)
    # 32 rows per CTA -> 2188 CTAs x 128 x 512 floats, far beyond the fixed scratch array
    rc = lib.xnn_gemm_reduce_tf32x3_noalloc(70000, 128, 512, X.data_ptr(), 128, D.data_ptr(), 512, 32, 1.0,
                                            out.data_ptr(), None)
    assert rc == ERR_SCRATCH
    assert b"scratch" in lib.xnn_gemm_reduce_noalloc_error_string(rc)
    torch.cuda.synchronize()
    assert bool((out == 3.0).all())  # nothing was launched


def test_noalloc_rejects_unsupported_widths():
    lib = _lib()
    dev = torch.device("cuda:0")
    X = torch.zeros(1024, 64, device=dev)
    # above 256 columns the product runs as two halves that must each be a multiple of 16
    for N in (272, 8, 528):
        D = torch.zeros(1024, N, device=dev)
        out = torch.full((64, N), 3.0, device=dev)
        rc = lib.xnn_gemm_reduce_tf32x3_noalloc(1024, 64, N, X.data_ptr(), 64, D.data_ptr(), N, 0, 1.0,
                                                out.data_ptr(), None)
        assert rc == ERR_SHAPE, (N, rc)
        assert b"multiple of 32" in lib.xnn_gemm_reduce_noalloc_error_string(rc)
        torch.cuda.synchronize()
        assert bool((out == 3.0).all())
