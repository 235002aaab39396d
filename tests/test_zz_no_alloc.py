"""tb_linear_static_scratch: the split-K projection for callers that cannot
allocate device memory (code inside a custom allocator, or next to a
framework that has reserved all device memory for its own pool).  Its
partial tiles live in an array built into the library instead of
caller-provided scratch.

Checked through the C ABI against tb_linear with caller-owned scratch on the
same inputs, for two calls in a row (the second reuses the array the first
left behind), plus the size limit.  This file is collected last so a failure
here never hides the rest of the suite; it also passes on its own in a fresh
process.
"""
from __future__ import annotations

import ctypes
import math
from ctypes import c_float, c_int, c_size_t, c_void_p

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

from tinybatch_b200 import _native  # noqa: E402

TB_STATIC_SCRATCH_BYTES = 8 << 20


def _lib():
    lib = _native.load()
    fn = lib.tb_linear_static_scratch
    fn.restype = c_int
    fn.argtypes = [c_void_p, c_int, c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_int, c_int,
                   c_float, c_float, c_void_p, c_int, c_int, c_int, c_int, c_void_p]
    return lib


def _static(lib, x, w, out, bn, splits):
    M, K = x.shape
    N = w.shape[0]
    return lib.tb_linear_static_scratch(x.data_ptr(), K, w.data_ptr(), K, M, N, K, None, 0, 0,
                                        0.0, 0.0, out.data_ptr(), out.stride(0), 1, bn, splits,
                                        torch.cuda.current_stream().cuda_stream)


def _reference(lib, x, w, out, bn, splits):
    M, K = x.shape
    N = w.shape[0]
    need = lib.tb_gemm_scratch_bytes(M, N, bn, splits)
    ws = torch.zeros(max(need, 256), dtype=torch.uint8, device="cuda")
    rc = lib.tb_linear(x.data_ptr(), K, w.data_ptr(), K, M, N, K, None, 0, 0, 0.0, 0.0,
                       out.data_ptr(), out.stride(0), 1, bn, splits, ws.data_ptr(), ws.numel(),
                       None, torch.cuda.current_stream().cuda_stream)
    return rc


def _inputs(M, N, K, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16).cuda()
    w = (torch.randn(N, K, generator=g) / math.sqrt(K)).to(torch.bfloat16).cuda()
    return x, w


def test_static_scratch_matches_caller_scratch_twice():
    lib = _lib()
    _native.status(clear=True)
    for seed, (M, N, K, bn, splits) in enumerate([(128, 512, 2048, 128, 4),
                                                  (100, 384, 1024, 64, 3)]):
        x, w = _inputs(M, N, K, seed)
        got = torch.full((M, N), float("nan"), device="cuda")
        want = torch.full((M, N), float("nan"), device="cuda")
        assert _static(lib, x, w, got, bn, splits) == 0, lib.tb_last_error()
        assert _reference(lib, x, w, want, bn, splits) == 0, lib.tb_last_error()
        torch.cuda.synchronize()
        torch.testing.assert_close(got, want, atol=2e-3, rtol=2e-3)
        torch.testing.assert_close(got, x.float() @ w.float().t(), atol=2e-3, rtol=2e-3)
    assert _native.status(clear=True) == 0


def test_static_scratch_rejects_oversized_calls():
    lib = _lib()
    M, N, K, bn, splits = 128, 8192, 1024, 256, 4     # 32 tiles x 4 splits x 128 KiB > 8 MiB
    x, w = _inputs(M, N, K, 7)
    out = torch.empty(M, N, device="cuda")
    rc = _static(lib, x, w, out, bn, splits)
    assert rc == 1
    assert b"built-in array" in lib.tb_last_error()
