"""tcgen05 GEMM (mg_gemm_bf16) against an fp32 PyTorch product of the same bf16 inputs.

Products of bf16 values are exact in fp32, so the only difference is the
summation order of the fp32 accumulation: |C - ref| <= 1e-5 * K * max|A||B|.
"""

from __future__ import annotations

import ctypes

import pytest

from mogemma_b200 import _core

pytestmark = pytest.mark.gpu

_lib = _core.lib()
_lib.mg_gemm_bf16.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p,
                              ctypes.c_int64, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_void_p,
                              ctypes.c_void_p]
_lib.mg_gemm_bf16.restype = ctypes.c_int


def _gemm(torch, a, b, n_cols=None):
    M, K = a.shape
    N = b.shape[0]
    c = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = _lib.mg_gemm_bf16(a.data_ptr(), a.stride(0), b.data_ptr(), b.stride(0), c.data_ptr(), c.stride(0), M, N, K,
                           err.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert rc == 0, _lib.mg_last_error().decode()
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    return c


# Fewer 128 x 256 tiles than SMs: one 128 x 128 tile per CTA; otherwise the
# persistent kernel (128 x 256 tiles, two TMEM accumulators), here with several
# tiles per CTA (288, 320 and 160 tiles on 148 SMs) and ragged rows / columns.
@pytest.mark.parametrize(("M", "N", "K"), [(128, 128, 64), (256, 384, 1152), (300, 700, 512), (1, 1536, 1152),
                                           (513, 129, 6912), (4096, 2304, 768), (8191, 1280, 1152),
                                           (5000, 1000, 256)])
def test_gemm_matches_fp32_product(M: int, N: int, K: int) -> None:
    torch = pytest.importorskip("torch")
    g = torch.Generator(device="cpu").manual_seed(M * 7 + N)
    a = (torch.randn(M, K, generator=g) * 0.5).to(torch.bfloat16).cuda()
    b = (torch.randn(N, K, generator=g) * 0.02).to(torch.bfloat16).cuda()
    c = _gemm(torch, a, b)
    ref = a.float() @ b.float().T
    tol = 1e-5 * K * float(a.float().abs().max()) * float(b.float().abs().max())
    assert float((c - ref).abs().max()) <= tol


def test_gemm_rejects_bad_k() -> None:
    torch = pytest.importorskip("torch")
    a = torch.zeros(4, 100, dtype=torch.bfloat16, device="cuda")
    c = torch.zeros(4, 4, dtype=torch.float32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = _lib.mg_gemm_bf16(a.data_ptr(), 100, a.data_ptr(), 100, c.data_ptr(), 4, 4, 4, 100, err.data_ptr(), None)
    assert rc == 1 and "multiple of 64" in _lib.mg_last_error().decode()
