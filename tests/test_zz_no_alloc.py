"""The allocation-free split-K GEMM entry point (mfb200_splitk_gemm_noalloc).

It exists for callers that cannot allocate GPU memory (code living inside
another framework's memory pool, or a search thread that must not take the
driver's allocation locks mid-game): its scratch is a fixed device array inside
the library. This test calls it through the C ABI several times in a row, with
different shapes (a ragged M, more slices than K blocks), and compares each
result with an fp64 host product of the same bf16 operands plus the bias,
within the split-K tolerance of tests/test_gemm_gpu.py; the first shape is
also checked against the library's existing GEMM entry point
(mfb200_debug_gemm, unsplit, fp32 output). The test allocates its own
input/output buffers (with torch); the entry point itself allocates nothing.
It sits in its own file, collected last.
"""
import ctypes

import numpy as np
import pytest

from metalfish_b200._lib import lib
from metalfish_b200.bf16 import from_bf16_bits, to_bf16_bits

pytestmark = pytest.mark.gpu


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def _reference(Ab, Wb, b, M, N, K):
    out = np.zeros((M, N), np.float32)
    st = ctypes.c_uint(0)
    rc = lib().mfb200_debug_gemm(M, N, K, 256 if N >= 256 else 64, 0, _p(Ab), _p(Wb), _p(b), 0, 0,
                                 None, ctypes.c_float(1.0), None, None, ctypes.c_float(0.0), None,
                                 ctypes.c_float(1.0), 1, 1, _p(out), ctypes.byref(st))
    assert rc == 0, f"debug gemm rc={rc}"
    return out


@pytest.mark.parametrize("shapes", [[(1024, 256, 2048, 7), (64, 128, 1024, 16),
                                     (300, 96, 256, 8), (130, 512, 1024, 3)]])
def test_noalloc_splitk_matches_existing_gemm(shapes):
    import torch
    L = lib()
    L.mfb200_splitk_gemm_noalloc.restype = ctypes.c_int
    L.mfb200_splitk_gemm_noalloc.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
                                             ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                             ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    L.mfb200_noalloc_last_error.restype = ctypes.c_char_p
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    rng = np.random.default_rng(7)
    for i, (M, N, K, splits) in enumerate(shapes):  # calls in a row: none may see stale scratch
        A = rng.standard_normal((M, K), dtype=np.float32)
        W = rng.standard_normal((N, K), dtype=np.float32) / np.float32(np.sqrt(K))
        b = (0.1 * rng.standard_normal(N)).astype(np.float32)
        Ab, Wb = to_bf16_bits(A), to_bf16_bits(W)
        dA = torch.from_numpy(Ab.view(np.int16)).to(dev)
        dW = torch.from_numpy(Wb.view(np.int16)).to(dev)
        db = torch.from_numpy(b).to(dev)
        dout = torch.full((M, N), float("nan"), dtype=torch.float32, device=dev)
        torch.cuda.synchronize(dev)
        rc = L.mfb200_splitk_gemm_noalloc(dA.data_ptr(), dW.data_ptr(), M, N, K, splits,
                                          db.data_ptr(), dout.data_ptr(), None)
        assert rc == 0, L.mfb200_noalloc_last_error().decode()
        torch.cuda.synchronize(dev)
        got = dout.cpu().numpy()
        exact = (from_bf16_bits(Ab).astype(np.float64) @ from_bf16_bits(Wb).astype(np.float64).T
                 + b.astype(np.float64))
        np.testing.assert_allclose(got, exact, rtol=1e-4, atol=1e-3)
        if i == 0:
            np.testing.assert_allclose(got, _reference(Ab, Wb, b, M, N, K), rtol=1e-4, atol=1e-3)


def test_noalloc_rejects_oversize():
    L = lib()
    L.mfb200_splitk_gemm_noalloc.restype = ctypes.c_int
    L.mfb200_noalloc_last_error.restype = ctypes.c_char_p
    rc = L.mfb200_splitk_gemm_noalloc(ctypes.c_void_p(16), ctypes.c_void_p(16), 4096, 1024, 1024,
                                      4, None, ctypes.c_void_p(16), None)
    assert rc != 0
    assert b"exceeds" in L.mfb200_noalloc_last_error()
