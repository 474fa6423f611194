"""tcgen05 GEMM kernel vs a float64 host product of the same bf16 inputs."""
import ctypes

import numpy as np
import pytest

from metalfish_b200._lib import lib
from metalfish_b200.bf16 import from_bf16_bits, round_bf16, to_bf16_bits

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True, params=[1, 0], ids=["pairs", "single"])
def gemm_kernel(request):
    """Every GEMM case runs through the CTA-pair kernel (where the shape
    selects it) and through the single-CTA kernel."""
    lib().mfb200_debug_set_gemm_pairs(request.param)
    yield request.param
    lib().mfb200_debug_set_gemm_pairs(1)


def _p(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def mish(x):
    return x * np.tanh(np.log1p(np.exp(x)))


def run_gemm(M, N, K, bn, mode=0, act=0, bias=True, alpha=0.5, seed=0, out_f32=False, k_splits=1,
             out_f16=False):
    rng = np.random.default_rng(seed)
    A = rng.standard_normal((M, K), dtype=np.float32)
    W = rng.standard_normal((N, K), dtype=np.float32) / np.float32(np.sqrt(K))
    b = rng.standard_normal(N, dtype=np.float32) * 0.1
    R = rng.standard_normal((M, N), dtype=np.float32)
    g = (1 + 0.1 * rng.standard_normal(N)).astype(np.float32)
    be = (0.1 * rng.standard_normal(N)).astype(np.float32)
    Ab, Wb = to_bf16_bits(A), to_bf16_bits(W)
    if k_splits > 1:
        bias, out_f32 = False, True
    b = b if bias else None
    out = np.zeros((k_splits, M, N), np.float32 if out_f32 else np.uint16)
    fmt = 2 if out_f16 else int(out_f32)
    st = ctypes.c_uint(0)
    rc = lib().mfb200_debug_gemm(M, N, K, bn, 0, _p(Ab), _p(Wb), _p(b), mode, act, _p(R),
                                 ctypes.c_float(alpha), _p(g), _p(be), ctypes.c_float(1e-3),
                                 None, ctypes.c_float(1.0), fmt, k_splits, _p(out),
                                 ctypes.byref(st))
    assert rc == 0, f"rc={rc} status={st.value}"
    acc = from_bf16_bits(Ab).astype(np.float64) @ from_bf16_bits(Wb).astype(np.float64).T
    if b is not None:
        acc = acc + b
    if mode in (1, 3):
        # in place (3), the residual is first rounded to the output format
        ref = (R.astype(np.float16).astype(np.float64) if (mode == 3 and out_f16) else R) + alpha * acc
    else:
        ref = {0: acc, 2: np.maximum(acc, 0) ** 2, 5: acc / (1 + np.exp(-acc)), 6: mish(acc)}[act]
    got = out.sum(0) if out_f32 else (out[0].view(np.float16).astype(np.float32) if out_f16 else
                                      from_bf16_bits(out[0]))
    return got, ref


@pytest.mark.parametrize("M,N,K,bn", [
    (128, 256, 64, 256),     # one tile, one k-block
    (128, 64, 64, 64),
    (256, 512, 1024, 256),
    (300, 3104, 1024, 256),  # ragged M, N not a multiple of the tile
    (512, 416, 1024, 256),   # partial last tile of 160 columns
    (384, 288, 1536, 256),   # partial last tile of 32 columns
    (1000, 1536, 1024, 128),
    (64, 4096, 256, 256),    # M smaller than one tile
    (517, 64, 192, 64),
])
def test_gemm_store(M, N, K, bn):
    got, ref = run_gemm(M, N, K, bn)
    err = np.abs(got - ref)
    tol = 1e-2 + 1e-2 * np.abs(ref)
    bad = err > tol
    assert not bad.any(), f"{bad.sum()} bad of {bad.size}; max err {err.max()} first {np.argwhere(bad)[:5]}"


@pytest.mark.parametrize("act", [2, 6])
def test_gemm_activation(act):
    got, ref = run_gemm(384, 1536, 1024, 256, act=act)
    np.testing.assert_allclose(got, ref, rtol=1e-2, atol=1e-2)


def test_gemm_residual():
    got, ref = run_gemm(257, 1024, 1536, 256, mode=1, alpha=0.427)
    np.testing.assert_allclose(got, ref, rtol=1e-2, atol=2e-2)


def test_gemm_residual_fp32_out():
    """fp32 residual stream: accumulate error only (no output rounding)."""
    got, ref = run_gemm(300, 1024, 1024, 256, mode=1, alpha=0.427, out_f32=True)
    np.testing.assert_allclose(got, ref, rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("M,N,K,bn", [(300, 1024, 1024, 256), (128, 768, 1536, 128), (517, 64, 192, 64)])
def test_gemm_accumulate_in_place(M, N, K, bn):
    """The residual GEMM of the forward: the fp32 residual stream is the output
    buffer and the TMA unit adds alpha*(A.W^T + bias) into it."""
    got, ref = run_gemm(M, N, K, bn, mode=3, alpha=0.427, out_f32=True)
    np.testing.assert_allclose(got, ref, rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("M,N,K,bn", [(300, 1024, 1024, 256), (517, 64, 192, 64)])
def test_gemm_accumulate_in_place_fp16(M, N, K, bn):
    """fp16 residual stream: one fp16 rounding of the sum (2^-11 relative)."""
    got, ref = run_gemm(M, N, K, bn, mode=3, alpha=0.427, out_f16=True)
    np.testing.assert_allclose(got, ref, rtol=2e-3, atol=2e-3)


@pytest.mark.parametrize("M,K,splits", [(1024, 2048, 16), (64, 2048, 32), (300, 1024, 5)])
def test_gemm_split_k(M, K, splits):
    """Split-K partial products sum to the full product (smolgen dense1 path)."""
    got, ref = run_gemm(M, 256, K, 256, k_splits=splits)
    np.testing.assert_allclose(got, ref, rtol=1e-4, atol=1e-3)


@pytest.mark.parametrize("M,N,K,bn", [(128, 256, 128, 256), (300, 1024, 1024, 256), (1000, 3104, 1024, 256),
                                      (200, 64, 512, 64)])
def test_gemm_fp8(M, N, K, bn):
    """kind::f8f6f4 e4m3 operands with per-column weight scales and an
    activation scale, vs float64 on the decoded operands."""
    from metalfish_b200.bf16 import from_e4m3_bits, to_e4m3_bits
    rng = np.random.default_rng(1)
    A = rng.standard_normal((M, K)).astype(np.float32) * 3
    W = rng.standard_normal((N, K)).astype(np.float32)
    a8, w8 = to_e4m3_bits(A), to_e4m3_bits(W)
    cs = (0.01 + 0.02 * rng.random(N)).astype(np.float32)
    b = (0.1 * rng.standard_normal(N)).astype(np.float32)
    a_scale = 0.5
    out = np.zeros((1, M, N), np.float32)
    st = ctypes.c_uint(0)
    rc = lib().mfb200_debug_gemm(M, N, K, bn, 1, _p(a8), _p(w8), _p(b), 0, 0, None, ctypes.c_float(1.0),
                                 None, None, ctypes.c_float(0.0), _p(cs), ctypes.c_float(a_scale), 1, 1,
                                 _p(out), ctypes.byref(st))
    assert rc == 0, f"rc={rc} status={st.value}"
    ref = (from_e4m3_bits(a8).astype(np.float64) @ from_e4m3_bits(w8).astype(np.float64).T) * a_scale * cs + b
    np.testing.assert_allclose(out[0], ref, rtol=1e-4, atol=1e-3)


@pytest.mark.parametrize("M,N,K,bn", [(128, 256, 256, 256), (300, 512, 1024, 256), (1000, 1024, 1536, 256),
                                      (200, 128, 512, 128), (4096, 1024, 1024, 256)])
def test_gemm_residual_layernorm(M, N, K, bn):
    """Fused residual + LayerNorm epilogue; a row spans N/bn cluster CTAs that
    exchange row statistics (the deepnorm LN(x + alpha*f) of every encoder
    layer)."""
    rng = np.random.default_rng(3)
    A = rng.standard_normal((M, K), dtype=np.float32)
    W = rng.standard_normal((N, K), dtype=np.float32) / np.float32(np.sqrt(K))
    b = (0.1 * rng.standard_normal(N)).astype(np.float32)
    R = (rng.standard_normal((M, N)) + 0.3).astype(np.float32)
    g = (1 + 0.1 * rng.standard_normal(N)).astype(np.float32)
    be = (0.1 * rng.standard_normal(N)).astype(np.float32)
    alpha = 0.427
    Ab, Wb = to_bf16_bits(A), to_bf16_bits(W)
    out = np.zeros((M, N), np.float32)
    out16 = np.zeros((M, N), np.uint16)
    st = ctypes.c_uint(0)
    rc = lib().mfb200_debug_gemm_ln(M, N, K, bn, _p(Ab), _p(Wb), _p(b), _p(R), ctypes.c_float(alpha),
                                    _p(g), _p(be), ctypes.c_float(1e-3), _p(out), _p(out16), ctypes.byref(st))
    assert rc == 0, f"rc={rc} status={st.value}"
    y = R + alpha * (from_bf16_bits(Ab).astype(np.float64) @ from_bf16_bits(Wb).astype(np.float64).T + b)
    mu = y.mean(1, keepdims=True)
    ref = (y - mu) / np.sqrt(y.var(1, keepdims=True) + 1e-3) * g + be
    np.testing.assert_allclose(out, ref, rtol=1e-3, atol=2e-3)
    np.testing.assert_allclose(from_bf16_bits(out16), ref, rtol=1e-2, atol=2e-2)


@pytest.mark.parametrize("M,N,K,bn", [(300, 1024, 1024, 256), (1000, 3104, 1024, 256), (517, 64, 192, 64)])
def test_gemm_fp16_operands(M, N, K, bn):
    """fp16 A and W (the GEMMs that read the fp16 residual stream)."""
    rng = np.random.default_rng(7)
    A = rng.standard_normal((M, K)).astype(np.float16)
    W = (rng.standard_normal((N, K)) / np.sqrt(K)).astype(np.float16)
    b = (rng.standard_normal(N) * 0.1).astype(np.float32)
    out = np.zeros((M, N), np.uint16)
    st = ctypes.c_uint(0)
    rc = lib().mfb200_debug_gemm(M, N, K, bn, 2, _p(A), _p(W), _p(b), 0, 0, None,
                                 ctypes.c_float(1.0), None, None, ctypes.c_float(1e-3),
                                 None, ctypes.c_float(1.0), 0, 1, _p(out), ctypes.byref(st))
    assert rc == 0, f"rc={rc} status={st.value}"
    ref = A.astype(np.float64) @ W.astype(np.float64).T + b
    np.testing.assert_allclose(from_bf16_bits(out), ref, rtol=1e-2, atol=1e-2)
