"""The bounded-wait error path of the tcgen05 GEMMs, exercised without a GPU
fault: a test-only launch announces the bytes of one pipeline stage on its
mbarrier but never issues the loads (a barrier that nothing completes), with
every wait limited to 1 ms. The waits on that stage run out; the kernel
records a timeout code in the device status word, drains what it issued,
frees its TMEM and returns, and the context stays usable: ordinary GEMMs and
forwards afterwards are correct.
"""
import ctypes

import numpy as np
import pytest

from metalfish_b200 import synthetic
from metalfish_b200._lib import lib
from metalfish_b200.network import create_network
from tests.conftest import load_golden

pytestmark = pytest.mark.gpu

TIMEOUT_CODES = {1: "producer", 2: "mma", 3: "epilogue", 4: "drain", 5: "row statistics"}
LIMIT_NS = 1_000_000  # 1 ms


def gemm_ok(M, N, K, pair):
    """An ordinary GEMM on the same context matches an fp64 host product."""
    rng = np.random.default_rng(M + N + K)
    a = rng.standard_normal((M, K), dtype=np.float32)
    w = rng.standard_normal((N, K), dtype=np.float32) / np.sqrt(K)
    from metalfish_b200.bf16 import to_bf16_bits, from_bf16_bits
    ab, wb = to_bf16_bits(a), to_bf16_bits(w)
    out = np.empty((M, N), np.uint16)
    st = ctypes.c_uint(0)
    lib().mfb200_debug_set_gemm_pairs(1 if pair else 0)
    try:
        rc = lib().mfb200_debug_gemm(M, N, K, 256, 0, ab.ctypes.data, wb.ctypes.data, None, 0, 0,
                                     None, 1.0, None, None, 0.0, None, 1.0, 0, 1, out.ctypes.data,
                                     ctypes.byref(st))
    finally:
        lib().mfb200_debug_set_gemm_pairs(1)
    assert rc == 0 and st.value == 0
    ref = from_bf16_bits(ab).astype(np.float64) @ from_bf16_bits(wb).astype(np.float64).T
    np.testing.assert_allclose(from_bf16_bits(out), ref, atol=2e-2, rtol=1e-2)


@pytest.mark.parametrize("pair", [0, 1])
def test_withheld_stage_times_out_and_context_recovers(pair):
    M, N, K = 512, 512, 1024
    st = ctypes.c_uint(0)
    rc = lib().mfb200_debug_gemm_withheld(M, N, K, pair, LIMIT_NS, ctypes.byref(st))
    assert rc == 0, f"withheld launch rc={rc}"
    assert st.value in TIMEOUT_CODES, f"status {st.value}"
    gemm_ok(M, N, K, pair)  # the next ordinary GEMM runs and is correct


def test_forward_with_withheld_stage_reports_timeout_then_recovers(positions):
    g = load_golden("small")
    cfg = synthetic.CONFIGS[str(g["config"])]
    t = synthetic.generate(cfg, int(g["weight_seed"]), bool(g["perturb_norms"]))
    net = create_network(cfg, t, max_batch=64)
    rc = lib().mfb200_debug_forward_withheld(net._h, 64, LIMIT_NS)
    assert rc != 0
    assert "timed out" in lib().mfb200_last_error(net._h).decode()
    out = net.evaluate_packed(positions.slice(0, 64))  # the same handle, an ordinary call
    assert np.abs(out.policy - g["policy"]).max() <= 5e-2
    assert np.abs(out.wdl - g["wdl"]).max() <= 1e-2
    net.close()
