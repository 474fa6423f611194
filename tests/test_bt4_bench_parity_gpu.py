"""BT4 parity at the batch sizes the benchmark configurations run.

The fixture ``tests/golden/ref_bt4_1024.npz`` holds the reference CPU
backend's outputs (``Cpu::CpuNetwork``, compiled unmodified from the
reference sources) for the BT4-shaped network the bench measures (weight
seed 3) on the first 1024 fixture positions: full policy logits for the
first 256, and for all 1024 the WDL, moves-left, top-1 policy index and the
top-1/top-2 logit gap.

* bf16 (configs 1 and the bench line): max |policy logit diff| <= 5e-2 and
  max |WDL diff| <= 1e-2, evaluated as one batch of 256 (config 1) and as
  one batch of 1024 (the bench's batch; the full-policy check covers the
  first 256 of them, WDL / moves-left / top-1 all 1024), and at the small
  MCTS batches 1, 2 and 16 (split-K GEMMs with their reduction kernels).
* 8-bit (config 2): top-1 policy agreement >= 99% and max |WDL diff| <= 2e-2
  against the fp32 reference. Top-1 is counted over the positions whose
  reference top-1/top-2 gap exceeds 0.1 logits: the random-init policies
  have near ties (gaps down to ~1e-3) where bf16 itself flips.
  - INT8 handles (signed 8-bit operands, per-row activation and per-channel
    weight scales, int32 accumulation; the two GEMMs that read the FFN hidden
    in bf16) meet both bounds.
  - FP8-e4m3 handles with e4m3 in every encoder GEMM do not: e4m3 keeps 3
    mantissa bits, and the rounding noise of 60 GEMMs compounds to
    |WDL diff| ~0.05 whatever the scale granularity (per tensor, per row or
    per 32-element block all give 0.045-0.065 in a CPU emulation). That
    configuration is held to its measured bounds below.
"""
import numpy as np
import pytest

from metalfish_b200 import synthetic
from metalfish_b200.network import create_network
from tests.conftest import load_golden

pytestmark = pytest.mark.gpu

POLICY_TOL = 5e-2
WDL_TOL = 1e-2
GAP = 0.1

_nets = {}


def bt4_net(precision="bf16", fp8_gemms=0, positions=None):
    key = (precision, fp8_gemms)
    if key not in _nets:
        _nets.clear()  # one BT4 handle at a time
        t = synthetic.generate(synthetic.BT4, 3)
        _nets[key] = create_network(
            synthetic.BT4, t, max_batch=1024, precision=precision, fp8_gemms=fp8_gemms,
            calibration=positions.slice(1024, 2048) if precision != "bf16" else None)
    return _nets[key]


@pytest.fixture(scope="module")
def golden():
    g = load_golden("bt4_1024")
    t = synthetic.generate(synthetic.BT4, 3)
    from tests.golden.make_golden import weights_digest
    assert weights_digest(t) == str(g["weights_sha256"]), "weight generator drifted"
    return g


def stats(out, g, n):
    full = min(n, int(g["full_policy_positions"]))
    dp = float(np.abs(out.policy[:full] - g["policy"][:full]).max())
    dw = float(np.abs(out.wdl - g["wdl"][:n]).max())
    dm = np.abs(out.moves_left - g["moves_left"][:n])
    clear = g["gap"][:n] > GAP
    hits = (out.policy.argmax(1) == g["top1"][:n])[clear]
    top1 = float(hits.mean()) if hits.size else 1.0  # no clear position among the first n
    msg = (f"n={n} policy max {dp:.4g} wdl max {dw:.4g} mlh max {dm.max():.4g} "
           f"top1 {top1:.4f} over {int(clear.sum())} clear positions")
    print(msg)
    return dp, dw, dm, top1, msg


@pytest.mark.parametrize("batch", [1, 2, 16, 256, 1024])
def test_bt4_bf16_matches_reference_at_bench_batch(batch, positions, golden):
    out = bt4_net(positions=positions).evaluate_packed(positions.slice(0, batch))
    dp, dw, dm, top1, msg = stats(out, golden, batch)
    assert dp <= POLICY_TOL, msg
    assert dw <= WDL_TOL, msg
    assert (dm <= 5e-2 + 2e-2 * np.abs(golden["moves_left"][:batch])).all(), msg
    np.testing.assert_allclose(out.value, out.wdl[:, 0] - out.wdl[:, 2], atol=1e-6)


def test_bt4_int8_meets_north_star_8bit_tolerance(positions, golden):
    out = bt4_net("int8", positions=positions).evaluate_packed(positions.slice(0, 1024))
    _, dw, _, top1, msg = stats(out, golden, 1024)
    assert top1 >= 0.99, msg
    assert dw <= 2e-2, msg


def test_bt4_fp8_e4m3_all_encoder_gemms_measured_bounds(positions, golden):
    out = bt4_net("fp8", positions=positions).evaluate_packed(positions.slice(0, 1024))
    _, dw, _, top1, msg = stats(out, golden, 1024)
    # measured on B200: top-1 90.5% of 474 clear positions, max |WDL diff| 0.083
    assert top1 >= 0.88, msg
    assert dw <= 0.1, msg
