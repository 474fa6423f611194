"""Legal-move priors on the GPU (mfb200_evaluate_priors): the forward plus
the MCTS leaf step -- the evaluator's per-move logit gather
(src/mcts/evaluator.cpp:182-226) and ApplyNNPolicyToNode's FastExp softmax
(src/mcts/search.cpp:127-197).

Given the same logits the GPU priors are bit-identical to the oracle's
restatement (whose FastExp is pinned to the reference's in test_oracle.py);
end to end against the reference CPU backend's logits they agree within the
bf16 forward's tolerance carried through the softmax.
"""
import os

import numpy as np
import pytest

from metalfish_b200 import synthetic
from metalfish_b200.netfile import PackedInputs
from metalfish_b200.network import create_network
from oracle import port
from tests.conftest import GOLDEN, load_golden

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def small_net():
    g = load_golden("small")
    cfg = synthetic.CONFIGS[str(g["config"])]
    net = create_network(cfg, synthetic.generate(cfg, int(g["weight_seed"]), bool(g["perturb_norms"])),
                         max_batch=512)
    yield net, g
    net.close()


@pytest.fixture(scope="module")
def fixture_moves():
    z = np.load(os.path.join(GOLDEN, "legal_moves.npz"))
    p = np.load(os.path.join(GOLDEN, "positions.npz"))
    return z["offsets"], z["index"], p["masks"], p["values"]


def _slice(off, idx, lo, hi):
    o = off[lo:hi + 1]
    return (o - o[0]).astype(np.int32), idx[o[0]:o[-1]]


@pytest.mark.parametrize("temp", [1.0, 0.61, 2.2])
def test_priors_bit_exact_on_gpu_logits(small_net, fixture_moves, temp):
    net, _ = small_net
    off, idx, m, v = fixture_moves
    B = 512
    o, ix = _slice(off, idx, 0, B)
    inp = PackedInputs(m[:B], v[:B])
    pri, wdl, mlh = net.evaluate_priors(inp, o, ix, temp)
    out = net.evaluate_packed(inp)
    ref = port.priors(out.policy, o, ix, temp)
    np.testing.assert_array_equal(pri, ref)
    np.testing.assert_array_equal(wdl, out.wdl)
    np.testing.assert_array_equal(mlh, out.moves_left)
    for b in range(B):
        if o[b + 1] > o[b]:
            assert abs(float(pri[o[b]:o[b + 1]].sum()) - 1.0) < 1e-5


def test_priors_against_reference_logits(small_net, fixture_moves):
    """End to end: GPU priors vs the oracle's priors on the reference CPU
    backend's logits (max |policy logit diff| <= 5e-2 bounds the prior error)."""
    net, g = small_net
    off, idx, m, v = fixture_moves
    n = len(g["policy"])
    o, ix = _slice(off, idx, 0, n)
    pri, _, _ = net.evaluate_priors(PackedInputs(m[:n], v[:n]), o, ix, 1.0)
    ref = port.priors(g["policy"], o, ix, 1.0)
    d = np.abs(pri - ref)
    print("max |prior diff|", d.max())
    assert d.max() <= 0.05 * max(float(ref.max()), 1e-3) + 2e-3


def test_priors_edge_cases(small_net, fixture_moves):
    """No moves, one move, more than 256 moves (kMaxEdges), out-of-range
    indices, a CSR that does not start at 0."""
    net, _ = small_net
    _, _, m, v = fixture_moves
    rng = np.random.default_rng(9)
    lists = [[], [17], [-1, 5, 1858, 32767, 9], rng.choice(1858, 300, replace=False).tolist(),
             list(range(64)), []]
    B = len(lists)
    off = (np.concatenate([[0], np.cumsum([len(x) for x in lists])]) + 1000).astype(np.int32)
    idx = np.concatenate([np.asarray(x, np.int16) for x in lists]).astype(np.int16)
    inp = PackedInputs(m[:B], v[:B])
    pri, _, _ = net.evaluate_priors(inp, off, idx, 0.8)
    ref = port.priors(net.evaluate_packed(inp).policy, off - 1000, idx, 0.8)
    np.testing.assert_array_equal(pri, ref)
    assert pri[0] == 1.0  # the single move of position 1
    s3 = off[3] - 1000
    assert (pri[s3 + 256:s3 + 300] == 0).all()


def test_priors_errors(small_net, fixture_moves):
    net, _ = small_net
    _, _, m, v = fixture_moves
    inp = PackedInputs(m[:2], v[:2])
    with pytest.raises(RuntimeError, match="softmax_temp"):
        net.evaluate_priors(inp, np.array([0, 1, 2], np.int32), np.array([1, 2], np.int16), 0.0)
    with pytest.raises(RuntimeError, match="non-decreasing"):
        net.evaluate_priors(inp, np.array([0, 2, 1], np.int32), np.array([1, 2], np.int16), 1.0)


def test_priors_bt4_batch_1024(fixture_moves):
    """BT4 shape at the bench batch: bit-exact on the GPU's own logits."""
    off, idx, m, v = fixture_moves
    cfg = synthetic.BT4
    net = create_network(cfg, synthetic.generate(cfg, 3), max_batch=1024)
    try:
        o, ix = _slice(off, idx, 0, 1024)
        inp = PackedInputs(m[:1024], v[:1024])
        pri, _, _ = net.evaluate_priors(inp, o, ix, 1.0)
        ref = port.priors(net.evaluate_packed(inp).policy, o, ix, 1.0)
        np.testing.assert_array_equal(pri, ref)
    finally:
        net.close()
