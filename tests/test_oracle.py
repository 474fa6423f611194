"""Pins the C restatement oracle against the reference itself.

The golden fixtures were produced by the reference's own Cpu::CpuNetwork
(compiled unmodified from the reference sources; tests/golden/make_golden.py).
The oracle keeps the reference's per-row accumulation order, so it must match
those outputs bit for bit.
"""
import os

import numpy as np
import pytest

from tests.conftest import GOLDEN, load_golden
from metalfish_b200 import layout, netfile, synthetic
from metalfish_b200.synthetic import CONFIGS
from oracle import port
from tests.golden.make_golden import weights_digest


def test_slot_tables_match_oracle_enums():
    assert port.slot_counts() == (len(layout.GLOBAL_SLOTS), len(layout.LAYER_SLOTS))


def test_policy_gather_table_matches_reference():
    ref = np.load(os.path.join(GOLDEN, "attn_policy_map.npy"))
    ours = port.build_policy_map()
    assert ref.shape == (4288,)
    assert np.array_equal(ours, ref)
    assert (ours >= 0).sum() == 1858


def test_policy_map_known_answer():
    """Port of the reference KAT tests/test_mcts_module.cpp:2620-2651 (fixture
    :443-505): identity embedding and policy projection, wq = plane 0, wk =
    plane 1, ppo = [1, 3, 5, 0]. The planes go through the input packing, which
    keeps only the FIRST nonzero value of a plane (plane 1 = {5 @ b1, 7 @ a8}
    packs to 5 on both squares). Expected: policy[0] (a1b1) = 2*5 = 10 and the
    mixed promotion logit policy[1793] = 5 * (3 + 0) = 15."""
    planes = np.zeros((1, 112, 64), np.float32)
    planes[0, 0, 0] = 2.0
    planes[0, 1, 1] = 5.0
    planes[0, 0, 48] = 2.0
    planes[0, 1, 56] = 7.0
    packed = netfile.pack_planes(planes)
    dense = netfile.unpack_planes(packed)[0]
    q = np.maximum(dense[0], 0)[:, None]   # relu default activation
    k = np.maximum(dense[1], 0)[:, None]
    ppo = np.array([[1.0], [3.0], [5.0], [0.0]], np.float32)
    out = port.policy_map(q, k, ppo)
    assert abs(out[0] - 10.0) < 1e-5
    assert abs(out[1793] - 15.0) < 1e-5


def test_pack_unpack_matches_reference_fixture(positions):
    """Unpacking the reference-packed positions and packing them again must
    reproduce the reference's masks and values exactly."""
    sub = positions.slice(0, 256)
    again = netfile.pack_planes(netfile.unpack_planes(sub))
    np.testing.assert_array_equal(again.masks, sub.masks)
    np.testing.assert_array_equal(again.values, sub.values)


@pytest.mark.parametrize("name", ["tiny", "small", "small_perturbed"])
def test_oracle_bit_exact_vs_reference(name, positions):
    g = load_golden(name)
    cfg = CONFIGS[str(g["config"])]
    tensors = synthetic.generate(cfg, int(g["weight_seed"]), bool(g["perturb_norms"]))
    assert weights_digest(tensors) == str(g["weights_sha256"]), "weight generator drifted"
    n = int(g["positions"])
    out = port.forward(cfg, tensors, positions.slice(0, n))
    np.testing.assert_array_equal(out.policy, g["policy"])
    np.testing.assert_array_equal(out.wdl, g["wdl"])
    np.testing.assert_array_equal(out.value, g["value"])
    np.testing.assert_array_equal(out.moves_left, g["moves_left"])


def test_oracle_bit_exact_vs_reference_bt4(positions):
    g = load_golden("bt4")
    cfg = synthetic.BT4
    tensors = synthetic.generate(cfg, int(g["weight_seed"]), bool(g["perturb_norms"]))
    assert weights_digest(tensors) == str(g["weights_sha256"])
    n = 4
    out = port.forward(cfg, tensors, positions.slice(0, n), threads=4)
    np.testing.assert_array_equal(out.policy, g["policy"][:n])
    np.testing.assert_array_equal(out.wdl, g["wdl"][:n])
    np.testing.assert_array_equal(out.moves_left, g["moves_left"][:n])


def test_golden_outputs_are_sane():
    for name in ("tiny", "small", "small_perturbed", "bt4"):
        g = load_golden(name)
        assert np.isfinite(g["policy"]).all()
        np.testing.assert_allclose(g["wdl"].sum(1), 1.0, atol=1e-5)
        np.testing.assert_allclose(g["value"], g["wdl"][:, 0] - g["wdl"][:, 2], atol=1e-6)
        assert (g["moves_left"] >= 0).all()


# ---------------------------------------------------------------- MCTS leaf priors
def test_fast_exp_matches_reference():
    """The oracle's FastExp is bit-identical to the reference's
    (src/mcts/core.h:38-44) on a grid, random values and the clamp/NaN/inf edges."""
    z = np.load(os.path.join(GOLDEN, "fastexp.npz"))
    got = port.fast_exp(z["x"])
    np.testing.assert_array_equal(got.view(np.uint32), z["y"].view(np.uint32))


def test_legal_move_fixture_is_consistent():
    z = np.load(os.path.join(GOLDEN, "legal_moves.npz"))
    off, idx = z["offsets"], z["index"]
    assert off[0] == 0 and off[-1] == len(idx) and len(off) == 4097
    n = np.diff(off)
    assert n.min() == 0 and n.max() <= 218  # mates/stalemates have no moves
    assert idx.min() >= 0 and idx.max() < 1858
    for b in range(0, 4096, 97):  # each move maps to its own policy entry
        s = idx[off[b]:off[b + 1]]
        assert len(set(s.tolist())) == len(s)


def _priors_py(pol, off, idx, temp):
    """Float32 restatement in numpy of the same loop, for the oracle's own check."""
    out = np.zeros(off[-1] - off[0], np.float32)
    inv_t = np.float32(1.0) / np.float32(temp)
    for b in range(len(off) - 1):
        lo, moves = off[b] - off[0], off[b + 1] - off[b]
        n = min(moves, 256)
        if n == 0:
            continue
        l = np.array([pol[b, i] if 0 <= i < 1858 else 0.0 for i in idx[lo:lo + n]], np.float32)
        e = port.fast_exp((l - l.max()) * inv_t)
        s = np.float32(0)
        for v in e:
            s = np.float32(s + v)
        out[lo:lo + n] = e * (np.float32(1) / s) if s > 0 else np.float32(1) / np.float32(n)
    return out


def test_oracle_priors_semantics():
    rng = np.random.default_rng(4)
    B = 6
    pol = rng.standard_normal((B, 1858)).astype(np.float32) * 3
    lists = [[], [17], list(range(40)), [-1, 5, 1858, 32767, 9],
             rng.choice(1858, 300, replace=False).tolist(), rng.choice(1858, 31).tolist()]
    off = np.concatenate([[0], np.cumsum([len(x) for x in lists])]).astype(np.int32)
    idx = np.concatenate([np.asarray(x, np.int16) for x in lists]).astype(np.int16)
    for temp in (1.0, 0.7, 2.3):
        got = port.priors(pol, off, idx, temp)
        np.testing.assert_array_equal(got, _priors_py(pol, off, idx, temp))
        for b in range(B):
            n = min(off[b + 1] - off[b], 256)
            if n:
                assert abs(float(got[off[b]:off[b] + n].sum()) - 1.0) < 1e-5
        assert (got[off[4] + 256:off[5]] == 0).all()  # past kMaxEdges
    # an out-of-range index reads logit 0
    p0 = port.priors(np.zeros((1, 1858), np.float32), np.array([0, 2], np.int32),
                     np.array([-1, 3], np.int16), 1.0)
    np.testing.assert_array_equal(p0, np.array([0.5, 0.5], np.float32))


# ---------------------------------------------------------------- position encoder
FORMATS = (1, 2, 3, 4, 5, 132, 133)


def _history_sets():
    z = np.load(os.path.join(GOLDEN, "history.npz"))
    names = sorted({k.split("/")[0] for k in z.files})
    return {n: {k.split("/")[1]: z[k] for k in z.files if k.startswith(n + "/")} for n in names}


def test_encoder_restatement_matches_reference_all_formats():
    """bt4o_encode on the reference's own board records reproduces the
    reference encoder's packed planes and transforms bit for bit, in every
    input format, including pawnless games that reach every transform."""
    seen = set()
    for name, d in _history_sets().items():
        for fmt in FORMATS:
            ref_m = d[f"masks_{fmt}"]
            n = len(ref_m)
            m, v, t = port.encode(d["boards"], d["offsets"][:n + 1], fmt)
            np.testing.assert_array_equal(m, ref_m, err_msg=f"{name} format {fmt}")
            np.testing.assert_array_equal(v, d[f"values_{fmt}"], err_msg=f"{name} format {fmt}")
            np.testing.assert_array_equal(t, d[f"transforms_{fmt}"], err_msg=f"{name} format {fmt}")
            seen.update(t.tolist())
    assert seen == set(range(8))  # flip, mirror, transpose and their combinations


def test_encoder_restatement_matches_position_fixture():
    """The V2 encoding of the 1024 start games equals positions.npz (the
    reference's encoding the parity fixtures are built on)."""
    d = _history_sets()["start"]
    m, v, t = port.encode(d["boards"], d["offsets"], 5)
    z = np.load(os.path.join(GOLDEN, "positions.npz"))
    np.testing.assert_array_equal(m, z["masks"][:len(m)])
    np.testing.assert_array_equal(v, z["values"][:len(v)])
    np.testing.assert_array_equal(t, d["transforms_v2"])
