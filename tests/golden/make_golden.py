#!/usr/bin/env python3
"""Regenerate the golden fixtures in tests/golden/ from the REFERENCE itself.

Needs the reference source tree, named by the MF_REFERENCE environment
variable (the script stops when it is unset), and builds oracle/_ref/ with ``make -C oracle ref``; it is run
by hand in the development container, never by the tests. Outputs:

* ``attn_policy_map.npy``  -- the reference's 4288-entry gather table
  (src/nn/tables/attention_policy_map.h:15), dumped by oracle/dump_policy_map.
* ``positions.npz``        -- 4096 seeded random-playout positions (seed 20251201),
  generated and packed by the reference's own encoder (oracle/ref_harness
  gen-inputs). Used as parity inputs and as the bench's synthetic inputs.
* ``legal_moves.npz``     -- for the same positions, the policy index of every
  legal move as the reference evaluator maps it (oracle/ref_harness gen-moves:
  MoveList<LEGAL>, the black-side mirror, NN::MoveToNNIndex with the encoder's
  transform), CSR ``offsets`` / ``index``.
  ``raw`` holds each move itself (from | to << 6 | promotion << 12).
* ``move_index.npz``      -- NN::MoveToNNIndex (src/nn/policy_map.cpp:316-360)
  for every transform, promotion kind and (from, to) pair.
* ``fastexp.npz``         -- inputs and outputs of the reference's FastExp
  (src/mcts/core.h:38-44), the exponential of the MCTS policy softmax.
* ``history.npz``         -- game histories as board records (the GPU
  encoder's input, include/mfb200.h mfb200_board), read through the
  reference's Position accessors (oracle/ref_harness gen-history), with the
  reference encoder's packed planes and transforms for all seven input
  formats: the first 1024 fixture games (formats on the first 256) and three
  sets of 64 games from pawnless starts, which reach every canonical transform.
* ``ref_bt4_1024.npz``    -- the BT4 net of ``ref_bt4`` (weight seed 3, the
  weights bench.py measures) on the first 1024 positions: full policy logits
  for the first 256 (``policy``), and for all 1024 the WDL, value, moves-left,
  the reference's top-1 policy index and its top-1/top-2 logit gap
  (``top1`` / ``gap``). ``--bt4-large`` regenerates only this file.
* ``ref_<config>.npz``     -- outputs of the reference ``Cpu::CpuNetwork`` on the
  first N of those positions, for seeded synthetic weights; plus a SHA-256 of
  the weights so a numpy change that alters the generator is caught.
"""
import hashlib
import os
import subprocess
import sys
import tempfile

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
from metalfish_b200 import netfile, synthetic  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.environ.get("MF_REFERENCE", "")
HARNESS = os.path.join(ROOT, "oracle", "_ref", "ref_harness")
POSITION_SEED = 20251201
POSITIONS = 4096

# (fixture name, config, weight seed, perturb_norms, positions evaluated)
CASES = [
    ("tiny", synthetic.TINY, 11, True, 32),
    ("small", synthetic.SMALL, 1, False, 64),
    ("small_perturbed", synthetic.SMALL, 2, True, 16),
    ("bt4", synthetic.BT4, 3, False, 16),
]


def weights_digest(tensors) -> str:
    h = hashlib.sha256()
    for name in sorted(tensors):
        h.update(name.encode())
        h.update(np.ascontiguousarray(tensors[name], np.float32).tobytes())
    return h.hexdigest()


def read_moves(path):
    b = open(path, "rb").read()
    assert b[:4] == b"MFMV", "bad legal-move file"
    count = int(np.frombuffer(b[8:12], np.uint32)[0])
    offsets = np.frombuffer(b[12:12 + 4 * (count + 1)], np.int32).copy()
    o = 12 + 4 * (count + 1)
    n = int(offsets[-1])
    index = np.frombuffer(b[o:o + 2 * n], np.int16).copy()
    raw = np.frombuffer(b[o + 2 * n:o + 4 * n], np.uint16).copy()
    return offsets, index, raw


PAWNLESS_FENS = ["8/8/3k4/8/8/4K3/8/R6Q w - - 0 1", "2kr4/8/8/8/8/8/8/4K1NB b - - 0 1",
                 "8/2q5/8/3k4/8/8/8/B3K1R1 w - - 0 1"]


def read_history(path):
    b = open(path, "rb").read()
    assert b[:4] == b"MFHB", "bad history file"
    cnt = int(np.frombuffer(b[8:12], np.uint32)[0])
    o = 12
    off = np.frombuffer(b[o:o + 4 * (cnt + 1)], np.int32).copy()
    o += 4 * (cnt + 1)
    nb = int(off[-1])
    boards = np.frombuffer(b[o:o + 112 * nb], np.uint8).reshape(nb, 112).copy()
    o += 112 * nb
    tr = np.frombuffer(b[o:o + 4 * cnt], np.int32).copy()
    o += 4 * cnt
    na = int(np.frombuffer(b[o:o + 4], np.uint32)[0])
    o += 4
    out = {"offsets": off, "boards": boards, "transforms_v2": tr}
    for _ in range(7):
        code = int(np.frombuffer(b[o:o + 4], np.int32)[0])
        o += 4
        out[f"masks_{code}"] = np.frombuffer(b[o:o + 8 * na * 112], np.uint64).reshape(na, 112).copy()
        o += 8 * na * 112
        out[f"values_{code}"] = np.frombuffer(b[o:o + 4 * na * 112], np.float32).reshape(na, 112).copy()
        o += 4 * na * 112
        out[f"transforms_{code}"] = np.frombuffer(b[o:o + 4 * na], np.int32).copy()
        o += 4 * na
    return out


def make_history(tmp) -> None:
    sets = {}
    p = os.path.join(tmp, "h0.mfhb")
    subprocess.run([HARNESS, "gen-history", str(POSITION_SEED), "1024", "256", p], check=True)
    sets["start"] = read_history(p)
    for k, fen in enumerate(PAWNLESS_FENS):
        p = os.path.join(tmp, f"h{k + 1}.mfhb")
        subprocess.run([HARNESS, "gen-history", str(7 + k), "64", "64", p, fen], check=True)
        sets[f"pawnless{k}"] = read_history(p)
    flat = {f"{name}/{key}": val for name, d in sets.items() for key, val in d.items()}
    np.savez_compressed(os.path.join(HERE, "history.npz"), **flat)


def make_moves_and_fastexp(tmp) -> None:
    mv = os.path.join(tmp, "moves.mfmv")
    subprocess.run([HARNESS, "gen-moves", str(POSITION_SEED), str(POSITIONS), mv], check=True)
    offsets, index, raw = read_moves(mv)
    np.savez_compressed(os.path.join(HERE, "legal_moves.npz"), offsets=offsets, index=index,
                        raw=raw, seed=POSITION_SEED)
    mi = os.path.join(tmp, "move_index.i16")
    subprocess.run([HARNESS, "dump-move-index", mi], check=True)
    np.savez_compressed(os.path.join(HERE, "move_index.npz"),
                        table=np.fromfile(mi, np.int16).reshape(8, 5, 64, 64))
    rng = np.random.default_rng(5)
    x = np.concatenate([
        np.linspace(-100.0, 100.0, 20001, dtype=np.float32),
        (rng.standard_normal(20000) * 8.0).astype(np.float32),
        np.array([-88.0, 88.0, -88.00001, 88.00001, 0.0, -0.0, 1e-30, -1e-30, np.inf, -np.inf,
                  np.nan], np.float32)])
    xin, yout = os.path.join(tmp, "fx.f32"), os.path.join(tmp, "fy.f32")
    x.tofile(xin)
    subprocess.run([HARNESS, "fastexp", xin, yout], check=True)
    np.savez_compressed(os.path.join(HERE, "fastexp.npz"), x=x, y=np.fromfile(yout, np.float32))


def make_bt4_large(tmp, pos) -> None:
    """BT4 reference outputs at the bench's batch (1024 positions)."""
    n, full = 1024, 256
    tensors = synthetic.generate(synthetic.BT4, 3, perturb_norms=False)
    net = os.path.join(tmp, "bt4.mfnt")
    netfile.write_net(net, synthetic.BT4.header(), tensors)
    out = os.path.join(tmp, "bt4_1024.mfot")
    threads = os.cpu_count() or 1
    r = subprocess.run([HARNESS, "eval", net, pos, out, str(threads), "0", str(n)],
                       check=True, capture_output=True, text=True)
    print("bt4_1024", r.stdout.strip())
    o = netfile.read_outputs(out)
    srt = np.sort(o.policy, axis=1)
    np.savez_compressed(os.path.join(HERE, "ref_bt4_1024.npz"), policy=o.policy[:full],
                        wdl=o.wdl, value=o.value, moves_left=o.moves_left,
                        top1=np.argmax(o.policy, axis=1).astype(np.int16),
                        gap=(srt[:, -1] - srt[:, -2]).astype(np.float32),
                        config=synthetic.BT4.name, weight_seed=3, perturb_norms=False,
                        positions=n, full_policy_positions=full,
                        weights_sha256=weights_digest(tensors))


def main() -> None:
    if not REF or not os.path.isdir(os.path.join(REF, "src", "nn")):
        sys.exit("set MF_REFERENCE to the reference source tree")
    if sys.argv[1:] == ["--bt4-large"]:
        subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "oracle"), f"REF={REF}", "ref"],
                       check=True)
        with tempfile.TemporaryDirectory() as tmp:
            pos = os.path.join(tmp, "pos.mfin")
            subprocess.run([HARNESS, "gen-inputs", str(POSITION_SEED), str(POSITIONS), pos],
                           check=True)
            inp = netfile.read_inputs(pos)
            z = np.load(os.path.join(HERE, "positions.npz"))
            assert np.array_equal(inp.masks, z["masks"]) and np.array_equal(inp.values, z["values"])
            make_bt4_large(tmp, pos)
        return
    if sys.argv[1:] == ["--moves-only"]:  # legal moves, FastExp and histories only
        subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "oracle"), f"REF={REF}", "ref"],
                       check=True)
        with tempfile.TemporaryDirectory() as tmp:
            make_moves_and_fastexp(tmp)
            make_history(tmp)
        return
    subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "oracle"), f"REF={REF}", "ref"],
                   check=True)
    with tempfile.TemporaryDirectory() as tmp:
        table = os.path.join(tmp, "apm.bin")
        subprocess.run([os.path.join(ROOT, "oracle", "_ref", "dump_policy_map"), table], check=True)
        np.save(os.path.join(HERE, "attn_policy_map.npy"), np.fromfile(table, np.int16))

        pos = os.path.join(tmp, "pos.mfin")
        subprocess.run([HARNESS, "gen-inputs", str(POSITION_SEED), str(POSITIONS), pos], check=True)
        inp = netfile.read_inputs(pos)
        np.savez_compressed(os.path.join(HERE, "positions.npz"), masks=inp.masks,
                            values=inp.values, seed=POSITION_SEED)
        make_moves_and_fastexp(tmp)
        make_history(tmp)

        threads = os.cpu_count() or 1
        for name, cfg, seed, perturb, n in CASES:
            tensors = synthetic.generate(cfg, seed, perturb_norms=perturb)
            net = os.path.join(tmp, f"{name}.mfnt")
            netfile.write_net(net, cfg.header(), tensors)
            out = os.path.join(tmp, f"{name}.mfot")
            r = subprocess.run([HARNESS, "eval", net, pos, out, str(threads), "0", str(n)],
                               check=True, capture_output=True, text=True)
            print(name, r.stdout.strip())
            o = netfile.read_outputs(out)
            np.savez_compressed(os.path.join(HERE, f"ref_{name}.npz"), policy=o.policy, wdl=o.wdl,
                                value=o.value, moves_left=o.moves_left, config=cfg.name,
                                weight_seed=seed, perturb_norms=perturb, positions=n,
                                weights_sha256=weights_digest(tensors))
        make_bt4_large(tmp, pos)


if __name__ == "__main__":
    main()
