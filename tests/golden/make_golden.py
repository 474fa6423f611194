#!/usr/bin/env python3
"""Regenerate the golden fixtures in tests/golden/ from the REFERENCE itself.

Needs the reference source tree (default /root/reference, override with
MF_REFERENCE) and builds oracle/_ref/ with ``make -C oracle ref``; it is run
by hand in the development container, never by the tests. Outputs:

* ``attn_policy_map.npy``  -- the reference's 4288-entry gather table
  (src/nn/tables/attention_policy_map.h:15), dumped by oracle/dump_policy_map.
* ``positions.npz``        -- 4096 seeded random-playout positions (seed 20251201),
  generated and packed by the reference's own encoder (oracle/ref_harness
  gen-inputs). Used as parity inputs and as the bench's synthetic inputs.
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
REF = os.environ.get("MF_REFERENCE", "/root/reference")
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


def main() -> None:
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


if __name__ == "__main__":
    main()
