"""The C++ drop-in: the reference harness (reference NN sources, compiled
unmodified) builds a WeightsFile and evaluates it through the B200 Network
subclass (metalfish_b200/host/b200_network.cpp) -- the path MetalFish's
CreateNetwork takes for backend "b200". Checked against the reference CPU
backend's golden outputs with the bf16 tolerances."""
import os
import subprocess

import numpy as np
import pytest

from metalfish_b200 import netfile, synthetic
from tests.conftest import load_golden

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HARNESS = os.path.join(ROOT, "oracle", "_ref", "b200_harness")


@pytest.mark.skipif(not os.path.exists(HARNESS), reason="b200_harness not built (needs the reference tree)")
@pytest.mark.parametrize("name", ["tiny", "small"])
def test_cpp_network_subclass_matches_reference(name, positions, tmp_path):
    g = load_golden(name)
    cfg = synthetic.CONFIGS[str(g["config"])]
    t = synthetic.generate(cfg, int(g["weight_seed"]), bool(g["perturb_norms"]))
    n = int(g["positions"])
    net, pos, out = tmp_path / "n.mfnt", tmp_path / "p.mfin", tmp_path / "o.mfot"
    netfile.write_net(str(net), cfg.header(), t)
    netfile.write_inputs(str(pos), positions.slice(0, n))
    r = subprocess.run([HARNESS, "eval-backend", "b200", str(net), str(pos), str(out)],
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    assert "b200" in r.stdout
    o = netfile.read_outputs(str(out))
    assert np.abs(o.policy - g["policy"][:n]).max() <= 5e-2
    assert np.abs(o.wdl - g["wdl"][:n]).max() <= 1e-2
    np.testing.assert_allclose(o.value, o.wdl[:, 0] - o.wdl[:, 2], atol=1e-6)


@pytest.mark.skipif(not os.path.exists(HARNESS), reason="b200_harness not built (needs the reference tree)")
def test_cpp_evaluate_priors_matches_python_api(positions, tmp_path):
    """B200Network::EvaluatePriors (the C++ MCTS leaf step) gives the same
    priors, bit for bit, as the Python mirror of the same C ABI call."""
    from metalfish_b200.network import create_network
    g = load_golden("small")
    cfg = synthetic.CONFIGS[str(g["config"])]
    t = synthetic.generate(cfg, int(g["weight_seed"]), bool(g["perturb_norms"]))
    z = np.load(os.path.join(ROOT, "tests", "golden", "legal_moves.npz"))
    n = 64
    off = z["offsets"][:n + 1].astype(np.int32)
    idx = z["index"][:off[-1]].astype(np.int16)
    net, pos, mv, out = (tmp_path / "n.mfnt", tmp_path / "p.mfin", tmp_path / "m.mfmv",
                         tmp_path / "o.f32")
    netfile.write_net(str(net), cfg.header(), t)
    netfile.write_inputs(str(pos), positions.slice(0, n))
    with open(mv, "wb") as f:
        f.write(b"MFMV")
        f.write(np.array([1, n], np.uint32).tobytes())
        f.write(off.tobytes())
        f.write(idx.tobytes())
    r = subprocess.run([HARNESS, "priors-b200", str(net), str(pos), str(mv), "0.9", str(out)],
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    cpp = np.fromfile(str(out), np.float32)
    py_net = create_network(cfg, t, max_batch=n)
    try:
        py, _, _ = py_net.evaluate_priors(positions.slice(0, n), off, idx, 0.9)
    finally:
        py_net.close()
    np.testing.assert_array_equal(cpp, py)


@pytest.mark.skipif(not os.path.exists(HARNESS), reason="b200_harness not built (needs the reference tree)")
def test_cpp_evaluate_leaves_from_engine_positions(tmp_path):
    """B200Network::EvaluateLeaves on the engine's own Position objects and
    MoveList<LEGAL> moves (the reference's game replay in the harness) gives
    the priors the Python mirror computes from the committed board records
    and raw moves of the same games, bit for bit."""
    from metalfish_b200.network import create_network
    g = load_golden("small")
    cfg = synthetic.CONFIGS[str(g["config"])]
    t = synthetic.generate(cfg, int(g["weight_seed"]), bool(g["perturb_norms"]))
    n = 64
    net, out = tmp_path / "n.mfnt", tmp_path / "o.f32"
    netfile.write_net(str(net), cfg.header(), t)
    r = subprocess.run([HARNESS, "leaves-b200", str(net), "20251201", str(n), "0.9", str(out)],
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    cpp = np.fromfile(str(out), np.float32)
    h = np.load(os.path.join(ROOT, "tests", "golden", "history.npz"))
    lm = np.load(os.path.join(ROOT, "tests", "golden", "legal_moves.npz"))
    hoff = h["start/offsets"][:n + 1]
    moff = lm["offsets"][:n + 1].astype(np.int32)
    py_net = create_network(cfg, t, max_batch=n)
    try:
        py, _, _ = py_net.evaluate_leaves(h["start/boards"][:hoff[-1]], hoff, lm["raw"][:moff[-1]],
                                          moff, 0.9)
    finally:
        py_net.close()
    np.testing.assert_array_equal(cpp, py)
