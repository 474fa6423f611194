"""One handle over two GPUs: the batch is sharded contiguously (one host
thread per GPU), weights replicated, no collective. Results must equal a
single-GPU handle's (same kernels, same per-position arithmetic)."""
import numpy as np
import pytest

from metalfish_b200 import synthetic
from metalfish_b200.network import create_network

pytestmark = pytest.mark.gpu


def test_two_gpu_handle_matches_one_gpu(positions):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    cfg = synthetic.SMALL
    t = synthetic.generate(cfg, 1)
    inp = positions.slice(0, 100)
    one = create_network(cfg, t, max_batch=128).evaluate_packed(inp)
    two_net = create_network(cfg, t, max_batch=128, num_devices=2)
    assert two_net.get_backend_capabilities().num_devices == 2
    two = two_net.evaluate_packed(inp)
    np.testing.assert_array_equal(two.policy, one.policy)
    np.testing.assert_array_equal(two.wdl, one.wdl)
    np.testing.assert_array_equal(two.moves_left, one.moves_left)
