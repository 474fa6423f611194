"""One handle over two GPUs: the batch is sharded contiguously (one host
thread per GPU), weights replicated, no collective. Results match a
single-GPU handle's within the tolerances the reference applies between
batch sizes on its CUDA transformer backend (policy 7.5e-2, value 2e-3,
moves-left 1.25e-1; tests/test_nn_comparison.cpp:825-832): a shard's smaller
batch can split a GEMM's K differently (small-batch split-K), which changes
the fp32 summation order."""
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
    np.testing.assert_allclose(two.policy, one.policy, rtol=0, atol=7.5e-2)
    np.testing.assert_allclose(two.wdl, one.wdl, rtol=0, atol=2e-3)
    np.testing.assert_allclose(two.value, one.value, rtol=0, atol=2e-3)
    np.testing.assert_allclose(two.moves_left, one.moves_left, rtol=0, atol=1.25e-1)
