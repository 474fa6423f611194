"""One handle over two GPUs: the batch is sharded contiguously (one host
thread per GPU), weights replicated, no collective. Each shard runs the
same plan a one-GPU handle runs for a batch of that size, so the two-GPU
result must equal, bit for bit, a one-GPU handle evaluating the two halves as
separate batches."""
import numpy as np
import pytest

from metalfish_b200 import synthetic
from metalfish_b200.network import create_network

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("batch", [100, 64, 7])
def test_two_gpu_handle_matches_one_gpu_per_shard(batch, positions):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    cfg = synthetic.SMALL
    t = synthetic.generate(cfg, 1)
    half = (batch + 1) // 2  # the first shard's size (shards are ceil(batch / 2))
    one_net = create_network(cfg, t, max_batch=128)
    parts = [one_net.evaluate_packed(positions.slice(0, half)),
             one_net.evaluate_packed(positions.slice(half, batch))]
    two_net = create_network(cfg, t, max_batch=128, num_devices=2)
    assert two_net.get_backend_capabilities().num_devices == 2
    two = two_net.evaluate_packed(positions.slice(0, batch))
    for field in ("policy", "wdl", "value", "moves_left"):
        want = np.concatenate([getattr(p, field) for p in parts])
        np.testing.assert_array_equal(getattr(two, field), want, err_msg=field)
    one_net.close()
    two_net.close()
