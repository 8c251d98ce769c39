"""Host-side multi-GPU logic on CPU ranks (gloo): the head partition, the
verification gather, and failure reporting."""
import numpy as np
import pytest

from splash_attention.shard import partition, launch
from helpers import make_inputs, oracle_run
import shard_workers


@pytest.mark.parametrize("BH,world", [(64, 8), (7, 2), (32, 3), (5, 8), (0, 2), (1, 1)])
def test_partition_covers_every_head_once(BH, world):
    parts = partition(BH, world)
    assert len(parts) == world
    seen = [h for s, e in parts for h in range(s, e)]
    assert seen == list(range(BH))
    sizes = [e - s for s, e in parts]
    assert max(sizes) - min(sizes) <= 1


def test_two_ranks_gloo_equal_single_process():
    BH, N, d = 5, 96, 16
    res = launch(shard_workers.oracle_slice, 2, args=(BH, N, d), backend="gloo", port=29561)
    Q, K, V, dO, Qi, Ki = make_inputs(1, BH, N, N, d, seed=5)
    full = oracle_run(Q, K, V, dO, Qi, Ki, 32, 32, 4, 1.5, 0.2, grads=False)
    for r in res:
        np.testing.assert_array_equal(r[0], full["O"])


def test_failed_rank_is_reported():
    with pytest.raises(RuntimeError, match="rank 1 failed.*injected failure"):
        launch(shard_workers.fails_on_rank1, 2, backend="gloo", port=29562, timeout=120)


@pytest.mark.parametrize("shape", [(2, 3, 40), (6, 40), (40,)])
def test_local_positions_accepts_every_position_layout(shape):
    import torch
    from splash_attention.shard import _local_positions, partition
    X = torch.zeros(2, 3, 40, 8)
    idx = torch.arange(2 * 3 * 40).reshape(6, 40) if len(shape) > 1 else torch.arange(40)
    idx = idx.reshape(shape)
    for rank in range(4):
        got = _local_positions(idx, X, rank, 4)
        if len(shape) == 1:
            assert got is idx
            continue
        s, e = partition(6, 4)[rank]
        assert torch.equal(got, idx.reshape(6, 40)[s:e])


def test_local_positions_rejects_mismatched_shapes():
    import torch
    from splash_attention.shard import _local_positions
    with pytest.raises(ValueError, match="positions must be"):
        _local_positions(torch.zeros(5, 40), torch.zeros(2, 3, 40, 8), 0, 2)
