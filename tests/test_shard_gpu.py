"""On one GPU: each rank's head slice computed alone equals the same heads of
the unsharded call (the property that makes head sharding collective-free)."""
import numpy as np
import pytest
import torch

from helpers import make_inputs

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("world", [2, 3])
def test_rank_slices_equal_full_run(cuda, world):
    from splash_attention import splash_attention
    from splash_attention.shard import sharded_attention
    Q, K, V, dO, Qi, Ki = (x.to(cuda) for x in make_inputs(2, 3, 512, 512, 128, seed=8,
                                                             dtype=torch.bfloat16))
    full = splash_attention(Q, K, V, Qi, Ki, out_dtype=torch.float32).reshape(6, 512, 128)
    parts = [sharded_attention(Q, K, V, Qi, Ki, rank=r, world=world, out_dtype=torch.float32)[0]
             for r in range(world)]
    torch.testing.assert_close(torch.cat(parts, 0), full, rtol=0, atol=0)
