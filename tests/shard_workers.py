"""Worker functions for the multi-process shard tests (importable by spawned
ranks)."""
import numpy as np
import torch


def oracle_slice(rank, world, BH, N, d):
    """Each rank runs the oracle on its head slice and all-gathers the
    outputs over gloo."""
    from splash_attention.shard import partition, gather_heads
    from helpers import make_inputs, oracle_run
    Q, K, V, dO, Qi, Ki = make_inputs(1, BH, N, N, d, seed=5)
    s, e = partition(BH, world)[rank]
    sl = lambda x: x[:, s:e].contiguous()
    r = oracle_run(sl(Q), sl(K), sl(V), sl(dO), Qi[s:e], Ki[s:e], 32, 32, 4, 1.5, 0.2)
    local = torch.from_numpy(r["O"]).unsqueeze(0)
    return gather_heads(local, world).numpy()


def fails_on_rank1(rank, world):
    if rank == 1:
        raise ValueError("injected failure on rank 1")
    return rank
