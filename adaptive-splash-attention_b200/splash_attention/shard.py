"""Head-sharded multi-GPU launch: one process per GPU, each rank owning a
contiguous range of the B·H independent heads.

The reference has no multi-GPU code.  Heads never interact in the τ solve,
the mask, the forward or the backward, so sharding needs no collective on
the data path: each rank runs the same C ABI on its own device and keeps its
outputs.  Collectives appear only outside the hot path (timing max, optional
verification gathers).
"""
import os
import traceback

import torch


def partition(BH, world):
    """Contiguous [start, end) head ranges for `world` ranks covering 0..BH-1
    exactly once; sizes differ by at most one (earlier ranks take the extra)."""
    if BH < 0 or world < 1:
        raise ValueError("partition: BH >= 0 and world >= 1 required")
    base, extra = divmod(BH, world)
    out, start = [], 0
    for r in range(world):
        n = base + (1 if r < extra else 0)
        out.append((start, start + n))
        start += n
    return out


def local_heads(t, rank, world):
    """Rows of a [B, H, N, d] (or [B*H, N]) tensor owned by `rank`, as a
    contiguous [1, h, N, d] (or [h, N]) view over the flattened heads."""
    if t.dim() == 4:
        B, H = t.shape[:2]
        s, e = partition(B * H, world)[rank]
        return t.reshape(B * H, *t.shape[2:])[s:e].unsqueeze(0)
    s, e = partition(t.shape[0], world)[rank]
    return t[s:e]


def sharded_attention(Q, K, V, Q_idx, K_idx, rank=None, world=None, **kw):
    """Run splash_attention on this rank's heads (autograd included).
    Inputs are the full [B, H, N, d] tensors (or views of them on this rank's
    device); returns this rank's [1, h, N, d] output."""
    from . import splash_attention
    if rank is None:
        rank = int(os.environ.get("RANK", 0))
    if world is None:
        world = int(os.environ.get("WORLD_SIZE", 1))
    q, k, v = (local_heads(x, rank, world) for x in (Q, K, V))
    return splash_attention(q, k, v, _local_positions(Q_idx, Q, rank, world),
                            _local_positions(K_idx, K, rank, world), **kw)


def _local_positions(idx, X, rank, world):
    """This rank's rows of a position tensor: [N] broadcasts to every head;
    [B*H, N] and [B, H, N] are flattened to heads and sliced."""
    if idx is None or idx.dim() == 1:
        return idx
    B, H, N = X.shape[0], X.shape[1], X.shape[2]
    if idx.dim() not in (2, 3) or idx.numel() != B * H * N:
        raise ValueError(f"sharded_attention: positions must be [N], [B*H, N] or [B, H, N] "
                         f"with B*H = {B * H} and N = {N}; got {tuple(idx.shape)}")
    return local_heads(idx.reshape(B * H, N), rank, world)


def gather_heads(local, world, group=None):
    """All-gather every rank's [1, h_r, N, d] output into [1, B*H, N, d]
    (outside the hot path: verification only).  Works with NCCL or gloo."""
    import torch.distributed as dist
    sizes = [torch.zeros(1, dtype=torch.long, device=local.device) for _ in range(world)]
    dist.all_gather(sizes, torch.tensor([local.shape[1]], device=local.device), group=group)
    hmax = int(max(s.item() for s in sizes))
    pad = torch.zeros(1, hmax, *local.shape[2:], dtype=local.dtype, device=local.device)
    pad[:, :local.shape[1]] = local
    parts = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(parts, pad, group=group)
    return torch.cat([p[:, :int(s.item())] for p, s in zip(parts, sizes)], dim=1)


def _worker(rank, world, fn, args, port, backend, queue):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    import torch.distributed as dist
    try:
        dist.init_process_group(backend, rank=rank, world_size=world)
        result = fn(rank, world, *args)
        queue.put((rank, "ok", result))
    except BaseException as e:  # report every failure to the launcher
        queue.put((rank, "error", f"{type(e).__name__}: {e}\n{traceback.format_exc()}"))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def launch(fn, world, args=(), backend="gloo", port=29541, timeout=300.0):
    """Run fn(rank, world, *args) in `world` spawned processes (one per GPU
    for NCCL, CPU ranks for gloo).  Returns the per-rank results; if any rank
    fails, the others are terminated and RuntimeError names the failed rank.
    The failure is detected on the host (the worker's exception), never by
    faulting a device."""
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, fn, args, port, backend, q))
             for r in range(world)]
    for p in procs:
        p.start()
    results, errors = {}, {}
    import queue as _queue
    import time
    deadline = time.time() + timeout
    try:
        while len(results) + len(errors) < world:
            try:
                rank, status, payload = q.get(timeout=max(0.1, deadline - time.time()))
            except _queue.Empty:
                errors[-1] = "timeout waiting for ranks"
                break
            (results if status == "ok" else errors)[rank] = payload
            if errors:
                break
    finally:
        for p in procs:
            if errors and p.is_alive():
                p.terminate()
        for p in procs:
            p.join(timeout=10)
    if errors:
        r = sorted(errors)[0]
        raise RuntimeError(f"rank {r} failed: {errors[r]}")
    return [results[r] for r in range(world)]
