#!/usr/bin/env python
"""Benchmark of the α-entmax block-sparse attention hot path on B200.

One step = forward (τ solve + block mask + tile lists + block-sparse
forward) + backward (dQ, dK, dV) of one configuration of BASELINE.json
through the splash_attention autograd surface, with inputs resident in HBM
(C1 is forward-only, as its config states).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config C1..C5]
                    [--scaling weak|strong] [--sweep]
    python bench.py --impl reference ...   # the reference-math CPU arm

Multi-GPU (torchrun, one process per GPU): heads are independent, so the
global B*H heads are split over the ranks with splash_attention.shard.partition
and every rank runs its own contiguous head range, with no collective on
the data path; the step time is the max over ranks of CUDA-event times.
``--scaling weak`` (default; C4 defaults to strong) makes the global batch N
times the configuration's heads, so every rank holds one configuration's
worth; ``strong`` splits the configuration's own heads.  Rank 0 prints one
JSON line.

Inputs: global head h draws its Q, K, V, dO from its own CUDA generator
(seed 1234 + h), so a rank can make its slice without the others'; the C4
cluster centroids come from one shared generator (seed 999).
"""
import argparse
import json
import os
import statistics
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "adaptive-splash-attention_b200"))
sys.path.insert(0, ROOT)

METRIC = "α-entmax attn fwd+bwd ms & effective TFLOP/s at N=4K/32K, 1–8 B200"

# BASELINE.json configs[0..4]; C3 is the single-GPU headline.  C1/C2 are the
# reference's fp32 cases (its own tile sizes: 64x64 for C1, the default
# 32x64 for C2), which run on the CUDA-core kernels.
CONFIGS = {
    "C1": dict(B=1, H=2, N=256, d=64, alpha=1.5, k_keep=8, causal=True, sigma=1.0,
               sm_scale=0.125, BM=64, BN=64, centroids=0, dtype="f32", fwd_only=True),
    "C2": dict(B=2, H=8, N=1024, d=64, alpha=1.5, k_keep=8, causal=True, sigma=1.0,
               sm_scale=0.125, BM=32, BN=64, centroids=0, dtype="f32", fwd_only=False),
    "C3": dict(B=4, H=16, N=4096, d=128, alpha=1.5, k_keep=8, causal=True, sigma=1.0,
               sm_scale=128 ** -0.5, BM=128, BN=128, centroids=0, dtype="bf16", fwd_only=False),
    "C4": dict(B=1, H=32, N=32768, d=128, alpha=2.0, k_keep=8, causal=True, sigma=1.0,
               sm_scale=128 ** -0.5, BM=128, BN=128, centroids=64, dtype="bf16", fwd_only=False),
    "C5": dict(B=8, H=16, N=8192, d=64, alpha=1.5, k_keep=16, causal=False, sigma=1.0,
               sm_scale=0.125, BM=128, BN=128, centroids=0, dtype="bf16", fwd_only=False),
}
C5_SWEEP = [(a, s) for a in (1.25, 1.5, 2.0) for s in (0.5, 1.0, 2.0)]

# Algorithmic FLOPs per active tile, in units of BM*BN*d, by launch label:
# every matmul counts 2 (tau_mask is charged per visible pair instead).
TILE_UNITS = {"forward": 4, "bwd_rowstats": 4, "bwd_dq": 6, "bwd_dkdv": 8, "bwd_pre": 0}


def load_peaks():
    """(bf16 burst TFLOP/s, bf16 sustained TFLOP/s, HBM GB/s, source)."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return p["bf16_tflops"], p["bf16_tflops_sustained"], p["hbm_gbs"], "measured"
    except Exception:
        return 1590.0, 1400.0, 6650.0, "fallback"


def load_traffic(label, cfg_name, head_frac=1.0):
    """Per-launch DRAM bytes of `label` copied from a committed ncu capture
    (profiles/traffic.txt: `label config bytes_per_launch source`, bytes of
    a launch over the configuration's B*H heads), times `head_frac` (this
    rank's heads / B*H: every head's tensors are read and written once), or
    None.  Not measured by this run: ncu cannot run inside a timed bench."""
    path = os.path.join(ROOT, "profiles", "traffic.txt")
    if not os.path.exists(path):
        return None
    for line in open(path):
        f = line.split()
        if len(f) >= 3 and not line.startswith("#") and f[0] == label and f[1] == cfg_name:
            return {"bytes": float(f[2]) * head_frac, "source": " ".join(f[3:]) or "profiles/traffic.txt"}
    return None


def head_range(c, rank, world, scaling):
    """(global heads, this rank's [h0, h1)) under the given scaling."""
    from splash_attention.shard import partition
    per_cfg = c.get("heads") or c["B"] * c["H"]
    total = per_cfg * world if scaling == "weak" else per_cfg
    return total, partition(total, world)[rank]


def make_inputs(c, h0, h1, device):
    """Seeded synthetic inputs of global heads [h0, h1): Q, K, V, dO as
    [1, h1-h0, N, d] in the config's dtype plus int32 arange positions
    [h1-h0, N].  Head h uses generator seed 1234 + h (order Q, K, V, dO;
    N(0, σ²) for Q and K, N(0, 1) for V and dO, drawn in fp32, then cast);
    C4 adds to every key the centroid of its cluster, c(j) = ⌊64 j / N⌋
    (contiguous 512-key runs), centroids 2·N(0, 1) from seed 999."""
    import torch
    N, d = c["N"], c["d"]
    dt = torch.float32 if c["dtype"] == "f32" else torch.bfloat16
    cent = None
    if c["centroids"]:
        gc = torch.Generator(device=device).manual_seed(999)
        cent = 2.0 * torch.randn(c["centroids"], d, generator=gc, device=device)
        cent = cent[(torch.arange(N, device=device) * c["centroids"]) // N]
    out = [torch.empty(1, h1 - h0, N, d, device=device, dtype=dt) for _ in range(4)]
    for i, h in enumerate(range(h0, h1)):
        g = torch.Generator(device=device).manual_seed(1234 + h)
        q = torch.randn(N, d, generator=g, device=device) * c["sigma"]
        k = torch.randn(N, d, generator=g, device=device) * c["sigma"]
        if cent is not None:
            k = k + cent
        v = torch.randn(N, d, generator=g, device=device)
        do = torch.randn(N, d, generator=g, device=device)
        for t, x in zip(out, (q, k, v, do)):
            t[0, i] = x.to(dt)
    idx = torch.arange(N, device=device, dtype=torch.int32).expand(h1 - h0, N).contiguous()
    return (*out, idx)


def settings(c, backend="auto", precision="split", fused=True):
    return dict(alpha=c["alpha"], sm_scale=c["sm_scale"], k_keep=c["k_keep"], block_m=c["BM"],
                block_n=c["BN"], causal=c["causal"], backend=backend, precision=precision,
                fused_forward=fused)


class Clocks:
    """SM clock and throttle reasons sampled through NVML every 5 ms by a
    background thread while the timed region runs (a 200 ms nvidia-smi poll
    sees nothing of a 50 ms region).  Read-only: no clock or power setting
    is touched."""

    NAMES = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, device_index, period_s=0.005):
        import threading
        self.dev = device_index
        self.period = period_s
        self.samples = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        self._nvml = None

    def _run(self):
        nv, h = self._nvml
        bits = (nv.nvmlClocksEventReasonHwSlowdown, nv.nvmlClocksEventReasonHwThermalSlowdown,
                nv.nvmlClocksEventReasonSwThermalSlowdown, nv.nvmlClocksEventReasonSwPowerCap)
        while not self._stop.is_set():
            try:
                mhz = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                r = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                self.samples.append((mhz, tuple(n for n, b_ in zip(self.NAMES, bits) if r & b_)))
            except Exception:
                return
            self._stop.wait(self.period)

    def __enter__(self):
        try:
            import threading
            import pynvml as nv
            nv.nvmlInit()
            bus = None
            try:
                import torch
                pr = torch.cuda.get_device_properties(self.dev)
                bus = f"{pr.pci_domain_id:08X}:{pr.pci_bus_id:02X}:{pr.pci_device_id:02X}.0"
            except Exception:
                pass
            h = (nv.nvmlDeviceGetHandleByPciBusId(bus) if bus
                 else nv.nvmlDeviceGetHandleByIndex(self.dev))
            self.max_mhz = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
            self._nvml = (nv, h)
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        except Exception:
            self._thread = None
        return self

    def __exit__(self, *a):
        if self._thread:
            self._stop.set()
            self._thread.join(timeout=2)
        return False

    def summary(self):
        if not self.samples:
            return None
        reasons = sorted({n for _, rs in self.samples for n in rs})
        return {"sm_mhz": statistics.median(m for m, _ in self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(self.samples), "source": "nvml, 5 ms"}



def cpu_baseline(c, heads=1, max_n=8192):
    """The oracle (C restatement of the reference arithmetic, OpenMP over all
    host cores) on a bounded sample: `heads` heads of the configuration at
    sequence length capped at max_n (the GPU arm's per-head seeds, drawn by
    torch's CPU generator; a capped C4 sample keeps its 512-key cluster
    runs), forward (+ backward unless the config is forward-only).
    Returns (effective TFLOP/s, s/step, sample description, threads)."""
    from oracle import oracle as orc
    c = dict(c)
    n_full = c["N"]
    if c["N"] > max_n:   # bounded sample: a shorter sequence, same cluster run length
        c["centroids"] = c["centroids"] * max_n // c["N"]
        c["N"] = max_n
    N, d = c["N"], c["d"]
    Q, K, V, dO, idx = make_inputs(c, 0, heads, "cpu")
    f = lambda x: x.float().reshape(heads, N, d).numpy()
    cfg = orc.Config(heads, N, N, d, c["BM"], c["BN"], c["k_keep"], c["alpha"], c["sm_scale"],
                     c["causal"])
    t0 = time.perf_counter()
    r = orc.run_all(cfg, f(Q), f(K), f(V), idx.numpy(), idx.numpy(),
                    None if c["fwd_only"] else f(dO))
    t = time.perf_counter() - t0
    T = int(r["M"].sum())
    units = 4 if c["fwd_only"] else 14
    flops = units * c["BM"] * c["BN"] * d * T
    threads = len(os.sched_getaffinity(0))
    sample = (f"{heads} of {c['B'] * c['H']} heads (N={N}"
              + (f" of {n_full}" if N != n_full else "") + f", d={d}), "
              f"{'fwd' if c['fwd_only'] else 'fwd+bwd'}, fp32 math on the "
              f"{'bf16-rounded ' if c['dtype'] == 'bf16' else ''}inputs")
    return flops / t / 1e12, t, sample, threads


def use_all_host_cores():
    """The CPU arms use every core this process may run on: torchrun sets
    OMP_NUM_THREADS=1 for its ranks, which would leave the OpenMP oracle on
    one core.  Must run before the oracle library is first loaded."""
    os.environ["OMP_NUM_THREADS"] = str(len(os.sched_getaffinity(0)))


def run_reference_arm(a, c, rank, world):
    if rank != 0:
        return 0
    use_all_host_cores()
    heads = c["B"] * c["H"] if a.config in ("C1", "C2") else 1
    for _ in range(a.warmup):
        cpu_baseline(c, heads)
    vals, secs = [], []
    for _ in range(a.steps):
        v, t, sample, threads = cpu_baseline(c, heads)
        vals.append(v)
        secs.append(t)
    v = statistics.median(vals)
    out = {"impl": "reference", "metric": METRIC, "value": v, "unit": "TFLOP/s",
           "n_gpus": world, "steps": a.steps, "warmup": a.warmup,
           "ms_per_step": statistics.median(secs) * 1e3, "higher_is_better": True,
           "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
           "config": {"workload": f"{a.config} ({sample})", **{k: c[k] for k in c}},
           "cpu_baseline": {"value": v, "unit": "TFLOP/s", "cores": threads, "kind": "port",
                            "sample": sample},
           "e2e": {"value": v, "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                   "d2h_bytes_per_step": 0},
           "note": "the reference ships no CPU path; this arm runs the oracle's C restatement "
                   "of its arithmetic (oracle/asa_oracle.c) on all host cores"}
    print(json.dumps(out), flush=True)
    return 0


def measure(a, c, name, rank, world, dev, scaling, dist, with_extras=True):
    """Time a.steps steps of config c on this rank's heads; returns the
    JSON record (rank 0) or None."""
    import torch
    import splash_attention as sa
    from splash_attention import ops

    total_heads, (h0, h1) = head_range(c, rank, world, scaling)
    Q, K, V, dO, idx = make_inputs(c, h0, h1, dev)
    st = settings(c, a.backend, a.precision, not a.unfused)
    q, k, v = (x.detach().requires_grad_(not c["fwd_only"]) for x in (Q, K, V))

    def step():
        if c["fwd_only"]:
            with torch.no_grad():
                return sa.splash_attention(q, k, v, idx, idx, **st)
        q.grad = k.grad = v.grad = None
        O = sa.splash_attention(q, k, v, idx, idx, **st)
        O.backward(dO)
        return O

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x):
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def sum_over_ranks(x):
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(t)
        return float(t.item())

    for _ in range(a.warmup):
        step()
    torch.cuda.synchronize()
    # active tiles of this rank's heads (outside the timed region)
    _, saved = ops.forward_saved(Q, K, V, idx, idx, ops.Settings(**st), need_o32=False)
    T_local = int(saved.M.sum().item())
    backend = ops.resolved_backend(saved.params[0])
    del saved
    N, BM, BN = c["N"], c["BM"], c["BN"]
    nqb, nkb = -(-N // BM), -(-N // BN)
    T = int(sum_over_ranks(T_local))
    if c["causal"]:
        per_head = sum(min(nkb, ((qb + 1) * BM - 1) // BN + 1) for qb in range(nqb))
    else:
        per_head = nqb * nkb
    T_bound = total_heads * per_head

    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    launches0 = ops.launch_count()
    with Clocks(dev.index) as clk:
        e0.record(stream)
        for _ in range(a.steps):
            step()
        e1.record(stream)
        torch.cuda.synchronize()
    launches = ops.launch_count() - launches0
    barrier()
    ms_max = max_over_ranks(e0.elapsed_time(e1) / a.steps)

    units = 4 if c["fwd_only"] else 14
    unit_flops = BM * BN * c["d"]
    eff_flops = units * unit_flops * T
    value = eff_flops / (ms_max * 1e-3) / 1e12
    rec = {"metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": a.steps,
           "warmup": a.warmup, "ms_per_step": ms_max, "higher_is_better": True,
           "scaling": scaling, "vs_baseline": None, "dtype": c["dtype"],
           "data": "synthetic: per-head seeded N(0,σ²) Q/K, N(0,1) V/dO, arange positions"
                   + (", 64 contiguous key clusters" if c["centroids"] else ""),
           "config": {"workload": name, "global_heads": total_heads,
                      "heads_per_rank": h1 - h0, "N": N, "d": c["d"], "alpha": c["alpha"],
                      "sigma": c["sigma"], "k_keep": c["k_keep"], "causal": c["causal"],
                      "tiles": f"{BM}x{BN}", "step": "fwd" if c["fwd_only"] else "fwd+bwd",
                      "global_batch": total_heads, "parallelism": f"heads-sharded x{world}",
                      "backend": backend, "precision": a.precision},
           "active_tiles": T, "active_fraction": T / T_bound,
           "flops_counted": f"{units}*BM*BN*d per active tile "
                            + ("(fwd)" if c["fwd_only"] else "(fwd 4 + bwd 10)")
                            + "; tau/mask pass timed, not counted",
           "gpu_launches": launches, "clocks": clk.summary()}
    in_bytes = sum(x.numel() * x.element_size() for x in (Q, K, V, dO))
    rec["config"]["fused_forward"] = st["fused_forward"]
    rec["config"]["l2"] = (f"inputs {in_bytes / 2**20:.0f} MiB per rank "
                           + ("exceed the 126 MB L2; no flush" if in_bytes > 126e6
                              else "fit in L2: L2 flushed between steps is NOT done; small case"))
    if not with_extras:
        return rec if rank == 0 else None

    # per-kernel device time of one more step (events around each launch)
    with ops.profile() as prof:
        step()
    kern = prof.result
    fwd_labels = ("tau_mask", "tile_lists", "forward", "forward_fused")
    rec["fwd_ms"] = sum(kern.get(x, (0, 0))[0] for x in fwd_labels)
    rec["bwd_ms"] = sum(v_[0] for k_, v_ in kern.items() if k_ not in fwd_labels)
    peak_b, peak_s, hbm, peak_kind = load_peaks()
    dom_label, (dom_ms, dom_n) = max(kern.items(), key=lambda kv: kv[1][0])
    h_local = h1 - h0
    pairs = h_local * (N * (N + 1) // 2 if c["causal"] else N * N)
    if dom_label == "tau_mask":
        dom_flops = 2.0 * c["d"] * pairs
    elif dom_label == "forward_fused":   # the τ/mask pass's S over visible pairs + the forward
        dom_flops = 2.0 * c["d"] * pairs + TILE_UNITS["forward"] * unit_flops * T_local
    else:
        dom_flops = TILE_UNITS.get(dom_label, 0) * unit_flops * T_local
    per_launch_ms = dom_ms / max(dom_n, 1)
    achieved = dom_flops / max(dom_n, 1) / (per_launch_ms * 1e-3) / 1e12
    traffic = load_traffic(dom_label, name, (h1 - h0) / (c["B"] * c["H"]))
    # kernels are timed inside one short step (milliseconds), so the burst
    # peak is the denominator
    rec["roofline"] = {"kernel": dom_label, "bound": "tensor", "achieved": achieved,
                       "peak": peak_b, "unit": "TFLOP/s", "frac": achieved / peak_b,
                       "frac_of_sustained": achieved / peak_s,
                       "traffic": traffic["bytes"] if traffic else None,
                       "traffic_source": (f"copied from an ncu capture ({traffic['source']}); "
                                          "not measured by this run") if traffic else None,
                       "peak_kind": f"{peak_kind} bf16 burst (of measured)",
                       "kernels_ms": {k_: round(v_[0], 4) for k_, v_ in kern.items()}}
    if "tau_mask" in kern:
        # the τ/mask pass (all its launches: bounds, top-k + mask, τ solve):
        # compulsory HBM bytes (Q and K read once, τ and M written)
        tm_ms = kern["tau_mask"][0]
        elt = 4 if c["dtype"] == "f32" else 2
        tm_bytes = h_local * (2 * N * c["d"] * elt + N * 4 + nqb * nkb)
        rec["tau_mask"] = {"ms": tm_ms, "hbm_gbs": tm_bytes / (tm_ms * 1e-3) / 1e9,
                           "hbm_frac": tm_bytes / (tm_ms * 1e-3) / 1e9 / hbm,
                           "tflops": 2.0 * c["d"] * pairs / (tm_ms * 1e-3) / 1e12,
                           "bytes": tm_bytes}

    # end to end through the public API with pinned host buffers: every
    # step copies Q, K, V, dO in and O, dQ, dK, dV out; the head chunks'
    # copies overlap the kernels (splash_attention.forward_backward_host)
    if not a.no_e2e:
        hQ, hK, hV, hdO = (x.cpu().pin_memory() for x in (Q, K, V, dO))
        hidx = idx.cpu()
        if c["fwd_only"]:
            hO = torch.empty(Q.shape, dtype=Q.dtype).pin_memory()
            h2d = sum(x.numel() * x.element_size() for x in (hQ, hK, hV))
            d2h = hO.numel() * hO.element_size()

            def e2e_step():
                dq, dk, dv = (x.to(dev, non_blocking=True) for x in (hQ, hK, hV))
                di = hidx.to(dev, non_blocking=True)
                with torch.no_grad():
                    o = sa.splash_attention(dq, dk, dv, di, di, **st)
                hO.copy_(o, non_blocking=True)
            api = "splash_attention.splash_attention (pinned host in/out)"
        else:
            outs = tuple(torch.empty(Q.shape, dtype=Q.dtype).pin_memory() for _ in range(4))
            h2d = sum(x.numel() * x.element_size() for x in (hQ, hK, hV, hdO))
            d2h = sum(x.numel() * x.element_size() for x in outs)

            # heads per chunk: the API's default (chunks of at least 32 MiB
            # of inputs) unless --e2e-chunk names a count
            chunk = a.e2e_chunk

            def e2e_step():
                sa.forward_backward_host(hQ, hK, hV, hdO, hidx, hidx, out=outs,
                                         heads_per_chunk=chunk, synchronize=False, **st)
            api = ("splash_attention.forward_backward_host (pinned host in/out, "
                   + (f"{chunk} heads per chunk" if chunk else "chunks of >= 32 MiB of inputs")
                   + ", copies overlapped with kernels)")
        for _ in range(2):
            e2e_step()
        torch.cuda.synchronize()
        barrier()
        n_e2e = max(2, a.steps // 2)
        e0.record(stream)
        for _ in range(n_e2e):
            e2e_step()
        e1.record(stream)
        torch.cuda.synchronize()
        e2e_ms = max_over_ranks(e0.elapsed_time(e1) / n_e2e)
        rec["e2e"] = {"value": eff_flops / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
                      "ms_per_step": e2e_ms, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                      "api": api}
    else:
        rec["e2e"] = None

    rec["cpu_baseline"] = None
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        use_all_host_cores()
        heads = c["B"] * c["H"] if name in ("C1", "C2") else 1
        v_, t_, sample, threads = cpu_baseline(c, heads)
        rec["cpu_baseline"] = {"value": v_, "unit": "TFLOP/s", "cores": threads, "kind": "port",
                               "sample": sample, "seconds": t_}
    return rec if rank == 0 else None


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--config", default="C3", choices=sorted(CONFIGS))
    ap.add_argument("--scaling", default=None, choices=["weak", "strong"])
    ap.add_argument("--sweep", action="store_true",
                    help="C5: one line per (alpha, sigma) point of the sweep")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--backend", default="auto")
    ap.add_argument("--precision", default="split")
    ap.add_argument("--unfused", action="store_true",
                    help="separate τ/mask, tile-list and forward launches instead of the fused forward")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--heads", type=int, default=None,
                    help="global heads per configuration instead of B*H (small profiling cases; "
                         "the line's config then names the reduced count)")
    ap.add_argument("--e2e-chunk", type=int, default=None,
                    help="heads per chunk in the e2e leg (default: chunks of at least 32 MiB of inputs)")
    a = ap.parse_args()
    c = dict(CONFIGS[a.config])
    if a.heads:
        c["heads"] = a.heads
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    if a.impl == "reference":
        return run_reference_arm(a, c, rank, world)
    scaling = a.scaling or ("strong" if a.config == "C4" else "weak")

    import torch
    import torch.distributed as dist
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)
    if a.sweep:
        if a.config != "C5":
            raise SystemExit("--sweep applies to C5")
        for alpha, sigma in C5_SWEEP:
            cc = dict(c, alpha=alpha, sigma=sigma)
            rec = measure(a, cc, "C5", rank, world, dev, scaling, dist, with_extras=False)
            if rec:
                rec["config"]["workload"] = f"C5 sweep alpha={alpha} sigma={sigma}"
                print(json.dumps(rec), flush=True)
    else:
        rec = measure(a, c, a.config, rank, world, dev, scaling, dist)
        if rec:
            print(json.dumps(rec), flush=True)
    if world > 1:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
