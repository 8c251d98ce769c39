#!/usr/bin/env python
"""Benchmark of the α-entmax block-sparse attention hot path on B200.

One step = forward (τ solve + block mask + tile lists + block-sparse
forward) + backward (dQ, dK, dV) of the headline configuration, through the
splash_attention autograd surface, with inputs resident in HBM.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config C3|C4|C5]
    python bench.py --impl reference ...   # the reference-math CPU arm

Multi-GPU (torchrun, one process per GPU): heads are independent, so every
rank runs its own shard of B*H heads (the headline batch per rank: weak
scaling) with no collective on the data path; the step time is the max over
ranks.  Rank 0 prints one JSON line.
"""
import argparse
import json
import math
import os
import statistics
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "adaptive-splash-attention_b200"))
sys.path.insert(0, ROOT)

METRIC = "α-entmax attn fwd+bwd ms & effective TFLOP/s at N=4K/32K, 1–8 B200"

# BASELINE.json configs[2..4]; C3 is the single-GPU headline.
CONFIGS = {
    "C3": dict(B=4, H=16, N=4096, d=128, alpha=1.5, k_keep=8, causal=True, sigma=1.0,
               sm_scale=128 ** -0.5, BM=128, BN=128, centroids=0),
    "C4": dict(B=1, H=32, N=32768, d=128, alpha=2.0, k_keep=8, causal=True, sigma=1.0,
               sm_scale=128 ** -0.5, BM=128, BN=128, centroids=64),
    "C5": dict(B=8, H=16, N=8192, d=64, alpha=1.5, k_keep=16, causal=False, sigma=1.0,
               sm_scale=0.125, BM=128, BN=128, centroids=0),
}

# Algorithmic FLOPs per active 128x128 tile, in units of BM*BN*d, by launch
# label: every matmul counts 2 (tau_mask is charged per visible pair instead).
TILE_UNITS = {"forward": 4, "backward": 10, "bwd_rowstats": 4, "bwd_dq": 6, "bwd_dkdv": 8,
              "bwd_pre": 0}


def load_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return p["bf16_tflops"], p["bf16_tflops_sustained"], p["hbm_gbs"], "measured"
    except Exception:
        return 1590.0, 1400.0, 6650.0, "fallback"


def load_traffic(label, cfg_name):
    """Per-launch DRAM bytes of `label` from the committed ncu summary
    (profiles/traffic.txt: `label config bytes_per_launch`), or None."""
    path = os.path.join(ROOT, "profiles", "traffic.txt")
    if not os.path.exists(path):
        return None
    for line in open(path):
        f = line.split()
        if len(f) >= 3 and not line.startswith("#") and f[0] == label and f[1] == cfg_name:
            return float(f[2])
    return None


def make_inputs(c, rank, device, torch):
    g = torch.Generator(device=device).manual_seed(1234 + rank)
    B, H, N, d = c["B"], c["H"], c["N"], c["d"]
    Q = (torch.randn(B, H, N, d, generator=g, device=device) * c["sigma"]).bfloat16()
    K = torch.randn(B, H, N, d, generator=g, device=device) * c["sigma"]
    if c["centroids"]:
        cent = 2.0 * torch.randn(c["centroids"], d, generator=g, device=device)
        K = K + cent[(torch.arange(N, device=device) * c["centroids"]) // N]
    K = K.bfloat16()
    V = torch.randn(B, H, N, d, generator=g, device=device).bfloat16()
    dO = torch.randn(B, H, N, d, generator=g, device=device).bfloat16()
    idx = torch.arange(N, device=device, dtype=torch.int32).expand(B * H, N).contiguous()
    return Q, K, V, dO, idx


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


def cpu_baseline(c, steps=1):
    """The oracle (C restatement of the reference arithmetic, OpenMP over all
    host cores) on a bounded sample: one head of the configuration at full
    sequence length, forward + backward.  Returns (effective TFLOP/s, s/step,
    sample description, threads)."""
    import numpy as np
    import torch
    from oracle import oracle as orc
    N, d = c["N"], c["d"]
    g = torch.Generator().manual_seed(7)
    Q = (torch.randn(1, N, d, generator=g) * c["sigma"]).bfloat16().float().numpy()
    K = torch.randn(1, N, d, generator=g) * c["sigma"]
    if c["centroids"]:
        cent = 2.0 * torch.randn(c["centroids"], d, generator=g)
        K = K + cent[(torch.arange(N) * c["centroids"]) // N]
    K = K.bfloat16().float().numpy()
    V = torch.randn(1, N, d, generator=g).bfloat16().float().numpy()
    dO = torch.randn(1, N, d, generator=g).bfloat16().float().numpy()
    idx = np.arange(N, dtype=np.int32)[None]
    cfg = orc.Config(1, N, N, d, c["BM"], c["BN"], c["k_keep"], c["alpha"], c["sm_scale"],
                     c["causal"])
    times, T = [], 0
    for _ in range(steps):
        t0 = time.perf_counter()
        r = orc.run_all(cfg, Q, K, V, idx, idx, dO)
        times.append(time.perf_counter() - t0)
        T = int(r["M"].sum())
    t = statistics.median(times)
    flops = 14.0 * c["BM"] * c["BN"] * d * T
    threads = len(os.sched_getaffinity(0))
    sample = f"1 of {c['B'] * c['H']} heads (B=1,H=1,N={N},d={d}), fwd+bwd, fp32 math on bf16-rounded inputs"
    return flops / t / 1e12, t, sample, threads


def run_reference_arm(a, c, rank, world):
    if rank != 0:
        return 0
    for _ in range(a.warmup):
        cpu_baseline(c, 1)
    vals, secs = [], []
    for _ in range(a.steps):
        v, t, sample, threads = cpu_baseline(c, 1)
        vals.append(v)
        secs.append(t)
    v = statistics.median(vals)
    out = {"impl": "reference", "metric": METRIC, "value": v, "unit": "TFLOP/s",
           "n_gpus": world, "steps": a.steps, "warmup": a.warmup,
           "ms_per_step": statistics.median(secs) * 1e3, "higher_is_better": True,
           "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
           "config": {"workload": a.config + " (one-head sample)", **{k: c[k] for k in c}},
           "cpu_baseline": {"value": v, "unit": "TFLOP/s", "cores": threads, "kind": "port",
                            "sample": sample},
           "e2e": {"value": v, "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                   "d2h_bytes_per_step": 0},
           "note": "the reference ships no CPU path; this arm runs the oracle's C restatement "
                   "of its arithmetic (oracle/asa_oracle.c) on all host cores"}
    print(json.dumps(out), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--config", default="C3", choices=sorted(CONFIGS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--backend", default="auto")
    ap.add_argument("--precision", default="split")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--e2e-chunk", type=int, default=4, help="heads per chunk in the e2e leg")
    a = ap.parse_args()
    c = dict(CONFIGS[a.config])
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    if a.impl == "reference":
        return run_reference_arm(a, c, rank, world)

    import torch
    import torch.distributed as dist
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)
    import splash_attention as sa
    from splash_attention import ops

    Q, K, V, dO, idx = make_inputs(c, rank, dev, torch)
    st = dict(alpha=c["alpha"], sm_scale=c["sm_scale"], k_keep=c["k_keep"], block_m=c["BM"],
              block_n=c["BN"], causal=c["causal"], backend=a.backend, precision=a.precision)
    q, k, v = (x.detach().requires_grad_() for x in (Q, K, V))

    def step(q, k, v, dO):
        q.grad = k.grad = v.grad = None
        O = sa.splash_attention(q, k, v, idx, idx, **st)
        O.backward(dO)
        return O

    def barrier():
        if world > 1:
            dist.barrier()

    for _ in range(a.warmup):
        step(q, k, v, dO)
    torch.cuda.synchronize()
    # active tiles of this rank's inputs (outside the timed region)
    _, saved = ops.forward_saved(Q, K, V, idx, idx, ops.Settings(**st), need_o32=False)
    T = int(saved.M.sum().item())
    BH, N = c["B"] * c["H"], c["N"]
    nb = (N + c["BM"] - 1) // c["BM"]
    T_bound = BH * (nb * (nb + 1) // 2 if c["causal"] else nb * nb)
    backend = ops.resolved_backend(saved.params[0])
    del saved

    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    launches0 = ops.launch_count()
    with Clocks(local) as clk:
        e0.record(stream)
        for _ in range(a.steps):
            step(q, k, v, dO)
        e1.record(stream)
        torch.cuda.synchronize()
    launches = ops.launch_count() - launches0
    barrier()
    ms = e0.elapsed_time(e1) / a.steps
    t = torch.tensor([ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())

    # per-kernel device time of one more step (events around each launch)
    with ops.profile() as prof:
        step(q, k, v, dO)
    kern = prof.result
    fwd_ms = sum(kern.get(x, (0, 0))[0] for x in ("tau_mask", "tile_lists", "forward"))
    bwd_ms = sum(v_[0] for k_, v_ in kern.items() if k_ not in ("tau_mask", "tile_lists", "forward"))

    unit_flops = c["BM"] * c["BN"] * c["d"]
    eff_flops = 14.0 * unit_flops * T * world
    value = eff_flops / (ms_max * 1e-3) / 1e12
    peak_b, peak_s, hbm, peak_kind = load_peaks()
    # dominant kernel and its roofline
    dom = max(kern.items(), key=lambda kv: kv[1][0])
    dom_label, (dom_ms, dom_n) = dom[0], dom[1]
    pairs = BH * (N * (N + 1) // 2 if c["causal"] else N * N)
    if dom_label == "tau_mask":
        dom_flops = 2.0 * c["d"] * pairs
    else:
        dom_flops = TILE_UNITS.get(dom_label, 0) * unit_flops * T
    per_launch_ms = dom_ms / max(dom_n, 1)
    achieved = dom_flops / max(dom_n, 1) / (per_launch_ms * 1e-3) / 1e12
    traffic = load_traffic(dom_label, a.config)
    roofline = {"kernel": dom_label, "bound": "tensor", "achieved": achieved, "peak": peak_s,
                "unit": "TFLOP/s", "frac": achieved / peak_s, "traffic": traffic,
                "peak_kind": f"{peak_kind} sustained bf16",
                "kernels_ms": {k_: round(v_[0], 4) for k_, v_ in kern.items()}}

    # end to end through the public API with pinned host buffers: every
    # step copies Q, K, V, dO in and O, dQ, dK, dV out; the head chunks'
    # copies overlap the kernels (splash_attention.forward_backward_host)
    e2e = None
    if not a.no_e2e:
        hQ, hK, hV, hdO = (x.cpu().pin_memory() for x in (Q, K, V, dO))
        outs = tuple(torch.empty(Q.shape, dtype=Q.dtype).pin_memory() for _ in range(4))
        h2d = sum(x.numel() * x.element_size() for x in (hQ, hK, hV, hdO))
        d2h = sum(x.numel() * x.element_size() for x in outs)
        hidx = idx.cpu()

        def e2e_step():
            sa.forward_backward_host(hQ, hK, hV, hdO, hidx, hidx, out=outs,
                                     heads_per_chunk=a.e2e_chunk, synchronize=False, **st)

        for _ in range(2):
            e2e_step()
        torch.cuda.synchronize()
        barrier()
        e0.record(stream)
        n_e2e = max(2, a.steps // 2)
        for _ in range(n_e2e):
            e2e_step()
        e1.record(stream)
        torch.cuda.synchronize()
        t = torch.tensor([e0.elapsed_time(e1) / n_e2e], device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
        e2e = {"value": eff_flops / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
               "ms_per_step": e2e_ms, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
               "api": "splash_attention.forward_backward_host (pinned host in/out, "
                      f"{a.e2e_chunk} heads per chunk, copies overlapped with kernels)"}

    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        v_, t_, sample, threads = cpu_baseline(c, 1)
        cpu = {"value": v_, "unit": "TFLOP/s", "cores": threads, "kind": "port",
               "sample": sample, "seconds": t_}

    if rank == 0:
        out = {
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world,
            "steps": a.steps, "warmup": a.warmup, "ms_per_step": ms_max,
            "fwd_ms": fwd_ms, "bwd_ms": bwd_ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic: seeded N(0,1) Q/K/V/dO (bf16), causal arange positions",
            "config": {"workload": a.config, "B_per_rank": c["B"], "H": c["H"], "N": N,
                       "d": c["d"], "alpha": c["alpha"], "k_keep": c["k_keep"],
                       "causal": c["causal"], "tiles": f"{c['BM']}x{c['BN']}",
                       "global_batch": c["B"] * world, "parallelism": f"heads-sharded x{world}",
                       "backend": backend, "precision": a.precision,
                       "l2": "inputs 4x64 MiB per rank exceed the 126 MB L2; no flush"},
            "active_tiles": T, "active_fraction": T / T_bound,
            "flops_counted": "14*BM*BN*d per active tile (fwd 4 + bwd 10); tau/mask pass timed, not counted",
            "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": launches,
            "clocks": clk.summary(),
        }
        print(json.dumps(out), flush=True)
    if world > 1:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
