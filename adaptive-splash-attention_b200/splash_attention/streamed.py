"""Forward + backward for host-resident tensors with the PCIe transfers
overlapped with the kernels.

Heads are independent, so the B*H heads are processed in chunks: chunk c's
inputs are copied in on one stream while chunk c-1 computes on a second and
chunk c-2's outputs are copied out on a third.  The results equal those of
the device API on the whole batch; only the copies move.
"""
import ctypes

import torch

from . import _lib as L
from .ops import Settings, make_params, _workspace, _ptr, _torch_dtype


def forward_backward_host(Q, K, V, dO, Q_idx=None, K_idx=None, out=None, heads_per_chunk=None,
                          slots=3, synchronize=True, **settings):
    """Q, K, V, dO: pinned host tensors [B, H, N, d] (bfloat16 or float32).
    Q_idx / K_idx: positions [B*H, N] (host or device; [N] broadcasts).
    out: optional pinned host tensors (O, dQ, dK, dV) to fill; allocated
    (pinned) when omitted.  settings: as splash_attention (alpha, sm_scale,
    k_keep, causal, ...).  Runs on the current CUDA device and returns
    (O, dQ, dK, dV) on the host; with synchronize=False the current stream
    is only made to wait for the copies, so the caller must synchronize
    before reading them."""
    for t in (Q, K, V, dO):
        if t.is_cuda or not t.is_pinned():
            raise ValueError("forward_backward_host: Q, K, V, dO must be pinned host tensors")
    B, H, NQ, d = Q.shape
    NK = K.shape[2]
    BH = B * H
    st = Settings(**settings)
    dev = torch.device("cuda", torch.cuda.current_device())
    if out is None:
        out_dt = st.out_dtype if st.out_dtype is not None else Q.dtype
        out = tuple(torch.empty(shape, dtype=out_dt, pin_memory=True)
                    for shape in (Q.shape, Q.shape, K.shape, K.shape))
    hO, hdQ, hdK, hdV = (t.view(BH, t.shape[2], d) for t in out)
    hq, hk, hv, hdo = (t.reshape(BH, t.shape[2], d) for t in (Q, K, V, dO))

    def positions(idx, N):
        if idx is None:
            return None
        idx = torch.as_tensor(idx)
        if idx.dim() == 1:
            idx = idx.unsqueeze(0).expand(BH, N)
        return idx.reshape(BH, N).to(device=dev, dtype=torch.int32, non_blocking=True).contiguous()

    main = torch.cuda.current_stream()
    qi, ki = positions(Q_idx, NQ), positions(K_idx, NK)
    s_in, s_comp, s_out = (torch.cuda.Stream(device=dev) for _ in range(3))
    for s_ in (s_in, s_comp, s_out):
        s_.wait_stream(main)
    if heads_per_chunk is None:
        # chunks of at least 32 MiB of inputs: smaller chunks leave most SMs
        # idle behind each kernel's longest (causal) block, larger ones
        # lengthen the first copy-in and the last copy-out, which nothing
        # overlaps (C3 on a B200: 4-head chunks 7.0 ms, 8-head 6.7 ms,
        # 16-head 7.3 ms per step)
        head_bytes = (2 * NQ + 2 * NK) * d * Q.element_size()
        heads_per_chunk = max(1, -(-(32 << 20) // head_bytes))
    if isinstance(heads_per_chunk, int):
        hc = max(1, min(heads_per_chunk, BH))
        chunks = [(c0, min(c0 + hc, BH)) for c0 in range(0, BH, hc)]
    else:
        sizes = [int(n) for n in heads_per_chunk]
        if any(n <= 0 for n in sizes) or sum(sizes) != BH:
            raise ValueError(f"forward_backward_host: chunk sizes {sizes} must be positive and sum to B*H = {BH}")
        chunks, a = [], 0
        for n in sizes:
            chunks.append((a, a + n))
            a += n
        hc = max(sizes)
    nslots = min(slots, len(chunks))
    # Everything a chunk needs is allocated once per slot, and the C ABI is
    # called directly: per chunk the host only enqueues copies and two calls.
    params = {}

    def chunk_params(n):
        if n not in params:
            shp_q = torch.empty(1, n, NQ, d, device="meta", dtype=Q.dtype)
            shp_k = torch.empty(1, n, NK, d, device="meta", dtype=Q.dtype)
            p = make_params(shp_q, shp_k, st)
            params[n] = (p, _workspace(p, dev))
        return params[n]

    p_full, (fwd_b, bwd_b) = chunk_params(hc)
    out_dt = _torch_dtype(p_full.out_dtype)
    nqb, nkb = -(-NQ // p_full.block_m), -(-NK // p_full.block_n)

    def slot_buffers():
        e = lambda *shape, dt=torch.float32: torch.empty(*shape, device=dev, dtype=dt)
        return dict(q=e(hc, NQ, d, dt=Q.dtype), k=e(hc, NK, d, dt=Q.dtype), v=e(hc, NK, d, dt=Q.dtype),
                    do=e(hc, NQ, d, dt=Q.dtype), O=e(hc, NQ, d, dt=out_dt),
                    O32=e(hc, NQ, d) if out_dt != torch.float32 else None,
                    tau=e(hc, NQ), M=e(hc, nqb, nkb, dt=torch.uint8), ptr=e(hc, nqb + 1, dt=torch.int32),
                    idx=e(hc, nqb * nkb, dt=torch.int32), rn=e(hc, NQ),
                    dQ=e(hc, NQ, d, dt=out_dt), dK=e(hc, NK, d, dt=out_dt), dV=e(hc, NK, d, dt=out_dt),
                    wf=e(fwd_b, dt=torch.uint8), wb=e(bwd_b, dt=torch.uint8))

    bufs = [slot_buffers() for _ in range(nslots)]
    lib = L.lib()
    comp_stream = ctypes.c_void_p(s_comp.cuda_stream)
    comp_done, out_done = [], []
    for c, (a, b) in enumerate(chunks):
        n = b - a
        B_ = bufs[c % nslots]
        p, (fwd_n, bwd_n) = chunk_params(n)
        with torch.cuda.stream(s_in):
            if c >= nslots:
                s_in.wait_event(comp_done[c - nslots])     # this slot is free again
            for key, src in (("q", hq), ("k", hk), ("v", hv), ("do", hdo)):
                B_[key][:n].copy_(src[a:b], non_blocking=True)
            ev_in = torch.cuda.Event()
            ev_in.record(s_in)
        s_comp.wait_event(ev_in)
        if c >= nslots:
            s_comp.wait_event(out_done[c - nslots])       # this slot's outputs copied out
        pq = _ptr(qi[a:b]) if qi is not None else None
        pk = _ptr(ki[a:b]) if ki is not None else None
        O32 = B_["O32"] if B_["O32"] is not None else B_["O"]
        L.check(lib.asa_forward(ctypes.byref(p), _ptr(B_["q"]), _ptr(B_["k"]), _ptr(B_["v"]), pq, pk,
                                _ptr(B_["O"]), _ptr(O32), _ptr(B_["tau"]), _ptr(B_["M"]), _ptr(B_["ptr"]),
                                _ptr(B_["idx"]), _ptr(B_["rn"]), _ptr(B_["wf"]), fwd_n, comp_stream),
                "asa_forward")
        L.check(lib.asa_backward(ctypes.byref(p), _ptr(B_["q"]), _ptr(B_["k"]), _ptr(B_["v"]), pq, pk,
                                 _ptr(O32), _ptr(B_["tau"]), _ptr(B_["M"]), _ptr(B_["ptr"]), _ptr(B_["idx"]),
                                 _ptr(B_["rn"]), _ptr(B_["do"]), _ptr(B_["dQ"]), _ptr(B_["dK"]),
                                 _ptr(B_["dV"]), _ptr(B_["wb"]), bwd_n, comp_stream),
                "asa_backward")
        ev_c = torch.cuda.Event()
        ev_c.record(s_comp)
        comp_done.append(ev_c)
        with torch.cuda.stream(s_out):
            s_out.wait_event(ev_c)
            for dst, key in ((hO, "O"), (hdQ, "dQ"), (hdK, "dK"), (hdV, "dV")):
                dst[a:b].copy_(B_[key][:n], non_blocking=True)
            ev_o = torch.cuda.Event()
            ev_o.record(s_out)
            out_done.append(ev_o)
    main.wait_stream(s_out)
    main.wait_stream(s_in)
    main.wait_stream(s_comp)
    if synchronize:
        main.synchronize()
    return out
