"""Forward + backward for host-resident tensors with the PCIe transfers
overlapped with the kernels.

Heads are independent, so the B*H heads are processed in chunks: chunk c's
inputs are copied in on one stream while chunk c-1 computes on a second and
chunk c-2's outputs are copied out on a third.  The results equal those of
the device API on the whole batch; only the copies move.
"""
import torch

from .ops import Settings, forward_saved, backward_saved


def forward_backward_host(Q, K, V, dO, Q_idx=None, K_idx=None, out=None, heads_per_chunk=8,
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
    hc = max(1, min(heads_per_chunk, BH))
    chunks = [(c0, min(c0 + hc, BH)) for c0 in range(0, BH, hc)]
    bufs = [tuple(torch.empty(hc, n, d, device=dev, dtype=Q.dtype) for n in (NQ, NK, NK, NQ))
            for _ in range(min(slots, len(chunks)))]
    comp_done = []
    for c, (a, b) in enumerate(chunks):
        n = b - a
        slot = bufs[c % len(bufs)]
        with torch.cuda.stream(s_in):
            if c >= len(bufs):
                s_in.wait_event(comp_done[c - len(bufs)])     # this slot's inputs consumed
            for dst, src in zip(slot, (hq, hk, hv, hdo)):
                dst[:n].copy_(src[a:b], non_blocking=True)
            ev_in = torch.cuda.Event()
            ev_in.record(s_in)
        with torch.cuda.stream(s_comp):
            s_comp.wait_event(ev_in)
            q, k, v, do = (x[:n].unsqueeze(0) for x in slot)
            O, saved = forward_saved(q, k, v, qi[a:b] if qi is not None else None,
                                     ki[a:b] if ki is not None else None, st)
            dQ, dK, dV = backward_saved(q, k, v, do, saved)
            ev_c = torch.cuda.Event()
            ev_c.record(s_comp)
            comp_done.append(ev_c)
        with torch.cuda.stream(s_out):
            s_out.wait_event(ev_c)
            for dst, src in zip((hO, hdQ, hdK, hdV), (O, dQ, dK, dV)):
                src.record_stream(s_out)
                dst[a:b].copy_(src.reshape(n, src.shape[2], d), non_blocking=True)
    main.wait_stream(s_out)
    main.wait_stream(s_in)
    main.wait_stream(s_comp)
    if synchronize:
        main.synchronize()
    return out
