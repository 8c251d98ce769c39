"""Float64 torch restatement of the reference notebook's top-k-only
("stable") operator (AdaSplashNotebook.ipynb file lines 303-450), used as
the autograd reference for its gradient (test infrastructure).  The
bisection's decisions are comparisons, so autograd through the bracket
arithmetic gives the operator's gradient almost everywhere."""
import torch


def stable_attention_f64(Q, K, V, Qi, Ki, alpha, sm_scale, k, causal=True):
    """Q, K, V: [BH, N, d] float64 (with requires_grad as wanted)."""
    alpha = min(max(alpha, 1.01), 3.0)
    am1, inv = alpha - 1.0, 1.0 / (alpha - 1.0)
    s = torch.clamp(sm_scale * torch.einsum("bqd,bkd->bqk", Q, K), -10.0, 10.0)
    if causal:
        s = s.masked_fill(~(Ki[:, None, :] <= Qi[:, :, None]), float("-inf"))
    top, idx = torch.topk(s, k, dim=-1)                     # descending, distinct keys
    dead = torch.isinf(top)
    top = torch.where(dead, torch.full_like(top, -1e6), top)  # the notebook's sentinel
    idx = torch.where(dead, torch.full_like(idx, -1), idx)
    smax, smin = top[..., 0], top[..., -1]
    lo, hi = am1 * smin - 1.0, am1 * smax + 1.0
    tau = 0.5 * (lo + hi)
    done = torch.zeros_like(tau, dtype=torch.bool)
    for _ in range(5):
        u = am1 * top - tau[..., None]
        # the notebook's loop stops at the first u <= 0 (scores are sorted)
        alive = torch.cumprod((u > 0).to(u.dtype), dim=-1).bool()
        up = torch.where(alive, torch.clamp(u, min=1e-8) ** inv, torch.zeros_like(u))
        f = up.sum(-1) - 1.0
        done = done | (f.abs() < 1e-4)
        pos = f > 0
        lo = torch.where(~done & pos, tau, lo)
        hi = torch.where(~done & ~pos, tau, hi)
        tn = 0.5 * (lo + hi)
        tn = torch.maximum(tn, smin * am1 - 10.0)
        tn = torch.minimum(tn, smax * am1 + 10.0)
        tau = torch.where(done, tau, tn)
    u = am1 * top - tau[..., None]
    p = torch.where(u > 1e-8, torch.clamp(u, min=1e-8) ** inv, torch.zeros_like(u))
    w = p / torch.clamp(p.sum(-1, keepdim=True), min=1e-8)
    Vg = torch.gather(V[:, None, :, :].expand(-1, Q.shape[1], -1, -1), 2,
                      idx.clamp(min=0)[..., None].expand(-1, -1, -1, V.shape[-1]))
    Vg = Vg * (idx >= 0)[..., None]
    return torch.einsum("bqj,bqjd->bqd", w, Vg), tau, idx
