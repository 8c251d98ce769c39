"""Float64 torch reference for the engine's opt-in modes (test
infrastructure): α-entmax attention with the threshold τ defined
implicitly by the row mass, and its autograd gradient.

    s   = clamp(sm_scale · q·k, -10, 10) over the visible keys (causal:
          K_idx <= Q_idx; `keys`, if given, restricts them further)
    p_j = [(α-1) s_j - τ]_+^{1/(α-1)},  τ such that Σ_j p_j = mass
    O   = Σ_j p_j v_j / (Σ_j p_j + 1e-8)

mass = 1 is exact α-entmax (tau_mode="exact").  τ is found by bisection
without autograd; one Newton step from it, with autograd, then carries the
implicit-function derivative dτ/ds = -(∂F/∂s)/(∂F/∂τ) into the gradient
(at the root the step's own value change is zero), which is what
grad_mode="jacobian" computes.
"""
import torch


def _solve_tau(u0, vis, am1, mass, iters=200):
    """τ with Σ_vis relu(u0 - τ)^{1/(α-1)} = mass per row (u0 = (α-1)s)."""
    inv = 1.0 / am1
    neg = torch.finfo(u0.dtype).min
    mx = torch.where(vis, u0, torch.full_like(u0, neg)).max(dim=-1).values
    hi = mx.clone()
    lo = mx - torch.clamp(mass, min=1e-30) ** am1 - 1.0
    for _ in range(iters):
        mid = 0.5 * (lo + hi)
        F = (torch.clamp(u0 - mid[..., None], min=0) ** inv * vis).sum(-1)
        big = F >= mass
        lo = torch.where(big, mid, lo)
        hi = torch.where(big, hi, mid)
    return 0.5 * (lo + hi)


def entmax_attention(Q, K, V, Qi, Ki, alpha, sm_scale, causal=True, keys=None, mass=None):
    """Q, K, V: [BH, N, d] float64 (requires_grad as wanted); Qi/Ki: [BH, N].
    keys: optional bool [BH, NQ, NK] restricting the keys; mass: optional
    [BH, NQ] row masses (default 1).  Returns O [BH, NQ, d] and τ."""
    am1 = alpha - 1.0
    inv = 1.0 / am1
    s = torch.clamp(sm_scale * torch.einsum("bqd,bkd->bqk", Q, K), -10.0, 10.0)
    vis = torch.ones_like(s, dtype=torch.bool)
    if causal:
        vis = Ki[:, None, :] <= Qi[:, :, None]
    if keys is not None:
        vis = vis & keys
    visf = vis.to(s.dtype)
    u0 = am1 * s
    if mass is None:
        mass = torch.ones(s.shape[:2], dtype=s.dtype)
    with torch.no_grad():
        tau0 = _solve_tau(u0.detach(), vis, am1, mass)
    F = (torch.clamp(u0 - tau0[..., None], min=0) ** inv * visf).sum(-1)
    dF = -inv * (torch.clamp(u0 - tau0[..., None], min=0) ** (inv - 1.0) *
                 (u0 > tau0[..., None]) * visf).sum(-1)
    tau = tau0 - (F - mass) / dF
    p = torch.clamp(u0 - tau[..., None], min=0) ** inv * visf
    n = p.sum(-1, keepdim=True)
    O = torch.einsum("bqk,bkd->bqd", p, V) / (n + 1e-8)
    return O, tau
