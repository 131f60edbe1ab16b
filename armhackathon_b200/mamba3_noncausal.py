"""Non-causal Mamba-3 aggregation, 1D and 2D
(reference python/arm_scan/mamba3_noncausal.py).

Unrolling the recurrence gives y_t = sum_s M[t,s] (q_t . k_s) v_s + D v_t with
M[t,s] = exp(L_t - L_s) * scale_s; the decay factorises, so the sum over all s
is a forward scan plus a backward scan minus the s == t term counted twice:

    non-causal = forward + backward - diagonal

``noncausal_scan`` computes exactly that with two kernel traversals;
``noncausal_scan_dense`` is the explicit O(L^2) mask form (plain torch), kept
as an independent check.  The diagonal needs q_t . k_t, which RoPE leaves
unchanged (both vectors rotate by the same angle), so it is computed from the
unrotated tensors.
"""

import torch

from .ss2d import _MERGES, grid_to_views
from .ss2d_mamba3 import grid_to_views_time_major, views_to_grid_time_major


def _diagonal_term(q, k, v, dt, trap, q_bias, k_bias, D=None, z=None):
    """(D + gamma_t (q_t . k_t)) v_t, gated -- the s == t contribution."""
    if q.dim() == 4:
        q = q[:, :, 0, :]
    if k.dim() == 4:
        k = k[:, :, 0, :]
    b, length, dqk = q.shape
    h = v.shape[2]
    qb = q.unsqueeze(2) + q_bias.view(1, 1, h, dqk)
    kb = k.unsqueeze(2) + k_bias.view(1, 1, h, dqk)
    qk = (qb * kb).sum(-1)
    gamma = dt * torch.sigmoid(trap)
    coef = gamma.permute(0, 2, 1) * qk
    if D is not None:
        coef = coef + D.view(1, 1, h)
    out = coef.unsqueeze(-1) * v
    if z is not None:
        out = out * (z * torch.sigmoid(z))
    return out


def noncausal_scan(q, k, v, adt, dt, trap, q_bias, k_bias, angles=None, D=None, z=None,
                   cos=None, sin=None):
    """Non-causal 1D aggregation via two scans, (b, l, h, dv)."""
    from .mamba3 import mamba3_scan_pair
    fwd, bwd = mamba3_scan_pair(q, k, v, adt, dt, trap, q_bias, k_bias, angles=angles, D=D,
                                z=z, cos=cos, sin=sin)
    diag = _diagonal_term(q.to(fwd.device, torch.float32), k.to(fwd.device, torch.float32),
                          v.to(fwd.device, torch.float32), dt.to(fwd.device, torch.float32),
                          trap.to(fwd.device, torch.float32),
                          q_bias.to(fwd.device, torch.float32),
                          k_bias.to(fwd.device, torch.float32),
                          None if D is None else D.to(fwd.device, torch.float32),
                          None if z is None else z.to(fwd.device, torch.float32))
    return fwd + bwd - diag


def noncausal_scan_dense(q, k, v, adt, dt, trap, q_bias, k_bias, angles=None, D=None,
                         z=None, cos=None, sin=None, causal=False):
    """Non-causal (or, with causal=True, causal) aggregation through the
    explicit (L, L) mask, y = (M o (Q K^T)) V + D V, gated.  Plain torch, O(L^2);
    an independent check of the scan route, not a product path."""
    from .mamba3 import angles_to_cos_sin
    if q.dim() == 3:
        q = q.unsqueeze(2)
    if k.dim() == 3:
        k = k.unsqueeze(2)
    b, length, _, dqk = q.shape
    h = v.shape[2]
    half = dqk // 2
    if cos is None:
        if angles is None:
            raise ValueError("pass either `angles` or both `cos` and `sin`")
        cos, sin = angles_to_cos_sin(angles, dt, half)
    qb = q[:, :, 0, :].unsqueeze(2) + q_bias.view(1, 1, h, dqk)
    kb = k[:, :, 0, :].unsqueeze(2) + k_bias.view(1, 1, h, dqk)

    def rope(t):
        v0, v1 = t[..., 0::2], t[..., 1::2]
        out = torch.empty_like(t)
        out[..., 0::2] = v0 * cos - v1 * sin
        out[..., 1::2] = v0 * sin + v1 * cos
        return out

    qr, kr = rope(qb), rope(kb)
    lam = torch.sigmoid(trap)
    gamma = dt * lam

    def half_mask(reverse):
        a, d_, l_ = adt, dt, lam
        if reverse:
            a, d_, l_ = (torch.flip(x, dims=[-1]) for x in (a, d_, l_))
        sh = torch.zeros_like(d_)
        sh[..., :-1] = d_[..., 1:] * (1.0 - l_[..., 1:])
        sc = d_ * l_ + sh
        cum = torch.cumsum(a, dim=-1)
        m = torch.exp(cum.unsqueeze(-1) - cum.unsqueeze(-2)) * sc.unsqueeze(-2)
        m = m * torch.tril(torch.ones(length, length, dtype=m.dtype, device=m.device), -1)
        return torch.flip(m, dims=[-1, -2]) if reverse else m

    M = half_mask(False) + torch.diag_embed(gamma)
    if not causal:
        M = M + half_mask(True)
    qk = torch.einsum("bthd,bshd->bhts", qr, kr)
    out = torch.einsum("bhts,bhts,bshp->bthp", M, qk, v)
    if D is not None:
        out = out + D.view(1, 1, h, 1) * v
    if z is not None:
        out = out * (z * torch.sigmoid(z))
    return out


def ss2d_noncausal_mamba3(q, k, v, adt, dt, trap, q_bias, k_bias, angles, D=None, z=None,
                          merge="sum"):
    """Four-direction non-causal 2D aggregation: per ordering
    (fwd + bwd - diag), then rows + cols.  merge "none" returns (rows, cols),
    each (b, H, W, h, dv)."""
    if merge not in _MERGES:
        raise ValueError(f"merge must be one of {_MERGES}, got {merge!r}")
    from .mamba3 import mamba3_scan_pair
    b, hh, ww = q.shape[:3]
    qv, kv, vv = (grid_to_views_time_major(t) for t in (q, k, v))
    dtv, trapv = grid_to_views(dt), grid_to_views(trap)
    zv = None if z is None else grid_to_views_time_major(z)
    fwd, bwd = mamba3_scan_pair(qv, kv, vv, grid_to_views(adt), dtv, trapv, q_bias, k_bias,
                                angles=grid_to_views_time_major(angles), D=D, z=zv)
    dev = fwd.device
    f32 = lambda t: None if t is None else t.to(dev, torch.float32)  # noqa: E731
    diag = _diagonal_term(f32(qv), f32(kv), f32(vv), f32(dtv), f32(trapv), f32(q_bias),
                          f32(k_bias), f32(D), f32(zv))
    nc = fwd + bwd - diag
    rows, cols = views_to_grid_time_major(nc[:b], nc[b:], hh, ww)
    if merge == "none":
        return rows, cols
    out = rows + cols
    return out if merge == "sum" else out * 0.5
