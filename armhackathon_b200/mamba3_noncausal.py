"""Non-causal Mamba-3 aggregation, 1D and on a token grid (the surface of the
reference's python/arm_scan/mamba3_noncausal.py).

Every token aggregates every other: with the forward mask
M[t, s] = exp(l_t - l_s) * scale_s for s < t (l the cumulative log decay,
scale the trapezoid weight), its mirror image for s > t from the reverse
traversal, and (D + gamma_t) on the diagonal, y = (M o QK^T) V gated by
silu(z).  Both half-masks are exactly what a forward and a reverse scan
compute, and each includes the diagonal, so

    non-causal = forward scan + reverse scan - diagonal term.

``noncausal_scan`` / ``ss2d_noncausal_mamba3`` run that identity in one
library call (arm_scan_mamba3_noncausal_f32_async): the scans accumulate
into one output in place and a kernel subtracts the diagonal term per token
-- no eager broadcast.  ``noncausal_scan_dense`` builds M explicitly, O(L^2),
as an independent check of the scan route (not a product path).
"""

from typing import Optional

import torch

from .ss2d import _MERGES


@torch.library.custom_op("arm_scan::mamba3_noncausal", mutates_args=())
def _noncausal_op(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, adt: torch.Tensor,
                  dt: torch.Tensor, trap: torch.Tensor, q_bias: torch.Tensor,
                  k_bias: torch.Tensor, angles: Optional[torch.Tensor],
                  cos: Optional[torch.Tensor], sin: Optional[torch.Tensor],
                  d_skip: Optional[torch.Tensor], z: Optional[torch.Tensor],
                  grid_w: int) -> torch.Tensor:
    from . import _ffi
    from .op import _CALLS, _on_device, _ptr, _stream
    b, length, _, dqk = q.shape
    h, dv = v.shape[2], v.shape[3]
    out = v.new_empty((b, length, h, dv))
    dims = _ffi.ArmMamba3Dims(b, h, dv, dqk, length, 1)
    with _on_device(v):
        _ffi.noncausal_raw(dims, grid_w, [q.data_ptr(), k.data_ptr(), v.data_ptr(),
                                          adt.data_ptr(), dt.data_ptr(), trap.data_ptr(),
                                          q_bias.data_ptr(), k_bias.data_ptr(), _ptr(angles)],
                           0 if angles is None else angles.shape[-1], _ptr(cos), _ptr(sin),
                           _ptr(d_skip), _ptr(z), out.data_ptr(), _stream(v))
    _CALLS["n"] += 1
    return out


@_noncausal_op.register_fake
def _(q, k, v, adt, dt, trap, q_bias, k_bias, angles, cos, sin, d_skip, z, grid_w):
    return v.new_empty((q.shape[0], q.shape[1], v.shape[2], v.shape[3]))


def _call(q, k, v, adt, dt, trap, q_bias, k_bias, angles, cos, sin, D, z, grid_w):
    """Everything to contiguous fp32 on a CUDA device (CPU inputs go to the
    current CUDA device and the result comes back), then one library call."""
    home = v.device
    dev = home if home.type == "cuda" else torch.device("cuda", torch.cuda.current_device())
    f = lambda t: None if t is None else t.to(dev, torch.float32).contiguous()  # noqa: E731
    b, length = q.shape[:2]
    q4 = f(q).reshape(b, length, 1, q.shape[-1])
    k4 = f(k).reshape(b, length, 1, k.shape[-1])
    out = _noncausal_op(q4, k4, f(v), f(adt), f(dt), f(trap), f(q_bias), f(k_bias), f(angles),
                        f(cos), f(sin), f(D), f(z), grid_w)
    return out.to(home)


def noncausal_scan(q, k, v, adt, dt, trap, q_bias, k_bias, angles=None, D=None, z=None,
                   cos=None, sin=None):
    """Non-causal 1D aggregation, (b, l, h, dv).  q, k (b, l, [1,] dqk);
    v, z (b, l, h, dv); adt, dt, trap (b, h, l); raw angles (b, l, h, r) or
    cos/sin (b, l, h, dqk/2).  Two scans and the diagonal correction in one
    library call."""
    if (cos is None) != (sin is None):
        raise ValueError("pass cos and sin together, or neither")
    if cos is None and angles is None:
        raise ValueError("pass either `angles` or both `cos` and `sin`")
    length = q.shape[1]
    return _call(q, k, v, adt, dt, trap, q_bias, k_bias, None if cos is not None else angles,
                 cos, sin, D, z, length)


def _dense_mask(adt, dt, trap, causal):
    """M[b, h, t, s] of the unrolled recurrence (diagonal: gamma_t)."""
    lam = torch.sigmoid(trap)
    gamma = dt * lam
    L = adt.shape[-1]
    zero = torch.zeros_like(dt[..., :1])
    # trapezoid weight of step s seen from later steps (forward) and from
    # earlier steps (reverse): its own gamma plus the neighbour's (1 - lam) dt
    scale_f = gamma + torch.cat([dt[..., 1:] * (1 - lam[..., 1:]), zero], -1)
    scale_r = gamma + torch.cat([zero, dt[..., :-1] * (1 - lam[..., :-1])], -1)
    cum = torch.cumsum(adt, -1)                              # l_t, inclusive
    cum_prev = cum - adt                                     # l_{t-1}
    t = torch.arange(L, device=adt.device)
    below = (t[:, None] > t[None, :])                        # s < t
    above = (t[:, None] < t[None, :])                        # s > t
    # forward: decays alpha_{s+1} .. alpha_t = exp(l_t - l_s)
    fwd = torch.exp((cum[..., :, None] - cum[..., None, :]).masked_fill(~below, 0.0))
    M = torch.where(below, fwd * scale_f[..., None, :], torch.zeros_like(fwd))
    if not causal:
        # reverse: decays alpha_t .. alpha_{s-1} = exp(l_{s-1} - l_{t-1})
        rev = torch.exp((cum_prev[..., None, :] - cum_prev[..., :, None]).masked_fill(~above, 0.0))
        M = M + torch.where(above, rev * scale_r[..., None, :], torch.zeros_like(rev))
    return M + torch.diag_embed(gamma)


def noncausal_scan_dense(q, k, v, adt, dt, trap, q_bias, k_bias, angles=None, D=None,
                         z=None, cos=None, sin=None, causal=False):
    """The same aggregation (causal=True: the forward scan) through the
    explicit (L, L) mask, y = (M o Q_r K_r^T) V + D V, gated; interleaved RoPE
    as in the SISO scan.  Plain torch, O(L^2), for checking."""
    from .mamba3 import angles_to_cos_sin
    q3 = q if q.dim() == 3 else q[:, :, 0, :]
    k3 = k if k.dim() == 3 else k[:, :, 0, :]
    h, dqk = v.shape[2], q3.shape[-1]
    if cos is None:
        if angles is None:
            raise ValueError("pass either `angles` or both `cos` and `sin`")
        cos, sin = angles_to_cos_sin(angles, dt, dqk // 2)

    def rotated(x, bias):
        xb = x[:, :, None, :] + bias[None, None]              # (b, l, h, dqk)
        pairs = xb.reshape(*xb.shape[:-1], dqk // 2, 2)
        c, s = cos[..., :dqk // 2], sin[..., :dqk // 2]
        re = pairs[..., 0] * c - pairs[..., 1] * s
        im = pairs[..., 0] * s + pairs[..., 1] * c
        return torch.stack([re, im], -1).reshape(xb.shape)

    qk = torch.einsum("bthn,bshn->bhts", rotated(q3, q_bias), rotated(k3, k_bias))
    y = torch.einsum("bhts,bshp->bthp", _dense_mask(adt, dt, trap, causal) * qk, v)
    if D is not None:
        y = y + D[None, None, :, None] * v
    if z is not None:
        y = y * torch.nn.functional.silu(z)
    return y


def ss2d_noncausal_mamba3(q, k, v, adt, dt, trap, q_bias, k_bias, angles, D=None, z=None,
                          merge="sum"):
    """Non-causal aggregation over a token grid, row-major and column-major
    orderings: layouts as ``ss2d_scan_mamba3`` (q, k (b, H, W, 1, dqk);
    v, z, angles (b, H, W, h, *); adt, dt, trap (b, h, H, W)).  merge "sum" /
    "mean" run in one library call; "none" returns (rows, cols), each
    (b, H, W, h, dv)."""
    if merge not in _MERGES:
        raise ValueError(f"merge must be one of {_MERGES}, got {merge!r}")
    b, H, W = q.shape[:3]
    L = H * W
    flat = lambda t: None if t is None else t.reshape(b, L, *t.shape[3:])  # noqa: E731
    hm = lambda t: t.reshape(b, t.shape[1], L)  # noqa: E731
    if merge != "none":
        out = _call(flat(q), flat(k), flat(v), hm(adt), hm(dt), hm(trap), q_bias, k_bias,
                    flat(angles), None, None, D, flat(z), W)
        out = out.reshape(b, H, W, *v.shape[3:])
        return out if merge == "sum" else out * 0.5
    # one ordering at a time: the row-major sequence, then the column-major
    # one as a contiguous transposed copy
    rows = _call(flat(q), flat(k), flat(v), hm(adt), hm(dt), hm(trap), q_bias, k_bias,
                 flat(angles), None, None, D, flat(z), L).reshape(b, H, W, *v.shape[3:])
    tg = lambda t: None if t is None else t.transpose(1, 2).reshape(b, L, *t.shape[3:])  # noqa: E731
    th = lambda t: t.transpose(2, 3).reshape(b, t.shape[1], L)  # noqa: E731
    cols = _call(tg(q), tg(k), tg(v), th(adt), th(dt), th(trap), q_bias, k_bias, tg(angles),
                 None, None, D, tg(z), L).reshape(b, W, H, *v.shape[3:]).transpose(1, 2)
    return rows, cols
