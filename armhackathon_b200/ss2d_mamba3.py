"""SS2D on the Mamba-3 recurrence (reference python/arm_scan/ss2d_mamba3.py).

Same topology as ``ss2d``: row-major and column-major orderings stacked on the
batch axis, each traversed forward and backward by ``mamba3_scan_pair``.
Mamba-3 tensors come in two layout families:

    time-major   q, k (b, H, W, g, dqk); v, z (b, H, W, h, dv);
                 angles (b, H, W, h, r)        -> (2b, H*W, ...)
    head-major   adt, dt, trap (b, h, H, W)    -> (2b, h, H*W)

The angle pre-pass accumulates along the traversal order, so it runs on the
views (each ordering gets its own theta), never on the grid.
"""

from typing import Optional

import torch

from .ss2d import _MERGES, grid_to_views


def grid_to_views_time_major(t):
    """(b, H, W, *rest) -> (2b, H*W, *rest): row-major over column-major."""
    if t.dim() < 3:
        raise ValueError(f"expected (b, H, W, ...), got {tuple(t.shape)}")
    b, h, w = t.shape[:3]
    rest = t.shape[3:]
    rows = t.reshape(b, h * w, *rest)
    cols = t.transpose(1, 2).reshape(b, w * h, *rest)
    return torch.cat((rows, cols), dim=0)


def views_to_grid_time_major(row_seq, col_seq, h, w):
    """Inverse of ``grid_to_views_time_major``' two halves."""
    b = row_seq.shape[0]
    rest = row_seq.shape[2:]
    rows = row_seq.reshape(b, h, w, *rest)
    cols = col_seq.reshape(b, w, h, *rest).transpose(1, 2)
    return rows, cols


def scan_pair_mamba3(q, k, v, adt, dt, trap, q_bias, k_bias, angles=None, D=None, z=None):
    """Default two-direction primitive: ``mamba3_scan_pair``."""
    from .mamba3 import mamba3_scan_pair
    return mamba3_scan_pair(q, k, v, adt, dt, trap, q_bias, k_bias, angles=angles, D=D, z=z)


def _check_grid(name, t, b, h, w, dim, head_major=False):
    if t.dim() != dim:
        raise ValueError(f"{name} must be {dim}-D "
                         f"{'(b, heads, H, W)' if head_major else '(b, H, W, ...)'}, "
                         f"got {tuple(t.shape)}")
    got = (t.shape[0], t.shape[2], t.shape[3]) if head_major else tuple(t.shape[:3])
    if got != (b, h, w):
        raise ValueError(f"{name} grid axes {got} do not match (b, H, W) = {(b, h, w)}; "
                         f"full shape {tuple(t.shape)}")


@torch.library.custom_op("arm_scan::ss2d_mamba3_fused", mutates_args=())
def _ss2d_fused_op(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, adt: torch.Tensor,
                   dt: torch.Tensor, trap: torch.Tensor, q_bias: torch.Tensor, k_bias: torch.Tensor,
                   angles: torch.Tensor, d_skip: Optional[torch.Tensor], z: Optional[torch.Tensor],
                   grid_w: int) -> torch.Tensor:
    from . import _ffi
    from .op import _on_device, _ptr, _stream, _CALLS
    b, length, _, dqk = q.shape
    h, dv = v.shape[2], v.shape[3]
    dims = _ffi.ArmMamba3Dims(b, h, dv, dqk, length, 1)
    out = v.new_empty((b, length, h, dv))
    with _on_device(v):
        _ffi.ss2d_mamba3_raw(
            dims, grid_w, [q.data_ptr(), k.data_ptr(), v.data_ptr(), adt.data_ptr(),
                           dt.data_ptr(), trap.data_ptr(), q_bias.data_ptr(), k_bias.data_ptr(),
                           angles.data_ptr()],
            angles.shape[3], _ptr(d_skip), _ptr(z), out.data_ptr(), _stream(v))
    _CALLS["n"] += 1
    return out


@_ss2d_fused_op.register_fake
def _(q, k, v, adt, dt, trap, q_bias, k_bias, angles, d_skip, z, grid_w):
    return v.new_empty((q.shape[0], q.shape[1], v.shape[2], v.shape[3]))


def _ss2d_fused(q, k, v, adt, dt, trap, q_bias, k_bias, angles, D, z, h, w):
    """All four traversals in one library call reading the grid in place;
    returns the sum (b, H, W, heads, dv)."""
    b = q.shape[0]
    f = lambda t: t.to(torch.float32).contiguous()  # noqa: E731
    L = h * w
    out = _ss2d_fused_op(
        f(q).reshape(b, L, 1, q.shape[-1]), f(k).reshape(b, L, 1, k.shape[-1]),
        f(v).reshape(b, L, v.shape[3], v.shape[4]), f(adt).reshape(b, adt.shape[1], L),
        f(dt).reshape(b, dt.shape[1], L), f(trap).reshape(b, trap.shape[1], L), f(q_bias),
        f(k_bias), f(angles).reshape(b, L, angles.shape[3], angles.shape[4]),
        None if D is None else f(D), None if z is None else f(z).reshape(b, L, *z.shape[3:]), w)
    return out.reshape(b, h, w, v.shape[3], v.shape[4])


def ss2d_scan_mamba3(q, k, v, adt, dt, trap, q_bias, k_bias, angles, D=None, z=None,
                     merge="sum", scan_pair=None):
    """Four-direction cross-scan over a token grid with Mamba-3 SISO.

    Layouts in the module docstring; q_bias, k_bias (h, dqk); D (h,).
    merge "sum" / "mean", or "none" for (row_fwd, row_bwd, col_fwd, col_bwd),
    each (b, H, W, h, dv).  D and z apply inside every direction.
    """
    if merge not in _MERGES:
        raise ValueError(f"merge must be one of {_MERGES}, got {merge!r}")
    if q.dim() != 5:
        raise ValueError(f"q must be (b, H, W, groups, dqk), got {tuple(q.shape)}")
    b, h, w = q.shape[:3]
    for name, t in (("q", q), ("k", k), ("v", v), ("angles", angles)):
        _check_grid(name, t, b, h, w, 5)
    for name, t in (("adt", adt), ("dt", dt), ("trap", trap)):
        _check_grid(name, t, b, h, w, 4, head_major=True)
    if z is not None:
        _check_grid("z", z, b, h, w, 5)
    if (scan_pair is None and merge in ("sum", "mean") and q.shape[3] == 1
            and all(t.is_cuda for t in (q, k, v, adt, dt, trap, angles))
            and 1 <= angles.shape[4] <= q.shape[4] // 2):
        out = _ss2d_fused(q, k, v, adt, dt, trap, q_bias, k_bias, angles, D, z, h, w)
        return out if merge == "sum" else out * 0.25
    if scan_pair is None:
        scan_pair = scan_pair_mamba3
    fwd, bwd = scan_pair(
        grid_to_views_time_major(q), grid_to_views_time_major(k), grid_to_views_time_major(v),
        grid_to_views(adt), grid_to_views(dt), grid_to_views(trap), q_bias, k_bias,
        angles=grid_to_views_time_major(angles), D=D,
        z=None if z is None else grid_to_views_time_major(z))
    row_f, col_f = views_to_grid_time_major(fwd[:b], fwd[b:], h, w)
    row_b, col_b = views_to_grid_time_major(bwd[:b], bwd[b:], h, w)
    if merge == "none":
        return row_f, row_b, col_f, col_b
    out = row_f + row_b + col_f + col_b
    return out if merge == "sum" else out * 0.25
