"""SS2D: the four-direction 2D cross-scan on the Mamba-1 recurrence
(reference python/arm_scan/ss2d.py:102-167).

The four directions are two traversal pairs over two token orderings:
row-major (h, w) and column-major (w, h), each scanned forward and backward.
Merged ("sum" / "mean") on CUDA grids, all four are one library call that
reads the grids in place (``selective_scan_ss2d``: the row-major pair as a
bidirectional sum over the grid's own order, the column-major pair as
per-column segments, split in time when the columns are too few to fill
the GPU).  Otherwise (merge "none", a custom scan pair, d_state > 16) both
orderings are stacked on the batch axis as views, so one bidirectional call
covers all four directions.  Time-varying inputs arrive grid-shaped.
"""

import torch

_MERGES = ("sum", "mean", "none")


def grid_to_views(t):
    """(b, c, h, w) -> (2b, c, h*w): row-major stacked over column-major."""
    b, c, h, w = t.shape
    rows = t.reshape(b, c, h * w)
    cols = t.transpose(2, 3).reshape(b, c, w * h)
    return torch.cat((rows, cols), dim=0)


def views_to_grid(row_seq, col_seq, h, w):
    """Inverse of ``grid_to_views``' two halves, back to (b, c, h, w)."""
    b, c, _ = row_seq.shape
    rows = row_seq.reshape(b, c, h, w)
    cols = col_seq.reshape(b, c, w, h).transpose(2, 3)
    return rows, cols


def scan_pair_arm(u, delta, A, B, C, D=None, delta_bias=None, delta_softplus=True):
    """(fwd, bwd) from one fused bidirectional call."""
    from .bidirectional import bidirectional_scan
    return bidirectional_scan(u, delta, A, B, C, D=D, delta_bias=delta_bias,
                              delta_softplus=delta_softplus, merge="none")


def scan_fn_arm(u, delta, A, B, C, D=None, delta_bias=None, delta_softplus=True):
    """Single-direction scan (the seam four-separate-scans models use)."""
    from .op import selective_scan
    return selective_scan(u, delta, A, B, C, D=D, delta_bias=delta_bias,
                          delta_softplus=delta_softplus)


def _in_place_fits(u, A, B):
    """Whether the one-call in-place SS2D covers this shape: d_state <= 16
    and, with B/C groups, a multiple of 8 channels per group."""
    d = u.shape[1]
    groups = B.shape[1] if B.dim() == 5 else 1
    return A.shape[1] <= 16 and (groups == 1 or (d // groups) % 8 == 0)


def ss2d_scan(u, delta, A, B, C, D=None, delta_bias=None, delta_softplus=True,
              merge="sum", scan_pair=None):
    """Four-direction cross-scan over a token grid.

    u, delta : (b, d, h, w);  A : (d, n);  B, C : (b, n, h, w) or
    (b, groups, n, h, w);  D, delta_bias : (d,).
    merge "sum" / "mean" over (row_fwd, row_bwd, col_fwd, col_bwd), or "none"
    for the four planes, each (b, d, h, w).  D applies in every direction.
    """
    if merge not in _MERGES:
        raise ValueError(f"merge must be one of {_MERGES}, got {merge!r}")
    if u.dim() != 4:
        raise ValueError(f"u must be (b, d, h, w), got {tuple(u.shape)}")
    if delta.shape != u.shape:
        raise ValueError(f"delta {tuple(delta.shape)} must match u {tuple(u.shape)}")
    if scan_pair is None:
        scan_pair = scan_pair_arm
    b, _, h, w = u.shape
    for name, t in (("B", B), ("C", C)):
        if t.shape[0] != b or tuple(t.shape[-2:]) != (h, w):
            raise ValueError(f"{name} must be (b={b}, ..., {h}, {w}), got {tuple(t.shape)}")

    def _views(t):
        if t.dim() == 5:
            bb, g, n, hh, ww = t.shape
            v = grid_to_views(t.reshape(bb, g * n, hh, ww))
            return v.reshape(2 * bb, g, n, hh * ww)
        return grid_to_views(t)

    if scan_pair is scan_pair_arm and merge != "none" and u.device.type == "cuda" \
            and _in_place_fits(u, A, B):
        # one library call: all four traversals over the grids in place
        from .op import selective_scan_ss2d
        return selective_scan_ss2d(u, delta, A, B, C, D=D, delta_bias=delta_bias,
                                   delta_softplus=delta_softplus, merge=merge)
    fwd, bwd = scan_pair(grid_to_views(u), grid_to_views(delta), A, _views(B), _views(C),
                         D=D, delta_bias=delta_bias, delta_softplus=delta_softplus)
    row_f, col_f = views_to_grid(fwd[:b], fwd[b:], h, w)
    row_b, col_b = views_to_grid(bwd[:b], bwd[b:], h, w)
    if merge == "none":
        return row_f, row_b, col_f, col_b
    out = row_f + row_b + col_f + col_b
    return out if merge == "sum" else out * 0.25


def use_arm_scan(module, enable=True):
    """Point every block of ``module`` exposing ``scan_pair_fn`` / ``scan_fn``
    at this package's kernels (enable=True).  Returns the number of blocks
    switched.  enable=False restores nothing by itself: the caller's own
    torch implementation must be reassigned by the caller."""
    n = 0
    for m in module.modules():
        touched = False
        if enable and hasattr(m, "scan_pair_fn"):
            m.scan_pair_fn = scan_pair_arm
            touched = True
        if enable and hasattr(m, "scan_fn"):
            m.scan_fn = scan_fn_arm
            touched = True
        n += int(touched)
    return n
