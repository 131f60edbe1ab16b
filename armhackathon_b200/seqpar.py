"""Sequence-parallel bidirectional Mamba-1 scan across ranks (one GPU each).

A long single sequence is split into contiguous segments, segment r on rank r
(rank order = time order).  The recurrence h_t = a_t * h_{t-1} + b_t is linear
in h, and the decay across a whole segment factorises per state:
prod_t exp(dt_t * A_n) = exp(A_n * sum_t dt_t).  So a segment is summarised by
(h_end from a zero start, sum dt) per (batch, channel): about
batch*dim*(state+1)*4 bytes per direction (~100 KB at dim 1536, state 16).

Per call:
  1. each rank computes the final states of its segment, forward and
     backward from zero, without outputs (selective_scan_final_state), and
     sum(dt) per row;
  2. one all_gather of those summaries (the only collective);
  3. rank r folds the summaries of ranks < r (forward) and > r (backward)
     into its incoming states;
  4. rank r scans its segment in both directions from those states.
With the library's own functions on CUDA tensors and merge "sum", steps 1
and 4 are the two phases of one ``BidirectionalSegment``: step 1 reads the
segment once for both directions' end states and the dt sum, keeping that
pass's per-chunk aggregates on the device, and step 4 rescans both
directions from the incoming states without a second pass to rebuild them.
The fold is exact algebra, so the result equals the unsplit bidirectional
scan up to fp32 rounding.  No rank waits on another except inside the
all_gather, whose timeout is the process group's.
"""

import torch
import torch.distributed as dist
import torch.nn.functional as F


def _segment_dt_sum(delta, delta_bias, delta_softplus):
    dt = delta.float()
    if delta_bias is not None:
        dt = dt + delta_bias.float()[:, None]
    if delta_softplus:
        dt = F.softplus(dt)  # threshold 20, the kernel's contract
    return dt.sum(-1)


def fold_carries(h_ends, dt_sums, A, rank, reverse):
    """Incoming state of segment ``rank`` from the other segments' summaries.

    h_ends (W, B, D, N) (or a list of W tensors): each segment's state after its traversal from zero;
    dt_sums (W, B, D); A (D, N).  Forward: h_in = sum over j < rank of
    exp(A * sum_{j < k < rank} dt_k) * h_end(j); reverse: the same over
    j > rank with the segments between j and rank.  Evaluated for all j at
    once (a handful of tensor ops whatever the number of segments): the
    decay from segment j to ``rank`` is exp(A * (C_between)), with C the
    cumulative dt sums over the segments."""
    if isinstance(h_ends, (list, tuple)):
        h_ends, dt_sums = torch.stack(list(h_ends)), torch.stack(list(dt_sums))
    W = h_ends.shape[0]
    idx = torch.arange(W, device=h_ends.device)
    cum = torch.cumsum(dt_sums, 0)                    # C_j = sum_{k <= j}
    if not reverse:
        upto = cum[rank - 1] if rank > 0 else torch.zeros_like(cum[0])
        between = upto[None] - cum                    # sum_{j < k < rank}
        mask = idx < rank
    else:
        between = cum[:-1] if W > 1 else cum[:0]      # sum_{rank < k < j} = C_{j-1} - C_rank
        between = torch.cat([torch.zeros_like(cum[:1]), between], 0) - cum[rank][None]
        mask = idx > rank
    w = torch.exp(A.float()[None, None] * between.clamp_min(0)[..., None])
    w = w * mask.view(W, *([1] * (w.dim() - 1)))
    return (w * h_ends).sum(0)


def segment_summary(u, delta, A, B, C, delta_bias, delta_softplus):
    """This segment's summary, packed (B, D, 2N + 1): forward end state,
    backward end state (both from zero) and the sum of dt, from one library
    call that reads the segment once."""
    from .op import selective_scan_segment_summary
    hf, hb, sdt = selective_scan_segment_summary(u, delta, A, B, C, delta_bias=delta_bias,
                                                 delta_softplus=delta_softplus)
    return torch.cat([hf, hb, sdt[..., None]], dim=-1).contiguous()


def bidirectional_scan_seqpar(u, delta, A, B, C, D=None, z=None, delta_bias=None,
                              delta_softplus=False, merge="sum", group=None, scan_fn=None,
                              state_fn=None):
    """Bidirectional scan of one sequence split over the ranks of ``group``.

    Every rank passes its own segment (same layouts as ``selective_scan``:
    u, delta, z (batch, dim, L_rank); B, C (batch, [groups,] state, L_rank);
    A (dim, state); D, delta_bias (dim,)).  Returns this rank's segment of the
    merged output ("sum") or (fwd, bwd) ("none").  ``scan_fn`` and
    ``state_fn`` default to this package's ``selective_scan`` and
    ``selective_scan_final_state``; tests substitute CPU references.
    """
    if merge not in ("sum", "none"):
        raise ValueError(f"merge must be 'sum' or 'none', got {merge!r}")
    if scan_fn is None:
        from .op import selective_scan as scan_fn
    if state_fn is None:
        from .op import selective_scan_final_state as state_fn
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    skw = dict(delta_bias=delta_bias, delta_softplus=delta_softplus)
    # the library's own functions on CUDA tensors: both directions' summaries
    # from one shared first pass, and both outputs summed by one call
    fused = merge == "sum" and u.device.type == "cuda" and getattr(
        scan_fn, "__module__", "") == __package__ + ".op" and getattr(
        state_fn, "__module__", "") == __package__ + ".op"
    if fused:
        from .op import BidirectionalSegment
        seg = BidirectionalSegment(u, delta, A, B, C, D=D, z=z, **skw)
        hf, hb, sdt = seg.summary()
        packed = torch.cat([hf, hb, sdt[..., None]], dim=-1).contiguous()
    else:
        hf = state_fn(u, delta, A, B, C, **skw)
        hb = state_fn(u, delta, A, B, C, reverse=True, **skw)
        sdt = _segment_dt_sum(delta, delta_bias, delta_softplus).to(hf.dtype)
        packed = torch.cat([hf, hb, sdt[..., None]], dim=-1).contiguous()
    parts = [torch.empty_like(packed) for _ in range(world)]
    dist.all_gather(parts, packed, group=group)
    allp = torch.stack(parts)
    N = (packed.shape[-1] - 1) // 2
    h_f, h_b, sums = allp[..., :N], allp[..., N:2 * N], allp[..., 2 * N]
    kw = dict(D=D, z=z, **skw)
    h_in_f = fold_carries(h_f, sums, A, rank, False) if rank > 0 else None
    h_in_b = fold_carries(h_b, sums, A, rank, True) if rank < world - 1 else None
    if fused:
        return seg.finish(h_in_f, h_in_b)
    yf = scan_fn(u, delta, A, B, C, initial_state=h_in_f, **kw)
    yb = scan_fn(u, delta, A, B, C, reverse=True, initial_state=h_in_b, **kw)
    return yf + yb if merge == "sum" else (yf, yb)
