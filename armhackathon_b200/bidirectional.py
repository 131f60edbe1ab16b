"""Bidirectional Mamba-1 scan: both time directions of the same projected
inputs, merged (reference python/arm_scan/bidirectional.py:98-175).

With tied weights and no ``last_state`` request the fused two-direction op
runs; untied backward weights (``reverse_params``) or a ``last_state`` request
take two ``selective_scan`` calls, the backward one with ``reverse=True``
(never a flipped copy of the inputs).

Merges: "sum" (out_fwd + out_bwd), "mean", "concat" (channel axis, giving
(batch, 2*dim, len)) and "none" (the pair, for a learned combine).  With a
shared D under "sum" the skip term is counted in both directions (2*D*u),
which is what per-direction mixers do; pass D=None to add it once yourself.
"""

import torch

from .op import selective_scan, selective_scan_bidirectional, selective_scan_bidirectional_sum

_MERGES = ("sum", "mean", "concat", "none")


def bidirectional_scan(u, delta, A, B, C, D=None, z=None, delta_bias=None,
                       delta_softplus=False, merge="sum", reverse_params=None,
                       return_last_state=False):
    """Scan forward and backward in time and merge.

    Layouts are ``selective_scan``'s.  ``reverse_params`` overrides any of
    "A", "D", "delta", "delta_bias", "B", "C" for the backward pass (given in
    forward time order).  With ``return_last_state`` each output is paired
    with its final state (the backward one is the state at t = 0).
    """
    if merge not in _MERGES:
        raise ValueError(f"merge must be one of {_MERGES}, got {merge!r}")
    if (reverse_params is None and not return_last_state and merge in ("sum", "mean")
            and u.device.type == "cuda"):
        # one library call: the traversals share their first pass and the
        # reverse one sums into the output in place
        out = selective_scan_bidirectional_sum(
            u, delta, A, B, C, D=D, z=z, delta_bias=delta_bias, delta_softplus=delta_softplus)
        return out if merge == "sum" else out.mul_(0.5)
    if reverse_params is None and not return_last_state:
        out_f, out_b = selective_scan_bidirectional(
            u, delta, A, B, C, D=D, z=z, delta_bias=delta_bias,
            delta_softplus=delta_softplus)
    else:
        p = reverse_params or {}
        rev = selective_scan(
            u, p.get("delta", delta), p.get("A", A), p.get("B", B), p.get("C", C),
            D=p.get("D", D), z=z, delta_bias=p.get("delta_bias", delta_bias),
            delta_softplus=delta_softplus, return_last_state=return_last_state,
            reverse=True)
        fwd = selective_scan(
            u, delta, A, B, C, D=D, z=z, delta_bias=delta_bias,
            delta_softplus=delta_softplus, return_last_state=return_last_state)
        if return_last_state:
            (out_f, last_f), (out_b, last_b) = fwd, rev
        else:
            out_f, out_b = fwd, rev
    if merge == "sum":
        out = out_f + out_b
    elif merge == "mean":
        out = (out_f + out_b) * 0.5
    elif merge == "concat":
        out = torch.cat((out_f, out_b), dim=1)
    else:
        out = (out_f, out_b)
    if not return_last_state:
        return out
    return (out, (last_f, last_b)) if merge != "none" else ((out_f, last_f), (out_b, last_b))
