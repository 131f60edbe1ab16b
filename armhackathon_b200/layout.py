"""Shape rules of the Mamba-1 scan arguments, shared by the torch ops
(op.py) and the numpy front-end (numpy_api.py); no torch import.

The layouts are the reference's (python/arm_scan/op.py:63-100,
kernel/arm-scan-core/src/lib.rs:9-16): u, delta, z (batch, dim, len); A
(dim, state); B, C (batch, state, len) or (batch, groups, state, len); D,
delta_bias (dim,); initial state (batch, dim, state).  The C ABI cannot see
buffer lengths, so every front-end checks the shapes here before a call.
"""

from dataclasses import dataclass
from typing import Optional, Sequence


@dataclass(frozen=True)
class M1Layout:
    batch: int
    dim: int
    length: int
    state: int
    groups: int

    @property
    def bc_shape(self):
        """B / C as the kernels read them: (batch, groups, state, len)."""
        return (self.batch, self.groups, self.state, self.length)


def _shape(x) -> Optional[tuple]:
    return None if x is None else tuple(int(d) for d in x)


def m1_layout(u: Sequence[int], delta: Sequence[int], A: Sequence[int], B: Sequence[int],
              C: Sequence[int], D=None, z=None, delta_bias=None,
              initial_state=None) -> M1Layout:
    """Check the argument shapes (tuples, or anything with ``len`` and
    indexing) and return the scan's dimensions; raises ValueError naming the
    first argument that does not fit."""
    u, delta, A, B, C = (_shape(s) for s in (u, delta, A, B, C))
    if len(u) != 3:
        raise ValueError(f"u must be (batch, dim, len), got {u}")
    batch, dim, length = u
    if len(A) != 2 or A[0] != dim:
        raise ValueError(f"A must be ({dim}, state), got {A}")
    state = A[1]
    groups = None
    for name, s in (("B", B), ("C", C)):
        if len(s) == 3 and s == (batch, state, length):
            g = 1
        elif len(s) == 4 and s[0] == batch and s[2:] == (state, length) and s[1] >= 1:
            g = s[1]
        else:
            raise ValueError(f"{name} must be ({batch}, {state}, {length}) or "
                             f"({batch}, groups, {state}, {length}), got {s}")
        if groups is not None and g != groups:
            raise ValueError(f"B and C disagree on the number of groups ({groups} vs {g})")
        groups = g
    if dim % groups:
        raise ValueError(f"groups ({groups}) must divide dim ({dim})")
    wants = (("delta", delta, (batch, dim, length)), ("z", _shape(z), (batch, dim, length)),
             ("D", _shape(D), (dim,)), ("delta_bias", _shape(delta_bias), (dim,)),
             ("initial_state", _shape(initial_state), (batch, dim, state)))
    for name, got, want in wants:
        if got is not None and got != want:
            raise ValueError(f"{name} must be {want}, got {got}")
    return M1Layout(batch, dim, length, state, groups)
