"""PyTorch front-end of the Mamba-1 selective scan.

Same surface as the reference's python/arm_scan/op.py: custom ops
``arm_scan::selective_scan`` and ``arm_scan::selective_scan_bidirectional``
with fake (meta) kernels, so they trace under ``torch.compile`` without a graph
break, and the Python wrappers ``selective_scan`` /
``selective_scan_bidirectional`` with the reference's argument names and
defaults.

Where the computation runs: always on the GPU, through libb200scan.so.
* CUDA tensors are passed as device pointers to the ``_async`` entry points on
  the current torch stream (no host synchronization).
* CPU tensors (what reference callers pass) go through the synchronous entry
  points, which copy them to the current CUDA device, run the kernel and copy
  the results back -- the reference's blocking contract.  Pinned host tensors
  make those copies faster.
There is no CPU implementation: without a GPU the call raises.

Inference only: no autograd formula is registered (as in the reference).
"""

from typing import Optional, Tuple

import torch

from . import _ffi
from .layout import m1_layout

_CALLS = {"n": 0}


def _prep(t: torch.Tensor, device) -> torch.Tensor:
    return t.to(device=device, dtype=torch.float32).contiguous()


def _ptr(t: Optional[torch.Tensor]) -> int:
    return 0 if t is None else t.data_ptr()


def _stream(t: torch.Tensor):
    """Stream handle for a CUDA tensor's device, None for host tensors."""
    if t.device.type == "cuda":
        return torch.cuda.current_stream(t.device).cuda_stream
    return None


class _on_device:
    """Make ``t``'s CUDA device current for the duration of a call."""

    def __init__(self, t):
        self.ctx = torch.cuda.device(t.device) if t.device.type == "cuda" else None

    def __enter__(self):
        if self.ctx is not None:
            self.ctx.__enter__()

    def __exit__(self, *exc):
        if self.ctx is not None:
            self.ctx.__exit__(*exc)


@torch.library.custom_op("arm_scan::selective_scan", mutates_args=())
def _selective_scan_op(
    u: torch.Tensor,
    delta: torch.Tensor,
    a: torch.Tensor,
    b: torch.Tensor,
    c: torch.Tensor,
    d_skip: Optional[torch.Tensor],
    z: Optional[torch.Tensor],
    delta_bias: Optional[torch.Tensor],
    h0: Optional[torch.Tensor],
    delta_softplus: bool,
    reverse: bool,
) -> Tuple[torch.Tensor, torch.Tensor]:
    batch, dim, length = u.shape
    state = a.shape[1]
    groups = b.shape[1] if b.dim() == 4 else 1
    out = torch.empty_like(u)
    last_state = u.new_empty((batch, dim, state))
    dims = _ffi.ArmScanDims(batch, dim, length, state, groups)
    with _on_device(u):
        _ffi.scan_raw(
            dims, u.data_ptr(), delta.data_ptr(), a.data_ptr(), b.data_ptr(), c.data_ptr(),
            _ptr(d_skip), _ptr(z), _ptr(delta_bias), delta_softplus, "auto", "auto",
            out.data_ptr(), last_state.data_ptr(), ptr_h0=_ptr(h0), reverse=reverse,
            stream=_stream(u))
    _CALLS["n"] += 1
    return out, last_state


@_selective_scan_op.register_fake
def _(u, delta, a, b, c, d_skip, z, delta_bias, h0, delta_softplus, reverse):
    return torch.empty_like(u), u.new_empty((u.shape[0], u.shape[1], a.shape[1]))


def _bc4(t, batch, state, length):
    return t.reshape(batch, 1, state, length) if t.dim() == 3 else t


def selective_scan(u, delta, A, B, C, D=None, z=None, delta_bias=None,
                   delta_softplus=False, return_last_state=False,
                   initial_state=None, reverse=False):
    """Mamba-1 selective scan.

    u, delta, z : (batch, dim, len);  A : (dim, state)
    B, C        : (batch, state, len) or (batch, groups, state, len)
    D, delta_bias : (dim,);  initial_state : (batch, dim, state) or None
    Returns out (batch, dim, len) [, last_state (batch, dim, state)], on u's
    device.  Inputs are converted to contiguous float32 on u's device, so
    transposed views and other devices' tensors are accepted.

    ``reverse`` walks the sequence backward: output index t is still step t,
    it equals flipping u/delta/B/C/z in time, scanning forward and flipping
    the result; ``last_state`` is then the state after consuming t = 0.
    """
    lay = m1_layout(u.shape, delta.shape, A.shape, B.shape, C.shape,
                    None if D is None else D.shape, None if z is None else z.shape,
                    None if delta_bias is None else delta_bias.shape,
                    None if initial_state is None else initial_state.shape)
    dev = u.device
    B = B.reshape(lay.bc_shape)
    C = C.reshape(lay.bc_shape)
    opt = lambda t: None if t is None else _prep(t, dev)  # noqa: E731
    out, last_state = _selective_scan_op(
        _prep(u, dev), _prep(delta, dev), _prep(A, dev), _prep(B, dev), _prep(C, dev),
        opt(D), opt(z), opt(delta_bias), opt(initial_state), bool(delta_softplus),
        bool(reverse))
    return (out, last_state) if return_last_state else out


@torch.library.custom_op("arm_scan::selective_scan_bidirectional", mutates_args=())
def _selective_scan_bidir_op(
    u: torch.Tensor,
    delta: torch.Tensor,
    a: torch.Tensor,
    b: torch.Tensor,
    c: torch.Tensor,
    d_skip: Optional[torch.Tensor],
    z: Optional[torch.Tensor],
    delta_bias: Optional[torch.Tensor],
    delta_softplus: bool,
) -> Tuple[torch.Tensor, torch.Tensor]:
    batch, dim, length = u.shape
    state = a.shape[1]
    out_fwd = torch.empty_like(u)
    out_bwd = torch.empty_like(u)
    dims = _ffi.ArmScanDims(batch, dim, length, state, b.shape[1] if b.dim() == 4 else 1)
    with _on_device(u):
        _ffi.scan_bidir_raw(
            dims, u.data_ptr(), delta.data_ptr(), a.data_ptr(), b.data_ptr(), c.data_ptr(),
            _ptr(d_skip), _ptr(z), _ptr(delta_bias), delta_softplus, "auto", "auto",
            out_fwd.data_ptr(), out_bwd.data_ptr(), stream=_stream(u))
    _CALLS["n"] += 1
    return out_fwd, out_bwd


@_selective_scan_bidir_op.register_fake
def _(u, delta, a, b, c, d_skip, z, delta_bias, delta_softplus):
    return torch.empty_like(u), torch.empty_like(u)


@torch.library.custom_op("arm_scan::selective_scan_bidirectional_sum", mutates_args=())
def _selective_scan_bidir_sum_op(
    u: torch.Tensor,
    delta: torch.Tensor,
    a: torch.Tensor,
    b: torch.Tensor,
    c: torch.Tensor,
    d_skip: Optional[torch.Tensor],
    z: Optional[torch.Tensor],
    delta_bias: Optional[torch.Tensor],
    delta_softplus: bool,
    h0_fwd: Optional[torch.Tensor] = None,
    h0_bwd: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    batch, dim, length = u.shape
    state = a.shape[1]
    out = torch.empty_like(u)
    dims = _ffi.ArmScanDims(batch, dim, length, state, b.shape[1] if b.dim() == 4 else 1)
    with _on_device(u):
        _ffi.scan_bidir_sum_raw(
            dims, u.data_ptr(), delta.data_ptr(), a.data_ptr(), b.data_ptr(), c.data_ptr(),
            _ptr(d_skip), _ptr(z), _ptr(delta_bias), delta_softplus, "auto", out.data_ptr(),
            ptr_h0_fwd=_ptr(h0_fwd), ptr_h0_bwd=_ptr(h0_bwd), stream=_stream(u))
    _CALLS["n"] += 1
    return out


@_selective_scan_bidir_sum_op.register_fake
def _(u, delta, a, b, c, d_skip, z, delta_bias, delta_softplus, h0_fwd=None, h0_bwd=None):
    return torch.empty_like(u)


def selective_scan_bidirectional_sum(u, delta, A, B, C, D=None, z=None, delta_bias=None,
                                     delta_softplus=False, initial_states=None):
    """out_fwd + out_bwd of ``selective_scan_bidirectional`` in one call, on
    CUDA tensors: the two traversals share their first pass and the reverse
    one adds into the output in place.  ``initial_states`` = (h0_fwd,
    h0_bwd), each (batch, dim, state) or None: the incoming state of each
    traversal (the reverse one's enters at the last step)."""
    if u.device.type != "cuda":
        raise ValueError("selective_scan_bidirectional_sum needs CUDA tensors")
    batch, dim, length = u.shape
    state = A.shape[1]
    dev = u.device
    B = _bc4(B, batch, state, length)
    C = _bc4(C, batch, state, length)
    opt = lambda t: None if t is None else _prep(t, dev)  # noqa: E731
    h0f, h0b = initial_states if initial_states is not None else (None, None)
    for t in (h0f, h0b):
        if t is not None and tuple(t.shape) != (batch, dim, state):
            raise ValueError(f"initial states must be {(batch, dim, state)}, got {tuple(t.shape)}")
    return _selective_scan_bidir_sum_op(
        _prep(u, dev), _prep(delta, dev), _prep(A, dev), _prep(B, dev), _prep(C, dev),
        opt(D), opt(z), opt(delta_bias), bool(delta_softplus), opt(h0f), opt(h0b))


@torch.library.custom_op("arm_scan::selective_scan_bidirectional_final_states", mutates_args=())
def _bidir_states_op(u: torch.Tensor, delta: torch.Tensor, a: torch.Tensor, b: torch.Tensor,
                     c: torch.Tensor, delta_bias: Optional[torch.Tensor],
                     delta_softplus: bool) -> Tuple[torch.Tensor, torch.Tensor]:
    batch, dim, length = u.shape
    state = a.shape[1]
    hf = u.new_empty((batch, dim, state))
    hb = u.new_empty((batch, dim, state))
    dims = _ffi.ArmScanDims(batch, dim, length, state, b.shape[1] if b.dim() == 4 else 1)
    with _on_device(u):
        _ffi.bidir_states_raw(dims, u.data_ptr(), delta.data_ptr(), a.data_ptr(), b.data_ptr(),
                              c.data_ptr(), _ptr(delta_bias), delta_softplus, "auto",
                              hf.data_ptr(), hb.data_ptr(), stream=_stream(u))
    _CALLS["n"] += 1
    return hf, hb


@_bidir_states_op.register_fake
def _(u, delta, a, b, c, delta_bias, delta_softplus):
    s = (u.shape[0], u.shape[1], a.shape[1])
    return u.new_empty(s), u.new_empty(s)


def selective_scan_bidirectional_final_states(u, delta, A, B, C, delta_bias=None,
                                              delta_softplus=False):
    """(h_fwd, h_bwd): the states after the forward and the reverse traversal
    from zero, without outputs, on CUDA tensors (one shared first pass where
    the two-pass kernel applies)."""
    if u.device.type != "cuda":
        raise ValueError("selective_scan_bidirectional_final_states needs CUDA tensors")
    batch, dim, length = u.shape
    state = A.shape[1]
    dev = u.device
    B = _bc4(B, batch, state, length)
    C = _bc4(C, batch, state, length)
    return _bidir_states_op(_prep(u, dev), _prep(delta, dev), _prep(A, dev), _prep(B, dev),
                            _prep(C, dev), None if delta_bias is None else _prep(delta_bias, dev),
                            bool(delta_softplus))


def selective_scan_segment_summary(u, delta, A, B, C, delta_bias=None, delta_softplus=False):
    """(h_fwd, h_bwd, dt_sum): the states after the forward and the reverse
    traversal from zero and the per-row sum of dt over the sequence, on CUDA
    tensors -- what a segment of a sequence split over devices contributes
    to the others (one shared pass where the lane kernel applies)."""
    if u.device.type != "cuda":
        raise ValueError("selective_scan_segment_summary needs CUDA tensors")
    batch, dim, length = u.shape
    state = A.shape[1]
    dev = u.device
    B = _bc4(B, batch, state, length)
    C = _bc4(C, batch, state, length)
    u, delta, A, B, C = (_prep(t, dev) for t in (u, delta, A, B, C))
    db = None if delta_bias is None else _prep(delta_bias, dev)
    hf = u.new_empty((batch, dim, state))
    hb = u.new_empty((batch, dim, state))
    sdt = u.new_empty((batch, dim))
    dims = _ffi.ArmScanDims(batch, dim, length, state, B.shape[1] if B.dim() == 4 else 1)
    with _on_device(u):
        _ffi.segment_summary_raw(dims, u.data_ptr(), delta.data_ptr(), A.data_ptr(), B.data_ptr(),
                                 C.data_ptr(), _ptr(db), delta_softplus, "auto", hf.data_ptr(),
                                 hb.data_ptr(), sdt.data_ptr(), stream=_stream(u))
    _CALLS["n"] += 1
    return hf, hb, sdt


class BidirectionalSegment:
    """The bidirectional sum of one segment of a sequence split over devices,
    in two phases around the exchange of segment summaries (CUDA tensors,
    the layouts of ``selective_scan``).

    ``summary()`` returns (h_fwd, h_bwd, dt_sum) as
    ``selective_scan_segment_summary`` does, from one shared pass that also
    leaves its per-segment aggregates in a workspace this object holds;
    ``finish(h0_fwd, h0_bwd)`` returns out_fwd + out_bwd from those incoming
    states as ``selective_scan_bidirectional_sum`` does, reusing the
    aggregates instead of re-reading the inputs for them.  The input tensors
    must not change between the two calls.  Where the two-phase kernels do
    not cover the shape (state > 16, length not a multiple of 4, unaligned
    tensors) both phases run the one-call functions instead."""

    def __init__(self, u, delta, A, B, C, D=None, z=None, delta_bias=None, delta_softplus=False):
        if u.device.type != "cuda":
            raise ValueError("BidirectionalSegment needs CUDA tensors")
        batch, dim, length = u.shape
        state = A.shape[1]
        dev = u.device
        B = _bc4(B, batch, state, length)
        C = _bc4(C, batch, state, length)
        opt = lambda t: None if t is None else _prep(t, dev)  # noqa: E731
        self.u, self.delta, self.A, self.B, self.C = (_prep(t, dev) for t in (u, delta, A, B, C))
        self.D, self.z, self.delta_bias = opt(D), opt(z), opt(delta_bias)
        self.delta_softplus = bool(delta_softplus)
        self.shape = (batch, dim, state)
        self.dims = _ffi.ArmScanDims(batch, dim, length, state, self.B.shape[1] if self.B.dim() == 4 else 1)
        self.ws_bytes = _ffi.bidirectional_workspace_bytes(self.dims)
        aligned = all(t is None or t.data_ptr() % 16 == 0
                      for t in (self.u, self.delta, self.A, self.B, self.C, self.D, self.z,
                                self.delta_bias))
        if not aligned:
            self.ws_bytes = 0
        self.ws = torch.empty(self.ws_bytes, dtype=torch.uint8, device=dev) if self.ws_bytes else None
        self._summarised = False

    def summary(self):
        if self.ws is None:
            self._summarised = True
            return selective_scan_segment_summary(self.u, self.delta, self.A, self.B, self.C,
                                                  delta_bias=self.delta_bias,
                                                  delta_softplus=self.delta_softplus)
        hf = self.u.new_empty(self.shape)
        hb = self.u.new_empty(self.shape)
        sdt = self.u.new_empty(self.shape[:2])
        with _on_device(self.u):
            _ffi.bidirectional_summary_raw(
                self.dims, self.u.data_ptr(), self.delta.data_ptr(), self.A.data_ptr(),
                self.B.data_ptr(), self.C.data_ptr(), _ptr(self.delta_bias), self.delta_softplus,
                self.ws.data_ptr(), self.ws_bytes, hf.data_ptr(), hb.data_ptr(), sdt.data_ptr(),
                _stream(self.u))
        _CALLS["n"] += 1
        self._summarised = True
        return hf, hb, sdt

    def finish(self, h0_fwd=None, h0_bwd=None):
        if not self._summarised:
            raise RuntimeError("BidirectionalSegment.finish() before summary()")
        dev = self.u.device
        h0 = [None if t is None else _prep(t, dev) for t in (h0_fwd, h0_bwd)]
        for t in h0:
            if t is not None and tuple(t.shape) != self.shape:
                raise ValueError(f"initial states must be {self.shape}, got {tuple(t.shape)}")
        if self.ws is None:
            return selective_scan_bidirectional_sum(self.u, self.delta, self.A, self.B, self.C,
                                                    D=self.D, z=self.z, delta_bias=self.delta_bias,
                                                    delta_softplus=self.delta_softplus,
                                                    initial_states=tuple(h0))
        out = torch.empty_like(self.u)
        with _on_device(self.u):
            _ffi.bidirectional_finish_raw(
                self.dims, self.u.data_ptr(), self.delta.data_ptr(), self.A.data_ptr(),
                self.B.data_ptr(), self.C.data_ptr(), _ptr(self.D), _ptr(self.z),
                _ptr(self.delta_bias), self.delta_softplus, self.ws.data_ptr(), self.ws_bytes,
                _ptr(h0[0]), _ptr(h0[1]), out.data_ptr(), _stream(self.u))
        _CALLS["n"] += 1
        return out


def selective_scan_ss2d(u, delta, A, B, C, D=None, delta_bias=None, delta_softplus=True,
                        merge="sum"):
    """The Mamba-1 SS2D cross-scan, merged "sum" or "mean", in one library call
    over CUDA grids read in place: u, delta (b, d, h, w); B, C (b, n, h, w)
    or (b, groups, n, h, w); A (d, n); D, delta_bias (d,).  The row-major
    traversals run as a bidirectional sum over the grid's natural order, the
    column-major ones as per-column segments (no transposed copies)."""
    if u.device.type != "cuda" or u.dim() != 4:
        raise ValueError("selective_scan_ss2d takes (b, d, h, w) CUDA grids")
    if merge not in ("sum", "mean"):
        raise ValueError(f"merge must be 'sum' or 'mean', got {merge!r}")
    b, d, h, w = u.shape
    state = A.shape[1]
    dev = u.device
    G = 1 if B.dim() == 4 else B.shape[1]
    bc = lambda t: _prep(t, dev).reshape(b, G, state, h * w)  # noqa: E731
    us, ds = _prep(u, dev), _prep(delta, dev)
    As, Bs, Cs = _prep(A, dev), bc(B), bc(C)
    Ds = None if D is None else _prep(D, dev)
    db = None if delta_bias is None else _prep(delta_bias, dev)
    out = torch.empty_like(us)
    dims = _ffi.ArmScanDims(b, d, h * w, state, G)
    with _on_device(us):
        _ffi.ss2d_raw(dims, h, w, us.data_ptr(), ds.data_ptr(), As.data_ptr(), Bs.data_ptr(),
                      Cs.data_ptr(), _ptr(Ds), _ptr(db), delta_softplus, merge == "mean",
                      out.data_ptr(), _stream(us))
    _CALLS["n"] += 1
    return out


def causal_conv1d_silu(x, weight, bias=None):
    """silu(causal depthwise conv1d(x) + bias) over (batch, dim, len) CUDA
    rows; weight (dim, kernel) or (dim, 1, kernel) as nn.Conv1d stores it.
    One kernel pass (the Mamba-1 mixer's input prologue)."""
    if x.device.type != "cuda" or x.dim() != 3:
        raise ValueError("causal_conv1d_silu takes a (batch, dim, len) CUDA tensor")
    batch, dim, length = x.shape
    w = weight.reshape(dim, -1)
    dev = x.device
    xs, ws = _prep(x, dev), _prep(w, dev)
    bs = None if bias is None else _prep(bias, dev)
    out = torch.empty_like(xs)
    with _on_device(xs):
        _ffi.conv_silu_raw(batch, dim, length, ws.shape[1], xs.data_ptr(), ws.data_ptr(),
                           _ptr(bs), out.data_ptr(), _stream(xs))
    return out


def selective_scan_bidirectional(u, delta, A, B, C, D=None, z=None,
                                 delta_bias=None, delta_softplus=False):
    """Forward and backward scans of the same inputs in one call.

    Layouts as ``selective_scan``; returns (out_fwd, out_bwd).  Equal to
    ``selective_scan`` plus ``selective_scan(..., reverse=True)``; merging
    the two directions is the caller's job (``bidirectional_scan``).
    """
    batch, dim, length = u.shape
    state = A.shape[1]
    dev = u.device
    B = _bc4(B, batch, state, length)
    C = _bc4(C, batch, state, length)
    opt = lambda t: None if t is None else _prep(t, dev)  # noqa: E731
    return _selective_scan_bidir_op(
        _prep(u, dev), _prep(delta, dev), _prep(A, dev), _prep(B, dev), _prep(C, dev),
        opt(D), opt(z), opt(delta_bias), bool(delta_softplus))


def kernel_calls() -> int:
    """How many times a native scan entry point has been invoked."""
    return _CALLS["n"]


@torch.library.custom_op("arm_scan::selective_state_update", mutates_args=("state",))
def _state_update_op(state: torch.Tensor, x: torch.Tensor, dt: torch.Tensor, A: torch.Tensor,
                     B: torch.Tensor, C: torch.Tensor, D: Optional[torch.Tensor],
                     z: Optional[torch.Tensor], dt_bias: Optional[torch.Tensor],
                     dt_softplus: bool) -> torch.Tensor:
    batch, dim, n = state.shape
    groups = B.shape[1]
    dims = _ffi.ArmScanDims(batch, dim, 1, n, groups)
    out = x.new_empty((batch, dim))
    with _on_device(state):
        _ffi.state_update_raw(dims, state.data_ptr(), x.data_ptr(), dt.data_ptr(), A.data_ptr(),
                              B.data_ptr(), C.data_ptr(), _ptr(D), _ptr(z), _ptr(dt_bias),
                              dt_softplus, out.data_ptr(), _stream(state))
    _CALLS["n"] += 1
    return out


@_state_update_op.register_fake
def _(state, x, dt, A, B, C, D, z, dt_bias, dt_softplus):
    return x.new_empty((state.shape[0], state.shape[1]))


def selective_state_update(state, x, dt, A, B, C, D=None, z=None, dt_bias=None,
                           dt_softplus=False):
    """One decode step of the Mamba-1 recurrence (mamba_ssm's
    ``selective_state_update``): updates ``state`` (batch, dim, d_state), a
    contiguous fp32 CUDA tensor, in place and returns y (batch, dim).

    x, dt, z : (batch, dim);  A : (dim, d_state);  B, C : (batch, d_state) or
    (batch, groups, d_state);  D, dt_bias : (dim,).  Equivalent to
    ``selective_scan`` over one step with ``initial_state=state`` and
    ``return_last_state=True``, without the scan's staging.
    """
    if state.device.type != "cuda" or state.dtype != torch.float32 or not state.is_contiguous():
        raise ValueError("state must be a contiguous float32 CUDA tensor (updated in place)")
    batch, dim, n = state.shape
    dev = state.device
    if B.dim() == 2:
        B, C = B.unsqueeze(1), C.unsqueeze(1)
    groups = B.shape[1]
    for name, t, want in (("x", x, (batch, dim)), ("dt", dt, (batch, dim)), ("A", A, (dim, n)),
                          ("B", B, (batch, groups, n)), ("C", C, (batch, groups, n))):
        if tuple(t.shape) != want:
            raise ValueError(f"{name} must be {want}, got {tuple(t.shape)}")
    if dim % groups:
        raise ValueError(f"dim ({dim}) must be a multiple of groups ({groups})")
    for name, t, want in (("D", D, (dim,)), ("dt_bias", dt_bias, (dim,)), ("z", z, (batch, dim))):
        if t is not None and tuple(t.shape) != want:
            raise ValueError(f"{name} must be {want}, got {tuple(t.shape)}")
    opt = lambda t: None if t is None else _prep(t, dev)  # noqa: E731
    return _state_update_op(state, _prep(x, dev), _prep(dt, dev), _prep(A, dev), _prep(B, dev),
                            _prep(C, dev), opt(D), opt(z), opt(dt_bias), bool(dt_softplus))


@torch.library.custom_op("arm_scan::selective_scan_final_state", mutates_args=())
def _final_state_op(u: torch.Tensor, delta: torch.Tensor, A: torch.Tensor, B: torch.Tensor,
                    C: torch.Tensor, delta_bias: Optional[torch.Tensor],
                    initial_state: Optional[torch.Tensor], delta_softplus: bool,
                    reverse: bool) -> torch.Tensor:
    batch, dim, length = u.shape
    state, groups = A.shape[1], B.shape[1]
    dims = _ffi.ArmScanDims(batch, dim, length, state, groups)
    last = u.new_empty((batch, dim, state))
    with _on_device(u):
        _ffi.final_state_raw(dims, u.data_ptr(), delta.data_ptr(), A.data_ptr(), B.data_ptr(),
                             C.data_ptr(), _ptr(delta_bias), delta_softplus, reverse,
                             _ptr(initial_state), last.data_ptr(), _stream(u))
    _CALLS["n"] += 1
    return last


@_final_state_op.register_fake
def _(u, delta, A, B, C, delta_bias, initial_state, delta_softplus, reverse):
    return u.new_empty((u.shape[0], u.shape[1], A.shape[1]))


def selective_scan_final_state(u, delta, A, B, C, delta_bias=None, delta_softplus=False,
                               initial_state=None, reverse=False):
    """The ``last_state`` of ``selective_scan`` with the same arguments,
    without computing the outputs (d_state <= 16).  The first step of a
    sequence-parallel scan; CUDA tensors only."""
    if u.device.type != "cuda":
        raise ValueError("selective_scan_final_state runs on CUDA tensors")
    batch, dim, length = u.shape
    state = A.shape[1]
    dev = u.device
    B = _bc4(B, batch, state, length)
    C = _bc4(C, batch, state, length)
    opt = lambda t: None if t is None else _prep(t, dev)  # noqa: E731
    return _final_state_op(_prep(u, dev), _prep(delta, dev), _prep(A, dev), _prep(B, dev),
                           _prep(C, dev), opt(delta_bias), opt(initial_state),
                           bool(delta_softplus), bool(reverse))
