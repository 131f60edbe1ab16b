"""NumPy front-end of the Mamba-1 scan (the reference's
python/arm_scan/numpy_api.py surface): host arrays in, host arrays out, no
torch.  The arrays are handed to the synchronous C entry point as host
pointers; the library stages them through the current CUDA device (for a
batch of two or more rows it pipelines per batch row over two streams, so
uploads overlap scans) and returns once the outputs are back in host
memory."""

import numpy as np

from . import _ffi
from .layout import m1_layout


def _host_f32(a):
    """A C-contiguous float32 view or copy, or None."""
    return None if a is None else np.ascontiguousarray(a, dtype=np.float32)


def _addr(a):
    return 0 if a is None else a.ctypes.data


def selective_scan_numpy(u, delta, A, B, C, D=None, z=None, delta_bias=None,
                         delta_softplus=False, return_last_state=False,
                         backend="auto", threading="auto", initial_state=None,
                         reverse=False):
    """Mamba-1 selective scan on numpy arrays; layouts and semantics as
    ``selective_scan``.  Returns out (batch, dim, len) [, last_state
    (batch, dim, state)], float32."""
    host = {k: _host_f32(v) for k, v in dict(u=u, delta=delta, A=A, B=B, C=C, D=D, z=z,
                                                delta_bias=delta_bias,
                                                h0=initial_state).items()}
    lay = m1_layout(*(None if host[k] is None else host[k].shape
                      for k in ("u", "delta", "A", "B", "C", "D", "z", "delta_bias", "h0")))
    host["B"] = host["B"].reshape(lay.bc_shape)
    host["C"] = host["C"].reshape(lay.bc_shape)
    out = np.empty((lay.batch, lay.dim, lay.length), np.float32)
    last = np.empty((lay.batch, lay.dim, lay.state), np.float32)
    _ffi.scan_raw(_ffi.ArmScanDims(lay.batch, lay.dim, lay.length, lay.state, lay.groups),
                  *(_addr(host[k]) for k in ("u", "delta", "A", "B", "C", "D", "z",
                                             "delta_bias")),
                  delta_softplus, backend, threading, out.ctypes.data, last.ctypes.data,
                  ptr_h0=_addr(host["h0"]), reverse=reverse)
    return (out, last) if return_last_state else out
