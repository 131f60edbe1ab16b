"""ctypes binding of libb200scan.so (the C ABI in include/b200scan.h).

Mirrors the reference loader python/arm_scan/_ffi.py: the library is looked up
via the ``ARM_SCAN_LIB`` environment variable first, then next to this
package; its ABI version is checked before any entry point is bound.  Pointers
are passed as integer addresses (0 = null).

Two call families:
* ``*_raw``       -- the synchronous v7-shaped entry points.  Every buffer must
  be host memory (the library stages it through the GPU) or every buffer
  device memory; the call returns once the results are in place.
* ``*_async_raw`` -- device pointers, enqueued on a CUDA stream handle.

There is no CPU implementation behind any of these: if the library or a GPU
is missing, the call raises.
"""

import ctypes
import os
import sys
from pathlib import Path

ABI_VERSION = 13

_LIB_NAMES = ["libb200scan.so"]

ERROR_NAMES = {
    0: "ok",
    1: "null pointer",
    2: "invalid dims/shapes",
    3: "backend unavailable",
    4: "bad backend/threading enum",
    5: "panic inside kernel",
    6: "CUDA error",
    7: "timeout",
}

BACKENDS = {"auto": 0, "scalar": 1, "sequential": 1, "neon": 2}
THREADING = {"auto": 0, "sequential": 1, "seq": 1, "rayon": 2}


class ArmScanDims(ctypes.Structure):
    _fields_ = [(n, ctypes.c_size_t) for n in ("batch", "dim", "len", "state", "groups")]


class ArmMamba3Dims(ctypes.Structure):
    _fields_ = [(n, ctypes.c_size_t) for n in ("batch", "heads", "dv", "dqk", "len", "rank")]


class ArmMamba3MixerDims(ctypes.Structure):
    _fields_ = [(n, ctypes.c_size_t) for n in ("batch", "len", "heads", "headdim", "d_state",
                                               "rank", "n_angles")]


class ArmMamba3TcOptions(ctypes.Structure):
    _fields_ = [("in_dtype", ctypes.c_int), ("out_dtype", ctypes.c_int),
                ("out_layout", ctypes.c_int), ("angles_shared", ctypes.c_int),
                ("n_angles", ctypes.c_size_t)]


DTYPE_F32, DTYPE_BF16 = 0, 1


def _candidate_paths():
    env = os.environ.get("ARM_SCAN_LIB")
    if env:
        yield Path(env)
    here = Path(__file__).resolve().parent
    for name in _LIB_NAMES:
        yield here / name


_lib = None
_lib_path = None

_VP = ctypes.c_void_p
_I = ctypes.c_int


def _bind(lib):
    lib.arm_scan_abi_version.restype = ctypes.c_uint32
    lib.arm_scan_last_error.restype = ctypes.c_char_p
    m1 = [ctypes.POINTER(ArmScanDims), *([_VP] * 8), _I, _I, _I, _I, _VP, _VP, _VP]
    lib.arm_scan_selective_scan_f32.argtypes = m1
    lib.arm_scan_selective_scan_f32_async.argtypes = m1 + [_VP]
    bi = [ctypes.POINTER(ArmScanDims), *([_VP] * 8), _I, _I, _I, _VP, _VP, _VP, _VP]
    lib.arm_scan_selective_scan_bidirectional_f32.argtypes = bi
    lib.arm_scan_selective_scan_bidirectional_f32_async.argtypes = bi + [_VP]
    m3 = [ctypes.POINTER(ArmMamba3Dims), *([_VP] * 15), _I, _I, _I, _VP, _VP, _VP]
    lib.arm_scan_mamba3_scan_f32.argtypes = m3
    lib.arm_scan_mamba3_scan_f32_async.argtypes = m3 + [_VP]
    lib.arm_scan_mamba3_angles_workspace_bytes.restype = ctypes.c_size_t
    lib.arm_scan_mamba3_angles_workspace_bytes.argtypes = [ctypes.POINTER(ArmMamba3Dims),
                                                           ctypes.c_size_t]
    lib.arm_scan_mamba3_angles_f32_async.restype = ctypes.c_int
    lib.arm_scan_mamba3_angles_f32_async.argtypes = [
        ctypes.POINTER(ArmMamba3Dims), _VP, ctypes.c_size_t, _VP, _VP, _VP, _VP,
        ctypes.c_size_t, _VP]
    lib.arm_scan_mamba3_angles_f32_noalloc.restype = ctypes.c_int
    lib.arm_scan_mamba3_angles_f32_noalloc.argtypes = [
        ctypes.POINTER(ArmMamba3Dims), _VP, ctypes.c_size_t, _VP, _VP, _VP, _VP]
    for f in ("arm_scan_selective_scan_f32", "arm_scan_selective_scan_f32_async",
              "arm_scan_selective_scan_bidirectional_f32",
              "arm_scan_selective_scan_bidirectional_f32_async",
              "arm_scan_mamba3_scan_f32", "arm_scan_mamba3_scan_f32_async",
              "arm_scan_tensor_status"):
        getattr(lib, f).restype = ctypes.c_int
    lib.arm_scan_mamba3_ss2d_f32_async.restype = ctypes.c_int
    lib.arm_scan_mamba3_ss2d_f32_async.argtypes = [
        ctypes.POINTER(ArmMamba3Dims), ctypes.c_size_t, *([_VP] * 9), ctypes.c_size_t,
        _VP, _VP, _VP, _VP]
    lib.arm_scan_mamba3_noncausal_f32_async.restype = ctypes.c_int
    lib.arm_scan_mamba3_noncausal_f32_async.argtypes = [
        ctypes.POINTER(ArmMamba3Dims), ctypes.c_size_t, *([_VP] * 9), ctypes.c_size_t,
        _VP, _VP, _VP, _VP, _VP, _VP]
    lib.arm_scan_causal_conv1d_silu_f32_async.restype = ctypes.c_int
    lib.arm_scan_causal_conv1d_silu_f32_async.argtypes = [ctypes.c_size_t] * 4 + [_VP] * 5
    lib.arm_scan_selective_scan_final_state_f32_async.restype = ctypes.c_int
    lib.arm_scan_selective_scan_final_state_f32_async.argtypes = [
        ctypes.POINTER(ArmScanDims), *([_VP] * 6), ctypes.c_int, ctypes.c_int, _VP, _VP, _VP]
    lib.arm_scan_selective_state_update_f32_async.restype = ctypes.c_int
    lib.arm_scan_selective_state_update_f32_async.argtypes = [
        ctypes.POINTER(ArmScanDims), *([_VP] * 9), ctypes.c_int, _VP, _VP]
    lib.arm_scan_kernel_launches.restype = ctypes.c_ulonglong
    lib.arm_scan_kernel_launches.argtypes = []
    lib.arm_scan_set_device.restype = ctypes.c_int
    lib.arm_scan_set_device.argtypes = [_I]
    lib.arm_scan_set_kernel_override.restype = ctypes.c_int
    lib.arm_scan_set_kernel_override.argtypes = [_I, _I]
    lib.arm_scan_selective_scan_bidirectional_sum_f32_async.restype = ctypes.c_int
    lib.arm_scan_selective_scan_bidirectional_sum_f32_async.argtypes = [
        ctypes.POINTER(ArmScanDims), *([_VP] * 8), _I, _I, _I, _VP, _VP, _VP, _VP, _VP, _VP]
    lib.arm_scan_selective_scan_bidirectional_final_states_f32_async.restype = ctypes.c_int
    lib.arm_scan_selective_scan_bidirectional_final_states_f32_async.argtypes = [
        ctypes.POINTER(ArmScanDims), *([_VP] * 6), _I, _I, _VP, _VP, _VP]
    lib.arm_scan_selective_scan_segment_summary_f32_async.restype = ctypes.c_int
    lib.arm_scan_selective_scan_segment_summary_f32_async.argtypes = [
        ctypes.POINTER(ArmScanDims), *([_VP] * 6), _I, _I, _VP, _VP, _VP, _VP]
    lib.arm_scan_selective_scan_bidirectional_workspace_bytes.restype = ctypes.c_size_t
    lib.arm_scan_selective_scan_bidirectional_workspace_bytes.argtypes = [ctypes.POINTER(ArmScanDims)]
    lib.arm_scan_selective_scan_bidirectional_summary_f32_async.restype = ctypes.c_int
    lib.arm_scan_selective_scan_bidirectional_summary_f32_async.argtypes = [
        ctypes.POINTER(ArmScanDims), *([_VP] * 6), _I, _VP, ctypes.c_size_t, _VP, _VP, _VP, _VP]
    lib.arm_scan_selective_scan_bidirectional_finish_f32_async.restype = ctypes.c_int
    lib.arm_scan_selective_scan_bidirectional_finish_f32_async.argtypes = [
        ctypes.POINTER(ArmScanDims), *([_VP] * 8), _I, _VP, ctypes.c_size_t, _VP, _VP, _VP, _VP]
    lib.arm_scan_selective_scan_ss2d_f32_async.restype = ctypes.c_int
    lib.arm_scan_selective_scan_ss2d_f32_async.argtypes = [
        ctypes.POINTER(ArmScanDims), ctypes.c_size_t, ctypes.c_size_t, *([_VP] * 7), _I, _I, _VP, _VP]
    lib.arm_scan_mamba3_mixer_prologue_f32_async.restype = ctypes.c_int
    lib.arm_scan_mamba3_mixer_prologue_f32_async.argtypes = [
        ctypes.POINTER(ArmMamba3MixerDims), *([_VP] * 4), ctypes.c_float, ctypes.c_float,
        *([_VP] * 9)]
    lib.arm_scan_mamba3_mimo_x_tc_async.restype = ctypes.c_int
    lib.arm_scan_mamba3_mimo_x_tc_async.argtypes = [
        ctypes.POINTER(ArmMamba3Dims), ctypes.POINTER(ArmMamba3TcOptions), *([_VP] * 8),
        ctypes.c_int, _VP, _VP, _VP]
    lib.arm_scan_mamba3_siso_tc_async.restype = ctypes.c_int
    lib.arm_scan_mamba3_siso_tc_async.argtypes = [
        ctypes.POINTER(ArmMamba3Dims), ctypes.POINTER(ArmMamba3TcOptions), *([_VP] * 11),
        ctypes.c_int, _VP, _VP, _VP, _VP]


def load():
    """Load (once) and return the ctypes library handle."""
    global _lib, _lib_path
    if _lib is not None:
        return _lib
    tried = []
    for path in _candidate_paths():
        tried.append(str(path))
        if path.is_file():
            lib = ctypes.CDLL(str(path))
            version = lib.arm_scan_abi_version()
            if version != ABI_VERSION:
                raise RuntimeError(
                    f"{path} has ABI version {version}, this package needs {ABI_VERSION}; "
                    f"rebuild with `python -m armhackathon_b200.build`")
            _bind(lib)
            _lib, _lib_path = lib, path
            return lib
    raise OSError("libb200scan.so not found; build it with `python -m armhackathon_b200.build` "
                  "(searched: " + ", ".join(tried) + ")")


def lib_path():
    load()
    return _lib_path


def _check(code, what):
    if code != 0:
        msg = load().arm_scan_last_error()
        msg = msg.decode() if msg else ""
        raise RuntimeError(f"{what} failed with code {code} ({ERROR_NAMES.get(code, 'unknown')})"
                           + (f": {msg}" if msg else ""))


def _n(p):
    return p or None


def scan_raw(dims, ptr_u, ptr_delta, ptr_a, ptr_b, ptr_c, ptr_d_skip, ptr_z,
             ptr_delta_bias, delta_softplus, backend, threading, ptr_out,
             ptr_last, ptr_h0=0, *, reverse=False, stream=None):
    """Mamba-1 scan.  ``stream`` None -> synchronous entry point (host or
    device pointers); an integer stream handle -> the _async entry point."""
    lib = load()
    args = (ctypes.byref(dims), ptr_u, ptr_delta, ptr_a, ptr_b, ptr_c, _n(ptr_d_skip), _n(ptr_z),
            _n(ptr_delta_bias), int(bool(delta_softplus)), int(bool(reverse)),
            BACKENDS[backend], THREADING[threading], ptr_out, _n(ptr_last), _n(ptr_h0))
    if stream is None:
        _check(lib.arm_scan_selective_scan_f32(*args), "arm_scan_selective_scan_f32")
    else:
        _check(lib.arm_scan_selective_scan_f32_async(*args, _n(stream)),
               "arm_scan_selective_scan_f32_async")


def scan_bidir_raw(dims, ptr_u, ptr_delta, ptr_a, ptr_b, ptr_c, ptr_d_skip, ptr_z,
                   ptr_delta_bias, delta_softplus, backend, threading, ptr_out_fwd,
                   ptr_out_bwd, ptr_last_fwd=0, ptr_last_bwd=0, *, stream=None):
    """Fused bidirectional Mamba-1 scan (forward + reverse of the same inputs)."""
    lib = load()
    args = (ctypes.byref(dims), ptr_u, ptr_delta, ptr_a, ptr_b, ptr_c, _n(ptr_d_skip), _n(ptr_z),
            _n(ptr_delta_bias), int(bool(delta_softplus)), BACKENDS[backend],
            THREADING[threading], ptr_out_fwd, ptr_out_bwd, _n(ptr_last_fwd), _n(ptr_last_bwd))
    if stream is None:
        _check(lib.arm_scan_selective_scan_bidirectional_f32(*args),
               "arm_scan_selective_scan_bidirectional_f32")
    else:
        _check(lib.arm_scan_selective_scan_bidirectional_f32_async(*args, _n(stream)),
               "arm_scan_selective_scan_bidirectional_f32_async")


def mamba3_raw(dims, ptrs, reverse, backend, threading, ptr_out, ptr_last_state,
               ptr_last_bx, *, stream=None):
    """Mamba-3 scan.  ``ptrs`` are the 15 input addresses in signature order:
    q, k, v, adt, dt, trap, q_bias, k_bias, cos, sin, d_skip, z, psi, zeta, phi
    (d_skip, z and the three MIMO projections may be 0)."""
    lib = load()
    if len(ptrs) != 15:
        raise ValueError(f"expected 15 input pointers, got {len(ptrs)}")
    args = (ctypes.byref(dims), *[_n(p) for p in ptrs], int(reverse), int(backend),
            int(threading), ptr_out, _n(ptr_last_state), _n(ptr_last_bx))
    if stream is None:
        _check(lib.arm_scan_mamba3_scan_f32(*args), "arm_scan_mamba3_scan_f32")
    else:
        _check(lib.arm_scan_mamba3_scan_f32_async(*args, _n(stream)),
               "arm_scan_mamba3_scan_f32_async")


def mamba3_tc_raw(dims, opts, ptrs, reverse, ptr_out, ptr_last_state, ptr_last_bx, stream):
    """Tensor-core Mamba-3 SISO with the angle pre-pass fused in.  ``ptrs``:
    q, k, v, adt, dt, trap, q_bias, k_bias, angles, d_skip, z (the last two
    may be 0).  Device pointers, stream-ordered."""
    if len(ptrs) != 11:
        raise ValueError(f"expected 11 input pointers, got {len(ptrs)}")
    _check(load().arm_scan_mamba3_siso_tc_async(
        ctypes.byref(dims), ctypes.byref(opts), *[_n(p) for p in ptrs], int(reverse), ptr_out,
        _n(ptr_last_state), _n(ptr_last_bx), _n(stream)), "arm_scan_mamba3_siso_tc_async")


def mamba3_mimo_x_raw(dims, opts, ptrs, reverse, ptr_out, ptr_last_state, stream):
    """Per-rank Mamba-3 MIMO on the tensor cores.  ``ptrs``: x, b, c, adt,
    dt, trap, angles, d_skip (the last two may be 0).  Device pointers,
    stream-ordered."""
    if len(ptrs) != 8:
        raise ValueError(f"expected 8 input pointers, got {len(ptrs)}")
    _check(load().arm_scan_mamba3_mimo_x_tc_async(
        ctypes.byref(dims), ctypes.byref(opts), *[_n(p) for p in ptrs], int(reverse), ptr_out,
        _n(ptr_last_state), _n(stream)), "arm_scan_mamba3_mimo_x_tc_async")


def angles_workspace_bytes(dims, n_angles):
    return int(load().arm_scan_mamba3_angles_workspace_bytes(ctypes.byref(dims), n_angles))


def angles_async_raw(dims, ptr_angles, n_angles, ptr_dt, ptr_cos, ptr_sin, ptr_ws, ws_bytes,
                     stream):
    """Mamba-3 angle pre-pass (device pointers, stream-ordered)."""
    _check(load().arm_scan_mamba3_angles_f32_async(
        ctypes.byref(dims), ptr_angles, n_angles, ptr_dt, ptr_cos, ptr_sin, ptr_ws, ws_bytes,
        _n(stream)), "arm_scan_mamba3_angles_f32_async")


def ss2d_mamba3_raw(dims, grid_w, ptrs, n_angles, ptr_d_skip, ptr_z, ptr_out, stream):
    """Four-direction Mamba-3 SISO cross-scan of a row-major token grid.
    ``ptrs``: q, k, v, adt, dt, trap, q_bias, k_bias, angles."""
    _check(load().arm_scan_mamba3_ss2d_f32_async(
        ctypes.byref(dims), int(grid_w), *[_n(p) for p in ptrs], int(n_angles),
        _n(ptr_d_skip), _n(ptr_z), ptr_out, _n(stream)), "arm_scan_mamba3_ss2d_f32_async")


def noncausal_raw(dims, grid_w, ptrs, n_angles, ptr_cos, ptr_sin, ptr_d_skip, ptr_z, ptr_out,
                  stream):
    """Non-causal Mamba-3 aggregation (1D when grid_w == len, else a grid).
    ``ptrs``: q, k, v, adt, dt, trap, q_bias, k_bias, angles (angles 0 when
    cos/sin are given)."""
    _check(load().arm_scan_mamba3_noncausal_f32_async(
        ctypes.byref(dims), int(grid_w), *[_n(p) for p in ptrs], int(n_angles), _n(ptr_cos),
        _n(ptr_sin), _n(ptr_d_skip), _n(ptr_z), ptr_out, _n(stream)),
        "arm_scan_mamba3_noncausal_f32_async")


def conv_silu_raw(batch, dim, length, kernel, ptr_x, ptr_w, ptr_bias, ptr_out, stream):
    """Causal depthwise conv1d + bias + SiLU (device pointers)."""
    _check(load().arm_scan_causal_conv1d_silu_f32_async(
        batch, dim, length, kernel, ptr_x, ptr_w, _n(ptr_bias), ptr_out, _n(stream)),
        "arm_scan_causal_conv1d_silu_f32_async")


def final_state_raw(dims, ptr_u, ptr_delta, ptr_a, ptr_b, ptr_c, ptr_delta_bias, softplus,
                    reverse, ptr_h0, ptr_last, stream):
    """Final state of a Mamba-1 scan without outputs (device pointers)."""
    _check(load().arm_scan_selective_scan_final_state_f32_async(
        ctypes.byref(dims), ptr_u, ptr_delta, ptr_a, ptr_b, ptr_c, _n(ptr_delta_bias),
        int(softplus), int(reverse), _n(ptr_h0), ptr_last, _n(stream)),
        "arm_scan_selective_scan_final_state_f32_async")


def state_update_raw(dims, ptr_state, ptr_x, ptr_dt, ptr_a, ptr_b, ptr_c, ptr_d_skip, ptr_z,
                     ptr_dt_bias, dt_softplus, ptr_out, stream):
    """One Mamba-1 decode step (device pointers, stream-ordered)."""
    _check(load().arm_scan_selective_state_update_f32_async(
        ctypes.byref(dims), ptr_state, ptr_x, ptr_dt, ptr_a, ptr_b, ptr_c, _n(ptr_d_skip),
        _n(ptr_z), _n(ptr_dt_bias), int(dt_softplus), ptr_out, _n(stream)),
        "arm_scan_selective_state_update_f32_async")


def mixer_prologue_raw(dims, ptr_proj, ptr_dt_bias, ptr_b_norm_w, ptr_c_norm_w, a_floor, eps,
                       ptr_z, ptr_x, ptr_q, ptr_k, ptr_dt, ptr_adt, ptr_trap, ptr_angles, stream):
    """Mamba-3 mixer prologue (device pointers, stream-ordered)."""
    _check(load().arm_scan_mamba3_mixer_prologue_f32_async(
        ctypes.byref(dims), ptr_proj, ptr_dt_bias, ptr_b_norm_w, ptr_c_norm_w, float(a_floor),
        float(eps), ptr_z, ptr_x, ptr_q, ptr_k, ptr_dt, ptr_adt, ptr_trap, ptr_angles,
        _n(stream)), "arm_scan_mamba3_mixer_prologue_f32_async")


def scan_bidir_sum_raw(dims, ptr_u, ptr_delta, ptr_a, ptr_b, ptr_c, ptr_d_skip, ptr_z,
                       ptr_delta_bias, delta_softplus, backend, ptr_out, ptr_last_fwd=0,
                       ptr_last_bwd=0, ptr_h0_fwd=0, ptr_h0_bwd=0, *, stream):
    """Bidirectional Mamba-1 scan summed into one output (device pointers)."""
    _check(load().arm_scan_selective_scan_bidirectional_sum_f32_async(
        ctypes.byref(dims), ptr_u, ptr_delta, ptr_a, ptr_b, ptr_c, _n(ptr_d_skip), _n(ptr_z),
        _n(ptr_delta_bias), int(bool(delta_softplus)), BACKENDS[backend], THREADING["auto"],
        ptr_out, _n(ptr_last_fwd), _n(ptr_last_bwd), _n(ptr_h0_fwd), _n(ptr_h0_bwd),
        _n(stream)), "arm_scan_selective_scan_bidirectional_sum_f32_async")


def bidir_states_raw(dims, ptr_u, ptr_delta, ptr_a, ptr_b, ptr_c, ptr_delta_bias,
                     delta_softplus, backend, ptr_last_fwd, ptr_last_bwd, *, stream):
    """Final states of both traversals of a bidirectional scan (device pointers)."""
    _check(load().arm_scan_selective_scan_bidirectional_final_states_f32_async(
        ctypes.byref(dims), ptr_u, ptr_delta, ptr_a, ptr_b, ptr_c, _n(ptr_delta_bias),
        int(bool(delta_softplus)), BACKENDS[backend], ptr_last_fwd, ptr_last_bwd, _n(stream)),
        "arm_scan_selective_scan_bidirectional_final_states_f32_async")


def segment_summary_raw(dims, ptr_u, ptr_delta, ptr_a, ptr_b, ptr_c, ptr_delta_bias,
                        delta_softplus, backend, ptr_last_fwd, ptr_last_bwd, ptr_dt_sum, stream):
    """Both final states and the per-row sum of dt of a segment (device pointers)."""
    _check(load().arm_scan_selective_scan_segment_summary_f32_async(
        ctypes.byref(dims), ptr_u, ptr_delta, ptr_a, ptr_b, ptr_c, _n(ptr_delta_bias),
        int(bool(delta_softplus)), BACKENDS[backend], ptr_last_fwd, ptr_last_bwd, ptr_dt_sum,
        _n(stream)), "arm_scan_selective_scan_segment_summary_f32_async")


def bidirectional_workspace_bytes(dims):
    """Workspace of the two-phase bidirectional form (0: shape not covered)."""
    return int(load().arm_scan_selective_scan_bidirectional_workspace_bytes(ctypes.byref(dims)))


def bidirectional_summary_raw(dims, ptr_u, ptr_delta, ptr_a, ptr_b, ptr_c, ptr_delta_bias,
                              delta_softplus, ptr_ws, ws_bytes, ptr_last_fwd, ptr_last_bwd,
                              ptr_dt_sum, stream):
    """Phase 1 of the two-phase bidirectional form (device pointers)."""
    _check(load().arm_scan_selective_scan_bidirectional_summary_f32_async(
        ctypes.byref(dims), ptr_u, ptr_delta, ptr_a, ptr_b, ptr_c, _n(ptr_delta_bias),
        int(bool(delta_softplus)), ptr_ws, int(ws_bytes), ptr_last_fwd, ptr_last_bwd, ptr_dt_sum,
        _n(stream)), "arm_scan_selective_scan_bidirectional_summary_f32_async")


def bidirectional_finish_raw(dims, ptr_u, ptr_delta, ptr_a, ptr_b, ptr_c, ptr_d, ptr_z,
                             ptr_delta_bias, delta_softplus, ptr_ws, ws_bytes, ptr_h0_fwd,
                             ptr_h0_bwd, ptr_out, stream):
    """Phase 2 of the two-phase bidirectional form (device pointers)."""
    _check(load().arm_scan_selective_scan_bidirectional_finish_f32_async(
        ctypes.byref(dims), ptr_u, ptr_delta, ptr_a, ptr_b, ptr_c, _n(ptr_d), _n(ptr_z),
        _n(ptr_delta_bias), int(bool(delta_softplus)), ptr_ws, int(ws_bytes), _n(ptr_h0_fwd),
        _n(ptr_h0_bwd), ptr_out, _n(stream)),
        "arm_scan_selective_scan_bidirectional_finish_f32_async")


def ss2d_raw(dims, h, w, ptr_u, ptr_delta, ptr_a, ptr_b, ptr_c, ptr_d, ptr_delta_bias,
             delta_softplus, merge_mean, ptr_out, stream):
    """Mamba-1 SS2D cross-scan of grids read in place (device pointers)."""
    _check(load().arm_scan_selective_scan_ss2d_f32_async(
        ctypes.byref(dims), int(h), int(w), ptr_u, ptr_delta, ptr_a, ptr_b, ptr_c, _n(ptr_d),
        _n(ptr_delta_bias), int(bool(delta_softplus)), int(bool(merge_mean)), ptr_out, _n(stream)),
        "arm_scan_selective_scan_ss2d_f32_async")


def set_device(ordinal):
    """Device the synchronous host-buffer calls of this thread run on (-1:
    the current CUDA device)."""
    _check(load().arm_scan_set_device(int(ordinal)), "arm_scan_set_device")


def kernel_launches():
    """GPU kernels the library has launched in this process so far."""
    return int(load().arm_scan_kernel_launches())


KNOBS = {"m1_kernel": 0, "m1_segments": 1, "m1_bidir_independent": 2, "m3_tc_split": 3,
         "m3_chunk_form": 4, "pdl_off": 5}
M1_KERNELS = {"auto": 0, "lane": 1, "tile": 2, "chunked": 3, "tile_timesplit": 4}


def set_kernel_override(knob, value):
    """Process-wide kernel-selection override (``KNOBS``; 0 = default)."""
    _check(load().arm_scan_set_kernel_override(KNOBS[knob], int(value)),
           "arm_scan_set_kernel_override")


class kernel_override:
    """Context manager: ``with kernel_override(m1_kernel=2, m1_segments=4): ...``
    sets the given knobs and puts every one back to 0 on exit."""

    def __init__(self, **knobs):
        self.knobs = knobs

    def __enter__(self):
        for k, v in self.knobs.items():
            set_kernel_override(k, v)
        return self

    def __exit__(self, *exc):
        for k in self.knobs:
            set_kernel_override(k, 0)
        return False


def tensor_status():
    """Raise if a tensor-core kernel's bounded wait expired since the last
    check (call after synchronizing the stream of an async launch)."""
    _check(load().arm_scan_tensor_status(), "arm_scan_tensor_status")


def exported_symbols():
    """Names of every entry point include/b200scan.h declares."""
    return ["arm_scan_abi_version", "arm_scan_last_error",
            "arm_scan_selective_scan_f32", "arm_scan_selective_scan_f32_async",
            "arm_scan_selective_scan_bidirectional_f32",
            "arm_scan_selective_scan_bidirectional_f32_async",
            "arm_scan_mamba3_scan_f32", "arm_scan_mamba3_scan_f32_async",
            "arm_scan_mamba3_angles_workspace_bytes", "arm_scan_mamba3_angles_f32_async",
            "arm_scan_mamba3_angles_f32_noalloc", "arm_scan_tensor_status",
            "arm_scan_mamba3_siso_tc_async", "arm_scan_kernel_launches",
            "arm_scan_selective_state_update_f32_async",
            "arm_scan_selective_scan_final_state_f32_async", "arm_scan_mamba3_ss2d_f32_async",
            "arm_scan_mamba3_mixer_prologue_f32_async",
            "arm_scan_selective_scan_bidirectional_sum_f32_async",
            "arm_scan_selective_scan_bidirectional_final_states_f32_async",
            "arm_scan_set_kernel_override", "arm_scan_mamba3_mimo_x_tc_async",
            "arm_scan_selective_scan_segment_summary_f32_async",
            "arm_scan_mamba3_noncausal_f32_async", "arm_scan_causal_conv1d_silu_f32_async",
            "arm_scan_set_device", "arm_scan_selective_scan_bidirectional_workspace_bytes",
            "arm_scan_selective_scan_bidirectional_summary_f32_async",
            "arm_scan_selective_scan_bidirectional_finish_f32_async",
            "arm_scan_selective_scan_ss2d_f32_async"]


if __name__ == "__main__":  # pragma: no cover
    print(lib_path(), load().arm_scan_abi_version(), file=sys.stderr)
