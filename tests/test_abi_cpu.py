"""C-ABI library checks that need no GPU: it loads, reports ABI v13, exports
every entry point include/b200scan.h declares, and rejects bad arguments with
the reference's codes before touching a device (reference
kernel/arm-scan-ffi/src/lib.rs:53-58 and its FFI unit tests)."""

import ctypes
import re
import subprocess

import pytest

from conftest import ROOT

from armhackathon_b200 import _ffi

HEADER = ROOT / "include" / "b200scan.h"


def declared_functions():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"\b(arm_scan_[a-z0-9_]+)\s*\(", text)))


def test_library_loads_with_abi_v13():
    lib = _ffi.load()
    assert lib.arm_scan_abi_version() == 13
    assert _ffi.lib_path().name == "libb200scan.so"


def test_every_declared_symbol_is_exported():
    out = subprocess.run(["nm", "-D", "--defined-only", str(_ffi.lib_path())],
                         capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r"\sT\s(\w+)", out))
    declared = declared_functions()
    assert declared, "header parse found nothing"
    missing = [f for f in declared if f not in exported]
    assert not missing, missing
    assert set(_ffi.exported_symbols()) <= set(declared)


def _m1_call(dims, ptrs=None, backend=0, threading=0, out=True):
    lib = _ffi.load()
    buf = (ctypes.c_float * 8)()
    p = ctypes.cast(buf, ctypes.c_void_p).value
    args = ptrs if ptrs is not None else [p] * 5
    return lib.arm_scan_selective_scan_f32(
        ctypes.byref(dims) if dims is not None else None, *args, None, None, None,
        1, 0, backend, threading, p if out else None, None, None)


def test_null_pointer_rejected():
    dims = _ffi.ArmScanDims(1, 1, 1, 1, 1)
    assert _m1_call(dims, out=False) == 1
    assert _m1_call(None) == 1
    assert "null" in _ffi.load().arm_scan_last_error().decode()


def test_bad_enum_and_neon_backend():
    dims = _ffi.ArmScanDims(1, 1, 1, 1, 1)
    assert _m1_call(dims, backend=7) == 4
    assert _m1_call(dims, threading=-1) == 4
    assert _m1_call(dims, backend=2) == 3


@pytest.mark.parametrize("bad", [(0, 1, 1, 1, 1), (1, 0, 1, 1, 1), (1, 1, 0, 1, 1),
                                 (1, 1, 1, 0, 1), (1, 1, 1, 1, 0), (1, 3, 4, 16, 2),
                                 (1, 4, 4, 257, 1)])
def test_invalid_dims_rejected(bad):
    assert _m1_call(_ffi.ArmScanDims(*bad)) == 2


def test_overflowing_dims_rejected():
    big = (1 << 63) + 1
    assert _m1_call(_ffi.ArmScanDims(big, 4, 4, 4, 1)) == 2


def test_bidir_half_carry_rejected():
    lib = _ffi.load()
    buf = (ctypes.c_float * 8)()
    p = ctypes.cast(buf, ctypes.c_void_p).value
    dims = _ffi.ArmScanDims(1, 1, 1, 1, 1)
    rc = lib.arm_scan_selective_scan_bidirectional_f32(
        ctypes.byref(dims), p, p, p, p, p, None, None, None, 1, 0, 0, p, p, p, None)
    assert rc == 2


def _m3(dims, mimo=0, last_state=False, last_bx=False, reverse=0):
    lib = _ffi.load()
    buf = (ctypes.c_float * 8)()
    p = ctypes.cast(buf, ctypes.c_void_p).value
    proj = [p if i < mimo else None for i in range(3)]
    return lib.arm_scan_mamba3_scan_f32(
        ctypes.byref(dims), p, p, p, p, p, p, p, p, p, p, None, None, *proj, reverse, 0, 0, p,
        p if last_state else None, p if last_bx else None)


def test_mamba3_argument_rules():
    siso = _ffi.ArmMamba3Dims(1, 1, 4, 4, 1, 1)
    assert _m3(siso, mimo=2) == 1                          # partial projections
    assert _m3(siso, last_state=True) == 1                 # half a carry
    assert _m3(_ffi.ArmMamba3Dims(1, 1, 4, 5, 1, 1)) == 2  # odd dqk
    assert _m3(_ffi.ArmMamba3Dims(1, 1, 4, 4, 1, 2)) == 2  # rank>1 without projections
    assert _m3(_ffi.ArmMamba3Dims(1, 1, 4, 4, 1, 2), mimo=3, last_state=True,
               last_bx=True) == 2                          # MIMO has no last_bx
    assert _m3(_ffi.ArmMamba3Dims(0, 1, 4, 4, 1, 1)) == 2  # zero dim


def _tc(dims, opts, angles=True, null_q=False, last_state=False, last_bx=False):
    """arm_scan_mamba3_siso_tc_async with dummy non-null pointers: every
    case here is rejected by the host checks before any device work."""
    lib = _ffi.load()
    p = ctypes.c_void_p(16)
    ptrs = [None if null_q else p] + [p] * 7 + [p if angles else None, None, None]
    return lib.arm_scan_mamba3_siso_tc_async(
        ctypes.byref(dims), opts if opts is None else ctypes.byref(opts), *ptrs, 0, p,
        p if last_state else None, p if last_bx else None, None)


def test_tensor_entry_argument_rules():
    good = _ffi.ArmMamba3Dims(1, 1, 64, 128, 1, 1)
    o = lambda i=0, out=0, lay=1, sh=1, n=64: _ffi.ArmMamba3TcOptions(i, out, lay, sh, n)  # noqa: E731
    assert _tc(good, None) == 1                                     # null opts
    assert _tc(good, o(), null_q=True) == 1                         # null q
    assert _tc(good, o(), angles=False) == 1                        # angles needed for n_angles > 0
    assert _tc(good, o(), last_state=True) == 1                     # half a carry
    assert _tc(good, o(i=2)) == 4                                   # bad dtype
    assert _tc(good, o(out=-1)) == 4
    assert _tc(good, o(lay=2)) == 4                                 # bad layout
    assert _tc(good, o(sh=3)) == 4
    assert _tc(good, o(n=65)) == 2                                  # more pairs than dqk/2
    assert _tc(_ffi.ArmMamba3Dims(1, 1, 64, 128, 1, 2), o()) == 2   # rank 2 (no projections)
    assert _tc(_ffi.ArmMamba3Dims(1, 1, 64, 64, 1, 1), o(n=32)) == 3  # dqk 64: not covered
    assert _tc(_ffi.ArmMamba3Dims(1, 1, 32, 128, 1, 1), o()) == 3   # dv 32: not covered
    assert b"tensor" in _ffi.load().arm_scan_last_error()


def test_lazy_exports_are_functions_after_submodule_import():
    import importlib
    import armhackathon_b200 as arm
    importlib.import_module("armhackathon_b200.hf_patch")
    for name in ("patch", "unpatch", "stats", "selective_scan", "mamba3_scan", "ss2d_scan"):
        assert callable(getattr(arm, name)) and not hasattr(getattr(arm, name), "__path__")
    assert type(arm.patch).__name__ == "function"


def test_state_update_argument_rules():
    """arm_scan_selective_state_update_f32_async: host checks before any
    device work (dummy pointers never dereferenced)."""
    lib = _ffi.load()
    p = ctypes.c_void_p(16)

    def call(dims, null_state=False):
        return lib.arm_scan_selective_state_update_f32_async(
            ctypes.byref(dims), None if null_state else p, p, p, p, p, p, None, None, None, 1, p,
            None)
    assert call(_ffi.ArmScanDims(1, 4, 1, 4, 1), null_state=True) == 1
    assert call(_ffi.ArmScanDims(0, 4, 1, 4, 1)) == 2
    assert call(_ffi.ArmScanDims(1, 6, 1, 4, 4)) == 2   # dim not a multiple of groups


def test_mixer_prologue_argument_rules():
    """arm_scan_mamba3_mixer_prologue_f32_async: host checks before any
    device work (dummy pointers never dereferenced)."""
    lib = _ffi.load()
    p = ctypes.c_void_p(16)

    def call(dims, null_proj=False):
        return lib.arm_scan_mamba3_mixer_prologue_f32_async(
            ctypes.byref(dims), None if null_proj else p, p, p, p, ctypes.c_float(1e-4),
            ctypes.c_float(1e-5), p, p, p, p, p, p, p, p, None)
    assert call(_ffi.ArmMamba3MixerDims(1, 4, 2, 8, 16, 1, 4), null_proj=True) == 1
    assert call(_ffi.ArmMamba3MixerDims(1, 4, 0, 8, 16, 1, 4)) == 2   # no heads
    assert call(_ffi.ArmMamba3MixerDims(1, 4, 2, 8, 16, 1, 9)) == 2   # n_angles > d_state / 2
    assert call(_ffi.ArmMamba3MixerDims(1, 1 << 62, 2, 8, 16, 1, 4)) == 2  # overflow


def test_bidirectional_sum_and_states_argument_rules():
    """The bidirectional sum / final-states entries: host checks before any
    device work (dummy pointers never dereferenced)."""
    lib = _ffi.load()
    p = ctypes.c_void_p(16)
    dims = _ffi.ArmScanDims(1, 4, 64, 4, 1)

    def sum_call(out=p, lf=None, lb=None, d=dims):
        return lib.arm_scan_selective_scan_bidirectional_sum_f32_async(
            ctypes.byref(d), p, p, p, p, p, None, None, None, 1, 0, 0, out, lf, lb, None, None,
            None)

    def states_call(lf=p, lb=p, backend=0, d=dims):
        return lib.arm_scan_selective_scan_bidirectional_final_states_f32_async(
            ctypes.byref(d), p, p, p, p, p, None, 1, backend, lf, lb, None)
    assert sum_call(out=None) == 1
    assert sum_call(lf=p) == 2                  # last states both-or-neither
    assert sum_call(d=_ffi.ArmScanDims(0, 4, 64, 4, 1)) == 2
    assert states_call(lb=None) == 1
    assert states_call(backend=2) == 3          # neon backend unavailable
    assert states_call(backend=9) == 4
    assert states_call(d=_ffi.ArmScanDims(1, 6, 64, 4, 4)) == 2  # dim not a multiple of groups


def test_no_alloc_angles_reject_problems_beyond_their_scratch():
    """The allocation-free angle entry checks the problem against its fixed
    4 MiB scratch before any CUDA call: 64 heads x 1024 chunks x 64 angles x
    4 B = 16 MiB is refused with code 2 (dummy non-null pointers, no GPU)."""
    lib = _ffi.load()
    dims = _ffi.ArmMamba3Dims(1, 64, 0, 128, 128 * 1024, 1)
    dummy = 16
    rc = lib.arm_scan_mamba3_angles_f32_noalloc(ctypes.byref(dims), dummy, 64, dummy, dummy,
                                                dummy, None)
    assert rc == 2
    assert b"scratch" in lib.arm_scan_last_error()


def test_set_device_rejects_ordinals_outside_the_machine():
    """arm_scan_set_device accepts -1 (the current device) and rejects an
    ordinal beyond the device count with code 2 (no GPU here: every ordinal
    >= 0 is outside)."""
    lib = _ffi.load()
    assert lib.arm_scan_set_device(-1) == 0
    assert lib.arm_scan_set_device(64) == 2
    assert lib.arm_scan_set_device(-2) == 2


def test_angle_entries_reject_lengths_beyond_the_grid():
    """The angle pre-pass launches one CTA per 128-step chunk: a length whose
    chunk count does not fit the grid is refused (code 2) before any CUDA call."""
    lib = _ffi.load()
    dims = _ffi.ArmMamba3Dims(1, 1, 0, 128, (1 << 31) * 128 + 1, 1)
    dummy = 16
    rc = lib.arm_scan_mamba3_angles_f32_async(ctypes.byref(dims), dummy, 64, dummy, dummy, dummy,
                                              dummy, 1 << 40, None)
    assert rc == 2
    assert b"chunks" in lib.arm_scan_last_error()


def test_bidirectional_workspace_bytes_host_only():
    """The two-phase form's workspace size is a host computation that needs
    no device for the shapes it does not cover (state > 16, length not a
    multiple of 4, no dims): 0.  (Covered shapes need the device's SM count
    for their segment plan; the GPU tests check those.)"""
    from armhackathon_b200 import _ffi
    lib = _ffi.load()
    f = lambda *d: _ffi.bidirectional_workspace_bytes(_ffi.ArmScanDims(*d))  # noqa: E731
    assert f(1, 64, 1027, 16, 1) == 0
    assert f(1, 64, 1024, 32, 1) == 0
    assert f(1, 64, 0, 16, 1) == 0
    assert lib.arm_scan_selective_scan_bidirectional_workspace_bytes(None) == 0


def test_ss2d_entry_rejects_before_device_work():
    """The one-call Mamba-1 SS2D entry: null pointers (code 1), a length that
    is not h x w (code 2), d_state > 16 and groups whose channel count is
    not a multiple of 8 (code 3) -- all host checks, no device touched."""
    lib = _ffi.load()
    buf = (ctypes.c_float * 8)()
    p = ctypes.cast(buf, ctypes.c_void_p).value

    def call(dims, h, w, out=p):
        return lib.arm_scan_selective_scan_ss2d_f32_async(
            ctypes.byref(dims), h, w, p, p, p, p, p, None, None, 1, 0, out, None)

    assert call(_ffi.ArmScanDims(1, 8, 12, 16, 1), 3, 4, out=None) == 1
    assert call(_ffi.ArmScanDims(1, 8, 12, 16, 1), 3, 5) == 2
    assert call(_ffi.ArmScanDims(1, 8, 12, 16, 1), 0, 12) == 2
    assert call(_ffi.ArmScanDims(1, 8, 12, 32, 1), 3, 4) == 3
    assert call(_ffi.ArmScanDims(1, 24, 12, 16, 2), 3, 4) == 3
    assert "multiple of 8" in lib.arm_scan_last_error().decode()


def test_bidirectional_phases_reject_before_device_work():
    """The two-phase bidirectional entries: null workspace or outputs (code
    1) and shapes the two-phase kernels do not cover (code 3), checked on
    the host."""
    lib = _ffi.load()
    buf = (ctypes.c_float * 8)()
    p = ctypes.cast(buf, ctypes.c_void_p).value
    dims = _ffi.ArmScanDims(1, 8, 64, 16, 1)
    s = lib.arm_scan_selective_scan_bidirectional_summary_f32_async
    f = lib.arm_scan_selective_scan_bidirectional_finish_f32_async
    assert s(ctypes.byref(dims), p, p, p, p, p, None, 1, None, 0, p, p, p, None) == 1
    assert s(ctypes.byref(dims), p, p, p, p, p, None, 1, p, 64, p, None, p, None) == 1
    assert f(ctypes.byref(dims), p, p, p, p, p, None, None, None, 1, p, 64, None, None, None,
             None) == 1
    odd = _ffi.ArmScanDims(1, 8, 63, 16, 1)
    assert f(ctypes.byref(odd), p, p, p, p, p, None, None, None, 1, p, 64, None, None, p,
             None) == 3
