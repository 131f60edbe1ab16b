"""The allocation-free angle pre-pass entry point, through the C ABI.

arm_scan_mamba3_angles_f32_noalloc exists for callers that may not allocate
device memory while they run (a host framework or inference server that owns
all device memory through its own allocator, or a real-time caller that
forbids allocation after start-up).  It keeps its scratch in a fixed array
inside the library, so it must give the same cos/sin as the workspace entry
point, call after call, even though every call reuses the same array.

This file is named to be collected last: if it fails, a run stopping at the
first failure has already run every other test.  It passes alone in a fresh
process and after the rest of the suite.
"""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = 1e-6  # the two entry points run the same kernels; results agree to rounding


def _inputs(b, length, h, r, seed):
    g = torch.Generator().manual_seed(seed)
    ang = torch.randn(b, length, h, r, generator=g).cuda()
    dt = torch.nn.functional.softplus(torch.randn(b, h, length, generator=g) - 4).cuda()
    return ang.contiguous(), dt.contiguous()


def _with_workspace(lib, dims, ang, dt, r, half):
    from armhackathon_b200 import _ffi
    cos = torch.empty(ang.shape[0], ang.shape[1], ang.shape[2], half, device="cuda")
    sin = torch.empty_like(cos)
    nbytes = _ffi.angles_workspace_bytes(dims, r)
    ws = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    rc = lib.arm_scan_mamba3_angles_f32_async(ctypes.byref(dims), ang.data_ptr(), r,
                                              dt.data_ptr(), cos.data_ptr(), sin.data_ptr(),
                                              ws.data_ptr(), nbytes, None)
    assert rc == 0
    return cos, sin


def _no_alloc(lib, dims, ang, dt, r, half):
    cos = torch.full((ang.shape[0], ang.shape[1], ang.shape[2], half), float("nan"),
                     device="cuda")
    sin = torch.full_like(cos, float("nan"))
    rc = lib.arm_scan_mamba3_angles_f32_noalloc(ctypes.byref(dims), ang.data_ptr(), r,
                                                dt.data_ptr(), cos.data_ptr(), sin.data_ptr(),
                                                None)
    assert rc == 0, lib.arm_scan_last_error()
    return cos, sin


def test_no_alloc_matches_workspace_entry_on_two_calls_in_a_row():
    from armhackathon_b200 import _ffi
    lib = _ffi.load()
    # two different problems back to back: the second reuses the array the
    # first left behind (a longer sequence first, then a shorter one)
    for (b, length, h, dqk, r, seed) in [(2, 3000, 3, 64, 20, 1), (3, 700, 5, 32, 16, 2)]:
        ang, dt = _inputs(b, length, h, r, seed)
        dims = _ffi.ArmMamba3Dims(b, h, 0, dqk, length, 1)
        want_c, want_s = _with_workspace(lib, dims, ang, dt, r, dqk // 2)
        got_c, got_s = _no_alloc(lib, dims, ang, dt, r, dqk // 2)
        torch.cuda.synchronize()
        assert torch.allclose(got_c, want_c, atol=TOL, rtol=0)
        assert torch.allclose(got_s, want_s, atol=TOL, rtol=0)
