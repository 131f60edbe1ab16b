"""armhackathon_b200 -- a B200-native selective-scan engine with the op
surface of the reference ``arm_scan`` package (AdityaP9116/ARMHackathon).

    import armhackathon_b200 as arm_scan
    arm_scan.patch()                       # HF transformers Mamba uses the GPU scan
    arm_scan.selective_scan(u, delta, A, B, C, D=..., z=...)
    arm_scan.bidirectional_scan(...) / ss2d_scan(...)
    arm_scan.mamba3_scan(...) / mamba3_scan_pair(...) / mamba3_mimo_scan(...)
    arm_scan.ss2d_scan_mamba3(...) / noncausal_scan(...) / ss2d_noncausal_mamba3(...)
    arm_scan.selective_scan_numpy(...)     # numpy in, numpy out (no torch)
    arm_scan.selective_state_update(state, x, dt, A, B, C, ...)  # one decode step
    arm_scan.mamba3_mixer_prologue(proj, ...) / mamba3_mixer_scan(proj, ...)  # Mamba-3 mixer

Every scan runs as sm_100a CUDA kernels in libb200scan.so, reached through
its C ABI (include/b200scan.h).  There is no CPU implementation.
"""

from ._ffi import lib_path
from .numpy_api import selective_scan_numpy

__all__ = [
    "selective_scan_numpy", "lib_path", "selective_scan", "selective_scan_bidirectional",
    "bidirectional_scan", "ss2d_scan", "use_arm_scan", "mamba3_scan", "mamba3_scan_pair",
    "mamba3_mimo_scan", "ss2d_scan_mamba3", "noncausal_scan", "noncausal_scan_dense",
    "ss2d_noncausal_mamba3", "angles_to_cos_sin", "patch", "unpatch", "stats", "kernel_calls",
    "selective_state_update", "selective_scan_final_state", "mamba3_mixer_prologue",
    "selective_scan_bidirectional_sum", "selective_scan_bidirectional_final_states",
    "mamba3_mixer_scan", "mamba3_mimo_x_scan", "selective_scan_segment_summary",
    "causal_conv1d_silu", "BidirectionalSegment", "selective_scan_ss2d",
]

_LAZY = {
    "selective_scan": ".op", "selective_scan_bidirectional": ".op", "kernel_calls": ".op",
    "selective_state_update": ".op", "selective_scan_final_state": ".op",
    "selective_scan_bidirectional_sum": ".op",
    "selective_scan_segment_summary": ".op", "causal_conv1d_silu": ".op",
    "BidirectionalSegment": ".op", "selective_scan_ss2d": ".op",
    "selective_scan_bidirectional_final_states": ".op",
    "bidirectional_scan": ".bidirectional",
    "ss2d_scan": ".ss2d", "use_arm_scan": ".ss2d",
    "mamba3_scan": ".mamba3", "mamba3_scan_pair": ".mamba3", "mamba3_mimo_scan": ".mamba3",
    "mamba3_mimo_x_scan": ".mamba3",
    "angles_to_cos_sin": ".mamba3",
    "ss2d_scan_mamba3": ".ss2d_mamba3",
    "noncausal_scan": ".mamba3_noncausal", "noncausal_scan_dense": ".mamba3_noncausal",
    "ss2d_noncausal_mamba3": ".mamba3_noncausal",
    "mamba3_mixer_prologue": ".mamba3_mixer", "mamba3_mixer_scan": ".mamba3_mixer",
    "patch": ".hf_patch", "unpatch": ".hf_patch", "stats": ".hf_patch",
}


def __getattr__(name):
    # torch-dependent modules load on first use, so numpy-only callers never
    # import torch
    import importlib
    if name in _LAZY:
        # importing a submodule binds it as a package attribute (``patch`` is
        # both a module and its function): rebind the function afterwards
        obj = getattr(importlib.import_module(_LAZY[name], __name__), name)
        globals()[name] = obj
        return obj
    raise AttributeError(f"module 'armhackathon_b200' has no attribute '{name}'")
