"""Mamba-3 mixer around the scan: the prologue between ``in_proj`` and the
scan call, fused into one CUDA kernel, and the mixer's forward from the
``in_proj`` output to the scan output.

Reference: apps/mamba3_lm/block.py.  ``Mamba3Mixer.forward`` (146-199) splits
the in_proj output into [z, x, B, C, dd_dt, dd_A, trap, angles] (116-121,
150-151), computes the data-dependent decay ``A = clamp(-heavy_tail(dd_A),
max=-A_floor)`` (52-62, 164-165), ``DT = softplus(dd_dt + dt_bias)`` (166),
``ADT = A * DT`` (167), transposes DT / ADT / trap to (b, h, l) (158,
168-169), broadcasts the angles over heads (174), RMS-normalizes B and C
(78-82, 176-177) and calls the scan with Q <- C, K <- B (179-199).  There
every step is a separate torch op; here ``mamba3_mixer_prologue`` does all of
them in one pass over ``proj`` (``arm_scan_mamba3_mixer_prologue_f32_async``)
and ``mamba3_mixer_scan`` feeds the result to ``mamba3_scan`` /
``mamba3_mimo_scan``.  One B/C group, as the reference's MIMO entry requires
(python/arm_scan/mamba3.py:289-294).
"""

from typing import NamedTuple, Optional

import torch

from . import _ffi
from .mamba3 import mamba3_mimo_scan, mamba3_scan
from .op import _on_device, _stream


class MixerPrologue(NamedTuple):
    z: torch.Tensor       # (b, l, h, p)
    x: torch.Tensor       # (b, l, h, p)
    q: torch.Tensor       # (b, l, r, n): RMSNorm(C) * C_norm weight
    k: torch.Tensor       # (b, l, r, n): RMSNorm(B) * B_norm weight
    dt: torch.Tensor      # (b, h, l)
    adt: torch.Tensor     # (b, h, l)
    trap: torch.Tensor    # (b, h, l), pre-sigmoid
    angles: torch.Tensor  # (b, l, n_angles)


def proj_width(nheads, headdim, d_state, mimo_rank, n_angles):
    """Width of one in_proj row (block.py:116-121, one B/C group)."""
    return 2 * nheads * headdim + 2 * mimo_rank * d_state + 3 * nheads + n_angles


def mamba3_mixer_prologue(proj, *, nheads, headdim, d_state, n_angles, dt_bias,
                          B_norm_weight, C_norm_weight, mimo_rank=1, A_floor=1e-4,
                          eps=1e-5) -> MixerPrologue:
    """The scan's inputs from the in_proj output ``proj`` (b, l, W), a float32
    CUDA tensor, in one kernel.  ``dt_bias`` (h,), the norm weights (d_state,).
    Raises on a CPU tensor: there is no host path."""
    if proj.device.type != "cuda":
        raise ValueError("mamba3_mixer_prologue needs a CUDA tensor (no host path)")
    if proj.dim() != 3:
        raise ValueError(f"proj must be (b, l, W), got {tuple(proj.shape)}")
    if n_angles > d_state // 2:
        raise ValueError(f"n_angles ({n_angles}) exceeds d_state / 2 ({d_state // 2})")
    b, l, w = proj.shape
    want = proj_width(nheads, headdim, d_state, mimo_rank, n_angles)
    if w != want:
        raise ValueError(f"proj rows are {w} wide; this mixer's are {want} (one B/C group)")
    dev = proj.device
    f32 = lambda t: t.detach().to(device=dev, dtype=torch.float32).contiguous()  # noqa: E731
    proj = f32(proj)
    dt_bias, bw, cw = f32(dt_bias), f32(B_norm_weight), f32(C_norm_weight)
    for name, t, n in (("dt_bias", dt_bias, nheads), ("B_norm_weight", bw, d_state),
                       ("C_norm_weight", cw, d_state)):
        if t.numel() != n:
            raise ValueError(f"{name} must have {n} elements, got {t.numel()}")
    new = lambda *s: torch.empty(s, device=dev, dtype=torch.float32)  # noqa: E731
    out = MixerPrologue(
        z=new(b, l, nheads, headdim), x=new(b, l, nheads, headdim),
        q=new(b, l, mimo_rank, d_state), k=new(b, l, mimo_rank, d_state),
        dt=new(b, nheads, l), adt=new(b, nheads, l), trap=new(b, nheads, l),
        angles=new(b, l, n_angles))
    dims = _ffi.ArmMamba3MixerDims(b, l, nheads, headdim, d_state, mimo_rank, n_angles)
    with _on_device(proj):
        _ffi.mixer_prologue_raw(
            dims, proj.data_ptr(), dt_bias.data_ptr(), bw.data_ptr(), cw.data_ptr(), A_floor,
            eps, out.z.data_ptr(), out.x.data_ptr(), out.q.data_ptr(), out.k.data_ptr(),
            out.dt.data_ptr(), out.adt.data_ptr(), out.trap.data_ptr(), out.angles.data_ptr(),
            _stream(proj))
    return out


def mamba3_mixer_scan(proj, *, nheads, headdim, d_state, n_angles, dt_bias, B_norm_weight,
                      C_norm_weight, D, B_bias, C_bias, mimo_rank=1, A_floor=1e-4, eps=1e-5,
                      psi: Optional[torch.Tensor] = None, zeta: Optional[torch.Tensor] = None,
                      phi: Optional[torch.Tensor] = None, precision="fp32"):
    """``Mamba3Mixer.forward`` from the in_proj output to the scan output
    (block.py:146-198): the fused prologue, then the SISO or MIMO scan with
    Q <- C, K <- B and the angles broadcast over heads.  ``B_bias`` /
    ``C_bias`` are (h, r, n) as in the checkpoint; ``psi``/``zeta``/``phi``
    (the mixer's mimo_x / mimo_z / mimo_o) are required for rank > 1.
    Returns y (b, l, h * p) (the out_proj input)."""
    pro = mamba3_mixer_prologue(
        proj, nheads=nheads, headdim=headdim, d_state=d_state, n_angles=n_angles,
        dt_bias=dt_bias, B_norm_weight=B_norm_weight, C_norm_weight=C_norm_weight,
        mimo_rank=mimo_rank, A_floor=A_floor, eps=eps)
    b, l = proj.shape[:2]
    angles = pro.angles.unsqueeze(-2).expand(-1, -1, nheads, -1)
    if mimo_rank > 1:
        if psi is None or zeta is None or phi is None:
            raise ValueError("a MIMO mixer needs psi, zeta and phi")
        y = mamba3_mimo_scan(
            q=pro.q, k=pro.k, v=pro.x, adt=pro.adt, dt=pro.dt, trap=pro.trap,
            q_bias=C_bias, k_bias=B_bias, psi=psi, zeta=zeta, phi=phi, angles=angles, D=D,
            z=pro.z, precision=precision)
    else:
        y = mamba3_scan(
            q=pro.q, k=pro.k, v=pro.x, adt=pro.adt, dt=pro.dt, trap=pro.trap,
            q_bias=C_bias.reshape(nheads, d_state), k_bias=B_bias.reshape(nheads, d_state),
            angles=angles, D=D, z=pro.z, precision=precision)
    return y.reshape(b, l, nheads * headdim)
