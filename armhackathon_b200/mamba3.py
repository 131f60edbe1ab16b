"""PyTorch front-end of the Mamba-3 scans (SISO and rank-r MIMO).

Same surface as the reference's python/arm_scan/mamba3.py: the custom op
``arm_scan::mamba3_scan`` (with a fake kernel), ``angles_to_cos_sin`` (the RoPE
angle pre-pass), ``mamba3_scan``, ``mamba3_scan_pair`` and
``mamba3_mimo_scan``, with the reference's argument names, layouts and shape
checks.  Extension: ``return_last_state=True`` also returns the final state
(batch, heads, dv, dqk), which the reference's op never exposes.

Contracts kept from the reference:
* ``trap`` is PRE-sigmoid; the kernel applies the sigmoid.
* angles arrive raw and ``angles_to_cos_sin`` accumulates
  theta = cumsum(tanh(angle) * pi * dt) along the traversal-order time axis;
  fewer angle pairs than dqk/2 are padded with the identity rotation.
* SISO rotates interleaved lane pairs, MIMO rotates split halves.
* the kernel writes head-major (b, h, l, dv); the op returns time-major
  (b, l, h, dv).
All tensors of a call live on one device; CPU tensors are computed on the
current CUDA device through the synchronous entry point.
"""

import math
from typing import Optional, Tuple

import torch

from . import _ffi
from .op import _CALLS, _on_device, _prep, _ptr, _stream
from .op import kernel_calls  # noqa: F401  (re-export, like the reference)


def angles_to_cos_sin(angles: torch.Tensor, dt: torch.Tensor,
                      half: int) -> Tuple[torch.Tensor, torch.Tensor]:
    """RoPE angle pre-pass: theta = cumsum(tanh(angle) * pi * dt) over time.

    angles (b, l, h, r) raw, dt (b, h, l) post-softplus, half = dqk // 2;
    returns cos, sin (b, l, h, half), computed at the angles' precision
    floored at float32; pairs r..half-1 get cos = 1, sin = 0.
    """
    if angles.dim() != 4:
        raise ValueError(f"angles must be (b, l, h, r), got {tuple(angles.shape)}")
    r = angles.shape[-1]
    if r > half:
        raise ValueError(f"angles has {r} rotation pairs but the head dim allows {half}")
    dtype = torch.promote_types(angles.dtype, torch.float32)
    if dtype == torch.float64:
        # f64 analysis path (the dense non-causal check): plain torch, at the
        # caller's precision, exactly as the reference computes it
        dt_blh = dt.permute(0, 2, 1).unsqueeze(-1).to(dtype)
        theta = torch.cumsum(torch.tanh(angles.to(dtype)) * math.pi * dt_blh, dim=1)
        cos, sin = torch.cos(theta), torch.sin(theta)
        if r < half:
            pad = (*theta.shape[:-1], half - r)
            cos = torch.cat([cos, torch.ones(pad, dtype=cos.dtype, device=cos.device)], dim=-1)
            sin = torch.cat([sin, torch.zeros(pad, dtype=sin.dtype, device=sin.device)], dim=-1)
        return cos, sin
    return _angles_gpu(angles, dt, half)


def _angles_gpu(angles, dt, half):
    """fp32 pre-pass through the library's CUDA kernel; CPU inputs are
    computed on the current CUDA device and returned on the CPU."""
    home = angles.device
    dev = home if home.type == "cuda" else torch.device("cuda", torch.cuda.current_device())
    a = angles.to(device=dev, dtype=torch.float32).contiguous()
    d = dt.to(device=dev, dtype=torch.float32).contiguous()
    b, length, h, r = a.shape
    cos = torch.empty((b, length, h, half), device=dev)
    sin = torch.empty_like(cos)
    dims = _ffi.ArmMamba3Dims(b, h, 0, 2 * half, length, 1)
    nbytes = _ffi.angles_workspace_bytes(dims, r)
    ws = torch.empty(max(nbytes, 4), dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        _ffi.angles_async_raw(dims, a.data_ptr(), r, d.data_ptr(), cos.data_ptr(),
                              sin.data_ptr(), ws.data_ptr(), nbytes,
                              torch.cuda.current_stream(dev).cuda_stream)
    if home.type != "cuda":
        cos, sin = cos.to(home), sin.to(home)
    return cos, sin


@torch.library.custom_op("arm_scan::mamba3_scan", mutates_args=())
def _mamba3_scan_op(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    adt: torch.Tensor,
    dt: torch.Tensor,
    trap: torch.Tensor,
    q_bias: torch.Tensor,
    k_bias: torch.Tensor,
    cos: torch.Tensor,
    sin: torch.Tensor,
    d_skip: Optional[torch.Tensor],
    z: Optional[torch.Tensor],
    reverse: bool,
    psi: Optional[torch.Tensor] = None,
    zeta: Optional[torch.Tensor] = None,
    phi: Optional[torch.Tensor] = None,
    backend: int = 0,
) -> Tuple[torch.Tensor, torch.Tensor]:
    # q is (b, l, 1, dqk) for SISO (axis 2 = the single B/C group) and
    # (b, l, rank, dqk) for MIMO (axis 2 = rank); the projections decide.
    b, length, rank, dqk = q.shape
    h, dv = v.shape[2], v.shape[3]
    mimo = psi is not None
    dims = _ffi.ArmMamba3Dims(b, h, dv, dqk, length, rank)
    out_hm = v.new_empty((b, h, length, dv))
    last_state = v.new_empty((b, h, dv, dqk))
    last_bx = None if mimo else v.new_empty((b, h, dqk))
    with _on_device(v):
        _ffi.mamba3_raw(
            dims,
            [q.data_ptr(), k.data_ptr(), v.data_ptr(), adt.data_ptr(), dt.data_ptr(),
             trap.data_ptr(), q_bias.data_ptr(), k_bias.data_ptr(), cos.data_ptr(),
             sin.data_ptr(), _ptr(d_skip), _ptr(z), _ptr(psi), _ptr(zeta), _ptr(phi)],
            1 if reverse else 0, backend, _ffi.THREADING["auto"],
            out_hm.data_ptr(), last_state.data_ptr(), _ptr(last_bx), stream=_stream(v))
    _CALLS["n"] += 1
    return out_hm.permute(0, 2, 1, 3).contiguous(), last_state


@_mamba3_scan_op.register_fake
def _(q, k, v, adt, dt, trap, q_bias, k_bias, cos, sin, d_skip, z, reverse,
      psi=None, zeta=None, phi=None, backend=0):
    b, length, _, dqk = q.shape
    h, dv = v.shape[2], v.shape[3]
    return v.new_empty((b, length, h, dv)), v.new_empty((b, h, dv, dqk))


@torch.library.custom_op("arm_scan::mamba3_scan_tc", mutates_args=())
def _mamba3_scan_tc_op(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    adt: torch.Tensor,
    dt: torch.Tensor,
    trap: torch.Tensor,
    q_bias: torch.Tensor,
    k_bias: torch.Tensor,
    angles: torch.Tensor,
    d_skip: Optional[torch.Tensor],
    z: Optional[torch.Tensor],
    reverse: bool,
) -> Tuple[torch.Tensor, torch.Tensor]:
    # q, k, v, z, angles share one dtype (fp32 or bf16); out has it too and
    # is written directly in (b, l, h, dv)
    b, length, _, dqk = q.shape
    h, dv = v.shape[2], v.shape[3]
    dims = _ffi.ArmMamba3Dims(b, h, dv, dqk, length, 1)
    bf16 = q.dtype == torch.bfloat16
    dtype = _ffi.DTYPE_BF16 if bf16 else _ffi.DTYPE_F32
    opts = _ffi.ArmMamba3TcOptions(dtype, dtype, 1, 1 if angles.shape[2] == 1 else 0,
                                   angles.shape[3])
    out = v.new_empty((b, length, h, dv))
    last_state = v.new_empty((b, h, dv, dqk), dtype=torch.float32)
    last_bx = v.new_empty((b, h, dqk), dtype=torch.float32)
    with _on_device(v):
        _ffi.mamba3_tc_raw(
            dims, opts,
            [q.data_ptr(), k.data_ptr(), v.data_ptr(), adt.data_ptr(), dt.data_ptr(),
             trap.data_ptr(), q_bias.data_ptr(), k_bias.data_ptr(), angles.data_ptr(),
             _ptr(d_skip), _ptr(z)],
            1 if reverse else 0, out.data_ptr(), last_state.data_ptr(), last_bx.data_ptr(),
            _stream(v))
    _CALLS["n"] += 1
    return out, last_state


@_mamba3_scan_tc_op.register_fake
def _(q, k, v, adt, dt, trap, q_bias, k_bias, angles, d_skip, z, reverse):
    b, length, _, dqk = q.shape
    h, dv = v.shape[2], v.shape[3]
    return v.new_empty((b, length, h, dv)), v.new_empty((b, h, dv, dqk), dtype=torch.float32)


def _mamba3_tc_angles(q, k, v, adt, dt, trap, q_bias, k_bias, angles, D, z, reverse):
    """precision="bf16" with raw angles: one tensor-core call with the angle
    pre-pass fused in.  q, k, v, z, angles run in bf16 when q is bf16 (else
    fp32); the output has that dtype."""
    b, length, _, dqk = q.shape
    h = v.shape[2]
    if angles.dim() != 4 or angles.shape[:2] != (b, length) or angles.shape[2] not in (1, h):
        raise ValueError(f"angles must be (b, l, h, r) or (b, l, 1, r), got {tuple(angles.shape)}")
    if angles.shape[3] > dqk // 2:
        raise ValueError(f"angles has {angles.shape[3]} pairs, more than dqk/2 = {dqk // 2}")
    if angles.shape[2] > 1 and angles.stride(2) == 0:
        # a head-broadcast view (angles.expand over heads): pass the one row
        # per (b, l) instead of materialising a copy per head
        angles = angles[:, :, :1, :]
    home = v.device
    dev = home if home.type == "cuda" else torch.device("cuda", torch.cuda.current_device())
    io = torch.bfloat16 if q.dtype == torch.bfloat16 else torch.float32
    big = lambda t: t.to(device=dev, dtype=io).contiguous()  # noqa: E731
    f32 = lambda t: None if t is None else t.to(device=dev, dtype=torch.float32).contiguous()  # noqa: E731
    out, last = _mamba3_scan_tc_op(
        big(q), big(k), big(v), f32(adt), f32(dt), f32(trap), f32(q_bias), f32(k_bias),
        big(angles), f32(D), None if z is None else big(z), bool(reverse))
    if home.type != "cuda":
        out, last = out.to(home), last.to(home)
    return out, last


def _check_shapes(q, k, v, adt, dt, trap, q_bias, k_bias, cos, sin, D, z):
    """Every tensor against the SISO layout contract.  The C entry point is
    told how many elements to read, so a short buffer would be an
    out-of-bounds read rather than an error: shapes are owned here."""
    b, length, groups, dqk = q.shape
    if groups != 1:
        raise ValueError(f"SISO expects one B/C group, got {groups}")
    if dqk % 2:
        raise ValueError(f"dqk must be even (RoPE lane pairs), got {dqk}")
    if v.dim() != 4:
        raise ValueError(f"v must be (b, l, h, dv), got {tuple(v.shape)}")
    h, dv = v.shape[2], v.shape[3]
    half = dqk // 2
    want = {
        "q": (b, length, 1, dqk), "k": (b, length, 1, dqk), "v": (b, length, h, dv),
        "adt": (b, h, length), "dt": (b, h, length), "trap": (b, h, length),
        "q_bias": (h, dqk), "k_bias": (h, dqk),
        "cos": (b, length, h, half), "sin": (b, length, h, half),
    }
    got = dict(q=q, k=k, v=v, adt=adt, dt=dt, trap=trap, q_bias=q_bias, k_bias=k_bias,
               cos=cos, sin=sin)
    if D is not None:
        want["D"], got["D"] = (h,), D
    if z is not None:
        want["z"], got["z"] = (b, length, h, dv), z
    for name, shape in want.items():
        actual = tuple(got[name].shape)
        if actual != shape:
            raise ValueError(f"{name} must be {shape}, got {actual}")


_PRECISION = {"fp32": 0, "bf16": 3}


def mamba3_scan(q, k, v, adt, dt, trap, q_bias, k_bias, angles=None,
                D=None, z=None, reverse=False, cos=None, sin=None,
                return_last_state=False, precision="fp32"):
    """Mamba-3 SISO selective scan.

    q, k : (b, l, 1, dqk) or (b, l, dqk);  v, z : (b, l, h, dv)
    adt, dt : (b, h, l) (adt = A*dt <= 0, dt post-softplus);  trap : (b, h, l)
    angles : (b, l, h, r) raw (the pre-pass runs here), or pass cos/sin
    q_bias, k_bias : (h, dqk);  D : (h,)
    returns (b, l, h, dv) [, last_state (b, h, dv, dqk)]

    precision "fp32" (default): fp32 arithmetic throughout.  "bf16": the
    tensor-core kernel -- q/k/v/W operands rounded to bf16, fp32
    accumulation and fp32 state (for bf16 models; covers dqk 128, dv 64).
    With raw ``angles`` it also fuses the angle pre-pass, accepts bf16 (or
    fp32) q/k/v/z/angles, returns the output in that dtype, and takes angles
    (b, l, 1, r) shared by all heads.
    """
    if precision not in _PRECISION:
        raise ValueError(f"precision must be one of {sorted(_PRECISION)}, got {precision!r}")
    if q.dim() == 3:
        q = q.unsqueeze(2)
    if k.dim() == 3:
        k = k.unsqueeze(2)
    if (cos is None) != (sin is None):
        raise ValueError("pass cos and sin together, or neither")
    half = q.shape[-1] // 2
    if precision == "bf16" and cos is None and angles is not None:
        if q.shape[2] != 1:
            raise ValueError(f"SISO expects one B/C group, got {q.shape[2]}")
        out, last = _mamba3_tc_angles(q, k, v, adt, dt, trap, q_bias, k_bias, angles, D, z,
                                      reverse)
        return (out, last) if return_last_state else out
    if cos is None:
        if angles is None:
            raise ValueError("pass either `angles` or both `cos` and `sin`")
        cos, sin = angles_to_cos_sin(angles, dt, half)
    _check_shapes(q, k, v, adt, dt, trap, q_bias, k_bias, cos, sin, D, z)
    dev = v.device
    opt = lambda t: None if t is None else _prep(t, dev)  # noqa: E731
    out, last = _mamba3_scan_op(
        _prep(q, dev), _prep(k, dev), _prep(v, dev), _prep(adt, dev), _prep(dt, dev),
        _prep(trap, dev), _prep(q_bias, dev), _prep(k_bias, dev), _prep(cos, dev),
        _prep(sin, dev), opt(D), opt(z), bool(reverse), backend=_PRECISION[precision])
    return (out, last) if return_last_state else out


def mamba3_scan_pair(q, k, v, adt, dt, trap, q_bias, k_bias, angles=None,
                     D=None, z=None, cos=None, sin=None):
    """Both traversal directions of the same inputs -> (fwd, bwd).

    The angle pre-pass runs once and is shared: a reverse traversal walks the
    same tokens backward, each keeping its own position's rotation.
    """
    if cos is None:
        if angles is None:
            raise ValueError("pass either `angles` or both `cos` and `sin`")
        cos, sin = angles_to_cos_sin(angles, dt, q.shape[-1] // 2)
    common = dict(q_bias=q_bias, k_bias=k_bias, D=D, z=z, cos=cos, sin=sin)
    fwd = mamba3_scan(q, k, v, adt, dt, trap, reverse=False, **common)
    bwd = mamba3_scan(q, k, v, adt, dt, trap, reverse=True, **common)
    return fwd, bwd


def mamba3_mimo_scan(q, k, v, adt, dt, trap, q_bias, k_bias, psi, zeta, phi,
                     angles=None, D=None, z=None, reverse=False, cos=None, sin=None,
                     return_last_state=False, precision="fp32"):
    """Mamba-3 MIMO (rank-r) selective scan.

    q, k : (b, l, r, 1, dqk) or (b, l, r, dqk);  v, z : (b, l, h, dv)
    adt, dt, trap : (b, h, l);  q_bias, k_bias : (h, r, dqk)
    psi, zeta, phi : (h, r, dv) input / gate / output projections
    angles : (b, l, h, a) raw;  D : (h,)
    returns (b, l, h, dv) [, last_state (b, h, dv, dqk)]

    Not a SISO call at r = 1: MIMO rotates split halves (i, i + dqk/2).

    precision "bf16": the tensor-core kernel (ranks 2 and 4, dqk 128, dv 64):
    q/k/x/W operands rounded to bf16, fp32 accumulation and fp32 state.
    """
    if precision not in _PRECISION:
        raise ValueError(f"precision must be one of {sorted(_PRECISION)}, got {precision!r}")
    if q.dim() == 5:
        if q.shape[3] != 1:
            raise ValueError(f"MIMO expects one B/C group, got {q.shape[3]}")
        q = q[:, :, :, 0, :]
    if k.dim() == 5:
        k = k[:, :, :, 0, :]
    if q.dim() != 4 or k.dim() != 4:
        raise ValueError(f"q/k must be (b, l, r, dqk) after squeezing the group axis; got "
                         f"{tuple(q.shape)} and {tuple(k.shape)}")
    rank, dqk = q.shape[2], q.shape[3]
    h, dv = v.shape[2], v.shape[3]
    if (cos is None) != (sin is None):
        raise ValueError("pass cos and sin together, or neither")
    if cos is None:
        if angles is None:
            raise ValueError("pass either `angles` or both `cos` and `sin`")
        cos, sin = angles_to_cos_sin(angles, dt, dqk // 2)
    for name, t, want in (
        ("q", q, (q.shape[0], q.shape[1], rank, dqk)),
        ("k", k, (q.shape[0], q.shape[1], rank, dqk)),
        ("q_bias", q_bias, (h, rank, dqk)),
        ("k_bias", k_bias, (h, rank, dqk)),
        ("psi", psi, (h, rank, dv)),
        ("zeta", zeta, (h, rank, dv)),
        ("phi", phi, (h, rank, dv)),
    ):
        if tuple(t.shape) != want:
            raise ValueError(f"{name} must be {want}, got {tuple(t.shape)}")
    if z is not None and tuple(z.shape) != tuple(v.shape):
        raise ValueError(f"z must match v {tuple(v.shape)}, got {tuple(z.shape)}")
    b, length = q.shape[0], q.shape[1]
    half = dqk // 2
    for name, t, want in (("adt", adt, (b, h, length)), ("dt", dt, (b, h, length)),
                          ("trap", trap, (b, h, length)), ("cos", cos, (b, length, h, half)),
                          ("sin", sin, (b, length, h, half))):
        if tuple(t.shape) != want:
            raise ValueError(f"{name} must be {want}, got {tuple(t.shape)}")
    if D is not None and tuple(D.shape) != (h,):
        raise ValueError(f"D must be ({h},), got {tuple(D.shape)}")
    dev = v.device
    opt = lambda t: None if t is None else _prep(t, dev)  # noqa: E731
    out, last = _mamba3_scan_op(
        _prep(q, dev), _prep(k, dev), _prep(v, dev), _prep(adt, dev), _prep(dt, dev),
        _prep(trap, dev), _prep(q_bias, dev), _prep(k_bias, dev), _prep(cos, dev),
        _prep(sin, dev), opt(D), opt(z), bool(reverse), _prep(psi, dev), _prep(zeta, dev),
        _prep(phi, dev), backend=_PRECISION[precision])
    return (out, last) if return_last_state else out


def mamba3_mimo_x_scan(x, B, C, adt, dt, trap, angles=None, D=None, reverse=False,
                       return_last_state=False, out_dtype=None):
    """Mamba-3 MIMO with the input given per rank (tensor cores, bf16 operands,
    fp32 state).  Per (batch, head), h (dv x dqk):

        h_t = a_t h_{t-1} + b_t X_{t-1} B_{t-1}^T + g_t X_t B_t^T,   Y_t = h_t C_t (+ D X_t)

    with a = exp(adt), g = dt * sigmoid(trap), b = a * dt * (1 - sigmoid(trap))
    (the gates of ``mamba3_scan``) and B, C RoPE-rotated split-halves by
    theta = cumsum(tanh(angles) * pi * dt).  This is ``mamba3_mimo_scan`` with
    x_r given directly instead of psi_r * v, and per-rank outputs instead of
    the zeta-gated, phi-weighted sum (reference python/arm_scan/mamba3.py:261-334).

    x : (b, l, h, dv, r) fp32 or bf16;  B, C : (b, l, dqk, r), same dtype
    adt, dt, trap : (b, h, l);  angles : (b, l, a) shared by the heads or
    (b, l, h, a), a <= dqk/2 (None: no rotation);  D : (h,) or None
    returns Y (b, l, h, dv, r) in ``out_dtype`` (default x's dtype)
    [, last_state (b, h, dv, dqk) fp32].  rank 2 or 4, dqk 128, dv 64.
    """
    if x.dim() != 5 or B.dim() != 4 or C.dim() != 4:
        raise ValueError("x must be (b, l, h, dv, r) and B, C (b, l, dqk, r)")
    b, length, h, dv, rank = x.shape
    dqk = B.shape[2]
    if tuple(B.shape) != (b, length, dqk, rank) or tuple(C.shape) != tuple(B.shape):
        raise ValueError(f"B and C must be {(b, length, dqk, rank)}, got {tuple(B.shape)} and "
                         f"{tuple(C.shape)}")
    if x.dtype not in (torch.float32, torch.bfloat16) or B.dtype != x.dtype or C.dtype != x.dtype:
        raise ValueError("x, B, C must share one dtype, float32 or bfloat16")
    for name, t in (("adt", adt), ("dt", dt), ("trap", trap)):
        if tuple(t.shape) != (b, h, length):
            raise ValueError(f"{name} must be {(b, h, length)}, got {tuple(t.shape)}")
    shared, n_angles = 1, 0
    if angles is not None:
        if angles.dim() == 3 and tuple(angles.shape[:2]) == (b, length):
            shared = 1
        elif angles.dim() == 4 and tuple(angles.shape[:3]) == (b, length, h):
            shared = 0
        else:
            raise ValueError(f"angles must be (b, l, a) or (b, l, h, a), got {tuple(angles.shape)}")
        n_angles = angles.shape[-1]
        if n_angles > dqk // 2:
            raise ValueError(f"angles has {n_angles} pairs, head dim allows {dqk // 2}")
    if D is not None and tuple(D.shape) != (h,):
        raise ValueError(f"D must be ({h},), got {tuple(D.shape)}")
    if x.device.type != "cuda":
        raise ValueError("mamba3_mimo_x_scan runs on CUDA tensors only")
    out_dtype = x.dtype if out_dtype is None else out_dtype
    if out_dtype not in (torch.float32, torch.bfloat16):
        raise ValueError("out_dtype must be float32 or bfloat16")
    f32 = lambda t: t.to(torch.float32).contiguous()  # noqa: E731
    xs, Bs, Cs = x.contiguous(), B.contiguous(), C.contiguous()
    adt_, dt_, trap_ = f32(adt), f32(dt), f32(trap)
    ang = f32(angles) if angles is not None else None
    Ds = f32(D) if D is not None else None
    out = torch.empty(b, length, h, dv, rank, dtype=out_dtype, device=x.device)
    last = torch.empty(b, h, dv, dqk, dtype=torch.float32, device=x.device) \
        if return_last_state else None
    dims = _ffi.ArmMamba3Dims(b, h, dv, dqk, length, rank)
    opts = _ffi.ArmMamba3TcOptions(
        _ffi.DTYPE_BF16 if x.dtype == torch.bfloat16 else _ffi.DTYPE_F32,
        _ffi.DTYPE_BF16 if out_dtype == torch.bfloat16 else _ffi.DTYPE_F32, 0, shared, n_angles)
    ptrs = [xs.data_ptr(), Bs.data_ptr(), Cs.data_ptr(), adt_.data_ptr(), dt_.data_ptr(),
            trap_.data_ptr(), ang.data_ptr() if ang is not None else 0,
            Ds.data_ptr() if Ds is not None else 0]
    with torch.cuda.device(x.device):
        _ffi.mamba3_mimo_x_raw(dims, opts, ptrs, bool(reverse), out.data_ptr(),
                               last.data_ptr() if last is not None else 0,
                               torch.cuda.current_stream(x.device).cuda_stream)
    return (out, last) if return_last_state else out
