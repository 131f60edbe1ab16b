"""TEST INFRASTRUCTURE ONLY -- numpy front-end of the CPU oracle.

Wraps liboracle.so (scan_oracle.cc, a C++ restatement of the reference's
scalar recurrences) and restates in numpy the Mamba-3 RoPE angle pre-pass of
the reference's Python layer (``angles_to_cos_sin``,
python/arm_scan/mamba3.py:41-89: theta = cumsum(tanh(angle) * pi * dt), padded
to dqk/2 pairs with cos=1, sin=0).

Only tests/, __graft_entry__.smoke() and the CPU-baseline leg of bench.py may
import this module.  The armhackathon_b200 package never does.
"""

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle.so"


class M1Dims(ctypes.Structure):
    _fields_ = [(n, ctypes.c_size_t) for n in ("batch", "dim", "len", "state", "groups")]


class M3Dims(ctypes.Structure):
    _fields_ = [(n, ctypes.c_size_t) for n in ("batch", "heads", "dv", "dqk", "len", "rank")]


_lib = None


def build():
    """Compile liboracle.so with the committed Makefile (g++ only)."""
    subprocess.run(["make", "-s", "-C", str(HERE), "liboracle.so"], check=True)


def lib():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        _lib = ctypes.CDLL(str(LIB_PATH))
    return _lib


def hw_threads():
    return int(lib().oracle_hw_threads()) or (os.cpu_count() or 1)


def _arr(x, dt):
    return None if x is None else np.ascontiguousarray(x, dtype=dt)


def _p(x):
    return None if x is None else x.ctypes.data_as(ctypes.c_void_p)


def _call(name, *args):
    rc = getattr(lib(), name)(*args)
    if rc != 0:
        raise ValueError(f"{name} rejected its arguments (code {rc})")


def m1_scan(u, delta, A, B, C, D=None, z=None, delta_bias=None,
            delta_softplus=False, reverse=False, h0=None, dtype=np.float64,
            nthreads=1):
    """Mamba-1 scan (kernel/arm-scan-core/src/scalar.rs:11-89).

    B, C may be (batch, state, len) or (batch, groups, state, len).
    Returns (out, last_state) in ``dtype``.
    """
    dt = np.dtype(dtype)
    suffix = "f64" if dt == np.float64 else "f32"
    u, delta, A = _arr(u, dt), _arr(delta, dt), _arr(A, dt)
    batch, dim, length = u.shape
    state = A.shape[1]
    B, C = _arr(B, dt), _arr(C, dt)
    groups = B.shape[1] if B.ndim == 4 else 1
    D, z, delta_bias, h0 = (_arr(x, dt) for x in (D, z, delta_bias, h0))
    out = np.empty((batch, dim, length), dt)
    last = np.empty((batch, dim, state), dt)
    dims = M1Dims(batch, dim, length, state, groups)
    _call(f"oracle_m1_scan_{suffix}", ctypes.byref(dims), _p(u), _p(delta), _p(A),
          _p(B), _p(C), _p(D), _p(z), _p(delta_bias), ctypes.c_int(bool(delta_softplus)),
          ctypes.c_int(bool(reverse)), _p(out), _p(last), _p(h0), ctypes.c_int(nthreads))
    return out, last


def m1_scan_bidir(u, delta, A, B, C, D=None, z=None, delta_bias=None,
                  delta_softplus=False, dtype=np.float64, nthreads=1):
    """Fused bidirectional Mamba-1 scan (scalar.rs:114-201).

    Returns (out_fwd, out_bwd, last_fwd, last_bwd).
    """
    dt = np.dtype(dtype)
    suffix = "f64" if dt == np.float64 else "f32"
    u, delta, A = _arr(u, dt), _arr(delta, dt), _arr(A, dt)
    batch, dim, length = u.shape
    state = A.shape[1]
    B, C = _arr(B, dt), _arr(C, dt)
    groups = B.shape[1] if B.ndim == 4 else 1
    D, z, delta_bias = (_arr(x, dt) for x in (D, z, delta_bias))
    of = np.empty((batch, dim, length), dt)
    ob = np.empty((batch, dim, length), dt)
    lf = np.empty((batch, dim, state), dt)
    lb = np.empty((batch, dim, state), dt)
    dims = M1Dims(batch, dim, length, state, groups)
    _call(f"oracle_m1_scan_bidir_{suffix}", ctypes.byref(dims), _p(u), _p(delta), _p(A),
          _p(B), _p(C), _p(D), _p(z), _p(delta_bias), ctypes.c_int(bool(delta_softplus)),
          _p(of), _p(ob), _p(lf), _p(lb), ctypes.c_int(nthreads))
    return of, ob, lf, lb


def angles_to_cos_sin(angles, dt, half):
    """RoPE pre-pass, python/arm_scan/mamba3.py:41-89, in float64.

    angles (b, l, h, r), dt (b, h, l) -> cos, sin (b, l, h, half).
    """
    angles = np.asarray(angles, np.float64)
    r = angles.shape[-1]
    if r > half:
        raise ValueError(f"angles has {r} pairs, head dim allows {half}")
    dt_blh = np.transpose(np.asarray(dt, np.float64), (0, 2, 1))[..., None]
    theta = np.cumsum(np.tanh(angles) * np.pi * dt_blh, axis=1)
    cos, sin = np.cos(theta), np.sin(theta)
    if r < half:
        pad = theta.shape[:-1] + (half - r,)
        cos = np.concatenate([cos, np.ones(pad)], -1)
        sin = np.concatenate([sin, np.zeros(pad)], -1)
    return cos, sin


def m3_mixer_prologue(proj, heads, headdim, d_state, rank, n_angles, dt_bias, B_norm_weight,
                      C_norm_weight, A_floor, eps):
    """Mamba-3 mixer prologue, apps/mamba3_lm/block.py:146-177, in float64.

    proj (b, l, W), one B/C group, split as block.py:116-121 / 150-151;
    heavy_tail (52-62), clamp (165), softplus (166, threshold 20), ADT (167),
    (b, l, h) -> (b, h, l) transposes (158, 168-169), RMSNorm (78-82; eps
    inside the sqrt) of B (-> k) and C (-> q).  Returns a dict of z, x
    (b, l, h, p), q, k (b, l, r, n), dt, adt, trap (b, h, l), angles (b, l, a).
    """
    proj = np.asarray(proj, np.float64)
    b, l, _ = proj.shape
    hp, rn = heads * headdim, rank * d_state
    cuts = np.cumsum([hp, hp, rn, rn, heads, heads, heads])
    z, x, B, C, dd_dt, dd_A, trap, ang = np.split(proj, cuts, axis=-1)
    neg, pos = np.minimum(dd_A, 0.0), np.maximum(dd_A, 0.0)
    A = np.minimum(-(pos + 1.0 / (1.0 - neg)), -float(A_floor))
    v = dd_dt + np.asarray(dt_bias, np.float64)
    dt = np.where(v > 20.0, v, np.log1p(np.exp(np.minimum(v, 20.0))))
    adt = A * dt

    def rms(t, w):
        t = t.reshape(b, l, rank, d_state)
        rstd = 1.0 / np.sqrt(np.mean(t * t, axis=-1, keepdims=True) + float(eps))
        return t * rstd * np.asarray(w, np.float64)

    tr = lambda t: np.ascontiguousarray(np.transpose(t, (0, 2, 1)))  # noqa: E731
    return dict(z=z.reshape(b, l, heads, headdim), x=x.reshape(b, l, heads, headdim),
                q=rms(C, C_norm_weight), k=rms(B, B_norm_weight), dt=tr(dt), adt=tr(adt),
                trap=tr(trap), angles=ang)


def m3_siso(q, k, v, adt, dt, trap, q_bias, k_bias, cos, sin, D=None, z=None,
            reverse=False, dtype=np.float64, nthreads=1, want_state=False):
    """Mamba-3 SISO scan (kernel/arm-scan-core/src/mamba3/scalar.rs:50-196).

    q, k (b, l, 1, dqk) or (b, l, dqk); returns out TIME-major (b, l, h, dv)
    (the reference op permutes its head-major kernel output the same way,
    python/arm_scan/mamba3.py:142), plus (last_state (b,h,dv,dqk), last_bx)
    when ``want_state``.
    """
    d_t = np.dtype(dtype)
    suffix = "f64" if d_t == np.float64 else "f32"
    q, k = _arr(q, d_t), _arr(k, d_t)
    if q.ndim == 3:
        q, k = q[:, :, None, :], k[:, :, None, :]
    v = _arr(v, d_t)
    b, length, heads, dv = v.shape
    dqk = q.shape[-1]
    args = [_arr(x, d_t) for x in (adt, dt, trap, q_bias, k_bias, cos, sin)]
    D, z = _arr(D, d_t), _arr(z, d_t)
    out = np.empty((b, heads, length, dv), d_t)
    ls = np.empty((b, heads, dv, dqk), d_t)
    lb = np.empty((b, heads, dqk), d_t)
    dims = M3Dims(b, heads, dv, dqk, length, 1)
    _call(f"oracle_m3_siso_{suffix}", ctypes.byref(dims), _p(q), _p(k), _p(v),
          *[_p(x) for x in args], _p(D), _p(z), ctypes.c_int(bool(reverse)),
          _p(out), _p(ls), _p(lb), ctypes.c_int(nthreads))
    out = np.ascontiguousarray(out.transpose(0, 2, 1, 3))
    return (out, ls, lb) if want_state else out


def m3_mimo(q, k, v, adt, dt, trap, q_bias, k_bias, cos, sin, psi, zeta, phi,
            D=None, z=None, reverse=False, dtype=np.float64, nthreads=1,
            want_state=False):
    """Mamba-3 MIMO scan (kernel/arm-scan-core/src/mamba3/mimo.rs:98-284).

    q, k (b, l, r, dqk) or (b, l, r, 1, dqk); returns out time-major
    (b, l, h, dv) (and last_state (b, h, dv, dqk) when ``want_state``).
    """
    d_t = np.dtype(dtype)
    suffix = "f64" if d_t == np.float64 else "f32"
    q, k = _arr(q, d_t), _arr(k, d_t)
    if q.ndim == 5:
        q, k = q[:, :, :, 0, :], k[:, :, :, 0, :]
    rank, dqk = q.shape[2], q.shape[3]
    v = _arr(v, d_t)
    b, length, heads, dv = v.shape
    args = [_arr(x, d_t) for x in (adt, dt, trap, q_bias, k_bias, cos, sin)]
    D, z = _arr(D, d_t), _arr(z, d_t)
    psi, zeta, phi = (_arr(x, d_t) for x in (psi, zeta, phi))
    out = np.empty((b, heads, length, dv), d_t)
    ls = np.empty((b, heads, dv, dqk), d_t)
    dims = M3Dims(b, heads, dv, dqk, length, rank)
    _call(f"oracle_m3_mimo_{suffix}", ctypes.byref(dims), _p(q), _p(k), _p(v),
          *[_p(x) for x in args], _p(D), _p(z), _p(psi), _p(zeta), _p(phi),
          ctypes.c_size_t(cos.shape[-1]), ctypes.c_int(bool(reverse)), _p(out),
          _p(ls), ctypes.c_int(nthreads))
    out = np.ascontiguousarray(out.transpose(0, 2, 1, 3))
    return (out, ls) if want_state else out


def m3_mimo_x(x, b, c, adt, dt, trap, cos, sin, D=None, reverse=False, dtype=np.float64,
              nthreads=1, want_state=False):
    """Mamba-3 MIMO with X given per rank (the h_t / Y_t = h_t C_t form):
    x (b, l, h, dv, r), b/c (b, l, dqk, r) -> out (b, l, h, dv, r) (and
    last_state (b, h, dv, dqk) when ``want_state``).  See
    oracle_m3_mimo_x in scan_oracle_body.h."""
    d_t = np.dtype(dtype)
    suffix = "f64" if d_t == np.float64 else "f32"
    x, b, c = _arr(x, d_t), _arr(b, d_t), _arr(c, d_t)
    bsz, length, heads, dv, rank = x.shape
    dqk = b.shape[2]
    args = [_arr(t, d_t) for t in (adt, dt, trap, cos, sin)]
    D = _arr(D, d_t)
    out = np.empty_like(x)
    ls = np.empty((bsz, heads, dv, dqk), d_t)
    dims = M3Dims(bsz, heads, dv, dqk, length, rank)
    _call(f"oracle_m3_mimo_x_{suffix}", ctypes.byref(dims), _p(x), _p(b), _p(c),
          *[_p(t) for t in args], ctypes.c_size_t(cos.shape[-1]), _p(D),
          ctypes.c_int(bool(reverse)), _p(out), _p(ls), ctypes.c_int(nthreads))
    return (out, ls) if want_state else out


def bf16_round(x):
    """Round-to-nearest-even to bfloat16, returned as float32."""
    x = np.ascontiguousarray(x, np.float32)
    bits = x.view(np.uint32).astype(np.uint64)
    bias = ((bits >> 16) & 1) + 0x7FFF
    return ((bits + bias) >> 16 << 16).astype(np.uint32).view(np.float32)


def bf16_ulps_at_scale(got, golden):
    """Worst |got - golden| in bf16 ULPs at the golden tensor's scale.

    Restates tests/verify_golden_mamba3.py:50-82 of the reference: one ULP is
    max|golden| * 2^-8, and ``got`` is rounded to bf16 first (like-for-like
    with a bf16-stored capture).
    """
    golden = np.asarray(golden, np.float64)
    ulp = max(float(np.abs(golden).max()), 1e-30) * 2.0 ** -8
    diff = np.abs(bf16_round(got).astype(np.float64) - golden)
    return float(diff.max() / ulp)
