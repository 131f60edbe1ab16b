"""Mamba-3 parity on the GPU: CUDA kernels through the C ABI against the
official-kernel captures (<= 8 / 12 bf16 ULPs at tensor scale, the reference's
gates in tests/verify_golden_mamba3.py and verify_golden_mamba3_mimo.py), the
reference's f64 oracle outputs stored in the fixtures (fp32 inputs: relative
error <= 1e-4), and the CPU oracle for reverse traversal, final states, pairs,
non-causal and 2D compositions."""

import json

import numpy as np
import pytest
import torch

import oracle
from conftest import GOLDEN

pytestmark = pytest.mark.gpu

IDX = json.loads((GOLDEN / "index.json").read_text())
REL_TOL = 1e-4


def arm():
    import armhackathon_b200 as a
    return a


def rel_err(got, want):
    want = np.asarray(want, np.float64)
    return float(np.abs(np.asarray(got, np.float64) - want).max()
                 / max(np.abs(want).max(), 1e-30))


def load(family, name):
    d = np.load(GOLDEN / family / f"{name}.npz")
    kw = {k[3:]: torch.from_numpy(d[k]).cuda() for k in d.files if k.startswith("kw_")}
    return kw, d


def siso(kw, reverse=False, state=False):
    return arm().mamba3_scan(kw["Q"], kw["K"], kw["V"], kw["ADT"], kw["DT"], kw["Trap"],
                             kw["Q_bias"], kw["K_bias"], angles=kw["Angles"], D=kw["D"],
                             z=kw["Z"], reverse=reverse, return_last_state=state)


@pytest.mark.parametrize("name", IDX["m3_siso"])
def test_siso_golden(name):
    kw, d = load("m3_siso", name)
    out, st = siso(kw, state=True)
    rev, rst = siso(kw, reverse=True, state=True)
    out, rev = out.cpu().numpy(), rev.cpu().numpy()
    assert oracle.bf16_ulps_at_scale(out, d["out"]) <= 8.0
    assert rel_err(out, d["ref_f64"]) <= REL_TOL
    assert rel_err(rev, d["ref_rev_f64"]) <= REL_TOL
    if "ref_state_f64" in d.files:
        assert rel_err(st.cpu().numpy(), d["ref_state_f64"]) <= REL_TOL
        assert rel_err(rst.cpu().numpy(), d["ref_rev_state_f64"]) <= REL_TOL


@pytest.mark.parametrize("name", IDX["m3_mimo"])
def test_mimo_golden(name):
    kw, d = load("m3_mimo", name)
    out = arm().mamba3_mimo_scan(kw["Q"], kw["K"], kw["V"], kw["ADT"], kw["DT"], kw["Trap"],
                                 kw["Q_bias"], kw["K_bias"], kw["MIMO_V"], kw["MIMO_Z"],
                                 kw["MIMO_Out"], angles=kw["Angles"], D=kw["D"], z=kw["Z"])
    out = out.cpu().numpy()
    assert oracle.bf16_ulps_at_scale(out, d["out"]) <= 12.0
    assert rel_err(out, d["ref_f64"]) <= REL_TOL


def random_siso(b, l, h, dv, dqk, r, seed=0):
    g = torch.Generator().manual_seed(seed)
    f = lambda *s: torch.randn(*s, generator=g)  # noqa: E731
    dt = torch.nn.functional.softplus(f(b, h, l) - 4)
    A = -torch.exp(torch.rand(h, generator=g) * np.log(16))
    return dict(q=f(b, l, 1, dqk) / dqk ** 0.5, k=f(b, l, 1, dqk) / dqk ** 0.5, v=f(b, l, h, dv),
                adt=A.view(1, h, 1) * dt, dt=dt, trap=f(b, h, l), q_bias=0.1 * f(h, dqk),
                k_bias=0.1 * f(h, dqk), angles=f(b, l, h, r), D=1 + 0.1 * f(h), z=f(b, l, h, dv))


@pytest.mark.parametrize("shape", [(2, 300, 3, 64, 128, 64), (1, 1, 2, 32, 64, 16),
                                   (3, 129, 5, 48, 32, 8), (1, 257, 4, 64, 64, 32)])
@pytest.mark.parametrize("reverse", [False, True])
def test_siso_random_vs_oracle(shape, reverse):
    b, l, h, dv, dqk, r = shape
    x = random_siso(b, l, h, dv, dqk, r, seed=l)
    cos, sin = oracle.angles_to_cos_sin(x["angles"].numpy(), x["dt"].numpy(), dqk // 2)
    want, wst, wbx = oracle.m3_siso(x["q"], x["k"], x["v"], x["adt"], x["dt"], x["trap"],
                                    x["q_bias"], x["k_bias"], cos, sin, D=x["D"], z=x["z"],
                                    reverse=reverse, want_state=True, nthreads=8)
    xc = {k: v.cuda() for k, v in x.items()}
    out, st = arm().mamba3_scan(**xc, reverse=reverse, return_last_state=True)
    assert rel_err(out.cpu().numpy(), want) <= REL_TOL
    assert rel_err(st.cpu().numpy(), wst) <= REL_TOL


def test_pair_and_noncausal():
    x = {k: v.cuda() for k, v in random_siso(2, 96, 3, 32, 64, 32, seed=11).items()}
    a = arm()
    fwd, bwd = a.mamba3_scan_pair(**x)
    assert torch.allclose(fwd, a.mamba3_scan(**x), atol=0, rtol=0)
    assert torch.allclose(bwd, a.mamba3_scan(**x, reverse=True), atol=0, rtol=0)
    nc = a.noncausal_scan(**x)
    dense = a.noncausal_scan_dense(**{k: v.double() for k, v in x.items()})
    assert rel_err(nc.cpu().numpy(), dense.cpu().numpy()) <= REL_TOL
    causal = a.noncausal_scan_dense(**{k: v.double() for k, v in x.items()}, causal=True)
    assert rel_err(fwd.cpu().numpy(), causal.cpu().numpy()) <= REL_TOL


def test_ss2d_mamba3_directions_vs_oracle():
    g = torch.Generator().manual_seed(4)
    b, H, W, h, dv, dqk, r = 2, 6, 9, 2, 32, 64, 16
    f = lambda *s: torch.randn(*s, generator=g)  # noqa: E731
    dt = torch.nn.functional.softplus(f(b, h, H, W) - 4)
    x = dict(q=f(b, H, W, 1, dqk) / 8, k=f(b, H, W, 1, dqk) / 8, v=f(b, H, W, h, dv),
             adt=-dt * 2.0, dt=dt, trap=f(b, h, H, W), q_bias=0.1 * f(h, dqk),
             k_bias=0.1 * f(h, dqk), angles=f(b, H, W, h, r), D=torch.ones(h), z=f(b, H, W, h, dv))
    a = arm()
    planes = a.ss2d_scan_mamba3(**{k: v.cuda() for k, v in x.items()}, merge="none")
    from armhackathon_b200.ss2d import grid_to_views
    from armhackathon_b200.ss2d_mamba3 import grid_to_views_time_major, views_to_grid_time_major
    tv = {k: grid_to_views_time_major(x[k]) for k in ("q", "k", "v", "angles", "z")}
    hv = {k: grid_to_views(x[k]) for k in ("adt", "dt", "trap")}
    cos, sin = oracle.angles_to_cos_sin(tv["angles"].numpy(), hv["dt"].numpy(), dqk // 2)
    outs = [oracle.m3_siso(tv["q"], tv["k"], tv["v"], hv["adt"], hv["dt"], hv["trap"],
                           x["q_bias"], x["k_bias"], cos, sin, D=x["D"], z=tv["z"], reverse=rv)
            for rv in (False, True)]
    rf, cf = views_to_grid_time_major(torch.from_numpy(outs[0][:b]), torch.from_numpy(outs[0][b:]), H, W)
    rb, cb = views_to_grid_time_major(torch.from_numpy(outs[1][:b]), torch.from_numpy(outs[1][b:]), H, W)
    for got, want in zip(planes, (rf, rb, cf, cb)):
        assert rel_err(got.cpu().numpy(), want.numpy()) <= REL_TOL
    nc_rows, nc_cols = a.ss2d_noncausal_mamba3(**{k: v.cuda() for k, v in x.items()}, merge="none")
    assert nc_rows.shape == (b, H, W, h, dv) and nc_cols.shape == (b, H, W, h, dv)
    # the one-call grid form (both orderings summed in place, diagonal
    # subtracted per ordering) against the per-ordering calls
    nc_sum = a.ss2d_noncausal_mamba3(**{k: v.cuda() for k, v in x.items()}, merge="sum")
    assert rel_err(nc_sum.cpu().numpy(), (nc_rows + nc_cols).cpu().numpy()) <= REL_TOL
    # and the row ordering against the dense mask on the row-major sequence
    rv = {k: grid_to_views_time_major(x[k])[:b] for k in ("q", "k", "v", "angles", "z")}
    rv.update({k: grid_to_views(x[k])[:b] for k in ("adt", "dt", "trap")})
    dense = a.noncausal_scan_dense(**{k: v.double() for k, v in rv.items()}, q_bias=x["q_bias"].double(),
                                   k_bias=x["k_bias"].double(), D=x["D"].double())
    assert rel_err(nc_rows.reshape(dense.shape).cpu().numpy(), dense.numpy()) <= REL_TOL


def test_noncausal_with_cos_sin():
    """The 1D non-causal call given precomputed cos / sin equals the one
    given raw angles."""
    x = {k: v.cuda() for k, v in random_siso(2, 130, 3, 32, 64, 16, seed=12).items()}
    a = arm()
    cos, sin = a.angles_to_cos_sin(x["angles"], x["dt"], 32)
    y1 = a.noncausal_scan(**x)
    xc = dict(x)
    xc.pop("angles")
    y2 = a.noncausal_scan(**xc, cos=cos, sin=sin)
    assert rel_err(y2.cpu().numpy(), y1.cpu().numpy()) <= REL_TOL


def test_mimo_random_state_and_reverse():
    g = torch.Generator().manual_seed(9)
    b, l, h, dv, dqk, R = 2, 70, 3, 32, 64, 4
    f = lambda *s: torch.randn(*s, generator=g)  # noqa: E731
    dt = torch.nn.functional.softplus(f(b, h, l) - 4)
    x = dict(q=f(b, l, R, dqk) / 8, k=f(b, l, R, dqk) / 8, v=f(b, l, h, dv), adt=-dt, dt=dt,
             trap=f(b, h, l), q_bias=0.1 * f(h, R, dqk), k_bias=0.1 * f(h, R, dqk),
             psi=f(h, R, dv), zeta=f(h, R, dv), phi=f(h, R, dv), angles=f(b, l, h, dqk // 4),
             D=torch.ones(h), z=f(b, l, h, dv))
    cos, sin = oracle.angles_to_cos_sin(x["angles"].numpy(), x["dt"].numpy(), dqk // 2)
    for rv in (False, True):
        want, wst = oracle.m3_mimo(x["q"], x["k"], x["v"], x["adt"], x["dt"], x["trap"],
                                   x["q_bias"], x["k_bias"], cos, sin, x["psi"], x["zeta"],
                                   x["phi"], D=x["D"], z=x["z"], reverse=rv, want_state=True)
        out, st = arm().mamba3_mimo_scan(**{k: v.cuda() for k, v in x.items()}, reverse=rv,
                                         return_last_state=True)
        assert rel_err(out.cpu().numpy(), want) <= REL_TOL
        assert rel_err(st.cpu().numpy(), wst) <= REL_TOL


@pytest.mark.parametrize("mimo", [False, True])
def test_sequential_backend_matches_oracle(mimo):
    """backend=1 selects the sequential-in-time kernel (the on-device
    restatement of the scalar loop); it must agree with the oracle too."""
    from armhackathon_b200 import _ffi
    g = torch.Generator().manual_seed(21)
    b, l, h, dv, dqk, R = 2, 77, 3, 32, 64, (2 if mimo else 1)
    f = lambda *s: torch.randn(*s, generator=g)  # noqa: E731
    dt = torch.nn.functional.softplus(f(b, h, l) - 4)
    q, k = f(b, l, R, dqk) / 8, f(b, l, R, dqk) / 8
    v, z, trap = f(b, l, h, dv), f(b, l, h, dv), f(b, h, l)
    qb, kb = 0.1 * f(h, R, dqk), 0.1 * f(h, R, dqk)
    proj = [f(h, R, dv) for _ in range(3)] if mimo else [None] * 3
    cos, sin = oracle.angles_to_cos_sin(f(b, l, h, dqk // 4).numpy(), dt.numpy(), dqk // 2)
    D = torch.ones(h)
    if mimo:
        want = oracle.m3_mimo(q, k, v, -dt, dt, trap, qb, kb, cos, sin, *proj, D=D, z=z)
    else:
        want = oracle.m3_siso(q, k, v, -dt, dt, trap, qb[:, 0], kb[:, 0], cos, sin, D=D, z=z)
    dev = lambda t: None if t is None else t.float().contiguous().cuda()  # noqa: E731
    ins = [dev(x) for x in (q, k, v, -dt, dt, trap, qb, kb, torch.from_numpy(cos),
                            torch.from_numpy(sin), D, z, *proj)]
    out = torch.empty(b, h, l, dv, device="cuda")
    dims = _ffi.ArmMamba3Dims(b, h, dv, dqk, l, R)
    _ffi.mamba3_raw(dims, [0 if t is None else t.data_ptr() for t in ins], 0, 1, 0,
                    out.data_ptr(), 0, 0)
    got = out.permute(0, 2, 1, 3).cpu().numpy()
    assert rel_err(got, want) <= REL_TOL


@pytest.mark.parametrize("shape", [(2, 5000, 3, 64, 20), (1, 1, 2, 128, 64), (3, 129, 4, 16, 8)])
def test_angle_prepass_kernel_vs_oracle(shape):
    """The CUDA angle pre-pass (theta = cumsum(tanh(angle) * pi * dt), cos/sin
    padded with the identity) against the f64 oracle restatement of the
    reference's angles_to_cos_sin; pairs beyond n_angles must be exactly
    (1, 0).  Tolerance 1e-4 absolute on cos/sin (the prefix sum is fp32, as
    in the reference's torch path)."""
    b, length, h, dqk, r = shape
    g = torch.Generator().manual_seed(length)
    ang = torch.randn(b, length, h, r, generator=g)
    dt = torch.nn.functional.softplus(torch.randn(b, h, length, generator=g) - 4)
    cos, sin = arm().angles_to_cos_sin(ang.cuda(), dt.cuda(), dqk // 2)
    wc, ws = oracle.angles_to_cos_sin(ang.numpy(), dt.numpy(), dqk // 2)
    assert np.abs(cos.cpu().numpy() - wc).max() < 1e-4
    assert np.abs(sin.cpu().numpy() - ws).max() < 1e-4
    if r < dqk // 2:
        assert torch.all(cos[..., r:] == 1) and torch.all(sin[..., r:] == 0)


BF16_TOL = 2e-2  # bf16 operands, fp32 accumulation and state (north_star bf16 bar)


@pytest.mark.parametrize("shape", [(1, 300, 2), (2, 128, 3), (1, 1, 1), (3, 517, 4)])
@pytest.mark.parametrize("reverse", [False, True])
def test_tensor_core_siso_vs_oracle(shape, reverse):
    """tcgen05 kernel (precision="bf16") against the f64 oracle: outputs and
    final states within the bf16 bar, including partial last chunks."""
    b, l, h = shape
    x = random_siso(b, l, h, 64, 128, 64, seed=l + 1)
    cos, sin = oracle.angles_to_cos_sin(x["angles"].numpy(), x["dt"].numpy(), 64)
    want, wst, _ = oracle.m3_siso(x["q"], x["k"], x["v"], x["adt"], x["dt"], x["trap"],
                                  x["q_bias"], x["k_bias"], cos, sin, D=x["D"], z=x["z"],
                                  reverse=reverse, want_state=True, nthreads=8)
    out, st = arm().mamba3_scan(**{k: v.cuda() for k, v in x.items()}, reverse=reverse,
                                return_last_state=True, precision="bf16")
    torch.cuda.synchronize()
    from armhackathon_b200 import _ffi
    _ffi.tensor_status()  # no bounded MMA wait expired
    assert rel_err(out.cpu().numpy(), want) <= BF16_TOL
    assert rel_err(st.cpu().numpy(), wst) <= BF16_TOL


@pytest.mark.parametrize("name", [n for n in IDX["m3_siso"] if n.endswith(("00", "01", "02", "03"))])
def test_tensor_core_siso_official_goldens(name):
    """The 24-head x 64 x 128 captures from the official (bf16) kernel, within
    the reference's 8 bf16-ULP gate."""
    kw, d = load("m3_siso", name)
    out = arm().mamba3_scan(kw["Q"], kw["K"], kw["V"], kw["ADT"], kw["DT"], kw["Trap"],
                            kw["Q_bias"], kw["K_bias"], angles=kw["Angles"], D=kw["D"],
                            z=kw["Z"], precision="bf16")
    assert oracle.bf16_ulps_at_scale(out.cpu().numpy(), d["out"]) <= 8.0


def _tc_case(b, l, h, r, seed, bf16, shared):
    """Inputs for the fused-angle tensor entry and the f64 oracle's answer on
    exactly those (bf16-rounded where bf16) values."""
    x = random_siso(b, l, h, 64, 128, r, seed=seed)
    if shared:
        x["angles"] = x["angles"][:, :, :1, :].contiguous()
    if bf16:
        for key in ("q", "k", "v", "z", "angles"):
            x[key] = x[key].to(torch.bfloat16)
    xf = {key: val.float() for key, val in x.items()}
    full = xf["angles"].expand(b, l, h, r).contiguous()
    cos, sin = oracle.angles_to_cos_sin(full.numpy(), xf["dt"].numpy(), 64)
    return x, xf, cos, sin


@pytest.mark.parametrize("bf16", [False, True])
@pytest.mark.parametrize("shared", [False, True])
@pytest.mark.parametrize("reverse", [False, True])
def test_tensor_core_fused_angles_vs_oracle(bf16, shared, reverse):
    """precision="bf16" with raw angles: angle pre-pass fused into the
    tensor-core kernel, bf16 or fp32 q/k/v/z/angles, output in that dtype
    and (b, l, h, dv) layout; against the f64 oracle within the bf16 bar."""
    b, l, h, r = 2, 389, 3, 64
    x, xf, cos, sin = _tc_case(b, l, h, r, 7 + l, bf16, shared)
    want, wst, _ = oracle.m3_siso(xf["q"], xf["k"], xf["v"], xf["adt"], xf["dt"], xf["trap"],
                                  xf["q_bias"], xf["k_bias"], cos, sin, D=xf["D"], z=xf["z"],
                                  reverse=reverse, want_state=True, nthreads=8)
    out, st = arm().mamba3_scan(**{k: v.cuda() for k, v in x.items()}, reverse=reverse,
                                return_last_state=True, precision="bf16")
    torch.cuda.synchronize()
    from armhackathon_b200 import _ffi
    _ffi.tensor_status()
    assert out.dtype == (torch.bfloat16 if bf16 else torch.float32)
    assert tuple(out.shape) == (b, l, h, 64) and out.is_contiguous()
    assert rel_err(out.float().cpu().numpy(), want) <= BF16_TOL
    assert rel_err(st.cpu().numpy(), wst) <= BF16_TOL


@pytest.mark.parametrize("shape", [(1, 1, 1, 64), (1, 128, 2, 48), (2, 1000, 2, 8),
                                   (3, 255, 2, 64)])
def test_tensor_core_fused_angles_shapes_and_carry(shape):
    """Ragged lengths, fewer rotated pairs than dqk/2, and the (last_state,
    last_bx) carry through the C entry point with head-major output."""
    import ctypes
    from armhackathon_b200 import _ffi
    b, l, h, r = shape
    x, xf, cos, sin = _tc_case(b, l, h, r, 3 * l + r, True, False)
    for reverse in (False, True):
        want, wst, wbx = oracle.m3_siso(xf["q"], xf["k"], xf["v"], xf["adt"], xf["dt"],
                                        xf["trap"], xf["q_bias"], xf["k_bias"], cos, sin,
                                        D=xf["D"], z=xf["z"], reverse=reverse,
                                        want_state=True, nthreads=8)
        c = {k: v.cuda().contiguous() for k, v in x.items()}
        out = torch.empty((b, h, l, 64), device="cuda")
        st = torch.empty((b, h, 64, 128), device="cuda")
        bx = torch.empty((b, h, 128), device="cuda")
        dims = _ffi.ArmMamba3Dims(b, h, 64, 128, l, 1)
        opts = _ffi.ArmMamba3TcOptions(_ffi.DTYPE_BF16, _ffi.DTYPE_F32, 0, 0, r)
        _ffi.mamba3_tc_raw(dims, opts, [c["q"].data_ptr(), c["k"].data_ptr(), c["v"].data_ptr(),
                                        c["adt"].data_ptr(), c["dt"].data_ptr(),
                                        c["trap"].data_ptr(), c["q_bias"].data_ptr(),
                                        c["k_bias"].data_ptr(), c["angles"].data_ptr(),
                                        c["D"].data_ptr(), c["z"].data_ptr()],
                           reverse, out.data_ptr(), st.data_ptr(), bx.data_ptr(),
                           torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        _ffi.tensor_status()
        got = out.permute(0, 2, 1, 3).cpu().numpy()
        assert rel_err(got, want) <= BF16_TOL
        assert rel_err(st.cpu().numpy(), wst) <= BF16_TOL
        assert rel_err(bx.cpu().numpy(), wbx) <= 1e-4  # fp32 carry, not an MMA operand


def test_tensor_core_fused_matches_cos_sin_entry():
    """Same fp32 inputs through the fused-angle entry and the reference-layout
    cos/sin entry (backend 3): both within the bf16 bar of each other."""
    b, l, h, r = 2, 640, 4, 64
    x = random_siso(b, l, h, 64, 128, r, seed=11)
    c = {k: v.cuda() for k, v in x.items()}
    a = arm().mamba3_scan(**c, precision="bf16")
    cos, sin = arm().angles_to_cos_sin(c["angles"], c["dt"], 64)
    c.pop("angles")
    bb = arm().mamba3_scan(**c, cos=cos, sin=sin, precision="bf16")
    assert rel_err(a.cpu().numpy(), bb.cpu().numpy()) <= BF16_TOL


@pytest.mark.parametrize("split", ["0", "1"])
def test_tensor_core_cos_sin_split_and_fused(split, knobs):
    """The reference-layout entry's two tensor-core forms (one persistent
    launch; three launches with B200SCAN_M3_TC_SPLIT=1) against the oracle."""
    knobs(m3_tc_split=int(split))
    x = random_siso(2, 700, 3, 64, 128, 64, seed=5)
    cos, sin = oracle.angles_to_cos_sin(x["angles"].numpy(), x["dt"].numpy(), 64)
    want, wst, _ = oracle.m3_siso(x["q"], x["k"], x["v"], x["adt"], x["dt"], x["trap"],
                                  x["q_bias"], x["k_bias"], cos, sin, D=x["D"], z=x["z"],
                                  want_state=True, nthreads=8)
    c = {k: v.cuda() for k, v in x.items()}
    c.pop("angles")
    out, st = arm().mamba3_scan(**c, cos=torch.from_numpy(cos).float().cuda(),
                                sin=torch.from_numpy(sin).float().cuda(), return_last_state=True,
                                precision="bf16")
    assert rel_err(out.cpu().numpy(), want) <= BF16_TOL
    assert rel_err(st.cpu().numpy(), wst) <= BF16_TOL


@pytest.mark.parametrize("R", [2, 4])
@pytest.mark.parametrize("shape", [(2, 300, 3), (1, 33, 2), (1, 1, 1)])
def test_tensor_core_mimo_vs_oracle(R, shape):
    """MIMO on the tensor cores (backend 3): rows = (step, rank), split-halves
    RoPE, psi/zeta/phi projections, forward and reverse, ragged lengths."""
    b, l, h = shape
    dv, dqk = 64, 128
    g = torch.Generator().manual_seed(17 * R + l)
    f = lambda *s: torch.randn(*s, generator=g)  # noqa: E731
    dt = torch.nn.functional.softplus(f(b, h, l) - 4)
    A = -torch.exp(torch.rand(h, generator=g) * np.log(16))
    x = dict(q=f(b, l, R, dqk) / (dqk * R) ** 0.5, k=f(b, l, R, dqk) / (dqk * R) ** 0.5,
             v=f(b, l, h, dv), adt=A.view(1, h, 1) * dt, dt=dt, trap=f(b, h, l),
             q_bias=0.1 * f(h, R, dqk), k_bias=0.1 * f(h, R, dqk), psi=f(h, R, dv),
             zeta=f(h, R, dv), phi=f(h, R, dv), angles=f(b, l, h, 64), D=1 + 0.1 * f(h),
             z=f(b, l, h, dv))
    cos, sin = oracle.angles_to_cos_sin(x["angles"].numpy(), x["dt"].numpy(), dqk // 2)
    for rv in (False, True):
        want, wst = oracle.m3_mimo(x["q"], x["k"], x["v"], x["adt"], x["dt"], x["trap"],
                                   x["q_bias"], x["k_bias"], cos, sin, x["psi"], x["zeta"],
                                   x["phi"], D=x["D"], z=x["z"], reverse=rv, want_state=True)
        out, st = arm().mamba3_mimo_scan(**{k: v.cuda() for k, v in x.items()}, reverse=rv,
                                         return_last_state=True, precision="bf16")
        torch.cuda.synchronize()
        from armhackathon_b200 import _ffi
        _ffi.tensor_status()
        assert rel_err(out.cpu().numpy(), want) <= BF16_TOL
        assert rel_err(st.cpu().numpy(), wst) <= BF16_TOL


def test_tensor_core_expanded_angles_view_is_shared():
    """Angles given as a head-broadcast view (b, l, 1, r).expand(b, l, h, r),
    as a Mamba-3 LM block passes them, give the same result as the explicit
    per-head copy."""
    b, l, h, r = 2, 300, 4, 64
    x = random_siso(b, l, h, 64, 128, r, seed=21)
    c = {k: v.cuda() for k, v in x.items()}
    row = c["angles"][:, :, :1, :]
    c["angles"] = row.expand(b, l, h, r)
    got = arm().mamba3_scan(**c, precision="bf16")
    c["angles"] = row.expand(b, l, h, r).contiguous()
    want = arm().mamba3_scan(**c, precision="bf16")
    assert torch.equal(got, want)


def test_chunk_kernel_unaligned_q_k_take_scalar_staging():
    """q, k that are not 16-byte aligned (a view one element into its
    storage) run the chunk kernels' element-by-element staging; same result."""
    x = random_siso(2, 300, 3, 64, 128, 64, seed=13)
    cos, sin = oracle.angles_to_cos_sin(x["angles"].numpy(), x["dt"].numpy(), 64)
    want = oracle.m3_siso(x["q"], x["k"], x["v"], x["adt"], x["dt"], x["trap"], x["q_bias"],
                          x["k_bias"], cos, sin, D=x["D"], z=x["z"], nthreads=8)
    c = {k: v.cuda() for k, v in x.items()}
    for name in ("q", "k"):
        t = c[name]
        buf = torch.empty(t.numel() + 1, device="cuda")
        shifted = buf[1:].view(t.shape)
        shifted.copy_(t)
        assert shifted.data_ptr() % 16 != 0
        c[name] = shifted
    out = arm().mamba3_scan(**c)
    assert rel_err(out.cpu().numpy(), want) <= REL_TOL


@pytest.mark.parametrize("grid", [(6, 9), (17, 23)])
@pytest.mark.parametrize("seq", ["0", "1"])
def test_ss2d_mamba3_fused_sum_vs_oracle(grid, seq, knobs):
    """merge="sum" / "mean" run all four traversals in one library call that
    reads the grid in place (column-major traversal by index mapping, the
    angle pre-pass per ordering, outputs summed in place), in both chunk-kernel
    forms, on non-square grids whose length is not a multiple of the chunk."""
    knobs(m3_chunk_form=1 if seq == "1" else 2)
    g = torch.Generator().manual_seed(sum(grid))
    b, (H, W), h, dv, dqk, r = 2, grid, 3, 32, 64, 16
    f = lambda *s: torch.randn(*s, generator=g)  # noqa: E731
    dt = torch.nn.functional.softplus(f(b, h, H, W) - 4)
    x = dict(q=f(b, H, W, 1, dqk) / 8, k=f(b, H, W, 1, dqk) / 8, v=f(b, H, W, h, dv),
             adt=-dt * 2.0, dt=dt, trap=f(b, h, H, W), q_bias=0.1 * f(h, dqk),
             k_bias=0.1 * f(h, dqk), angles=f(b, H, W, h, r), D=1 + 0.1 * f(h),
             z=f(b, H, W, h, dv))
    from armhackathon_b200.ss2d import grid_to_views
    from armhackathon_b200.ss2d_mamba3 import grid_to_views_time_major, views_to_grid_time_major
    tv = {k: grid_to_views_time_major(x[k]) for k in ("q", "k", "v", "angles", "z")}
    hv = {k: grid_to_views(x[k]) for k in ("adt", "dt", "trap")}
    cos, sin = oracle.angles_to_cos_sin(tv["angles"].numpy(), hv["dt"].numpy(), dqk // 2)
    want = 0
    for rv in (False, True):
        o = torch.from_numpy(oracle.m3_siso(tv["q"], tv["k"], tv["v"], hv["adt"], hv["dt"],
                                            hv["trap"], x["q_bias"], x["k_bias"], cos, sin,
                                            D=x["D"], z=tv["z"], reverse=rv, nthreads=8))
        rows, cols = views_to_grid_time_major(o[:b], o[b:], H, W)
        want = want + rows + cols
    c = {k: v.cuda() for k, v in x.items()}
    got = arm().ss2d_scan_mamba3(**c, merge="sum")
    assert tuple(got.shape) == (b, H, W, h, dv)
    assert rel_err(got.cpu().numpy(), want.numpy()) <= REL_TOL
    mean = arm().ss2d_scan_mamba3(**c, merge="mean")
    assert rel_err(mean.cpu().numpy(), 0.25 * want.numpy()) <= REL_TOL
