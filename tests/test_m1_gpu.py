"""Mamba-1 parity on the GPU: the CUDA kernels (through libb200scan.so's C ABI)
against the reference's golden vectors and the CPU oracle.

Tolerances: the reference's own gate for fp32 outputs against f64 ground
truth -- max |out - out_f64| < 1e-4 and < max(50 x the upstream f32 floor,
1e-6); last_state relative error < 1e-4 (reference tests/check_ffi.py:30-31,
82-83) -- plus the build's fp32 bar: max relative error <= 1e-4 against the
oracle, relative to the output's scale.
"""

import json

import numpy as np
import pytest
import torch

import oracle
from conftest import GOLDEN

pytestmark = pytest.mark.gpu

M1_CASES = json.loads((GOLDEN / "index.json").read_text())["m1"]
REL_TOL = 1e-4


def arm():
    import armhackathon_b200 as a
    return a


def load(name):
    d = np.load(GOLDEN / "m1" / f"{name}.npz")
    get = lambda k: d[k] if k in d.files else None  # noqa: E731
    inputs = dict(u=d["u"], delta=d["delta"], A=d["A"], B=d["B"], C=d["C"], D=get("D_skip"),
                  z=get("z"), delta_bias=get("delta_bias"),
                  delta_softplus=bool(d["delta_softplus"]))
    return inputs, d["out_f64"], d["last_state_f64"], float(d["f32_max_abs_err"])


def cuda(inputs):
    return {k: (torch.from_numpy(np.ascontiguousarray(v)).cuda() if isinstance(v, np.ndarray)
                else v) for k, v in inputs.items()}


def rel_err(got, want):
    want = np.asarray(want, np.float64)
    return float(np.abs(np.asarray(got, np.float64) - want).max()
                 / max(np.abs(want).max(), 1e-30))


def gate(out, last, out64, last64, floor):
    err = np.abs(out.astype(np.float64) - out64).max()
    assert err < 1e-4 and err < max(50 * floor, 1e-6), err
    lrel = np.abs(last.astype(np.float64) - last64).max() / max(1.0, np.abs(last64).max())
    assert lrel < 1e-4, lrel


@pytest.mark.parametrize("name", M1_CASES)
def test_golden_cuda_tensors(name):
    inputs, out64, last64, floor = load(name)
    out, last = arm().selective_scan(**cuda(inputs), return_last_state=True)
    torch.cuda.synchronize()
    gate(out.cpu().numpy(), last.cpu().numpy(), out64, last64, floor)


@pytest.mark.parametrize("name", ["tiny", "medium", "grouped_BC", "hf_mixer_layer0"])
def test_golden_host_buffers_numpy_api(name):
    """Host arrays through the synchronous C entry point (library-side staging)."""
    inputs, out64, last64, floor = load(name)
    out, last = arm().selective_scan_numpy(**inputs, return_last_state=True)
    gate(out, last, out64, last64, floor)


@pytest.mark.parametrize("name", ["small", "long_seq", "grouped_BC", "edge_L1"])
def test_sequential_backend_matches(name):
    inputs, out64, last64, floor = load(name)
    out, last = arm().selective_scan_numpy(**inputs, return_last_state=True, backend="scalar")
    gate(out, last, out64, last64, floor)


@pytest.mark.parametrize("name", ["small", "medium", "grouped_BC", "state13_neon_tail",
                                  "extreme_delta", "edge_L1", "no_z"])
def test_reverse_matches_oracle(name):
    inputs, *_ = load(name)
    want, want_last = oracle.m1_scan(**inputs, reverse=True)
    out, last = arm().selective_scan(**cuda(inputs), reverse=True, return_last_state=True)
    assert rel_err(out.cpu().numpy(), want) <= REL_TOL
    assert rel_err(last.cpu().numpy(), want_last) <= REL_TOL


def random_case(B, D, L, N, G=1, seed=0, z=True, dskip=True, bias=True):
    rng = np.random.default_rng(seed)
    f = lambda *s: rng.standard_normal(s).astype(np.float32)  # noqa: E731
    bc = (B, G, N, L) if G > 1 else (B, N, L)
    return dict(u=f(B, D, L), delta=(f(B, D, L) * 0.5).astype(np.float32),
                A=(-np.exp(rng.uniform(np.log(0.5), np.log(16), (D, N)))).astype(np.float32),
                B=f(*bc), C=f(*bc), D=f(D) if dskip else None, z=f(B, D, L) if z else None,
                delta_bias=rng.uniform(-6, -3, D).astype(np.float32) if bias else None,
                delta_softplus=True)


@pytest.mark.parametrize("shape", [(1, 7, 1001, 16, 1), (3, 40, 515, 13, 4), (2, 33, 4096, 16, 1),
                                   (1, 1536, 130, 16, 1), (2, 24, 3, 1, 2), (1, 5, 777, 64, 1)])
@pytest.mark.parametrize("reverse", [False, True])
def test_ragged_shapes_vs_oracle(shape, reverse):
    """Lengths off the vector width and the macro-chunk, odd channel counts,
    grouped B/C and unusual state sizes, forward and reverse."""
    B, D, L, N, G = shape
    inputs = random_case(B, D, L, N, G, seed=L)
    want, want_last = oracle.m1_scan(**inputs, reverse=reverse, nthreads=8)
    out, last = arm().selective_scan(**cuda(inputs), reverse=reverse, return_last_state=True)
    assert rel_err(out.cpu().numpy(), want) <= REL_TOL
    assert rel_err(last.cpu().numpy(), want_last) <= REL_TOL


def test_h0_streaming_resume():
    """Split scan resumed from last_state equals the one-shot scan."""
    inputs = random_case(2, 96, 1000, 16, seed=3)
    a = arm()
    full, last_full = a.selective_scan(**cuda(inputs), return_last_state=True)
    split = 333
    tv = ("u", "delta", "B", "C", "z")
    first = {k: (v[..., :split] if k in tv else v) for k, v in inputs.items()}
    second = {k: (v[..., split:] if k in tv else v) for k, v in inputs.items()}
    o1, s1 = a.selective_scan(**cuda(first), return_last_state=True)
    o2, s2 = a.selective_scan(**cuda(second), return_last_state=True, initial_state=s1)
    full = full.cpu().numpy()
    assert rel_err(torch.cat([o1, o2], -1).cpu().numpy(), full) <= REL_TOL
    assert rel_err(s2.cpu().numpy(), last_full.cpu().numpy()) <= REL_TOL


def test_bidirectional_fused_and_merges():
    inputs = random_case(2, 64, 777, 16, seed=5)
    a = arm()
    of, ob = a.selective_scan_bidirectional(**cuda(inputs))
    wf, wb, _, _ = oracle.m1_scan_bidir(**inputs, nthreads=8)
    assert rel_err(of.cpu().numpy(), wf) <= REL_TOL
    assert rel_err(ob.cpu().numpy(), wb) <= REL_TOL
    s = a.bidirectional_scan(**cuda(inputs), merge="sum")
    assert rel_err(s.cpu().numpy(), wf + wb) <= REL_TOL
    c = a.bidirectional_scan(**cuda(inputs), merge="concat")
    assert tuple(c.shape) == (2, 128, 777)
    (f2, lf), (b2, lb) = a.bidirectional_scan(**cuda(inputs), merge="none", return_last_state=True)
    assert rel_err(f2.cpu().numpy(), wf) <= REL_TOL and rel_err(b2.cpu().numpy(), wb) <= REL_TOL


@pytest.mark.parametrize("segments", ["1", "2", "4", "16"])
@pytest.mark.parametrize("shape", [(2, 70, 1024, 13, 2), (1, 64, 4096, 16, 1)])
def test_bidirectional_shared_first_pass(segments, shape, knobs):
    """The bidirectional entries on lengths the two-pass kernel takes: one
    forward walk per segment gives both traversals' segment aggregates (the
    reverse one from running products of the decays), then a carry and a
    rescan per direction; the sum entry adds the reverse traversal in place.
    Slowly decaying states so the carries matter; grouped B/C, ragged
    channel counts, d_state 13; final states through the C entry."""
    from armhackathon_b200 import _ffi
    knobs(m1_segments=int(segments))
    B, D, L, N, G = shape
    x = _slow_decay_case(B, D, L, N, seed=L + N)
    if G > 1:
        rng = np.random.default_rng(7)
        x["B"] = rng.standard_normal((B, G, N, L)).astype(np.float32)
        x["C"] = rng.standard_normal((B, G, N, L)).astype(np.float32)
    wf, wb, wlf, wlb = oracle.m1_scan_bidir(**x, nthreads=8)
    a = arm()
    t = cuda(x)
    of, ob = a.selective_scan_bidirectional(**t)
    assert rel_err(of.cpu().numpy(), wf) <= REL_TOL
    assert rel_err(ob.cpu().numpy(), wb) <= REL_TOL
    s = a.bidirectional_scan(**t, merge="sum")
    assert rel_err(s.cpu().numpy(), wf + wb) <= REL_TOL
    m = a.bidirectional_scan(**t, merge="mean")
    assert rel_err(m.cpu().numpy(), 0.5 * (wf + wb)) <= REL_TOL
    lf = torch.empty(B, D, N, device="cuda")
    lb = torch.empty(B, D, N, device="cuda")
    out = torch.empty(B, D, L, device="cuda")
    dims = _ffi.ArmScanDims(B, D, L, N, G)
    _ffi.scan_bidir_sum_raw(dims, t["u"].data_ptr(), t["delta"].data_ptr(), t["A"].data_ptr(),
                            t["B"].data_ptr(), t["C"].data_ptr(), t["D"].data_ptr(),
                            t["z"].data_ptr(), t["delta_bias"].data_ptr(), True, "auto",
                            out.data_ptr(), lf.data_ptr(), lb.data_ptr(),
                            stream=torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert rel_err(out.cpu().numpy(), wf + wb) <= REL_TOL
    assert rel_err(lf.cpu().numpy(), wlf) <= REL_TOL
    assert rel_err(lb.cpu().numpy(), wlb) <= REL_TOL


@pytest.mark.parametrize("shared", ["1", "0"])
def test_bidirectional_final_states_and_sum_with_h0(shared, knobs):
    """The two calls a sequence split over devices makes: both traversals'
    final states from zero (one shared first pass), then both outputs summed
    from given incoming states (forward one enters at t = 0, reverse one at
    t = L - 1); with and without the shared pass."""
    knobs(m1_bidir_independent=0 if shared == "1" else 1)
    B, D, L, N = 2, 70, 1024, 13
    x = _slow_decay_case(B, D, L, N, seed=11)
    a = arm()
    t = cuda(x)
    hf, hb = a.selective_scan_bidirectional_final_states(
        t["u"], t["delta"], t["A"], t["B"], t["C"], delta_bias=t["delta_bias"],
        delta_softplus=True)
    _, wlf = oracle.m1_scan(**x, nthreads=8)
    _, wlb = oracle.m1_scan(**x, reverse=True, nthreads=8)
    assert rel_err(hf.cpu().numpy(), wlf) <= REL_TOL
    assert rel_err(hb.cpu().numpy(), wlb) <= REL_TOL
    rng = np.random.default_rng(3)
    h0f, h0b = (rng.standard_normal((B, D, N)).astype(np.float32) for _ in range(2))
    out = a.selective_scan_bidirectional_sum(
        **t, initial_states=(torch.from_numpy(h0f).cuda(), torch.from_numpy(h0b).cuda()))
    wf, _ = oracle.m1_scan(**x, h0=h0f, nthreads=8)
    wb, _ = oracle.m1_scan(**x, reverse=True, h0=h0b, nthreads=8)
    assert rel_err(out.cpu().numpy(), wf + wb) <= REL_TOL


def test_bidirectional_sum_without_shared_pass(knobs):
    """The sum entry where the traversals run as independent scans (forced,
    and on a length the two-pass kernel does not take): second output in
    workspace, then an add kernel."""
    a = arm()
    for env, L in (("0", 1024), ("1", 777)):
        knobs(m1_bidir_independent=0 if env == "1" else 1)
        x = random_case(2, 64, L, 16, seed=9)
        wf, wb, _, _ = oracle.m1_scan_bidir(**x, nthreads=8)
        s = a.bidirectional_scan(**cuda(x), merge="sum")
        assert rel_err(s.cpu().numpy(), wf + wb) <= REL_TOL


def test_ss2d_golden_planes():
    a = arm()
    for name in json.loads((GOLDEN / "index.json").read_text())["m1_2d"]:
        d = np.load(GOLDEN / "m1_2d" / f"{name}.npz")
        t = lambda k: torch.from_numpy(d[k]).cuda()  # noqa: E731
        planes = a.ss2d_scan(t("u"), t("delta"), t("A"), t("B"), t("C"), D=t("D"),
                             delta_bias=t("delta_bias"), merge="none")
        for key, got in zip(("out_row_fwd", "out_row_bwd", "out_col_fwd", "out_col_bwd"), planes):
            err = np.abs(got.cpu().numpy().astype(np.float64) - d[key]).max()
            assert err < 1e-4, (name, key, err)
        want = sum(d[k] for k in ("out_row_fwd", "out_row_bwd", "out_col_fwd", "out_col_bwd"))
        for merge, scale in (("sum", 1.0), ("mean", 0.25)):
            for fn in (a.ss2d_scan, a.selective_scan_ss2d):
                got = fn(t("u"), t("delta"), t("A"), t("B"), t("C"), D=t("D"),
                         delta_bias=t("delta_bias"), merge=merge)
                err = np.abs(got.cpu().numpy().astype(np.float64) - scale * want).max()
                assert err < 4e-4, (name, merge, fn.__name__, err)


def test_config0_full_size_properties():
    """BASELINE config 0 at full size (B1 D1536 L2048 N16): against the
    oracle, and reverse == flip-forward-flip."""
    rng = np.random.default_rng(0)
    D, L, N = 1536, 2048, 16
    dt = np.exp(rng.uniform(np.log(1e-3), np.log(1e-1), D))
    inputs = dict(u=rng.standard_normal((1, D, L)).astype(np.float32),
                  delta=rng.standard_normal((1, D, L)).astype(np.float32),
                  A=np.tile(-np.arange(1, N + 1, dtype=np.float32), (D, 1)),
                  B=rng.standard_normal((1, N, L)).astype(np.float32),
                  C=rng.standard_normal((1, N, L)).astype(np.float32),
                  D=np.ones(D, np.float32), z=rng.standard_normal((1, D, L)).astype(np.float32),
                  delta_bias=np.log(np.expm1(dt)).astype(np.float32), delta_softplus=True)
    want, want_last = oracle.m1_scan(**inputs, dtype=np.float64, nthreads=8)
    out, last = arm().selective_scan(**cuda(inputs), return_last_state=True)
    assert rel_err(out.cpu().numpy(), want) <= REL_TOL
    assert rel_err(last.cpu().numpy(), want_last) <= REL_TOL
    fl = {k: (np.ascontiguousarray(np.flip(v, -1)) if k in ("u", "delta", "B", "C", "z") else v)
          for k, v in inputs.items()}
    rev = arm().selective_scan(**cuda(inputs), reverse=True)
    fwd_of_flip = arm().selective_scan(**cuda(fl))
    assert rel_err(torch.flip(rev, [-1]).cpu().numpy(), fwd_of_flip.cpu().numpy()) <= REL_TOL


def test_cpu_tensors_run_on_gpu_and_come_back():
    inputs, out64, last64, floor = load("medium")
    t = {k: (torch.from_numpy(v) if isinstance(v, np.ndarray) else v) for k, v in inputs.items()}
    out, last = arm().selective_scan(**t, return_last_state=True)
    assert out.device.type == "cpu"
    gate(out.numpy(), last.numpy(), out64, last64, floor)


def test_mixed_host_device_rejected():
    import ctypes
    from armhackathon_b200 import _ffi
    x = torch.zeros(1, 1, 4, device="cuda")
    h = torch.zeros(1, 1, 4)
    dims = _ffi.ArmScanDims(1, 1, 4, 1, 1)
    lib = _ffi.load()
    rc = lib.arm_scan_selective_scan_f32(ctypes.byref(dims), x.data_ptr(), h.data_ptr(),
                                         x.data_ptr(), x.data_ptr(), x.data_ptr(), None, None,
                                         None, 1, 0, 0, 0, x.data_ptr(), None, None)
    assert rc == 2


@pytest.mark.parametrize("kernel", ["lane", "tile", "chunked"])
@pytest.mark.parametrize("reverse", [False, True])
def test_every_kernel_vs_oracle(kernel, reverse, knobs):
    """Each Mamba-1 kernel the library can dispatch to (selected with the
    kernel override) against the oracle, on a grouped, h0-seeded case with a
    ragged row count."""
    from armhackathon_b200 import _ffi
    knobs(m1_kernel=_ffi.M1_KERNELS[kernel])
    inputs = random_case(3, 40, 1028, 16, 2, seed=7)
    rng = np.random.default_rng(1)
    h0 = rng.standard_normal((3, 40, 16)).astype(np.float32)
    want, want_last = oracle.m1_scan(**inputs, reverse=reverse, h0=h0, nthreads=8)
    out, last = arm().selective_scan(**cuda(inputs), reverse=reverse, return_last_state=True,
                                     initial_state=torch.from_numpy(h0).cuda())
    assert rel_err(out.cpu().numpy(), want) <= REL_TOL
    assert rel_err(last.cpu().numpy(), want_last) <= REL_TOL


def _slow_decay_case(B, D, L, N, seed):
    """Inputs whose state survives across thousands of steps (tiny dt, small
    |A|), so the time-split's carries between segments matter."""
    x = random_case(B, D, L, N, seed=seed)
    rng = np.random.default_rng(seed + 1)
    x["A"] = (-rng.uniform(0.05, 1.0, (D, N))).astype(np.float32)
    x["delta_bias"] = rng.uniform(-9, -7, D).astype(np.float32)
    return x


@pytest.mark.parametrize("segments", ["4", "8"])
@pytest.mark.parametrize("reverse", [False, True])
def test_time_split_vs_oracle(segments, reverse, knobs):
    """Few rows, long sequence, split in time (state-only pass, segment-decay
    fold, rescan from the carries): output, h0 resume and last_state."""
    knobs(m1_kernel=4, m1_segments=int(segments))
    B, D, L, N = 2, 24, 8192, 16
    x = _slow_decay_case(B, D, L, N, seed=int(segments))
    h0 = np.random.default_rng(3).standard_normal((B, D, N)).astype(np.float32)
    want, want_last = oracle.m1_scan(**x, reverse=reverse, h0=h0, nthreads=8)
    out, last = arm().selective_scan(**cuda(x), reverse=reverse, return_last_state=True,
                                     initial_state=torch.from_numpy(h0).cuda())
    assert rel_err(out.cpu().numpy(), want) <= REL_TOL
    assert rel_err(last.cpu().numpy(), want_last) <= REL_TOL


def test_time_split_chosen_automatically_and_bidirectional():
    """A one-sequence, few-channel, long problem takes the time split by
    itself; the fused bidirectional entry goes through it in both directions."""
    B, D, L, N = 1, 64, 32768, 16
    x = _slow_decay_case(B, D, L, N, seed=21)
    fwd, _ = oracle.m1_scan(**x, nthreads=8)
    bwd, _ = oracle.m1_scan(**x, reverse=True, nthreads=8)
    out = arm().selective_scan(**cuda(x))
    assert rel_err(out.cpu().numpy(), fwd) <= REL_TOL
    both = arm().bidirectional_scan(**cuda(x), merge="sum")
    assert rel_err(both.cpu().numpy(), fwd + bwd) <= REL_TOL


@pytest.mark.parametrize("shape", [(4, 512, 2048, 16, 1, False), (3, 256, 2048, 16, 2, True),
                                   (2, 64, 16384, 16, 1, True)])
def test_host_entry_pipelined_matches_device(shape):
    """The synchronous entry with host buffers pipelines per batch over two
    streams; every row's result is identical to the device-pointer path."""
    B, D, L, N, G, with_h0 = shape
    x = random_case(B, D, L, N, G, seed=B * D)
    h0 = (np.random.default_rng(1).standard_normal((B, D, N)).astype(np.float32)
          if with_h0 else None)
    out_h, last_h = arm().selective_scan_numpy(**x, initial_state=h0, return_last_state=True)
    xc = cuda(x)
    out_d, last_d = arm().selective_scan(
        **xc, initial_state=None if h0 is None else torch.from_numpy(h0).cuda(),
        return_last_state=True)
    assert np.array_equal(out_h, out_d.cpu().numpy())
    assert np.array_equal(last_h, last_d.cpu().numpy())


@pytest.mark.parametrize("shape", [(2, 40, 2048, 16, 2), (3, 130, 1024, 13, 1), (1, 8, 4096, 16, 1)])
@pytest.mark.parametrize("segments", ["1", "2", "4", "16"])
@pytest.mark.parametrize("reverse", [False, True])
def test_lane_kernel_segments_vs_oracle(shape, segments, reverse, knobs):
    """The lane kernel at forced segment counts (segment end states, exact
    segment-decay carries, rescan), with grouped B/C, ragged channel counts,
    d_state 13, h0 and slowly decaying states that carry across segments."""
    knobs(m1_kernel=1, m1_segments=int(segments))
    B, D, L, N, G = shape
    x = _slow_decay_case(B, D, L, N, seed=L + N)
    if G > 1:
        rng = np.random.default_rng(5)
        x["B"] = rng.standard_normal((B, G, N, L)).astype(np.float32)
        x["C"] = rng.standard_normal((B, G, N, L)).astype(np.float32)
    h0 = np.random.default_rng(2).standard_normal((B, D, N)).astype(np.float32)
    want, want_last = oracle.m1_scan(**x, reverse=reverse, h0=h0, nthreads=8)
    out, last = arm().selective_scan(**cuda(x), reverse=reverse, return_last_state=True,
                                     initial_state=torch.from_numpy(h0).cuda())
    assert rel_err(out.cpu().numpy(), want) <= REL_TOL
    assert rel_err(last.cpu().numpy(), want_last) <= REL_TOL


def test_library_counts_its_kernel_launches():
    """arm_scan_kernel_launches() advances by the kernels a call starts: three
    for the default fold-free form (pass 1, carries, pass 2)."""
    from armhackathon_b200 import _ffi
    x = cuda(random_case(2, 64, 2048, 16, seed=3))
    arm().selective_scan(**x)
    torch.cuda.synchronize()
    before = _ffi.kernel_launches()
    arm().selective_scan(**x)
    torch.cuda.synchronize()
    assert _ffi.kernel_launches() - before == 3


@pytest.mark.parametrize("groups", [1, 2])
def test_decode_steps_equal_the_scan(groups):
    """T chained selective_state_update steps from h0 reproduce the scan of
    the same T steps (outputs and final state), and one step matches the
    oracle."""
    B, D, T, N = 3, 40, 9, 16
    x = random_case(B, D, T, N, groups, seed=11)
    h0 = np.random.default_rng(4).standard_normal((B, D, N)).astype(np.float32)
    want, want_last = oracle.m1_scan(**x, h0=h0, nthreads=8)
    c = cuda(x)
    state = torch.from_numpy(h0).cuda().contiguous()
    ys = []
    for t in range(T):
        Bt = c["B"][..., t] if groups > 1 else c["B"][:, :, t]
        Ct = c["C"][..., t] if groups > 1 else c["C"][:, :, t]
        ys.append(arm().selective_state_update(
            state, c["u"][:, :, t], c["delta"][:, :, t], c["A"], Bt, Ct, D=c["D"],
            z=c["z"][:, :, t], dt_bias=c["delta_bias"], dt_softplus=True))
    y = torch.stack(ys, dim=-1)
    assert rel_err(y.cpu().numpy(), want) <= REL_TOL
    assert rel_err(state.cpu().numpy(), want_last) <= REL_TOL


@pytest.mark.parametrize("shape", [(2, 40, 2048, 16, 1), (1, 34, 1001, 13, 2)])
@pytest.mark.parametrize("reverse", [False, True])
def test_final_state_entry_equals_scan_last_state(shape, reverse):
    """selective_scan_final_state (no outputs: the two-pass kernel's first
    pass and carries, or the tile kernel's state-only mode) returns the scan's
    last_state."""
    B, D, L, N, G = shape
    x = random_case(B, D, L, N, G, seed=L)
    h0 = torch.from_numpy(np.random.default_rng(3).standard_normal((B, D, N)).astype(np.float32))
    c = cuda(x)
    _, want = arm().selective_scan(**c, reverse=reverse, initial_state=h0.cuda(),
                                   return_last_state=True)
    got = arm().selective_scan_final_state(c["u"], c["delta"], c["A"], c["B"], c["C"],
                                           delta_bias=c["delta_bias"], delta_softplus=True,
                                           initial_state=h0.cuda(), reverse=reverse)
    assert rel_err(got.cpu().numpy(), want.cpu().numpy()) <= 1e-5


@pytest.mark.parametrize("world", [2, 3])
def test_seqpar_fused_path_one_device(world, monkeypatch):
    """The sequence-parallel bidirectional scan on the library's own CUDA
    functions (segment summaries from one pass, then the sum entry with
    incoming states), every rank of a ``world``-way split run in this one process: the
    all_gather is replaced by the ranks' summaries computed here, so the
    result per segment must equal the unsplit bidirectional sum."""
    import torch.distributed as dist
    from armhackathon_b200 import seqpar
    B, D, L, N = 1, 96, 192 * world * 4, 16
    x = _slow_decay_case(B, D, L, N, seed=21)
    t = cuda(x)
    a = arm()
    full = a.bidirectional_scan(**t, merge="sum")
    seg = L // world
    sl = lambda v, r: v[..., r * seg:(r + 1) * seg].contiguous()  # noqa: E731
    summaries = [seqpar.segment_summary(sl(t["u"], r), sl(t["delta"], r), t["A"], sl(t["B"], r),
                                        sl(t["C"], r), t["delta_bias"], True)
                 for r in range(world)]
    # the summary's dt sum equals the torch restatement of softplus(delta + bias)
    for r in range(world):
        sdt = seqpar._segment_dt_sum(sl(t["delta"], r), t["delta_bias"], True)
        assert torch.allclose(summaries[r][..., -1], sdt, rtol=1e-5, atol=1e-6)
    rank = {"r": 0}

    def fake_all_gather(parts, packed, group=None):
        assert torch.allclose(packed, summaries[rank["r"]], rtol=1e-6, atol=1e-6)
        for p, s in zip(parts, summaries):
            p.copy_(s)

    monkeypatch.setattr(dist, "get_world_size", lambda group=None: world)
    monkeypatch.setattr(dist, "get_rank", lambda group=None: rank["r"])
    monkeypatch.setattr(dist, "all_gather", fake_all_gather)
    for r in range(world):
        rank["r"] = r
        y = seqpar.bidirectional_scan_seqpar(
            sl(t["u"], r), sl(t["delta"], r), t["A"], sl(t["B"], r), sl(t["C"], r), D=t["D"],
            z=sl(t["z"], r), delta_bias=t["delta_bias"], delta_softplus=True)
        assert rel_err(y.cpu().numpy(), sl(full, r).cpu().numpy()) <= REL_TOL


@pytest.mark.parametrize("shape", [(2, 48, 64, 4), (1, 7, 33, 4), (2, 16, 40, 3), (1, 5, 9, 6)])
def test_causal_conv1d_silu_matches_torch(shape):
    """The mixer prologue kernel (causal depthwise conv1d + bias + SiLU)
    against torch's conv1d with padding kernel-1 sliced to the sequence:
    vectorised (len multiple of 4, kernel <= 4) and general shapes."""
    import torch.nn.functional as F
    B, D, L, K = shape
    g = torch.Generator().manual_seed(L)
    x = torch.randn(B, D, L, generator=g).cuda()
    w = torch.randn(D, 1, K, generator=g).cuda()
    b = torch.randn(D, generator=g).cuda()
    want = F.silu(F.conv1d(x, w, b, padding=K - 1, groups=D)[..., :L])
    got = arm().causal_conv1d_silu(x, w, b)
    assert rel_err(got.cpu().numpy(), want.cpu().numpy()) <= 1e-5


@pytest.mark.parametrize("L", [1024, 1027])
def test_segment_summary_end_states_and_dt_sums(L):
    """The segment-summary entry (sequence parallelism): both traversals' end
    states from zero and the per-row sum of dt, on the lane kernel (length a
    multiple of 4: one shared pass) and on the fallback (1027: the row-tile
    scans plus a dt-sum kernel), against the oracle and a float64 sum."""
    B, D, N = 2, 40, 16
    x = _slow_decay_case(B, D, L, N, seed=L)
    t = cuda(x)
    hf, hb, sdt = arm().selective_scan_segment_summary(
        t["u"], t["delta"], t["A"], t["B"], t["C"], delta_bias=t["delta_bias"],
        delta_softplus=True)
    _, wlf = oracle.m1_scan(**x, nthreads=8)
    _, wlb = oracle.m1_scan(**x, reverse=True, nthreads=8)
    assert rel_err(hf.cpu().numpy(), wlf) <= REL_TOL
    assert rel_err(hb.cpu().numpy(), wlb) <= REL_TOL
    dt = np.logaddexp(0.0, x["delta"].astype(np.float64) + x["delta_bias"][None, :, None])
    assert rel_err(sdt.cpu().numpy(), dt.sum(-1)) <= REL_TOL


@pytest.mark.parametrize("segments,shape", [("auto", (2, 40, 1024, 16)), ("4", (2, 40, 1024, 16)),
                                            ("1", (1, 24, 512, 8)), ("auto", (1, 24, 1027, 16))])
def test_bidirectional_segment_two_phases(segments, shape, knobs):
    """The two-phase bidirectional form (summary, then finish from incoming
    states over the same workspace) equals the one-call functions it
    splits: the summary is bit-identical to the segment-summary entry and
    the finish to the sum entry with the same incoming states -- on the
    lane kernel with the automatic and forced segment counts, and on the
    one-call fallback (length not a multiple of 4)."""
    if segments != "auto":
        knobs(m1_segments=int(segments))
    B, D, L, N = shape
    x = _slow_decay_case(B, D, L, N, seed=L + N)
    t = cuda(x)
    a = arm()
    seg = a.BidirectionalSegment(t["u"], t["delta"], t["A"], t["B"], t["C"], D=t["D"], z=t["z"],
                                 delta_bias=t["delta_bias"], delta_softplus=True)
    assert (seg.ws_bytes > 0) == (L % 4 == 0)
    with pytest.raises(RuntimeError):
        seg.finish()
    got = seg.summary()
    want = a.selective_scan_segment_summary(t["u"], t["delta"], t["A"], t["B"], t["C"],
                                            delta_bias=t["delta_bias"], delta_softplus=True)
    for g, w in zip(got, want):
        assert torch.equal(g, w)
    g = torch.Generator().manual_seed(5)
    h0f = torch.randn(B, D, N, generator=g).cuda()
    h0b = torch.randn(B, D, N, generator=g).cuda()
    for init in [(h0f, h0b), (None, h0b), (h0f, None), (None, None)]:
        y = seg.finish(*init)
        ref = a.selective_scan_bidirectional_sum(**t, initial_states=init)
        assert torch.equal(y, ref)
    # and against the oracle: forward from h0f plus reverse from h0b
    yf, _ = oracle.m1_scan(**x, h0=h0f.cpu().numpy(), nthreads=8)
    yb, _ = oracle.m1_scan(**x, h0=h0b.cpu().numpy(), reverse=True, nthreads=8)
    assert rel_err(seg.finish(h0f, h0b).cpu().numpy(), yf + yb) <= REL_TOL


def _grid_views(x, h, w):
    """(b, c, h, w) numpy grid -> its row-major and column-major sequences."""
    b, c = x.shape[:2]
    return x.reshape(b, c, h * w), np.ascontiguousarray(x.transpose(0, 1, 3, 2)).reshape(b, c, w * h)


@pytest.mark.parametrize("shape", [(2, 32, 48, 40, 16, 2), (1, 12, 17, 33, 8, 1), (1, 8, 5, 64, 16, 1),
                                   (1, 24, 16, 20, 16, 2)])
def test_ss2d_in_place_vs_oracle(shape):
    """The one-call Mamba-1 SS2D (row-major traversals over the grid's own
    order, column-major ones per column, all summed into one output) against
    the f64 oracle run on the four traversal sequences: with groups, with
    d_state 8, with a grid whose length is not a multiple of 4 (the row
    traversals then take the fallback kernels), with columns longer than
    rows, and with groups of 12 channels, which the in-place call rejects
    (code 3) and ``ss2d_scan`` runs through stacked views.  These grids are
    too small to fill the GPU, so their columns are split in time (the
    sub-segment fold); the production-shape test covers unsplit columns."""
    B, D, H, W, N, G = shape
    rng = np.random.default_rng(H * W)
    f = lambda *s: rng.standard_normal(s).astype(np.float32)  # noqa: E731
    u, delta = f(B, D, H, W), (f(B, D, H, W) * 0.5).astype(np.float32)
    Bm, Cm = f(B, G, N, H, W), f(B, G, N, H, W)
    A = (-rng.uniform(0.1, 2.0, (D, N))).astype(np.float32)
    Dk, bias = f(D), (rng.uniform(-3, -1, D)).astype(np.float32)
    want = np.zeros((B, D, H, W))
    for order in ("row", "col"):
        pick = 0 if order == "row" else 1
        us, ds = _grid_views(u, H, W)[pick], _grid_views(delta, H, W)[pick]
        bs = _grid_views(Bm.reshape(B, G * N, H, W), H, W)[pick].reshape(B, G, N, H * W)
        cs = _grid_views(Cm.reshape(B, G * N, H, W), H, W)[pick].reshape(B, G, N, H * W)
        for rev in (False, True):
            y, _ = oracle.m1_scan(us, ds, A, bs, cs, D=Dk, delta_bias=bias, delta_softplus=True,
                                  reverse=rev, nthreads=8)
            y = y.reshape(B, D, H, W) if order == "row" else y.reshape(B, D, W, H).transpose(0, 1, 3, 2)
            want += y
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    args = (t(u), t(delta), t(A), t(Bm), t(Cm))
    kw = dict(D=t(Dk), delta_bias=t(bias))
    for merge, scale in (("sum", 1.0), ("mean", 0.25)):
        got = arm().ss2d_scan(*args, **kw, merge=merge)
        assert rel_err(got.cpu().numpy(), scale * want) <= REL_TOL
        if G > 1 and (D // G) % 8:
            with pytest.raises(RuntimeError, match="code 3"):
                arm().selective_scan_ss2d(*args, **kw, merge=merge)
        else:
            got = arm().selective_scan_ss2d(*args, **kw, merge=merge)
            assert rel_err(got.cpu().numpy(), scale * want) <= REL_TOL


def test_ss2d_production_shape_matches_planes():
    """The reference's SS2D workload shape (level-2 grid 192 x 160, inner
    dim 192, d_state 16): the in-place call's sum equals the sum of the four
    planes of merge="none" (transposed views through the bidirectional
    kernels), at batch 1 (columns split in time) and at batch 4 (one segment
    per column)."""
    g = torch.Generator(device="cuda").manual_seed(7)
    d, h, w, n = 192, 192, 160, 16
    r = lambda *s: torch.randn(*s, generator=g, device="cuda")  # noqa: E731
    a = arm()
    for b in (1, 4):
        u, delta = r(b, d, h, w), r(b, d, h, w) * 0.5
        Bm, Cm = r(b, n, h, w), r(b, n, h, w)
        A = -torch.rand(d, n, generator=g, device="cuda") * 2 - 0.1
        Dk, bias = r(d), torch.rand(d, generator=g, device="cuda") * 2 - 3
        planes = a.ss2d_scan(u, delta, A, Bm, Cm, D=Dk, delta_bias=bias, merge="none")
        calls = a.kernel_calls()
        got = a.ss2d_scan(u, delta, A, Bm, Cm, D=Dk, delta_bias=bias, merge="sum")
        assert a.kernel_calls() == calls + 1  # one library call
        want = sum(p.double() for p in planes)
        assert rel_err(got.cpu().numpy(), want.cpu().numpy()) <= REL_TOL
