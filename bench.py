"""Benchmark of the selective-scan hot path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--no-configs] [--no-prefill] [--no-e2e] [--no-cpu-baseline]

A step is one Mamba-1 ``selective_scan`` call over one batch of synthetic
input (fp32, seed = rank).  The headline workload ``prefill_scan`` is the
per-layer scan of BASELINE config 1 (HF Mamba-1 130M architecture prefill,
batch 8 x L 2048, d_inner 1536, d_state 16, softplus + delta_bias + D skip +
z gate, final state returned): 405.6 MB of algorithmic traffic per step,
larger than the 126 MB L2, so no flush is needed between steps.

value        -- algorithmic GB/s of the whole job (all ranks), inputs resident
                in HBM, CUDA-event timed, max over ranks.
e2e          -- the same metric through the reference-facing synchronous C
                entry point with pinned HOST buffers (H2D + kernels + D2H in
                the timed region).
roofline     -- the scan kernels' achieved algorithmic bandwidth against the
                measured HBM copy bandwidth (MEASURED_PEAKS.json).
cpu_baseline -- the oracle port of the reference's x86 CPU path (scalar
                recurrence, rows over all host threads), rank 0 only.
configs      -- (N = 1) every other BASELINE configuration as a sub-record:
                config 0, 2 (bf16 tensor path and fp32 path), 3 (per-rank
                MIMO, bf16), 4a (SS2D Mamba-3), 4b (bidirectional, L 262144)
                and config 1 (HF prefill tok/s), each with its time,
                algorithmic bytes and flops, roofline fraction and the CPU
                port timed on a stated sample (extrapolated linearly in L
                where the sample is shorter than the configuration).
                At N > 1: config 4b sequence-parallel over the ranks
                (strong scaling, one all_gather of segment carries).

Multi-GPU: one process per GPU (torchrun); each rank scans its own batch
(weak scaling over batch rows, no collective on the data path).
"""

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "scan GB/s & elems/s vs HBM roofline at 1/2/4/8 B200; Mamba-1 prefill tok/s"

PREFILL = dict(batch=8, dim=1536, len=2048, state=16,
               desc="Mamba-1 selective_scan at the 130M prefill shape (BASELINE config 1's "
                    "per-layer scan): batch 8 x L 2048, d_inner 1536, d_state 16, fp32")
CFG0 = dict(batch=1, dim=1536, len=2048, state=16,
            desc="BASELINE config 0: Mamba-1 selective_scan B1 D1536 L2048 N16 fp32")
CFG2 = dict(kind="siso", batch=4, heads=24, dv=64, dqk=128, len=4096, rank=1, pairs=64)
CFG4A = dict(kind="ss2d", batch=8, heads=6, dv=64, dqk=64, len=128 * 128, rank=1, pairs=32,
             grid=128)
CFG3 = dict(batch=8, heads=24, dv=64, dqk=128, len=8192, rank=4, pairs=64)
CFG4B = dict(batch=1, dim=1536, len=262144, state=16)
# the reference's SS2D workload (bench/bench_ss2d.py): level-1 grid, seed batch 4
M1SS2D = dict(batch=4, dim=96, h=384, w=320, state=16)


def m1_ss2d_inputs(dev):
    """Seeded grids of the SS2D workload: u, delta, A, B, C, D, delta_bias."""
    import torch
    w = M1SS2D
    g = torch.Generator(device=dev).manual_seed(0)
    rn = lambda *s: torch.randn(*s, generator=g, device=dev)  # noqa: E731
    gs = (w["batch"], w["dim"], w["h"], w["w"])
    u, delta = rn(*gs), rn(*gs) * 0.5
    Bm, Cm = rn(w["batch"], w["state"], w["h"], w["w"]), rn(w["batch"], w["state"], w["h"], w["w"])
    A = -torch.exp(torch.rand(w["dim"], w["state"], generator=g, device=dev) * 2)
    return (u, delta, A, Bm, Cm, torch.ones(w["dim"], device=dev),
            torch.full((w["dim"],), -2.0, device=dev))


def m1_ss2d_bytes(w):
    """u, delta and out (batch, dim, h, w) plus B, C (batch, state, h, w), fp32."""
    L = w["h"] * w["w"]
    return 4.0 * L * w["batch"] * (3 * w["dim"] + 2 * w["state"])

# algorithmic bytes and flops of the configurations (per call)
CFG_BYTES = {"cfg0": 50.80e6, "cfg2_bf16": 117.4e6, "cfg2_fp32": None, "cfg3": 1772e6,
             "cfg4a": 492.8e6, "cfg4b": 6.476e9}
CFG_FLOPS = {"cfg2_bf16": 22.5e9, "cfg2_fp32": 12.9e9, "cfg3": 824.6e9, "cfg4a": 51.5e9}


def m3_inputs(w, device, seed=0):
    """Synthetic Mamba-3 inputs with BASELINE config 2's distributions."""
    import torch
    g = torch.Generator(device=device).manual_seed(seed)
    B, H, P, N, L, R = w["batch"], w["heads"], w["dv"], w["dqk"], w["len"], w["rank"]
    rn = lambda *s: torch.randn(*s, generator=g, device=device)  # noqa: E731
    dt = torch.nn.functional.softplus(rn(B, H, L) - 4)
    A = -torch.exp(torch.rand(H, generator=g, device=device) * np.log(16))
    # per-step rotation tanh(angle) * pi ~ U[0, pi): angle = atanh(U[0, 1))
    ang = torch.atanh(torch.rand(B, L, H, w["pairs"], generator=g, device=device) * 0.999)
    x = dict(v=rn(B, L, H, P), adt=A.view(1, H, 1) * dt, dt=dt, trap=rn(B, H, L),
             D=1 + 0.1 * rn(H), angles=ang)
    if w["kind"] == "mimo":
        x.update(q=rn(B, L, R, N) / np.sqrt(N * R), k=rn(B, L, R, N) / np.sqrt(N * R),
                 q_bias=torch.zeros(H, R, N, device=device),
                 k_bias=torch.zeros(H, R, N, device=device),
                 psi=rn(H, R, P), zeta=rn(H, R, P), phi=rn(H, R, P), z=rn(B, L, H, P))
    else:
        x.update(q=rn(B, L, 1, N) / np.sqrt(N), k=rn(B, L, 1, N) / np.sqrt(N),
                 q_bias=torch.zeros(H, N, device=device), k_bias=torch.zeros(H, N, device=device))
    return x


def m3_bytes(w):
    B, H, P, N, L, R = w["batch"], w["heads"], w["dv"], w["dqk"], w["len"], w["rank"]
    # q, k, v, y, dt/adt/trap, angles (+ final state for SISO, z for MIMO)
    b = 2 * B * L * R * N + 2 * B * L * H * P + 3 * B * H * L + B * L * H * w["pairs"]
    if w["kind"] == "mimo":
        b += B * L * H * P
    if w["kind"] == "siso":
        b += B * H * P * N
    return 4 * b


def m3_bytes_bf16(w):
    """Config 2 as specified: q, k, v, y and angles (shared by the heads) in
    bf16; dt, adt, trap and the final state in fp32."""
    B, H, P, N, L = w["batch"], w["heads"], w["dv"], w["dqk"], w["len"]
    return (2 * (2 * B * L * N + 2 * B * L * H * P + B * L * w["pairs"])
            + 4 * (3 * B * H * L + B * H * P * N))


def mixer_inputs(w, device, seed=0):
    """Synthetic in_proj output and mixer parameters for the prologue."""
    import torch
    from armhackathon_b200.mamba3_mixer import proj_width
    g = torch.Generator(device=device).manual_seed(seed)
    B, H, P, N, L, R = w["batch"], w["heads"], w["dv"], w["dqk"], w["len"], w["rank"]
    W = proj_width(H, P, N, R, w["pairs"])
    rn = lambda *s: torch.randn(*s, generator=g, device=device)  # noqa: E731
    return dict(proj=rn(B, L, W), nheads=H, headdim=P, d_state=N, n_angles=w["pairs"],
                dt_bias=rn(H) - 2, B_norm_weight=1 + 0.1 * rn(N), C_norm_weight=1 + 0.1 * rn(N),
                mimo_rank=R)


def mixer_bytes(w):
    """Read one in_proj row, write the same number of floats (z, x, q, k,
    dt, adt, trap, angles), per (batch, step); parameters are negligible."""
    from armhackathon_b200.mamba3_mixer import proj_width
    W = proj_width(w["heads"], w["dv"], w["dqk"], w["rank"], w["pairs"])
    return 2 * 4 * w["batch"] * w["len"] * W


def torch_mixer_prologue(proj, nheads, headdim, d_state, n_angles, dt_bias, B_norm_weight,
                         C_norm_weight, mimo_rank, A_floor=1e-4, eps=1e-5):
    """The same prologue as separate torch ops on the GPU (how the reference's
    mixer runs it), for comparison with the fused kernel."""
    import torch
    import torch.nn.functional as F
    b, l, _ = proj.shape
    hp, rn = nheads * headdim, mimo_rank * d_state
    z, x, Bm, Cm, ddt, dda, trap, ang = torch.split(
        proj, [hp, hp, rn, rn, nheads, nheads, nheads, n_angles], dim=-1)
    a = -(dda.clamp_min(0) + torch.reciprocal(1 - dda.clamp_max(0)))
    a = a.clamp_max(-A_floor)
    dt = F.softplus(ddt + dt_bias)

    def rms(t, wt):
        t = t.reshape(b, l, mimo_rank, d_state)
        return t * torch.rsqrt(t.square().mean(-1, keepdim=True) + eps) * wt
    return (z.reshape(b, l, nheads, headdim).contiguous(),
            x.reshape(b, l, nheads, headdim).contiguous(), rms(Cm, C_norm_weight),
            rms(Bm, B_norm_weight), dt.permute(0, 2, 1).contiguous(),
            (a * dt).permute(0, 2, 1).contiguous(), trap.permute(0, 2, 1).contiguous(),
            ang.contiguous())


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def mufu_roofline(w, k_ms, clocks, launches_per_call):
    """The Mamba-1 scan's second roof: one exp per (batch, channel, step,
    state) is the algorithm's minimum (the reference computes exactly that);
    the MUFU unit issues 16 per clock per SM (nominal), at the SM clock
    sampled during the timed region.  One launch per call means the lane
    kernel ran unsplit, one exp per (step, state); three mean a time split
    (pass 1, carry, pass 2), whose rescan adds the exps of segments 1..S-2."""
    import torch
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    mhz = clocks.get("sm_mhz") or clocks.get("sm_max_mhz") or 1965.0
    exps = w["batch"] * w["dim"] * w["len"] * w["state"]
    achieved = exps / (k_ms * 1e-3) / 1e9
    peak = 16 * sms * mhz * 1e6 / 1e9
    return {"bound": "mufu", "achieved": achieved, "peak": peak, "unit": "Gexp/s",
            "frac": achieved / peak, "peak_source": "nominal 16/clk/SM x sampled SM clock",
            "launches_per_call": launches_per_call,
            "executed_per_algorithmic": 1.0 if launches_per_call == 1 else None,
            "note": "plus the softplus/silu transcendentals, 4 per (row, step)"}


def algorithmic_bytes(w):
    B, D, L, N = w["batch"], w["dim"], w["len"], w["state"]
    return 4 * (4 * B * D * L + 2 * B * N * L + D * N + 2 * D + B * D * N)


def make_inputs(w, device, seed=0):
    """Synthetic inputs with BASELINE config 0's distributions."""
    import torch
    g = torch.Generator(device=device).manual_seed(seed)
    B, D, L, N = w["batch"], w["dim"], w["len"], w["state"]
    rn = lambda *s: torch.randn(*s, generator=g, device=device)  # noqa: E731
    dt = torch.exp(torch.empty(D, device=device).uniform_(np.log(1e-3), np.log(1e-1),
                                                           generator=g))
    return dict(u=rn(B, D, L), delta=rn(B, D, L), z=rn(B, D, L),
                A=-torch.arange(1, N + 1, device=device, dtype=torch.float32).repeat(D, 1),
                B=rn(B, N, L), C=rn(B, N, L), D=torch.ones(D, device=device),
                delta_bias=torch.log(torch.expm1(dt)))


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None

    def __enter__(self):
        import tempfile
        self.path = tempfile.mktemp(suffix=".csv")
        try:
            # -f: nvidia-smi writes (and flushes) each sample to the file
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "100", "-f", self.path],
                stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            try:
                with open(self.path) as f:
                    self.lines = [ln for ln in f.read().splitlines() if ln.strip()]
                os.unlink(self.path)
            except OSError:
                pass

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in getattr(self, "lines", []):
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for name, val in zip(names, f[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def prefill_tok_s(dev, batch, length, steps=3, warmup=2):
    """random-init Mamba-1 130M architecture (24 layers,
    d_model 768, expand 2, d_state 16, d_conv 4, dt_rank 48, vocab 50280,
    weights N(0, 0.02), A_log = log(1..16), dt bias as config 0), fp32, HF
    transformers MambaForCausalLM with patch() routing the scan to this
    library; a full forward (logits included) over random token ids.  Returns
    tokens/s (CUDA events, median of `steps`)."""
    import torch
    from transformers import MambaConfig, MambaForCausalLM
    import armhackathon_b200 as arm
    cfg = MambaConfig(vocab_size=50280, hidden_size=768, state_size=16, num_hidden_layers=24,
                      expand=2, conv_kernel=4, time_step_rank=48, initializer_range=0.02,
                      use_cache=False)
    torch.manual_seed(0)
    model = MambaForCausalLM(cfg).to(dev).eval()
    with torch.no_grad():
        g = torch.Generator(device="cpu").manual_seed(0)
        for layer in model.backbone.layers:
            mx = layer.mixer
            mx.A_log.copy_(torch.log(torch.arange(1, 17, dtype=torch.float32)).repeat(
                mx.A_log.shape[0], 1))
            dt = torch.exp(torch.empty(mx.dt_proj.bias.shape).uniform_(
                np.log(1e-3), np.log(1e-1), generator=g))
            mx.dt_proj.bias.copy_(torch.log(torch.expm1(dt)))
    ids = torch.randint(0, 50280, (batch, length), device=dev)
    arm.patch()
    try:
        times = []
        with torch.no_grad():
            for i in range(warmup + steps):
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record()
                model(ids)
                b.record()
                torch.cuda.synchronize()
                if i >= warmup:
                    times.append(a.elapsed_time(b))
        engaged = arm.stats()["fast_calls"] > 0
    finally:
        arm.unpatch()
    del model
    torch.cuda.empty_cache()
    ms = statistics.median(times)
    return {"tok_s": batch * length / (ms * 1e-3), "ms": ms, "batch": batch, "len": length,
            "kernel_engaged": engaged}


def cpu_baseline(w):
    """Oracle port of the reference's CPU path on a bounded sample: all host
    threads, batch row 0 only (1/batch of the workload)."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle
    nthreads = oracle.hw_threads()
    rng = np.random.default_rng(0)
    D, L, N = w["dim"], w["len"], w["state"]
    f = lambda *s: rng.standard_normal(s).astype(np.float32)  # noqa: E731
    dt = np.exp(rng.uniform(np.log(1e-3), np.log(1e-1), D))
    inp = dict(u=f(1, D, L), delta=f(1, D, L), z=f(1, D, L),
               A=-np.tile(np.arange(1, N + 1, dtype=np.float32), (D, 1)), B=f(1, N, L),
               C=f(1, N, L), D=np.ones(D, np.float32),
               delta_bias=np.log(np.expm1(dt)).astype(np.float32))
    oracle.m1_scan(**inp, delta_softplus=True, dtype=np.float32, nthreads=nthreads)
    reps, t_total = 0, 0.0
    while t_total < 3.0 and reps < 50:
        t0 = time.perf_counter()
        oracle.m1_scan(**inp, delta_softplus=True, dtype=np.float32, nthreads=nthreads)
        t_total += time.perf_counter() - t0
        reps += 1
    t = t_total / reps
    sample = dict(w, batch=1)
    return {"value": algorithmic_bytes(sample) / t / 1e9, "unit": "GB/s", "cores": nthreads,
            "kind": "port",
            "sample": f"batch row 0 of the workload (1x{D}x{L}, N={N}), {reps} reps"}


def sm_peaks(clock_mhz=None):
    """Compute peaks for the roofline of a sub-record: measured bf16 tensor
    throughput (MEASURED_PEAKS.json, burst) and the nominal fp32 CUDA-core
    rate (148 SMs x 128 FMA x 2 at the SM clock)."""
    p = ROOT / "MEASURED_PEAKS.json"
    bf16 = 1590.0
    mhz = clock_mhz or 1965.0
    if p.exists():
        d = json.loads(p.read_text())
        bf16 = float(d.get("bf16_tflops", bf16))
        mhz = clock_mhz or float(d.get("sm_max_mhz", mhz))
    return bf16, 148 * 128 * 2 * mhz * 1e6 / 1e12


def time_call(fn, steps, warmup, graph=True):
    """Device time per call (ms), CUDA events around `steps` calls.  With
    graph=True the calls are captured once into a CUDA graph and replayed,
    so host-side launch overhead does not enter the figure of small ops;
    falls back to eager launches if capture fails."""
    import torch
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    g = None
    if graph:
        try:
            s = torch.cuda.Stream()
            s.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(s):
                fn()
            torch.cuda.current_stream().wait_stream(s)
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                for _ in range(steps):
                    fn()
            g.replay()
            torch.cuda.synchronize()
        except Exception:  # noqa: BLE001 -- eager timing below
            g = None
            torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    if g is not None:
        g.replay()
    else:
        for _ in range(steps):
            fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / steps, ("cuda graph" if g is not None else "eager")


def roof(ms, nbytes, flops, hbm, tc_peak_tflops):
    """Roofline of one sub-record: the slower of bytes / HBM and flops /
    compute peak, against the measured time."""
    t_mem = nbytes / (hbm * 1e9) if nbytes else 0.0
    t_cmp = flops / (tc_peak_tflops * 1e12) if flops else 0.0
    bound = "hbm" if t_mem >= t_cmp else "compute"
    t = max(t_mem, t_cmp)
    return {"bound": bound, "frac": t / (ms * 1e-3),
            "achieved_gbs": nbytes / (ms * 1e-3) / 1e9 if nbytes else None,
            "achieved_tflops": flops / (ms * 1e-3) / 1e12 if flops else None}


def cpu_port(kind, nthreads):
    """The oracle port of the reference's CPU path for one configuration on
    a bounded sample; returns (ms per full configuration, sample text)."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle
    rng = np.random.default_rng(0)
    f = lambda *s: rng.standard_normal(s).astype(np.float32)  # noqa: E731

    def clock(fn):
        fn()
        t0 = time.perf_counter()
        fn()
        return time.perf_counter() - t0

    if kind in ("cfg0", "cfg4b"):
        D, N = 1536, 16
        L = 2048 if kind == "cfg0" else 16384
        full_L = 2048 if kind == "cfg0" else 262144
        dt = np.exp(rng.uniform(np.log(1e-3), np.log(1e-1), D))
        inp = dict(u=f(1, D, L), delta=f(1, D, L), z=f(1, D, L),
                   A=-np.tile(np.arange(1, N + 1, dtype=np.float32), (D, 1)), B=f(1, N, L),
                   C=f(1, N, L), D=np.ones(D, np.float32),
                   delta_bias=np.log(np.expm1(dt)).astype(np.float32))
        if kind == "cfg0":
            t = clock(lambda: oracle.m1_scan(**inp, delta_softplus=True, dtype=np.float32,
                                             nthreads=nthreads))
        else:
            t = clock(lambda: oracle.m1_scan_bidir(**inp, delta_softplus=True, dtype=np.float32,
                                                   nthreads=nthreads))
        return t * 1e3 * full_L / L, f"1x{D}x{L} (x{full_L // L} extrapolated)"
    if kind in ("cfg2", "cfg4a"):
        w = CFG2 if kind == "cfg2" else CFG4A
        B, H, P, N = w["batch"], w["heads"], w["dv"], w["dqk"]
        L = 1024
        full = w["len"] * (4 if kind == "cfg4a" else 1)  # 4a: four traversals
        dt = np.log1p(np.exp(f(B, H, L) - 4))
        A = -np.exp(rng.uniform(0, np.log(16), H)).astype(np.float32)
        cos, sin = oracle.angles_to_cos_sin(f(B, L, H, w["pairs"]), dt, N // 2)
        args = (f(B, L, 1, N) / np.sqrt(N), f(B, L, 1, N) / np.sqrt(N), f(B, L, H, P),
                A[None, :, None] * dt, dt, f(B, H, L), np.zeros((H, N), np.float32),
                np.zeros((H, N), np.float32), cos, sin)
        t = clock(lambda: oracle.m3_siso(*args, D=np.ones(H, np.float32), dtype=np.float32,
                                         nthreads=nthreads))
        return t * 1e3 * full / L, f"{B}x{H} heads, L {L} (x{full / L:g} extrapolated)"
    if kind == "cfg3":
        w = CFG3
        B, H, P, N, R = w["batch"], w["heads"], w["dv"], w["dqk"], w["rank"]
        B, L = 1, 256
        dt = np.log1p(np.exp(f(B, H, L) - 4))
        A = -np.exp(rng.uniform(0, np.log(16), H)).astype(np.float32)
        cos, sin = oracle.angles_to_cos_sin(f(B, L, H, w["pairs"]), dt, N // 2)
        t = clock(lambda: oracle.m3_mimo_x(f(B, L, H, P, R), f(B, L, N, R), f(B, L, N, R),
                                           A[None, :, None] * dt, dt, f(B, H, L), cos, sin,
                                           dtype=np.float32, nthreads=nthreads))
        scale = w["batch"] * w["len"] / (B * L)
        return t * 1e3 * scale, f"1x{H} heads, L {L} (x{scale:g} extrapolated)"
    if kind == "m1_ss2d":
        w = M1SS2D
        d, n, L = 16, w["state"], w["h"] * w["w"]
        inp = dict(u=f(1, d, L), delta=f(1, d, L), A=-np.tile(np.arange(1, n + 1, dtype=np.float32),
                                                              (d, 1)),
                   B=f(1, n, L), C=f(1, n, L), D=np.ones(d, np.float32),
                   delta_bias=np.full(d, -2.0, np.float32))
        # two orderings, each a fused bidirectional pair (the reference's composition)
        t = 2 * clock(lambda: oracle.m1_scan_bidir(**inp, delta_softplus=True, dtype=np.float32,
                                                   nthreads=nthreads))
        scale = w["batch"] * w["dim"] / d
        return t * 1e3 * scale, f"1x{d} channels of the grid (x{scale:g} extrapolated)"
    raise ValueError(kind)


def config_suite(args, dev, hbm, clocks):
    """Every BASELINE configuration besides the headline, one sub-record each."""
    import torch
    import armhackathon_b200 as arm
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle
    nthreads = oracle.hw_threads()
    mhz = clocks.get("sm_mhz") if clocks else None
    bf16_peak, fp32_peak = sm_peaks(mhz)
    out = {}
    steps = max(3, min(args.steps, 20))

    def record(name, ms, how, nbytes, flops, peak, desc, cpu_kind):
        r = {"desc": desc, "ms": ms, "timing": how, "bytes": nbytes, "flops": flops,
             "roofline": roof(ms, nbytes, flops, hbm, peak)}
        if cpu_kind and not args.no_cpu_baseline:
            cms, sample = cpu_port(cpu_kind, nthreads)
            r["cpu_baseline"] = {"ms": cms, "cores": nthreads, "kind": "port", "sample": sample,
                                 "speedup": cms / ms}
        out[name] = r

    # config 0 (L2 flushed between calls is not possible inside the graph:
    # 50.8 MB fits L2, so the figure is an L2-warm one; the headline is not)
    x = make_inputs(CFG0, dev)
    f0 = lambda: arm.selective_scan(x["u"], x["delta"], x["A"], x["B"], x["C"], D=x["D"],  # noqa: E731
                                    z=x["z"], delta_bias=x["delta_bias"], delta_softplus=True,
                                    return_last_state=True)
    ms, how = time_call(f0, steps, args.warmup)
    record("cfg0", ms, how, CFG_BYTES["cfg0"], None, bf16_peak, CFG0["desc"] +
           " (L2-warm: the inputs fit the 126 MB L2)", "cfg0")
    del x

    # config 2: bf16 inputs on the tensor cores, and the fp32 chunk path
    x = m3_inputs(CFG2, dev)
    bf = torch.bfloat16
    xb = dict(x, q=x["q"].to(bf), k=x["k"].to(bf), v=x["v"].to(bf),
              angles=x["angles"][:, :, :1, :].to(bf).contiguous())
    ms, how = time_call(lambda: arm.mamba3_scan(**xb, return_last_state=True, precision="bf16"),
                        steps, args.warmup)
    record("cfg2_bf16", ms, how, CFG_BYTES["cfg2_bf16"], CFG_FLOPS["cfg2_bf16"], bf16_peak,
           "BASELINE config 2: Mamba-3 SISO B4 H24 P64 N128 L4096, bf16 inputs, fp32 state, "
           "tcgen05 kernel with the angle pre-pass fused", "cfg2")
    ms, how = time_call(lambda: arm.mamba3_scan(**x, return_last_state=True), steps, args.warmup)
    record("cfg2_fp32", ms, how, m3_bytes(CFG2), CFG_FLOPS["cfg2_fp32"], fp32_peak,
           "config 2's shape with fp32 inputs on the fp32 chunk kernels (CUDA cores; "
           "flops are the sequential form's)", None)
    del x, xb

    # config 3: per-rank MIMO, bf16
    w = CFG3
    g = torch.Generator(device=dev).manual_seed(0)
    rn = lambda *s: torch.randn(*s, generator=g, device=dev)  # noqa: E731
    B, L, H, P, N, R = w["batch"], w["len"], w["heads"], w["dv"], w["dqk"], w["rank"]
    dt = torch.nn.functional.softplus(rn(B, H, L) - 4)
    A = -torch.exp(torch.rand(H, generator=g, device=dev) * np.log(16))
    X = rn(B, L, H, P, R).to(bf)
    Bm = (rn(B, L, N, R) / (N * R) ** 0.5).to(bf)
    Cm = (rn(B, L, N, R) / (N * R) ** 0.5).to(bf)
    ang = torch.atanh(torch.rand(B, L, w["pairs"], generator=g, device=dev) * 0.999)
    trap, adt = rn(B, H, L), A.view(1, H, 1) * dt
    ms, how = time_call(lambda: arm.mamba3_mimo_x_scan(X, Bm, Cm, adt, dt, trap, angles=ang,
                                                       return_last_state=True),
                        max(2, steps // 4), 2)
    record("cfg3", ms, how, CFG_BYTES["cfg3"], CFG_FLOPS["cfg3"], bf16_peak,
           "BASELINE config 3: Mamba-3 MIMO r4 with X per rank (B8 H24 P64 N128 L8192), bf16 "
           "inputs, fp32 state, tcgen05 kernel (32-step tiles of 128 (step, rank) rows)", "cfg3")
    del X, Bm, Cm

    # config 4a: SS2D Mamba-3, fp32
    x = m3_inputs(CFG4A, dev)
    Bq, Hh, gd = CFG4A["batch"], CFG4A["heads"], CFG4A["grid"]
    grid = lambda t: t.reshape(Bq, gd, gd, *t.shape[2:])  # noqa: E731
    hm = lambda t: t.reshape(Bq, Hh, gd, gd)  # noqa: E731
    xs = dict(q=grid(x["q"]), k=grid(x["k"]), v=grid(x["v"]), angles=grid(x["angles"]),
              adt=hm(x["adt"]), dt=hm(x["dt"]), trap=hm(x["trap"]), q_bias=x["q_bias"],
              k_bias=x["k_bias"], D=x["D"])
    ms, how = time_call(lambda: arm.ss2d_scan_mamba3(**xs), max(2, steps // 4), 2)
    record("cfg4a", ms, how, CFG_BYTES["cfg4a"], CFG_FLOPS["cfg4a"], fp32_peak,
           "BASELINE config 4a: SS2D Mamba-3 SISO, 128x128 grid, B8 H6 P64 N64 fp32, four "
           "traversals summed in place", "cfg4a")
    del x, xs

    # config 4b: bidirectional Mamba-1, one sequence of 262144 steps
    x = make_inputs(CFG4B, dev)
    ms, how = time_call(lambda: arm.bidirectional_scan(
        x["u"], x["delta"], x["A"], x["B"], x["C"], D=x["D"], z=x["z"],
        delta_bias=x["delta_bias"], delta_softplus=True, merge="sum"), max(2, steps // 4), 2)
    record("cfg4b", ms, how, CFG_BYTES["cfg4b"], None, bf16_peak,
           "BASELINE config 4b: Mamba-1 bidirectional D1536 N16 L262144 fp32, summed, 1 GPU",
           "cfg4b")
    del x
    torch.cuda.empty_cache()

    # Mamba-1 SS2D at the reference's level-1 diffusion grid, one call
    w = M1SS2D
    u, delta, A, Bm, Cm, Dk, bias = m1_ss2d_inputs(dev)
    ms, how = time_call(lambda: arm.ss2d_scan(u, delta, A, Bm, Cm, D=Dk, delta_bias=bias),
                        steps, args.warmup)
    record("m1_ss2d", ms, how, m1_ss2d_bytes(w), None, bf16_peak,
           "Mamba-1 SS2D, four traversals summed, B4 D96 N16 on the reference's level-1 "
           "384x320 diffusion grid, fp32, grids read in place", "m1_ss2d")
    from armhackathon_b200.ss2d import grid_to_views, views_to_grid

    def views_path():
        both = arm.selective_scan_bidirectional_sum(
            grid_to_views(u), grid_to_views(delta), A, grid_to_views(Bm), grid_to_views(Cm), D=Dk,
            delta_bias=bias, delta_softplus=True)
        rs, cs = views_to_grid(both[:w["batch"]], both[w["batch"]:], w["h"], w["w"])
        return rs + cs
    out["m1_ss2d"]["views_path_ms"], _ = time_call(views_path, steps, args.warmup, graph=False)
    del u, delta, Bm, Cm

    # Mamba-3 mixer prologue (in_proj output -> scan inputs) at config 2's shape
    wm = dict(kind="mixer", batch=4, heads=24, dv=64, dqk=128, len=4096, rank=1, pairs=32)
    xm = mixer_inputs(wm, dev)
    ms, how = time_call(lambda: arm.mamba3_mixer_prologue(**xm), steps, args.warmup)
    t_ms, _ = time_call(lambda: torch_mixer_prologue(**xm), steps, args.warmup, graph=False)
    record("m3_mixer_prologue", ms, how, mixer_bytes(wm), None, bf16_peak,
           "Mamba-3 mixer prologue (split, softplus / heavy-tail gates, B/C RMSNorm, "
           "relayouts) at config 2's shape, 3432-wide in_proj rows, fp32, one kernel", None)
    out["m3_mixer_prologue"]["torch_ops_ms"] = t_ms
    del xm

    # config 1: HF prefill tokens/s
    if not args.no_prefill:
        out["cfg1_prefill"] = {
            "desc": "BASELINE config 1: random-init Mamba-1 130M architecture, fp32, patched HF "
                    "MambaForCausalLM full forward (logits included), 1 GPU",
            "runs": [prefill_tok_s(dev, 8, 2048), prefill_tok_s(dev, 1, 32768)]}
    return out


def run_seqpar_4b(args, dev, rank, world):
    """Config 4b sequence-parallel over the ranks (strong scaling)."""
    import torch
    import torch.distributed as dist
    from armhackathon_b200.seqpar import bidirectional_scan_seqpar
    seg = CFG4B["len"] // world
    x = make_inputs(dict(CFG4B, len=seg), dev, seed=rank)
    step = lambda: bidirectional_scan_seqpar(  # noqa: E731
        x["u"], x["delta"], x["A"], x["B"], x["C"], D=x["D"], z=x["z"],
        delta_bias=x["delta_bias"], delta_softplus=True)
    for _ in range(3):
        step()
    torch.cuda.synchronize()
    dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n = 5
    a.record()
    for _ in range(n):
        step()
    b.record()
    torch.cuda.synchronize()
    t = torch.tensor([a.elapsed_time(b) / n], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    return {"desc": f"BASELINE config 4b over {world} GPUs: one L 262144 sequence split in "
                    f"{world} segments (strong scaling; one all_gather of segment carries)",
            "ms": ms, "bytes": CFG_BYTES["cfg4b"], "GB_s": CFG_BYTES["cfg4b"] / (ms * 1e-3) / 1e9,
            "n_gpus": world}


def run_reference(args):
    """--impl reference: the reference's CPU path (scalar recurrence over rows
    on all host threads; the oracle port, as the Rust crate has no toolchain
    here) on the headline workload, plus every other configuration as a
    sub-record on a stated sample.  Rank 0 only."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle
    if int(os.environ.get("RANK", "0")) != 0:
        return
    nthreads = oracle.hw_threads()
    rng = np.random.default_rng(0)
    w = PREFILL
    B, D, L, N = w["batch"], w["dim"], w["len"], w["state"]
    f = lambda *s: rng.standard_normal(s).astype(np.float32)  # noqa: E731
    dt = np.exp(rng.uniform(np.log(1e-3), np.log(1e-1), D))
    # a step is one batch row of the workload (1/8 of it, bounded CPU time);
    # the line's value is that row's GB/s
    inp = dict(u=f(1, D, L), delta=f(1, D, L), z=f(1, D, L),
               A=-np.tile(np.arange(1, N + 1, dtype=np.float32), (D, 1)), B=f(1, N, L),
               C=f(1, N, L), D=np.ones(D, np.float32),
               delta_bias=np.log(np.expm1(dt)).astype(np.float32))
    for _ in range(args.warmup):
        oracle.m1_scan(**inp, delta_softplus=True, dtype=np.float32, nthreads=nthreads)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        oracle.m1_scan(**inp, delta_softplus=True, dtype=np.float32, nthreads=nthreads)
        times.append(time.perf_counter() - t0)
    t = statistics.median(times)
    gbs = algorithmic_bytes(dict(w, batch=1)) / t / 1e9
    line = {"impl": "reference", "metric": METRIC, "value": gbs, "unit": "GB/s", "n_gpus": 0,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": t * 1e3 * B,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seed 0, BASELINE config 0 distributions)",
            "config": {"workload": "prefill_scan", "desc": w["desc"], "batch": B, "dim": D,
                       "len": L, "state": N},
            "elems_per_s": D * L / t,
            "cpu_baseline": {"value": gbs, "unit": "GB/s", "cores": nthreads, "kind": "port",
                             "sample": f"batch row 0 of the workload (1x{D}x{L}, N={N}) per "
                                       "step; ms_per_step is scaled to the full batch"},
            "e2e": {"value": gbs, "unit": "GB/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    if not args.no_configs:
        line["configs"] = {}
        for k in ("cfg0", "cfg2", "cfg3", "cfg4a", "cfg4b", "m1_ss2d"):
            ms, sample = cpu_port(k, nthreads)
            line["configs"][k] = {"ms": ms, "cores": nthreads, "kind": "port", "sample": sample}
    print(json.dumps(line), flush=True)


def profile_case(case):
    """Three calls of one case, for ncu captures: prefill -- the headline
    scan; bidir_slice -- config 4b's bidirectional sum on 256 of its 1536
    channels (1.3 GB on the device); cfg3_eighth -- config 3's per-rank MIMO
    on B2 x L4096 (1/8 of it); cfg2_bf16 / cfg2_fp32 -- config 2 on the
    tensor-core and the fp32 chunk path; cfg4a -- config 4a's SS2D; mixer --
    the Mamba-3 mixer prologue at config 2's shape; tile_prefill -- the
    headline scan on the row-tile fallback kernel; m1_ss2d -- the Mamba-1
    SS2D workload (level-1 diffusion grid)."""
    import torch
    import armhackathon_b200 as arm
    dev = torch.device("cuda", 0)
    if case == "prefill":
        x = make_inputs(PREFILL, dev)
        f = lambda: arm.selective_scan(x["u"], x["delta"], x["A"], x["B"], x["C"], D=x["D"],  # noqa: E731
                                       z=x["z"], delta_bias=x["delta_bias"], delta_softplus=True,
                                       return_last_state=True)
    elif case == "bidir_slice":
        x = make_inputs(dict(CFG4B, dim=256), dev)
        f = lambda: arm.bidirectional_scan(x["u"], x["delta"], x["A"], x["B"], x["C"], D=x["D"],  # noqa: E731
                                           z=x["z"], delta_bias=x["delta_bias"],
                                           delta_softplus=True, merge="sum")
    elif case in ("cfg2_bf16", "cfg2_fp32"):
        x = m3_inputs(CFG2, dev)
        if case == "cfg2_bf16":
            bf = torch.bfloat16
            x = dict(x, q=x["q"].to(bf), k=x["k"].to(bf), v=x["v"].to(bf),
                     angles=x["angles"][:, :, :1, :].to(bf).contiguous())
            f = lambda: arm.mamba3_scan(**x, return_last_state=True, precision="bf16")  # noqa: E731
        else:
            f = lambda: arm.mamba3_scan(**x, return_last_state=True)  # noqa: E731
    elif case == "cfg4a":
        x = m3_inputs(CFG4A, dev)
        Bq, Hh, gd = CFG4A["batch"], CFG4A["heads"], CFG4A["grid"]
        grid = lambda t: t.reshape(Bq, gd, gd, *t.shape[2:])  # noqa: E731
        hm = lambda t: t.reshape(Bq, Hh, gd, gd)  # noqa: E731
        xs = dict(q=grid(x["q"]), k=grid(x["k"]), v=grid(x["v"]), angles=grid(x["angles"]),
                  adt=hm(x["adt"]), dt=hm(x["dt"]), trap=hm(x["trap"]), q_bias=x["q_bias"],
                  k_bias=x["k_bias"], D=x["D"])
        f = lambda: arm.ss2d_scan_mamba3(**xs)  # noqa: E731
    elif case == "mixer":
        wm = dict(kind="mixer", batch=4, heads=24, dv=64, dqk=128, len=4096, rank=1, pairs=32)
        xm = mixer_inputs(wm, dev)
        f = lambda: arm.mamba3_mixer_prologue(**xm)  # noqa: E731
    elif case == "m1_ss2d":
        u, delta, A, Bm, Cm, Dk, bias = m1_ss2d_inputs(dev)
        f = lambda: arm.ss2d_scan(u, delta, A, Bm, Cm, D=Dk, delta_bias=bias)  # noqa: E731
    elif case == "tile_prefill":
        from armhackathon_b200 import _ffi
        _ffi.set_kernel_override("m1_kernel", _ffi.M1_KERNELS["tile"])
        x = make_inputs(PREFILL, dev)
        f = lambda: arm.selective_scan(x["u"], x["delta"], x["A"], x["B"], x["C"], D=x["D"],  # noqa: E731
                                       z=x["z"], delta_bias=x["delta_bias"], delta_softplus=True,
                                       return_last_state=True)
    else:
        g = torch.Generator(device=dev).manual_seed(0)
        rn = lambda *s: torch.randn(*s, generator=g, device=dev)  # noqa: E731
        B, L, H, P, N, R = 2, 4096, 24, 64, 128, 4
        dt = torch.nn.functional.softplus(rn(B, H, L) - 4)
        X = rn(B, L, H, P, R).bfloat16()
        Bm = (rn(B, L, N, R) / (N * R) ** 0.5).bfloat16()
        Cm = (rn(B, L, N, R) / (N * R) ** 0.5).bfloat16()
        ang = torch.atanh(torch.rand(B, L, 64, generator=g, device=dev) * 0.999)
        trap = rn(B, H, L)
        f = lambda: arm.mamba3_mimo_x_scan(X, Bm, Cm, -dt, dt, trap, angles=ang,  # noqa: E731
                                           return_last_state=True)
    for _ in range(3):
        f()
    torch.cuda.synchronize()
    print(f"profile case {case}: 3 calls done", file=sys.stderr)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-configs", action="store_true",
                    help="skip the sub-records of the other BASELINE configurations")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-prefill", action="store_true",
                    help="skip the config-1 HF prefill tok/s measurement")
    ap.add_argument("--profile-case", choices=["prefill", "bidir_slice", "cfg3_eighth", "cfg2_bf16",
                                               "cfg2_fp32", "cfg4a", "mixer", "tile_prefill",
                                               "m1_ss2d"],
                    help="run three calls of one small case and exit (the program the ncu "
                         "captures in profiles/ run)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.profile_case:
        profile_case(args.profile_case)
        return
    if args.impl == "reference":
        run_reference(args)
        return

    # libraries may print banners to stdout (NCCL's version line); keep
    # stdout for the one JSON line: everything else goes to stderr until then
    sys.stdout.flush()
    json_fd = os.dup(1)
    os.dup2(2, 1)

    import torch
    import torch.distributed as dist
    import armhackathon_b200 as arm
    from armhackathon_b200 import _ffi

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)

    w = PREFILL
    x = make_inputs(w, dev, seed=rank)
    stream = torch.cuda.current_stream(dev)

    def step():
        return arm.selective_scan(x["u"], x["delta"], x["A"], x["B"], x["C"], D=x["D"], z=x["z"],
                                  delta_bias=x["delta_bias"], delta_softplus=True,
                                  return_last_state=True)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    # Eager steps, each bracketed by events (host dispatch of the Python op
    # included where it is slower than the kernel) ...
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    launches_before = _ffi.kernel_launches()
    for i in range(args.steps):
        starts[i].record(stream)
        step()
        ends[i].record(stream)
    torch.cuda.synchronize()
    launches = _ffi.kernel_launches() - launches_before  # GPU kernels, counted by the library
    eager_ms = statistics.mean(s.elapsed_time(e) for s, e in zip(starts, ends))
    # ... and the timed region proper: the K steps captured once into a CUDA
    # graph and replayed, so the figure is the device's, not the launcher's
    graph = None
    try:
        side = torch.cuda.Stream(dev)
        side.wait_stream(stream)
        with torch.cuda.stream(side):
            step()
        stream.wait_stream(side)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for _ in range(args.steps):
                step()
        graph.replay()
        torch.cuda.synchronize()
    except Exception:  # noqa: BLE001 -- eager launches instead
        graph = None
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t_begin = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        t_begin.record(stream)
        if graph is not None:
            graph.replay()
        else:
            for _ in range(args.steps):
                step()
        t_end.record(stream)
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    local_ms = t_begin.elapsed_time(t_end) / args.steps
    kernel_ms = [local_ms]
    t = torch.tensor([local_ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    step_ms = float(t.item())
    nbytes = algorithmic_bytes(w)
    value = world * nbytes / (step_ms * 1e-3) / 1e9
    elems = world * w["batch"] * w["dim"] * w["len"]

    # e2e: the reference-facing synchronous C entry point with pinned host buffers
    e2e = None
    if not args.no_e2e:
        host = {k: v.cpu().pin_memory() for k, v in x.items()}
        B, D, L, N = w["batch"], w["dim"], w["len"], w["state"]
        out_h = torch.empty((B, D, L)).pin_memory()
        last_h = torch.empty((B, D, N)).pin_memory()
        dims = _ffi.ArmScanDims(B, D, L, N, 1)

        def e2e_step():
            _ffi.scan_raw(dims, host["u"].data_ptr(), host["delta"].data_ptr(),
                          host["A"].data_ptr(), host["B"].data_ptr(), host["C"].data_ptr(),
                          host["D"].data_ptr(), host["z"].data_ptr(),
                          host["delta_bias"].data_ptr(), True, "auto", "auto",
                          out_h.data_ptr(), last_h.data_ptr())
        for _ in range(2):
            e2e_step()
        if world > 1:
            dist.barrier()
        e_steps = max(3, min(args.steps, 10))
        t0 = time.perf_counter()
        for _ in range(e_steps):
            e2e_step()
        e_ms = (time.perf_counter() - t0) * 1e3 / e_steps
        te = torch.tensor([e_ms], device=dev)
        if world > 1:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
        e_ms = float(te.item())
        h2d = sum(v.numel() * 4 for v in host.values())
        d2h = (out_h.numel() + last_h.numel()) * 4
        e2e = {"value": world * nbytes / (e_ms * 1e-3) / 1e9, "unit": "GB/s",
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": e_ms,
               "path": "arm_scan_selective_scan_f32 (synchronous C entry, pinned host buffers; "
                       "host wall clock, max over ranks)"}
        del host, out_h, last_h

    seqpar = run_seqpar_4b(args, dev, rank, world) if world > 1 and not args.no_configs else None

    if rank == 0:
        peak, peak_kind = peaks()
        k_ms = statistics.mean(kernel_ms)
        achieved = nbytes / (k_ms * 1e-3) / 1e9
        clocks = clk.summary()
        line = {
            "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seed = rank, BASELINE config 0 distributions)",
            "config": {"workload": "prefill_scan", "desc": w["desc"], "batch_per_gpu": w["batch"],
                       "dim": w["dim"], "len": w["len"], "state": w["state"],
                       "parallelism": f"dp{world} (batch rows per rank, no collective)",
                       "l2": "inputs larger than L2 (405.6 MB per step), no flush",
                       "timing": "K steps replayed from one CUDA graph" if graph is not None
                                 else "eager launches"},
            "eager_ms_per_step": eager_ms,
            "elems_per_s": elems / (step_ms * 1e-3),
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "peak_source": peak_kind,
                         "traffic": None,
                         "traffic_note": "not measurable inside the run; the ncu DRAM bytes of "
                                         "the same workload are in profiles/",
                         "bytes_per_launch": nbytes, "kernel_ms": k_ms},
            "mufu": mufu_roofline(w, k_ms, clocks, round(launches / args.steps)),
            "gpu_launches": launches,
            "e2e": e2e,
            "clocks": clocks,
        }
        if not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(w)
        if world == 1 and not args.no_configs:
            line["configs"] = config_suite(args, dev, peak, clocks)
        if seqpar:
            line["configs"] = {"cfg4b_seqpar": seqpar}
        sys.stdout.flush()
        os.write(json_fd, (json.dumps(line) + "\n").encode())
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
