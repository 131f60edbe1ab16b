"""Benchmark of the selective-scan hot path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload prefill_scan|cfg0|cfg2|cfg3|cfg4a|cfg4b]

A step is one Mamba-1 ``selective_scan`` call over one batch of synthetic
input (fp32, seed 0).  Default workload ``prefill_scan``: the per-layer scan
of BASELINE config 1 (HF Mamba-1 130M architecture prefill, batch 8 x
L 2048, d_inner 1536, d_state 16, softplus + delta_bias + D skip + z gate,
final state returned); 405.5 MB of algorithmic traffic per step, larger than
the 126 MB L2, so no flush is needed between steps.  ``cfg0`` is BASELINE
config 0 (batch 1) with an L2 flush between steps.

value      -- algorithmic GB/s of the whole job (all ranks), inputs resident
              in HBM, CUDA-event timed, max over ranks.
e2e        -- the same metric through the reference-facing synchronous C
              entry point with pinned HOST buffers (H2D + kernel + D2H inside
              the timed region).
roofline   -- the scan kernel's achieved algorithmic bandwidth against the
              measured HBM copy bandwidth.
cpu_baseline -- the oracle port of the reference's x86 CPU path (scalar
              recurrence, rows spread over all host threads), rank 0 only.

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

WORKLOADS = {
    "prefill_scan": dict(batch=8, dim=1536, len=2048, state=16, flush=False,
                         desc="Mamba-1 selective_scan at the 130M prefill shape (BASELINE "
                              "config 1's per-layer scan): batch 8 x L 2048, d_inner 1536, "
                              "d_state 16, fp32"),
    "cfg0": dict(batch=1, dim=1536, len=2048, state=16, flush=True,
                 desc="BASELINE config 0: Mamba-1 selective_scan B1 D1536 L2048 N16 fp32"),
}


M3_WORKLOADS = {
    "cfg2": dict(kind="siso", batch=4, heads=24, dv=64, dqk=128, len=4096, rank=1, pairs=64,
                 desc="BASELINE config 2: Mamba-3 SISO B4 H24 P64 N128 L4096 (fp32 on the C "
                      "ABI; the config's bf16 inputs are exactly representable)"),
    "cfg3": dict(kind="mimo", batch=8, heads=24, dv=64, dqk=128, len=8192, rank=4, pairs=64,
                 desc="BASELINE config 3 shape: Mamba-3 MIMO r4 B8 H24 P64 N128 L8192 through the "
                      "reference op formulation (psi/zeta/phi projections)"),
    "cfg4a": dict(kind="ss2d", batch=8, heads=6, dv=64, dqk=64, len=128 * 128, rank=1, pairs=32,
                  grid=128, desc="BASELINE config 4a: SS2D Mamba-3 SISO 128x128 grid B8 H6 P64 "
                                 "N64 fp32, 4 directions summed"),
    "m3_mixer": dict(kind="mixer", batch=4, heads=24, dv=64, dqk=128, len=4096, rank=1,
                     pairs=32, desc="Mamba-3 mixer prologue (in_proj output -> scan inputs: "
                                    "split, softplus/heavy-tail gates, B/C RMSNorm, relayouts) "
                                    "at config 2's shape with the checkpoint's 3432-wide in_proj "
                                    "rows (rope_fraction 0.5: 32 angles), fp32"),
    "cfg4b": dict(kind="bidir", batch=1, dim=1536, len=262144, state=16,
                  desc="BASELINE config 4b: Mamba-1 bidirectional D1536 N16 L262144 fp32, summed"),
}


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


def run_m3(args, w):
    """Time a Mamba-3 or bidirectional workload (recorded for the configs;
    the headline line is the Mamba-1 prefill scan)."""
    import torch
    import armhackathon_b200 as arm
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    if w["kind"] == "bidir":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        local = int(os.environ.get("LOCAL_RANK", "0"))
        dev = torch.device("cuda", local)
        torch.cuda.set_device(dev)
        seg = w["len"] // world  # strong scaling: one sequence split over the ranks
        x = make_inputs(dict(batch=1, dim=w["dim"], len=seg, state=w["state"]), dev, seed=rank)
        if world > 1:
            import torch.distributed as dist
            from armhackathon_b200.seqpar import bidirectional_scan_seqpar
            dist.init_process_group("nccl", device_id=dev)
            step = lambda: bidirectional_scan_seqpar(  # noqa: E731
                x["u"], x["delta"], x["A"], x["B"], x["C"], D=x["D"], z=x["z"],
                delta_bias=x["delta_bias"], delta_softplus=True)
        else:
            step = lambda: arm.bidirectional_scan(  # noqa: E731
                x["u"], x["delta"], x["A"], x["B"], x["C"], D=x["D"], z=x["z"],
                delta_bias=x["delta_bias"], delta_softplus=True, merge="sum")
        nbytes = 4 * (4 * w["dim"] * w["len"] + 2 * w["state"] * w["len"])
        for _ in range(args.warmup):
            step()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(args.steps):
            step()
        b.record()
        torch.cuda.synchronize()
        ms = torch.tensor([a.elapsed_time(b) / args.steps], device=dev)
        if world > 1:
            dist.all_reduce(ms, op=dist.ReduceOp.MAX)
            dist.destroy_process_group()
        if rank == 0:
            print(json.dumps({"metric": METRIC, "workload": args.workload, "desc": w["desc"],
                              "n_gpus": world, "scaling": "strong",
                              "ms_per_step": float(ms.item()),
                              "value": nbytes / (float(ms.item()) * 1e-3) / 1e9, "unit": "GB/s",
                              "bytes_per_step": nbytes,
                              "parallelism": f"sequence-parallel over {world} ranks, one "
                                             "all_gather of segment carries per call"}),
                  flush=True)
        return
    elif w["kind"] == "mixer":
        return run_mixer(args, w, dev)
    else:
        x = m3_inputs(w, dev)
        nbytes = m3_bytes(w)
        if w["kind"] == "mimo":
            prec = "bf16" if args.m3_bf16 else "fp32"
            step = lambda: arm.mamba3_mimo_scan(**x, precision=prec)  # noqa: E731
        elif w["kind"] == "siso" and args.m3_bf16:
            # bf16 model inputs, angles shared by all heads; the tensor-core
            # entry with the angle pre-pass fused in, output (b, l, h, dv) bf16
            bf = torch.bfloat16
            xb = dict(x, q=x["q"].to(bf), k=x["k"].to(bf), v=x["v"].to(bf),
                      angles=x["angles"][:, :, :1, :].to(bf).contiguous())
            nbytes = m3_bytes_bf16(w)
            step = lambda: arm.mamba3_scan(**xb, return_last_state=True,  # noqa: E731
                                           precision="bf16")
        elif w["kind"] == "siso":
            step = lambda: arm.mamba3_scan(**x, return_last_state=True)  # noqa: E731
        else:
            B, H, g = w["batch"], w["heads"], w["grid"]
            grid = lambda t: t.reshape(B, g, g, *t.shape[2:])  # noqa: E731
            hm = lambda t: t.reshape(B, H, g, g)  # noqa: E731
            xs = dict(q=grid(x["q"]), k=grid(x["k"]), v=grid(x["v"]), angles=grid(x["angles"]),
                      adt=hm(x["adt"]), dt=hm(x["dt"]), trap=hm(x["trap"]),
                      q_bias=x["q_bias"], k_bias=x["k_bias"], D=x["D"])
            step = lambda: arm.ss2d_scan_mamba3(**xs)  # noqa: E731
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(args.steps):
        step()
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / args.steps
    print(json.dumps({"metric": METRIC, "workload": args.workload, "desc": w["desc"],
                      "ms_per_step": ms, "value": nbytes / (ms * 1e-3) / 1e9, "unit": "GB/s",
                      "bytes_per_step": nbytes,
                      "note": "whole op incl. the torch angle pre-pass and output permute"}),
          flush=True)


def run_mixer(args, w, dev):
    """The fused Mamba-3 mixer prologue: HBM roofline of the one kernel, the
    same prologue as separate torch ops, and prologue + fp32 scan."""
    import torch
    import armhackathon_b200 as arm
    from armhackathon_b200 import _ffi
    x = mixer_inputs(w, dev)
    nbytes = mixer_bytes(w)
    H, N = w["heads"], w["dqk"]
    scan_kw = dict(D=torch.ones(H, device=dev), B_bias=torch.zeros(H, 1, N, device=dev),
                   C_bias=torch.zeros(H, 1, N, device=dev))

    def timed(fn, steps):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(steps):
            fn()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b) / steps

    n0 = _ffi.kernel_launches()
    with ClockSampler(dev.index or 0) as clk:
        ms = timed(lambda: arm.mamba3_mixer_prologue(**x), args.steps)
    clocks = clk.summary()
    per_call = (_ffi.kernel_launches() - n0) / (args.warmup + args.steps)
    launches = int(round(per_call * args.steps))  # kernels in the timed region
    torch_ms = timed(lambda: torch_mixer_prologue(**x), args.steps)
    full_ms = timed(lambda: arm.mamba3_mixer_scan(**x, **scan_kw), max(1, args.steps // 5))
    bf16_ms = timed(lambda: arm.mamba3_mixer_scan(**x, **scan_kw, precision="bf16"),
                    max(1, args.steps // 5))
    peak, peak_kind = peaks()
    gbs = nbytes / (ms * 1e-3) / 1e9
    print(json.dumps({
        "metric": METRIC, "workload": args.workload, "desc": w["desc"], "ms_per_step": ms,
        "value": gbs, "unit": "GB/s", "bytes_per_step": nbytes, "dtype": "f32",
        "roofline": {"bound": "hbm", "achieved": gbs, "peak": peak, "unit": "GB/s",
                     "frac": gbs / peak, "peak_source": peak_kind},
        "gpu_launches": launches, "clocks": clocks,
        "torch_ops_ms": torch_ms, "prologue_plus_fp32_scan_ms": full_ms,
        "prologue_plus_bf16_tensor_scan_ms": bf16_ms,
        "l2": "inputs larger than L2",
        "note": "the prologue alone (one kernel, CUDA events); torch_ops_ms = the same "
                "prologue as separate torch ops on this GPU"}), flush=True)


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def profiled_traffic(workload):
    """DRAM bytes of one scan op (all of its kernels) from the committed ncu
    summary (profiles/m1_seg2_<workload>.md, line 'traffic_bytes_per_launch:
    N'), or None when no capture of this workload is committed."""
    import re
    f = ROOT / "profiles" / f"m1_seg2_{workload}.md"
    if not f.exists():
        return None
    m = re.search(r"traffic_bytes_per_launch:\s*(\d+)", f.read_text())
    return int(m.group(1)) if m else None


def seg2_segments(w):
    """Segment count the default Mamba-1 kernel picks for this shape (the rule
    of m1_seg2_segments in armhackathon_b200/csrc/m1_seg2.cu)."""
    rows, L, S = w["batch"] * w["dim"], w["len"], 1
    while rows * S < 148 * 1024 and L % (2 * S) == 0 and L // (2 * S) >= 128 \
            and (L // (2 * S)) % 64 == 0:
        S *= 2
    return S


def mufu_roofline(w, k_ms, clocks):
    """The Mamba-1 scan's binding unit: one exp per (batch, channel, step,
    state) is the algorithm's minimum (the reference computes exactly that);
    the MUFU pipe issues 16 of them per clock per SM (nominal), taken at the
    SM clock sampled during the timed region."""
    import torch
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    mhz = clocks.get("sm_mhz") or clocks.get("sm_max_mhz") or 1965.0
    exps = w["batch"] * w["dim"] * w["len"] * w["state"]
    S = seg2_segments(w)
    achieved = exps / (k_ms * 1e-3) / 1e9
    peak = 16 * sms * mhz * 1e6 / 1e9
    return {"bound": "mufu", "achieved": achieved, "peak": peak, "unit": "Gexp/s",
            "frac": achieved / peak, "peak_source": "nominal 16/clk/SM x sampled SM clock",
            "executed_per_algorithmic": 2 * (S - 1) / S if S > 1 else 1.0, "segments": S,
            "note": "the default two-pass kernel computes the exps of segments 1 .. S-2 twice "
                    "(end states, then outputs), plus the softplus/silu exps per (row, step)"}


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


def run_reference(args, w):
    """--impl reference: the reference's CPU path (scalar recurrence over rows
    on all host threads; oracle port, the Rust crate has no toolchain here)."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    nthreads = oracle.hw_threads()
    rng = np.random.default_rng(0)
    B, D, L, N = w["batch"], w["dim"], w["len"], w["state"]
    f = lambda *s: rng.standard_normal(s).astype(np.float32)  # noqa: E731
    dt = np.exp(rng.uniform(np.log(1e-3), np.log(1e-1), D))
    inp = dict(u=f(B, D, L), delta=f(B, D, L), z=f(B, D, L),
               A=-np.tile(np.arange(1, N + 1, dtype=np.float32), (D, 1)), B=f(B, N, L),
               C=f(B, N, L), D=np.ones(D, np.float32),
               delta_bias=np.log(np.expm1(dt)).astype(np.float32))
    for _ in range(args.warmup):
        oracle.m1_scan(**inp, delta_softplus=True, dtype=np.float32, nthreads=nthreads)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        oracle.m1_scan(**inp, delta_softplus=True, dtype=np.float32, nthreads=nthreads)
        times.append(time.perf_counter() - t0)
    t = statistics.median(times)
    gbs = algorithmic_bytes(w) / t / 1e9
    line = {"impl": "reference", "metric": METRIC, "value": gbs, "unit": "GB/s", "n_gpus": 0,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": t * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seed 0, BASELINE config 0 distributions)",
            "config": {"workload": args.workload, "desc": w["desc"], "batch": B, "dim": D,
                       "len": L, "state": N},
            "elems_per_s": B * D * L / t,
            "cpu_baseline": {"value": gbs, "unit": "GB/s", "cores": nthreads, "kind": "port",
                             "sample": f"the full step workload ({B}x{D}x{L}, N={N}) per step"},
            "e2e": {"value": gbs, "unit": "GB/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


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


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="prefill_scan",
                    choices=sorted(WORKLOADS) + sorted(M3_WORKLOADS))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--m3-bf16", action="store_true",
                    help="Mamba-3 SISO/MIMO workloads on the tensor-core (bf16 operand) kernels")
    ap.add_argument("--no-prefill", action="store_true",
                    help="skip the config-1 HF prefill tok/s measurement")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.workload in M3_WORKLOADS:
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "workload": args.workload,
                              "unavailable": "reference arm is implemented for the Mamba-1 "
                                             "workloads only"}))
            return
        run_m3(args, M3_WORKLOADS[args.workload])
        return
    w = WORKLOADS[args.workload]
    if args.impl == "reference":
        run_reference(args, w)
        return

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

    x = make_inputs(w, dev, seed=rank)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev) if w["flush"] else None
    stream = torch.cuda.current_stream(dev)

    def step():
        return arm.selective_scan(x["u"], x["delta"], x["A"], x["B"], x["C"], D=x["D"], z=x["z"],
                                  delta_bias=x["delta_bias"], delta_softplus=True,
                                  return_last_state=True)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t_begin = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    from armhackathon_b200 import _ffi
    launches_before = _ffi.kernel_launches()
    with ClockSampler(local) as clk:
        t_begin.record(stream)
        for i in range(args.steps):
            if flush is not None:
                flush.fill_(i & 0xFF)
            starts[i].record(stream)
            step()
            ends[i].record(stream)
        t_end.record(stream)
        torch.cuda.synchronize()
    launches = _ffi.kernel_launches() - launches_before  # GPU kernels, counted by the library
    if world > 1:
        dist.barrier()
    kernel_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    step_ms = sum(kernel_ms) / len(kernel_ms) if flush is not None else \
        t_begin.elapsed_time(t_end) / args.steps
    t = torch.tensor([step_ms], device=dev)
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
               "path": "arm_scan_selective_scan_f32 (synchronous C entry, pinned host buffers)"}

    if rank == 0:
        peak, peak_kind = peaks()
        k_ms = statistics.mean(kernel_ms)
        achieved = nbytes / (k_ms * 1e-3) / 1e9
        line = {
            "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seed = rank, BASELINE config 0 distributions)",
            "config": {"workload": args.workload, "desc": w["desc"], "batch_per_gpu": w["batch"],
                       "dim": w["dim"], "len": w["len"], "state": w["state"],
                       "parallelism": f"dp{world} (batch rows per rank, no collective)",
                       "l2": "inputs larger than L2" if not w["flush"] else
                             "256 MB L2 flush between steps (outside the kernel events)"},
            "elems_per_s": elems / (step_ms * 1e-3),
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "peak_source": peak_kind,
                         "traffic": profiled_traffic(args.workload),
                         "traffic_source": "ncu dram__bytes_read+write summed over the op's "
                                           "kernels (profiles/m1_seg2_<workload>.md)",
                         "bytes_per_launch": nbytes,
                         "kernel_ms": k_ms},
            "gpu_launches": launches,
            "e2e": e2e,
            "clocks": clk.summary(),
        }
        line["mufu"] = mufu_roofline(w, k_ms, line["clocks"])
        if not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(w)
        if not args.no_prefill:
            line["prefill"] = {
                "metric": "Mamba-1 prefill tok/s (BASELINE config 1, fp32, patched HF, 1 GPU)",
                "runs": [prefill_tok_s(dev, 8, 2048), prefill_tok_s(dev, 1, 32768)]}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
