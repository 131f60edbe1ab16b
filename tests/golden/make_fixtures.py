"""Regenerate the committed golden fixtures from the reference checkout.

Run in a container that has the reference mounted (default path below, or
``--ref``).  The fixtures it writes are what the test-suite pins the CPU oracle
and the CUDA kernels against; the reference itself never travels to a GPU box.

What is produced, per family:

* ``m1/<case>.npz`` -- the reference's 16 Mamba-1 golden cases
  (tests/golden/*.npz in the reference: 15 synthetic draws from
  tests/golden_inputs.py:170-188 plus ``hf_mixer_layer0`` captured from a real
  mamba-130m layer).  Inputs and the f64 ground truth ``out_f64`` /
  ``last_state_f64`` are copied unchanged; ``f32_max_abs_err`` (the upstream
  f32 floor from tests/golden/manifest.json) rides along for the
  ``< 50 x floor`` gate of tests/check_ffi.py:30-31,82-83.
* ``m1_2d/<grid>.npz`` -- the six SS2D grids (tests/golden/2d) with their four
  per-direction f64 planes, unchanged.
* ``m3_siso/<case>.npz`` -- the Mamba-3 SISO captures from the official GPU
  kernel (tests/golden/mamba3/*.npz).  Cases longer than ``SISO_MAX_L`` tokens
  (``SISO_MAX_L_WIDE`` for the 24-head cases) are cut to their prefix: every input of a forward scan
  at step t only reaches outputs at steps >= t (the trapezoid reads t+1 only
  through ``scale_t``, which first acts on y_{t+1}; the angle pre-pass is a
  prefix sum), so the prefix of the captured output is exactly the output of
  the prefix.  Besides the captured ``out`` the file holds ``ref_f64`` /
  ``ref_rev_f64`` / ``ref_state_f64`` / ``ref_rev_state_f64`` (states only for
  the cases with small heads): the reference's own f64 oracle (tests/reference/mamba3_ref.py:150 ``mamba3_siso_ref``) run
  here on the same (cut) inputs, forward and with ``reverse=True``, stored rounded to
  f32; the final states come from a tiny restatement of that loop that also returns ``S``.
* ``m3_mimo/<case>.npz`` -- the MIMO captures (tests/golden/mamba3_mimo),
  cut to ``MIMO_MAX_L`` tokens the same way, plus ``ref_f64`` from
  ``mamba3_mimo_ref`` (mamba3_ref.py:305).

* ``m3_mimo_x/<case>.npz`` -- the MIMO scan with the input given per rank
  (BASELINE config 3's formulation: h_t = a_t h_{t-1} + b_t X_{t-1} B_{t-1}^T
  + g_t X_t B_t^T, Y_t = h_t C_t, per-rank outputs), pinned to the
  reference's own ``mamba3_mimo_ref``: seeded inputs whose per-rank X is
  psi_r * v (the form the reference op can express), the reference run once
  per rank with a one-hot output projection (phi selects rank r, no z), so
  that its output is rank r's Y (+ D X).  Stored in the per-rank layouts:
  x (b, l, h, p, r), b/c (b, l, n, r), raw angles (b, l, h, n/4); the
  reference's B is its K and C its Q; ``ref_f64`` (b, l, h, p, r).

* ``m3_mixer/<case>.npz`` -- the Mamba-3 mixer's prologue (everything between
  ``in_proj`` and the scan call, apps/mamba3_lm/block.py:146-177) run by the
  reference's own ``Mamba3Mixer`` on seeded random weights and inputs: its
  scan entry (``arm_scan.mamba3_scan`` / ``mamba3_mimo_scan``) is replaced by
  a stub that records the arguments it receives.  Stored: the ``in_proj``
  output ``proj``, the mixer's parameters, and the recorded q, k, v, z, adt,
  dt, trap and (head 0 of the broadcast) angles.

Usage:  python tests/golden/make_fixtures.py [--ref /path/to/reference]
"""

import argparse
import json
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
SISO_MAX_L = 128       # cut for cases with small heads (heads*dv <= 512)
SISO_MAX_L_WIDE = 32   # cut for the wide 24x64 cases
MIMO_MAX_L = 16
# final-state fixtures are kept only for cases whose state is this small
STATE_MAX_ELEMS = 1 << 16


def _save(path, **arrays):
    path.parent.mkdir(parents=True, exist_ok=True)
    np.savez_compressed(path, **arrays)


def make_m1(ref):
    src = ref / "tests" / "golden"
    manifest = json.loads((src / "manifest.json").read_text())
    keep = []
    for meta in manifest:
        d = np.load(src / f"{meta['name']}.npz")
        arrays = {k: d[k] for k in d.files if k != "meta_json"}
        arrays["delta_softplus"] = np.array(bool(meta["delta_softplus"]))
        arrays["f32_max_abs_err"] = np.array(float(meta["f32_max_abs_err"]))
        _save(HERE / "m1" / f"{meta['name']}.npz", **arrays)
        keep.append(meta["name"])
    return keep


def make_m1_2d(ref):
    src = ref / "tests" / "golden" / "2d"
    names = []
    for f in sorted(src.glob("*.npz")):
        d = np.load(f)
        _save(HERE / "m1_2d" / f.name, **{k: d[k] for k in d.files})
        names.append(f.stem)
    return names


def _siso_with_state(mod, kw, reverse):
    """``mamba3_siso_ref`` with the final state returned as well.

    Same algebra as mamba3_ref.py:150-263 (the function's body is re-run by
    calling it for ``out``); the state recursion below repeats its lines
    246-260 so ``S`` after the last traversal step can be recorded.  Used only
    to produce the ``*_state_f64`` fixtures, which pin the kernels' final-state
    output (the reference's Python op never requests it).
    """
    import torch
    out = mod.mamba3_siso_ref(**kw, reverse=reverse)
    dtype = torch.float64
    Q, K, V = (kw[k].to(dtype) for k in ("Q", "K", "V"))
    ADT, DT, Trap = (kw[k].to(dtype) for k in ("ADT", "DT", "Trap"))
    Q_bias, K_bias, Angles = (kw[k].to(dtype) for k in ("Q_bias", "K_bias", "Angles"))
    b, l, _, dv = V.shape
    h, dqk = Q_bias.shape
    q = Q[:, :, 0, :].unsqueeze(2) + Q_bias.view(1, 1, h, dqk)
    k = K[:, :, 0, :].unsqueeze(2) + K_bias.view(1, 1, h, dqk)
    theta = torch.cumsum(torch.tanh(Angles) * torch.pi
                         * DT.permute(0, 2, 1).unsqueeze(-1), dim=1)
    k = mod._rope(k, theta)
    if reverse:
        k, V = torch.flip(k, [1]), torch.flip(V, [1])
        ADT, DT, Trap = (torch.flip(t, [2]) for t in (ADT, DT, Trap))
    lam = torch.sigmoid(Trap)
    gamma = DT * lam
    shifted = torch.zeros_like(gamma)
    shifted[..., :-1] = DT[..., 1:] * (1.0 - lam[..., 1:])
    scale = gamma + shifted
    a = torch.exp(ADT)
    S = torch.zeros(b, h, dv, dqk, dtype=dtype)
    for t in range(l):
        S = (a[:, :, t].view(b, h, 1, 1) * S
             + scale[:, :, t].view(b, h, 1, 1)
             * V[:, t].unsqueeze(-1) * k[:, t].unsqueeze(-2))
    return out.numpy(), S.numpy()


def make_m3(ref):
    import torch
    sys.path.insert(0, str(ref / "tests"))
    from reference import mamba3_ref as mod  # noqa: E402

    names = {"siso": [], "mimo": []}
    siso_keys = ("Q", "K", "V", "ADT", "DT", "Trap", "Q_bias", "K_bias",
                 "Angles", "D", "Z")
    for f in sorted((ref / "tests" / "golden" / "mamba3").glob("mamba3_siso_combined_*.npz")):
        d = np.load(f)
        L, heads, dv = d["kw_V"].shape[1:4]
        cut = min(L, SISO_MAX_L if heads * dv <= 512 else SISO_MAX_L_WIDE)
        arrays = {}
        for k in siso_keys:
            a = d[f"kw_{k}"]
            if k in ("Q", "K", "V", "Angles", "Z"):
                a = a[:, :cut]
            elif k in ("ADT", "DT", "Trap"):
                a = a[:, :, :cut]
            arrays[f"kw_{k}"] = np.ascontiguousarray(a)
        arrays["out"] = np.ascontiguousarray(d["out"][:, :cut])
        arrays["orig_len"] = np.array(L)
        kw = {k: torch.from_numpy(arrays[f"kw_{k}"]) for k in siso_keys}
        fwd, s_f = _siso_with_state(mod, kw, False)
        bwd, s_b = _siso_with_state(mod, kw, True)
        # stored as f32: the f64 results rounded once (rel 6e-8), far below
        # every tolerance they are used with, at half the bytes
        arrays.update(ref_f64=fwd.astype(np.float32),
                      ref_rev_f64=bwd.astype(np.float32))
        if s_f.size <= STATE_MAX_ELEMS:
            arrays.update(ref_state_f64=s_f.astype(np.float32),
                          ref_rev_state_f64=s_b.astype(np.float32))
        _save(HERE / "m3_siso" / f.name, **arrays)
        names["siso"].append(f.stem)

    mimo_keys = ("Q", "K", "V", "ADT", "DT", "Trap", "Q_bias", "K_bias",
                 "MIMO_V", "MIMO_Z", "MIMO_Out", "Angles", "D", "Z")
    for f in sorted((ref / "tests" / "golden" / "mamba3_mimo").glob("mamba3_mimo_combined_*.npz")):
        d = np.load(f)
        L = d["kw_V"].shape[1]
        cut = min(L, MIMO_MAX_L)
        arrays = {}
        for k in mimo_keys:
            a = d[f"kw_{k}"]
            if k in ("Q", "K", "V", "Angles", "Z"):
                a = a[:, :cut]
            elif k in ("ADT", "DT", "Trap"):
                a = a[:, :, :cut]
            arrays[f"kw_{k}"] = np.ascontiguousarray(a)
        arrays["out"] = np.ascontiguousarray(d["out"][:, :cut])
        arrays["orig_len"] = np.array(L)
        kw = {k: torch.from_numpy(arrays[f"kw_{k}"]) for k in mimo_keys}
        arrays["ref_f64"] = mod.mamba3_mimo_ref(**kw).numpy().astype(np.float32)
        _save(HERE / "m3_mimo" / f.name, **arrays)
        names["mimo"].append(f.stem)
    return names


MIMO_X_CASES = {
    # name: (batch, len, heads, headdim, d_state, rank, with_D, seed)
    "r2_small": (1, 24, 2, 8, 16, 2, False, 11),
    "r4_wide": (2, 20, 3, 16, 32, 4, True, 12),
    "r4_long": (1, 96, 1, 8, 16, 4, True, 13),
}


def make_mimo_x(ref):
    import torch
    sys.path.insert(0, str(ref / "tests"))
    from reference import mamba3_ref as mod  # noqa: E402
    names = []
    for name, (b, l, h, p, n, r, with_d, seed) in MIMO_X_CASES.items():
        g = torch.Generator().manual_seed(seed)
        rn = lambda *sh: torch.randn(*sh, generator=g, dtype=torch.float64)  # noqa: E731
        v = rn(b, l, h, p)
        psi = rn(h, r, p)
        Q = rn(b, l, r, 1, n) / np.sqrt(n * r)     # C
        K = rn(b, l, r, 1, n) / np.sqrt(n * r)     # B
        dt = torch.nn.functional.softplus(rn(b, h, l) - 2)
        A = -torch.exp(torch.rand(h, generator=g, dtype=torch.float64) * np.log(16))
        adt = A.view(1, h, 1) * dt
        trap = rn(b, h, l)
        ang = torch.atanh(torch.rand(b, l, h, n // 4, generator=g, dtype=torch.float64) * 0.999)
        D = 1 + 0.1 * rn(h) if with_d else None
        zero = torch.zeros(h, r, n, dtype=torch.float64)
        outs = []
        for rk in range(r):
            phi = torch.zeros(h, r, p, dtype=torch.float64)
            phi[:, rk, :] = 1.0
            outs.append(mod.mamba3_mimo_ref(Q, K, v, adt, dt, trap, zero, zero, psi,
                                            torch.ones(h, r, p, dtype=torch.float64), phi,
                                            ang, D=D, Z=None))
        x = v.unsqueeze(-1) * psi.permute(1, 0, 2).reshape(1, 1, r, h, p).permute(0, 1, 3, 4, 2)
        arrays = dict(x=x, b=K[:, :, :, 0, :].permute(0, 1, 3, 2), c=Q[:, :, :, 0, :].permute(0, 1, 3, 2),
                      adt=adt, dt=dt, trap=trap, angles=ang, ref_f64=torch.stack(outs, -1))
        if D is not None:
            arrays["D"] = D
        _save(HERE / "m3_mimo_x" / f"{name}.npz",
              **{k: np.ascontiguousarray(t.numpy()) for k, t in arrays.items()})
        names.append(name)
    return names


MIXER_CASES = {
    # name: (Mamba3Mixer kwargs, batch, len, seed)
    "siso_rope_half": (dict(d_model=64, d_state=16, expand=2, headdim=16, rope_fraction=0.5), 2, 33, 1),
    "siso_rope_full": (dict(d_model=48, d_state=32, expand=2, headdim=8, rope_fraction=1.0), 1, 70, 2),
    "mimo_r2": (dict(d_model=64, d_state=16, expand=2, headdim=16, rope_fraction=0.5,
                     is_mimo=True, mimo_rank=2), 2, 21, 3),
    "mimo_r4": (dict(d_model=32, d_state=8, expand=2, headdim=8, rope_fraction=1.0,
                     is_mimo=True, mimo_rank=4, A_floor=0.05), 1, 40, 4),
}


def make_mixer(ref):
    import torch
    sys.path.insert(0, str(ref / "python"))
    sys.path.insert(0, str(ref))
    from apps.mamba3_lm import block  # noqa: E402

    seen = {}

    def record(**kw):
        seen.clear()
        seen.update(kw)
        return torch.zeros_like(kw["v"])

    block.arm_scan.mamba3_scan = record
    block.arm_scan.mamba3_mimo_scan = record
    names = []
    for name, (kw, b, l, seed) in MIXER_CASES.items():
        torch.manual_seed(seed)
        mix = block.Mamba3Mixer(**kw).float()
        with torch.no_grad():
            # the parameters' inits are constants; random values exercise them
            for prm in (mix.dt_bias, mix.D, mix.B_bias, mix.C_bias, mix.B_norm.weight,
                        mix.C_norm.weight):
                prm.copy_(torch.randn_like(prm) * 0.5 + 1.0)
            mix.in_proj.weight.mul_(3.0)  # dd_A on both sides of heavy_tail's kink
            u = torch.randn(b, l, kw["d_model"])
            proj = mix.in_proj(u)
            mix(u)
        r = mix.mimo_rank
        q = seen["q"].reshape(b, l, r, -1) if r > 1 else seen["q"].reshape(b, l, -1)
        k = seen["k"].reshape(b, l, r, -1) if r > 1 else seen["k"].reshape(b, l, -1)
        arrays = dict(
            proj=proj, dt_bias=mix.dt_bias, B_norm_weight=mix.B_norm.weight,
            C_norm_weight=mix.C_norm.weight, A_floor=torch.tensor(mix.A_floor),
            eps=torch.tensor(mix.B_norm.eps), heads=torch.tensor(mix.nheads),
            headdim=torch.tensor(mix.headdim), d_state=torch.tensor(mix.d_state),
            rank=torch.tensor(r), n_angles=torch.tensor(mix.num_rope_angles),
            D=mix.D, q_bias=seen["q_bias"], k_bias=seen["k_bias"],
            q=q, k=k, v=seen["v"], z=seen["z"], adt=seen["adt"], dt=seen["dt"],
            trap=seen["trap"], angles=seen["angles"][:, :, 0, :])
        if r > 1:
            arrays.update(psi=seen["psi"], zeta=seen["zeta"], phi=seen["phi"])
        _save(HERE / "m3_mixer" / f"{name}.npz",
              **{k: np.ascontiguousarray(v.detach().float().numpy()) for k, v in arrays.items()})
        names.append(name)
    return names


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("ARM_SCAN_REFERENCE"),
                    help="reference checkout, read-only (default: $ARM_SCAN_REFERENCE)")
    args = ap.parse_args()
    if not args.ref:
        ap.error("pass --ref or set ARM_SCAN_REFERENCE to the reference checkout")
    ref = Path(args.ref)
    index = {
        "source": "AdityaP9116/ARMHackathon tests/golden (+ its Python oracles)",
        "siso_max_len": [SISO_MAX_L, SISO_MAX_L_WIDE],
        "mimo_max_len": MIMO_MAX_L,
        "m1": make_m1(ref),
        "m1_2d": make_m1_2d(ref),
    }
    index.update({f"m3_{k}": v for k, v in make_m3(ref).items()})
    index["m3_mixer"] = make_mixer(ref)
    index["m3_mimo_x"] = make_mimo_x(ref)
    (HERE / "index.json").write_text(json.dumps(index, indent=1) + "\n")
    print(json.dumps({k: (len(v) if isinstance(v, list) else v)
                      for k, v in index.items()}))


if __name__ == "__main__":
    main()
