"""The dense (L x L mask) form of the Mamba-3 aggregation, on CPU against the
oracle's scans: causal == the forward scan, non-causal == forward + reverse
scans - the diagonal term (D + gamma_t q_t . k_t) v_t, gated.  The dense
form is the independent check the GPU tests hold the one-call non-causal
entry against."""

import numpy as np
import torch

import oracle


def case(b=2, l=40, h=3, dv=8, dqk=16, r=4, seed=3):
    g = torch.Generator().manual_seed(seed)
    f = lambda *s: torch.randn(*s, generator=g, dtype=torch.float64)  # noqa: E731
    dt = torch.nn.functional.softplus(f(b, h, l) - 2)
    A = -torch.exp(torch.rand(h, generator=g, dtype=torch.float64) * np.log(4))
    return dict(q=f(b, l, 1, dqk) / 4, k=f(b, l, 1, dqk) / 4, v=f(b, l, h, dv),
                adt=A.view(1, h, 1) * dt, dt=dt, trap=f(b, h, l), q_bias=0.1 * f(h, dqk),
                k_bias=0.1 * f(h, dqk), angles=f(b, l, h, r), D=1 + 0.1 * f(h),
                z=f(b, l, h, dv))


def test_dense_causal_equals_forward_scan_and_noncausal_identity():
    from armhackathon_b200.mamba3_noncausal import noncausal_scan_dense
    x = case()
    dqk = x["q"].shape[-1]
    cos, sin = oracle.angles_to_cos_sin(x["angles"].numpy(), x["dt"].numpy(), dqk // 2)
    n = {k: v.numpy() for k, v in x.items() if k != "angles"}
    fwd = oracle.m3_siso(n["q"], n["k"], n["v"], n["adt"], n["dt"], n["trap"], n["q_bias"],
                         n["k_bias"], cos, sin, D=n["D"], z=n["z"])
    bwd = oracle.m3_siso(n["q"], n["k"], n["v"], n["adt"], n["dt"], n["trap"], n["q_bias"],
                         n["k_bias"], cos, sin, D=n["D"], z=n["z"], reverse=True)
    causal = noncausal_scan_dense(**x, causal=True).numpy()
    assert np.abs(causal - fwd).max() <= 1e-10 * np.abs(fwd).max()
    qb = n["q"][:, :, 0, None, :] + n["q_bias"][None, None]
    kb = n["k"][:, :, 0, None, :] + n["k_bias"][None, None]
    gamma = (n["dt"] / (1 + np.exp(-n["trap"]))).transpose(0, 2, 1)
    silu = n["z"] / (1 + np.exp(-n["z"]))
    diag = ((qb * kb).sum(-1) * gamma + n["D"][None, None])[..., None] * n["v"] * silu
    nc = noncausal_scan_dense(**x).numpy()
    want = fwd + bwd - diag
    assert np.abs(nc - want).max() <= 1e-10 * np.abs(want).max()
