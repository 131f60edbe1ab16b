"""Mamba-3 mixer prologue on the GPU: the fused kernel through the C ABI
against the scan arguments the reference's own Mamba3Mixer.forward produced
(apps/mamba3_lm/block.py:146-199, recorded in tests/golden/m3_mixer), and the
mixer's scan output against the CPU oracle scan on those arguments."""

import json

import numpy as np
import pytest
import torch

import oracle
from conftest import GOLDEN
from test_oracle_golden import MIXER_KEYS, load_mixer

pytestmark = pytest.mark.gpu

MIXER = json.loads((GOLDEN / "index.json").read_text())["m3_mixer"]
REL_TOL = 1e-4


def arm():
    import armhackathon_b200 as a
    return a


def prologue(d, dims, proj):
    return arm().mamba3_mixer_prologue(
        proj, nheads=dims["heads"], headdim=dims["headdim"], d_state=dims["d_state"],
        n_angles=dims["n_angles"], dt_bias=torch.from_numpy(d["dt_bias"]).cuda(),
        B_norm_weight=torch.from_numpy(d["B_norm_weight"]).cuda(),
        C_norm_weight=torch.from_numpy(d["C_norm_weight"]).cuda(), mimo_rank=dims["rank"],
        A_floor=dims["A_floor"], eps=dims["eps"])


def check_prologue(got, d):
    for ok, fk in MIXER_KEYS:
        want = d[fk]
        g = getattr(got, ok).cpu().numpy().reshape(want.shape)
        if ok in ("z", "x", "trap", "angles"):
            assert np.array_equal(g, want), ok  # copies: bit-exact
        else:
            assert np.abs(g - want).max() <= 2e-6 * max(1.0, np.abs(want).max()), ok


@pytest.mark.parametrize("name", MIXER)
def test_mixer_prologue_matches_reference_block(name):
    d, dims = load_mixer(name)
    check_prologue(prologue(d, dims, torch.from_numpy(d["proj"]).cuda()), d)


@pytest.mark.parametrize("name", MIXER[:1] + MIXER[-1:])
def test_mixer_prologue_unaligned_rows(name):
    """A proj that starts 4 bytes past a 16-byte boundary takes the scalar
    copy path; results are the same."""
    d, dims = load_mixer(name)
    flat = torch.empty(d["proj"].size + 1, device="cuda")
    proj = flat[1:].view(d["proj"].shape)
    proj.copy_(torch.from_numpy(d["proj"]))
    assert proj.data_ptr() % 16 != 0
    check_prologue(prologue(d, dims, proj), d)


@pytest.mark.parametrize("name", MIXER)
def test_mixer_scan_vs_oracle(name):
    d, dims = load_mixer(name)
    h, p, n, r = dims["heads"], dims["headdim"], dims["d_state"], dims["rank"]
    cu = lambda k: torch.from_numpy(d[k]).cuda()  # noqa: E731
    kw = dict(nheads=h, headdim=p, d_state=n, n_angles=dims["n_angles"], dt_bias=cu("dt_bias"),
              B_norm_weight=cu("B_norm_weight"), C_norm_weight=cu("C_norm_weight"),
              D=cu("D"), B_bias=cu("k_bias"), C_bias=cu("q_bias"), mimo_rank=r,
              A_floor=dims["A_floor"], eps=dims["eps"])
    if r > 1:
        kw.update(psi=cu("psi"), zeta=cu("zeta"), phi=cu("phi"))
    y = arm().mamba3_mixer_scan(cu("proj"), **kw).cpu().numpy()
    b, l = d["proj"].shape[:2]
    ang = np.broadcast_to(d["angles"][:, :, None, :], (b, l, h, dims["n_angles"]))
    half = n // 2
    cos, sin = oracle.angles_to_cos_sin(ang, d["dt"], half)
    if r > 1:
        want = oracle.m3_mimo(d["q"], d["k"], d["v"], d["adt"], d["dt"], d["trap"], d["q_bias"],
                              d["k_bias"], cos, sin, d["psi"], d["zeta"], d["phi"], D=d["D"],
                              z=d["z"])
    else:
        want = oracle.m3_siso(d["q"][:, :, None, :], d["k"][:, :, None, :], d["v"], d["adt"],
                              d["dt"], d["trap"], d["q_bias"].reshape(h, n),
                              d["k_bias"].reshape(h, n), cos, sin, D=d["D"], z=d["z"])
    want = want.reshape(b, l, h * p)
    assert np.abs(y - want).max() / max(np.abs(want).max(), 1e-30) <= REL_TOL


def test_mixer_prologue_rejects_host_tensor_and_wrong_width():
    d, dims = load_mixer(MIXER[0])
    with pytest.raises(ValueError):
        prologue(d, dims, torch.from_numpy(d["proj"]))
    with pytest.raises(ValueError):
        prologue(d, dims, torch.from_numpy(d["proj"][..., :-1].copy()).cuda())


def test_mixer_scan_bf16_tensor_path():
    """A mixer at the tensor-core shape (d_state 128, headdim 64):
    precision "bf16" routes the prologue's outputs, with the angles passed
    broadcast over heads, to the tcgen05 scan; against the fp32 mixer scan at
    the bf16 tolerance of the tensor-core tests."""
    g = torch.Generator(device="cuda").manual_seed(4)
    H, P, N, NA, b, l = 3, 64, 128, 32, 2, 300
    from armhackathon_b200.mamba3_mixer import proj_width
    W = proj_width(H, P, N, 1, NA)
    proj = torch.randn(b, l, W, device="cuda", generator=g)
    rn = lambda *s: torch.randn(*s, device="cuda", generator=g)  # noqa: E731
    kw = dict(nheads=H, headdim=P, d_state=N, n_angles=NA, dt_bias=rn(H) - 2,
              B_norm_weight=1 + 0.1 * rn(N), C_norm_weight=1 + 0.1 * rn(N), D=rn(H),
              B_bias=0.1 * rn(H, 1, N), C_bias=0.1 * rn(H, 1, N))
    want = arm().mamba3_mixer_scan(proj, **kw).cpu().numpy()
    got = arm().mamba3_mixer_scan(proj, **kw, precision="bf16").float().cpu().numpy()
    assert np.abs(got - want).max() / np.abs(want).max() <= 2e-2
