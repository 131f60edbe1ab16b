"""Shared pytest set-up: the ``gpu`` marker and import paths."""

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
for p in (ROOT, ROOT / "oracle"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line(
        "markers", "gpu: needs a CUDA device (B200); run with -m gpu")


@pytest.fixture(scope="session")
def golden_dir():
    return GOLDEN


@pytest.fixture
def knobs():
    """Set library kernel-selection overrides (``_ffi.KNOBS``) for one test;
    every knob it set goes back to the default (0) afterwards."""
    from armhackathon_b200 import _ffi
    used = []

    def set_knobs(**kw):
        for k, v in kw.items():
            _ffi.set_kernel_override(k, v)
            used.append(k)

    yield set_knobs
    for k in used:
        _ffi.set_kernel_override(k, 0)
