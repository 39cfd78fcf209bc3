"""Shared test plumbing.

Markers: ``gpu`` -- needs a B200 and the built ``bunsen_b200/libgdr.so``; the
rest runs on any CPU. Tolerances are max relative errors, ``max|got - want| /
max|want|`` over a tensor (a norm-wise bound, so entries near zero do not
dominate): 1e-4 for f32 runs, 2e-2 on outputs and 1e-2 on states for bf16
inputs.
"""

from __future__ import annotations

import pathlib
import sys

import numpy as np
import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

TOL_F32 = 1e-4
TOL_BF16_OUT = 2e-2
TOL_BF16_STATE = 1e-2


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and libgdr.so")


def rel_err(got, want) -> float:
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    assert got.shape == want.shape, (got.shape, want.shape)
    scale = np.abs(want).max()
    return float(np.abs(got - want).max() / (scale if scale > 0 else 1.0))


@pytest.fixture(scope="session")
def golden():
    """The committed golden vectors (tests/golden/*.npz)."""
    d = ROOT / "tests" / "golden"
    return {p.stem: dict(np.load(p)) for p in sorted(d.glob("*.npz"))}
