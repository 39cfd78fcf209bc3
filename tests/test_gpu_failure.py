"""Failure detection without a GPU fault: a bounded device-side wait that runs
out is reported on the host, and the context stays usable; bad arguments are
refused before anything launches."""

from __future__ import annotations

import pytest
import torch

from bunsen_b200 import _lib
from bunsen_b200.rule import GatedDeltaRule

pytestmark = pytest.mark.gpu


def test_a_wait_that_runs_out_is_reported_and_the_context_survives():
    lib = _lib.load()
    assert lib.gdr_device_error() == _lib.GDR_OK
    assert lib.gdr_selftest_wait_timeout(2_000_000, None) == _lib.GDR_OK  # 2 ms
    torch.cuda.synchronize()
    assert lib.gdr_device_error() == _lib.GDR_ERR_TIMEOUT
    assert lib.gdr_device_error() == _lib.GDR_OK  # the record was cleared
    # The context still runs the rule.
    x = torch.randn(1, 70, 1, 128, device="cuda").bfloat16()
    g = -torch.rand(1, 70, 1, device="cuda")
    b = torch.rand(1, 70, 1, device="cuda")
    out, st = GatedDeltaRule().chunked(x, x, x, g, b)
    torch.cuda.synchronize()
    assert torch.isfinite(out.float()).all() and torch.isfinite(st).all()
    assert lib.gdr_device_error() == _lib.GDR_OK


def test_selftest_limit_is_bounded():
    lib = _lib.load()
    assert lib.gdr_selftest_wait_timeout(0, None) == _lib.GDR_ERR_INVALID
    assert lib.gdr_selftest_wait_timeout(10**9, None) == _lib.GDR_ERR_INVALID
