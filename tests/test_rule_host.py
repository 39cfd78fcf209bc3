"""The host-side GatedDeltaRule mirror raises on bunsen's contract
violations before it touches a device (delta_rule.rs:135-150, :233)."""

from __future__ import annotations

import pytest
import torch

from bunsen_b200.rule import GatedDeltaRule, check_shapes


def _x(*shape):
    return torch.zeros(*shape)


def test_defaults_are_bunsens():
    r = GatedDeltaRule()
    assert r.qk_l2norm_eps == 1e-6 and r.chunk_size == 64
    assert r.with_chunk_size(4).chunk_size == 4
    assert r.with_qk_l2norm_eps(None).qk_l2norm_eps is None


@pytest.mark.parametrize("args,match", [
    ((_x(2, 5, 3, 4), _x(2, 5, 3, 5), _x(2, 5, 3, 6), _x(2, 5, 3), _x(2, 5, 3)), "must match q"),
    ((_x(2, 5, 3, 4), _x(2, 5, 3, 4), _x(2, 4, 3, 6), _x(2, 5, 3), _x(2, 5, 3)), "leading dims"),
    ((_x(2, 5, 3, 4), _x(2, 5, 3, 4), _x(2, 5, 3, 6), _x(2, 5, 2), _x(2, 5, 3)), "`g` is"),
    ((_x(2, 5, 3, 4), _x(2, 5, 3, 4), _x(2, 5, 3, 6), _x(2, 5, 3), _x(2, 5)), "`beta` is"),
    ((_x(2, 5, 2, 4), _x(2, 5, 2, 4), _x(2, 5, 3, 6), _x(2, 5, 3), _x(2, 5, 3)), "divide"),
])
def test_shape_contracts(args, match):
    with pytest.raises(ValueError, match=match):
        check_shapes(*args, None, None)


def test_state_shape_contract():
    q = _x(2, 5, 3, 4)
    with pytest.raises(ValueError, match="Dk, Dv"):
        check_shapes(q, q, _x(2, 5, 3, 6), _x(2, 5, 3), _x(2, 5, 3), _x(2, 3, 6, 4), None)


def test_zero_chunk_panics_like_bunsen():
    q = _x(1, 2, 1, 4)
    with pytest.raises(AssertionError, match="at least one position"):
        GatedDeltaRule(chunk_size=0).chunked(q, q, q, _x(1, 2, 1), _x(1, 2, 1))


def test_cpu_tensors_are_refused():
    q = _x(1, 2, 1, 4)
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        GatedDeltaRule().chunked(q, q, q, _x(1, 2, 1), _x(1, 2, 1))
