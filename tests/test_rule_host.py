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


def test_layer_options_are_checked_before_the_device():
    """gates replace g and beta; the norm's gate is shaped and typed like v;
    both are refused on the host when malformed."""
    q = _x(1, 5, 2, 4)
    v = _x(1, 5, 4, 6)
    a = _x(1, 5, 4)
    gates = (a, a, _x(4), _x(4))
    with pytest.raises(ValueError, match="g and beta are None"):
        GatedDeltaRule().chunked(q, q, v, a, a, gates=gates)
    with pytest.raises(TypeError, match="share one dtype"):
        GatedDeltaRule().chunked(q, q, v, None, None, gates=(a, a.double(), _x(4), _x(4)))
    with pytest.raises(ValueError, match="shaped and typed like v"):
        GatedDeltaRule().chunked(q, q, v, a, a, norm=(_x(1, 5, 4, 5), _x(6), 1e-6))
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        GatedDeltaRule().chunked(q, q, v, None, None, gates=gates, norm=(v, _x(6), 1e-6))


def test_layer_module_refuses_host_tensors():
    from bunsen_b200.layer import causal_conv1d, gated_norm, state_reorder
    with pytest.raises(RuntimeError, match="CUDA"):
        causal_conv1d(_x(1, 4, 8), _x(8, 4))
    with pytest.raises(RuntimeError, match="CUDA"):
        gated_norm(_x(3, 8), _x(3, 8), _x(8), 1e-6)
    with pytest.raises(RuntimeError, match="CUDA"):
        state_reorder(_x(3, 8), torch.zeros(3, dtype=torch.int32))
