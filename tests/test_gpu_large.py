"""Tensors past 2^31 elements: every index the kernels form from positions,
heads and features must be 64-bit. Each case is checked by a property the
domain gives (a sequence, or a row, does not depend on the others), so the
last part of a large call must equal an independent small call on that part
alone -- bit for bit where the path is the same per-sequence computation.

About 15 GB of device memory at most; a few seconds each on a B200."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from bunsen_b200 import _lib, workloads
from bunsen_b200.layer import causal_conv1d, gated_norm
from bunsen_b200.rule import GatedDeltaRule
from tests.conftest import TOL_BF16_OUT, TOL_BF16_STATE, rel_err

pytestmark = pytest.mark.gpu
DEV = "cuda"
BIG = 2**31


def _ok():
    torch.cuda.synchronize()
    assert _lib.load().gdr_device_error() == _lib.GDR_OK


@pytest.fixture(autouse=True)
def _free():
    yield
    torch.cuda.empty_cache()


def _ragged(lens, seed):
    """bf16 q/k/v at 16 key / 32 value heads, d 128, with f32 states."""
    gen = torch.Generator(device=DEV).manual_seed(seed)
    t, hq, hv, d = sum(lens), 16, 32, 128
    x = {"q": torch.randn(t, hq, d, device=DEV, generator=gen, dtype=torch.bfloat16),
         "k": torch.randn(t, hq, d, device=DEV, generator=gen, dtype=torch.bfloat16),
         "v": torch.randn(t, hv, d, device=DEV, generator=gen, dtype=torch.bfloat16),
         "g": torch.log(torch.rand(t, hv, device=DEV, generator=gen) * 0.099 + 0.9),
         "beta": torch.sigmoid(torch.randn(t, hv, device=DEV, generator=gen)),
         "state": torch.randn(len(lens), hv, d, d, device=DEV, generator=gen) * 0.1,
         "cu_seqlens": torch.tensor(np.concatenate([[0], np.cumsum(lens)]), dtype=torch.int32,
                                    device=DEV)}
    return x


def _last_alone(x, lens):
    a = sum(lens[:-1])
    y = {k: x[k][a:] for k in ("q", "k", "v", "g", "beta")}
    y["state"] = x["state"][-1:]
    y["cu_seqlens"] = torch.tensor([0, lens[-1]], dtype=torch.int32, device=DEV)
    return a, y


@pytest.mark.parametrize("algo", ["tensor", "auto"])
def test_prefill_past_2_31_elements(algo):
    """v and out hold 32 heads x 128 features of 540 000 positions (2.2e9
    elements): the last sequence, whose rows sit past 2^31 elements, against
    the same sequence alone. The single-pass kernel gives the same bits; the
    split form plans the two calls differently, so it agrees to rounding."""
    lens = [300_000, 239_000, 1_000]
    assert sum(lens) * 32 * 128 > BIG
    x = _ragged(lens, seed=1)
    rule = GatedDeltaRule(algo=algo)
    out, st = rule.chunked(x["q"], x["k"], x["v"], x["g"], x["beta"], x["state"],
                           cu_seqlens=x["cu_seqlens"])
    _ok()
    a, y = _last_alone(x, lens)
    o1, s1 = rule.chunked(y["q"], y["k"], y["v"], y["g"], y["beta"], y["state"],
                          cu_seqlens=y["cu_seqlens"])
    _ok()
    if algo == "tensor":
        assert torch.equal(out[a:], o1) and torch.equal(st[-1:], s1)
    else:
        assert rel_err(workloads.to_numpy_f32(out[a:]), workloads.to_numpy_f32(o1)) < TOL_BF16_OUT
        assert rel_err(st[-1:].cpu().numpy(), s1.cpu().numpy()) < TOL_BF16_STATE


def test_conv_past_2_31_elements():
    """The layer's conv over 270 000 positions x 8192 channels (2.2e9
    elements in and out): the last sequence against itself alone, bit for bit."""
    lens = [200_000, 69_000, 1_000]
    c, taps = 8192, 4
    assert sum(lens) * c > BIG
    gen = torch.Generator(device=DEV).manual_seed(2)
    x = torch.randn(sum(lens), c, device=DEV, generator=gen, dtype=torch.bfloat16)
    w = (torch.randn(c, taps, device=DEV, generator=gen) * 0.5).bfloat16()
    s0 = torch.randn(len(lens), taps - 1, c, device=DEV, generator=gen)
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]), dtype=torch.int32, device=DEV)
    splits = (2048, 4096)
    (q, k, v), nxt = causal_conv1d(x, w, s0, cu_seqlens=cu, silu=True, splits=splits)
    _ok()
    a = sum(lens[:-1])
    cu1 = torch.tensor([0, lens[-1]], dtype=torch.int32, device=DEV)
    (q1, k1, v1), n1 = causal_conv1d(x[a:], w, s0[-1:], cu_seqlens=cu1, silu=True, splits=splits)
    _ok()
    assert torch.equal(q[a:], q1) and torch.equal(k[a:], k1) and torch.equal(v[a:], v1)
    assert torch.equal(nxt[-1:], n1)


def test_gated_norm_past_2_31_elements():
    """17 Mi rows of 128 bf16 features (2.2e9 elements): the last rows against
    the same rows alone, bit for bit."""
    rows = 17 * 2**20
    assert rows * 128 > BIG
    gen = torch.Generator(device=DEV).manual_seed(3)
    x = torch.randn(rows, 128, device=DEV, generator=gen, dtype=torch.bfloat16)
    z = torch.randn(rows, 128, device=DEV, generator=gen, dtype=torch.bfloat16)
    w = torch.rand(128, device=DEV, generator=gen) + 0.5
    y = gated_norm(x, z, w, 1e-6)
    _ok()
    tail = 4099
    y1 = gated_norm(x[-tail:].clone(), z[-tail:].clone(), w, 1e-6)
    _ok()
    assert torch.equal(y[-tail:], y1)


def test_decode_states_past_2_31_elements():
    """A decode step over 4200 rows x 32 heads of 128 x 128 f32 states (2.2e9
    elements, updated in place): the last rows against themselves alone."""
    rows, hq, hv, d = 4200, 16, 32, 128
    assert rows * hv * d * d > BIG
    gen = torch.Generator(device=DEV).manual_seed(4)
    st = torch.randn(rows, hv, d, d, device=DEV, generator=gen) * 0.1
    q = torch.randn(rows, 1, hq, d, device=DEV, generator=gen, dtype=torch.bfloat16)
    k = torch.randn(rows, 1, hq, d, device=DEV, generator=gen, dtype=torch.bfloat16)
    v = torch.randn(rows, 1, hv, d, device=DEV, generator=gen, dtype=torch.bfloat16)
    g = torch.log(torch.rand(rows, 1, hv, device=DEV, generator=gen) * 0.099 + 0.9)
    beta = torch.sigmoid(torch.randn(rows, 1, hv, device=DEV, generator=gen))
    tail = 7
    st_tail = st[-tail:].clone()
    rule = GatedDeltaRule()
    out, _ = rule.recurrent(q, k, v, g, beta, st, state_out=st)
    _ok()
    o1, s1 = rule.recurrent(q[-tail:], k[-tail:], v[-tail:], g[-tail:], beta[-tail:], st_tail)
    _ok()
    assert torch.equal(out[-tail:], o1) and torch.equal(st[-tail:], s1)


def test_mixed_pool_past_2_31_elements():
    """gdr_mixed with a pool of 4200 slots (2.2e9 f32 elements): a prefill
    segment and decode rows whose slots sit past 2^31 elements, against the
    same batch on a pool holding just those slots."""
    n_slots, hq, hv, d = 4200, 16, 32, 128
    assert n_slots * hv * d * d > BIG
    lens = [300, 1, 1, 1]
    x = _ragged(lens, seed=5)
    slots = torch.tensor([4199, 4100, 3000, 4198], dtype=torch.int32, device=DEV)
    pool = torch.zeros(n_slots, hv, d, d, device=DEV)
    pool[slots.long()] = x["state"]
    rule = GatedDeltaRule()
    out = rule.mixed(x["q"], x["k"], x["v"], x["g"], x["beta"], pool, cu_seqlens=x["cu_seqlens"],
                     state_slots=slots)
    _ok()
    small = x["state"].clone()
    out1 = rule.mixed(x["q"], x["k"], x["v"], x["g"], x["beta"], small,
                      cu_seqlens=x["cu_seqlens"])
    _ok()
    assert torch.equal(out, out1) and torch.equal(pool[slots.long()], small)
