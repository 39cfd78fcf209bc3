"""gdr_mixed -- prefill segments and decode rows of different sequences in one
launch, states in place in a slot pool -- against the CPU oracle's chunked
(prefill) and recurrent (decode) forms on the same inputs."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from bunsen_b200 import _lib, workloads
from bunsen_b200.rule import GatedDeltaRule
from oracle import oracle
from tests.conftest import TOL_BF16_OUT, TOL_BF16_STATE, rel_err

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _batch(lens, hq=2, hv=4, n_slots=None, seed=9):
    gen = torch.Generator(device=DEV).manual_seed(seed)
    t = sum(lens)
    f = dict(device=DEV, generator=gen)
    unit = lambda a: a / a.norm(dim=-1, keepdim=True)  # noqa: E731
    x = {"q": unit(torch.randn(t, hq, 128, **f)).to(torch.bfloat16),
         "k": unit(torch.randn(t, hq, 128, **f)).to(torch.bfloat16),
         "v": torch.randn(t, hv, 128, **f).to(torch.bfloat16),
         "g": torch.log(torch.rand(t, hv, **f) * 0.099 + 0.9),
         "beta": torch.sigmoid(torch.randn(t, hv, **f)),
         "cu_seqlens": torch.tensor(np.concatenate([[0], np.cumsum(lens)]), dtype=torch.int32,
                                    device=DEV)}
    n_slots = n_slots or len(lens) + 3
    x["pool"] = torch.randn(n_slots, hv, 128, 128, **f) * 0.1
    perm = torch.randperm(n_slots, generator=torch.Generator().manual_seed(seed))[:len(lens)]
    x["slots"] = perm.to(torch.int32).to(DEV)
    return x


def _expect(x, lens, pool0):
    """Oracle: chunked for segments longer than 1, recurrent for single tokens,
    each from its slot's state in `pool0` (the pool before the call); slots
    not named keep their state."""
    f = lambda t: t.detach().to("cpu", torch.float32).numpy()  # noqa: E731
    q, k, v, g, b = (f(x[n]) for n in ("q", "k", "v", "g", "beta"))
    pool = f(pool0).copy()
    out = np.zeros(v.shape, np.float32)
    cu = np.concatenate([[0], np.cumsum(lens)])
    slots = x["slots"].cpu().numpy()
    for s, (a, e) in enumerate(zip(cu[:-1], cu[1:])):
        if e == a:
            continue
        fn = oracle.chunked if e - a > 1 else oracle.recurrent
        o, st = fn(q[None, a:e], k[None, a:e], v[None, a:e], g[None, a:e], b[None, a:e],
                   pool[slots[s]][None])
        out[a:e] = o[0]
        pool[slots[s]] = st[0]
    return out, pool


@pytest.mark.parametrize("lens", [[200, 1, 1, 64, 1, 0, 130, 1], [1] * 9, [300, 65, 2]])
def test_mixed_against_oracle(lens):
    x = _batch(lens)
    pool0 = x["pool"].clone()
    out = GatedDeltaRule().mixed(x["q"], x["k"], x["v"], x["g"], x["beta"], x["pool"],
                                 cu_seqlens=x["cu_seqlens"], state_slots=x["slots"])
    torch.cuda.synchronize()
    assert _lib.load().gdr_device_error() == _lib.GDR_OK
    wo, wp = _expect(x, lens, pool0)
    got = out.float().cpu().numpy()
    assert rel_err(got, wo) < TOL_BF16_OUT
    assert rel_err(x["pool"].cpu().numpy(), wp) < TOL_BF16_STATE


def test_mixed_matches_separate_calls_at_benchmark_shape():
    """The mixed benchmark shape, scaled (2 prefill segments of 2048 tokens +
    128 decode rows, 16/32 heads): one gdr_mixed launch against gdr_chunked on
    the segments and gdr_recurrent on the rows."""
    w = workloads.get("mixed", scale=0.125)
    x = workloads.make_inputs(w, DEV, seed=12)
    pool = x["state"].clone()
    rule = GatedDeltaRule(algo="tensor")  # the one-pass kernel gdr_mixed's prefill runs
    out = rule.mixed(x["q"], x["k"], x["v"], x["g"], x["beta"], pool, cu_seqlens=x["cu_seqlens"])
    n_pre = sum(1 for L in w.seqlens if L > 1)
    t_pre = sum(L for L in w.seqlens if L > 1)
    cu = x["cu_seqlens"]
    o1, s1 = rule.chunked(x["q"][:t_pre], x["k"][:t_pre], x["v"][:t_pre], x["g"][:t_pre],
                          x["beta"][:t_pre], x["state"][:n_pre], cu_seqlens=cu[:n_pre + 1])
    dq = lambda t: t[t_pre:][:, None].contiguous()  # noqa: E731
    o2, s2 = rule.recurrent(dq(x["q"]), dq(x["k"]), dq(x["v"]), dq(x["g"]), dq(x["beta"]),
                            x["state"][n_pre:])
    torch.cuda.synchronize()
    assert torch.equal(out[:t_pre], o1) and torch.equal(pool[:n_pre], s1)
    assert torch.equal(out[t_pre:], o2[:, 0]) and torch.equal(pool[n_pre:], s2)


def test_mixed_bad_slot_is_reported_and_skipped():
    lens = [70, 1]
    x = _batch(lens, n_slots=4)
    x["slots"] = torch.tensor([1, 9], dtype=torch.int32, device=DEV)  # 9 is outside the pool
    before = x["pool"].clone()
    GatedDeltaRule().mixed(x["q"], x["k"], x["v"], x["g"], x["beta"], x["pool"],
                           cu_seqlens=x["cu_seqlens"], state_slots=x["slots"])
    torch.cuda.synchronize()
    assert _lib.load().gdr_device_error() == _lib.GDR_ERR_INVALID
    assert _lib.load().gdr_device_error() == _lib.GDR_OK  # the record was cleared
    assert not torch.equal(x["pool"][1], before[1])  # the good slot ran
    for s in (0, 2, 3):
        assert torch.equal(x["pool"][s], before[s])


def test_mixed_in_a_persistent_grid_with_more_items_than_ctas():
    """Many more (sequence, head) items than resident CTAs: every CTA pulls
    several items, prefill and decode, so one CTA runs several prefill items
    (each allocating and freeing TMEM) one after another."""
    rng = np.random.default_rng(3)
    lens = [int(x) for x in rng.integers(2, 80, 200)] + [1] * 300 + [130, 64]
    x = _batch(lens, hq=2, hv=4)
    pool0 = x["pool"].clone()
    out = GatedDeltaRule().mixed(x["q"], x["k"], x["v"], x["g"], x["beta"], x["pool"],
                                 cu_seqlens=x["cu_seqlens"], state_slots=x["slots"])
    torch.cuda.synchronize()
    assert _lib.load().gdr_device_error() == _lib.GDR_OK
    wo, wp = _expect(x, lens, pool0)
    assert rel_err(out.float().cpu().numpy(), wo) < TOL_BF16_OUT
    assert rel_err(x["pool"].cpu().numpy(), wp) < TOL_BF16_STATE


def test_mixed_rejects_a_short_workspace():
    x = _batch([5, 1])
    ws = torch.empty(4, dtype=torch.uint8, device=DEV)
    with pytest.raises(ValueError):
        GatedDeltaRule().mixed(x["q"], x["k"], x["v"], x["g"], x["beta"], x["pool"],
                               cu_seqlens=x["cu_seqlens"], state_slots=x["slots"], workspace=ws)
