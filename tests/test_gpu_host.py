"""gdr_chunked_host: the chunked rule on host tensors, streamed through the
GPU in groups of sequences, against the device call and the CPU oracle.

Tolerances as for every bf16 run: 2e-2 on outputs, 1e-2 on states; the host
call with the single-pass kernel is bit-identical to the device call (the
sequences are independent, so grouping them changes nothing)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from bunsen_b200 import workloads
from bunsen_b200.rule import GatedDeltaRule
from tests.conftest import TOL_BF16_OUT, TOL_BF16_STATE, rel_err
from tests.test_gpu_rule import _np, _oracle, _rand_bf16

pytestmark = pytest.mark.gpu


def _host(x):
    return {k: (v.cpu().pin_memory() if isinstance(v, torch.Tensor) else v) for k, v in x.items()}


def _both(x, rule):
    dev_o, dev_s = rule.chunked(x["q"], x["k"], x["v"], x["g"], x["beta"], x.get("state"),
                                cu_seqlens=x.get("cu_seqlens"))
    h = _host(x)
    host_o, host_s = rule.chunked_host(h["q"], h["k"], h["v"], h["g"], h["beta"], h.get("state"),
                                       cu_seqlens=h.get("cu_seqlens"))
    torch.cuda.synchronize()
    return _np(dev_o), _np(dev_s), _np(host_o), _np(host_s)


@pytest.mark.parametrize("state", [False, True])
def test_host_call_matches_device_call_and_oracle(state):
    lens = [700, 64 * 5 + 3, 1, 0, 1500, 129, 64, 2000, 33, 900]
    x = _rand_bf16(lens, state=state, seed=21)
    rule = GatedDeltaRule(algo="tensor")
    do, ds, ho, hs = _both(x, rule)
    assert (do == ho).all() and (ds == hs).all()
    wo, ws = _oracle("chunked", x)
    assert rel_err(ho, wo) < TOL_BF16_OUT and rel_err(hs, ws) < TOL_BF16_STATE


def test_host_call_dense_batch():
    x = _rand_bf16([300] * 20, state=True, packed=False, seed=22)
    do, ds, ho, hs = _both(x, GatedDeltaRule(algo="tensor"))
    assert (do == ho).all() and (ds == hs).all()


def test_host_call_at_ragged_scale_with_auto():
    """A quarter of the ragged pack, the default algorithm (each group of
    sequences may be split differently from the whole pack)."""
    w = workloads.get("ragged_prefill", scale=0.25)
    x = workloads.make_inputs(w, "cuda", seed=23)
    do, ds, ho, hs = _both(x, GatedDeltaRule())
    assert rel_err(ho, do) < TOL_BF16_OUT and rel_err(hs, ds) < TOL_BF16_STATE


def test_host_call_state_in_place_and_async():
    x = _host(_rand_bf16([400, 90, 1000], state=True, seed=24))
    rule = GatedDeltaRule(algo="tensor")
    o1, s1 = rule.chunked_host(x["q"], x["k"], x["v"], x["g"], x["beta"], x["state"],
                               cu_seqlens=x["cu_seqlens"])
    st = x["state"].clone().pin_memory()
    out = torch.empty_like(o1).pin_memory()
    rule.chunked_host(x["q"], x["k"], x["v"], x["g"], x["beta"], st, cu_seqlens=x["cu_seqlens"],
                      out=out, state_out=st, synchronize=False)
    torch.cuda.current_stream().synchronize()
    assert torch.equal(out, o1) and torch.equal(st, s1)
