"""Sequence-parallel prefill (``GDR_ALGO_TENSOR_SPLIT``) through the C ABI:
long sequences cut into segments whose state transitions are chained by a
scan, against the CPU oracle and against the one-pass tensor-core kernel.

Tolerances as for every bf16 run: 2e-2 on outputs, 1e-2 on states
(max |got - want| / max |want|)."""

from __future__ import annotations

import pytest
import torch

from bunsen_b200 import workloads
from bunsen_b200.rule import GatedDeltaRule
from tests.conftest import TOL_BF16_OUT, TOL_BF16_STATE, rel_err
from tests.test_gpu_rule import DEV, _gpu, _np, _oracle, _rand_bf16

pytestmark = pytest.mark.gpu

# Lengths with segments of every kind: whole chunks, a ragged tail, a
# sequence of one position, an empty one, and one just over a chunk.
LENS = [700, 64 * 5 + 3, 1, 0, 1500, 129, 64]


@pytest.mark.parametrize("split_chunks", [1, 2, 3, 5])
@pytest.mark.parametrize("state", [False, True])
def test_split_against_oracle(split_chunks, state):
    x = _rand_bf16(LENS, state=state, seed=11)
    o, s = _gpu("chunked", x, GatedDeltaRule(algo="tensor_split", split_chunks=split_chunks))
    wo, ws = _oracle("chunked", x)
    assert rel_err(o, wo) < TOL_BF16_OUT, rel_err(o, wo)
    assert rel_err(s, ws) < TOL_BF16_STATE, rel_err(s, ws)


def test_split_dense_batch_against_oracle():
    x = _rand_bf16([1000, 1000, 1000], state=True, packed=False, seed=12)
    o, s = _gpu("chunked", x, GatedDeltaRule(algo="tensor_split", split_chunks=4))
    wo, ws = _oracle("chunked", x)
    assert rel_err(o, wo) < TOL_BF16_OUT and rel_err(s, ws) < TOL_BF16_STATE


def test_split_long_sequence_many_segments():
    """4096 positions in 64 one-chunk segments: a 62-step scan."""
    x = _rand_bf16([4096], hq=1, hv=2, state=True, seed=13)
    o, s = _gpu("chunked", x, GatedDeltaRule(algo="tensor_split", split_chunks=1))
    wo, ws = _oracle("chunked", x)
    assert rel_err(o, wo) < TOL_BF16_OUT and rel_err(s, ws) < TOL_BF16_STATE


def test_split_chosen_length_matches_one_pass_at_full_ragged_size():
    """The full ragged pack (131072 positions, 64 sequences) with the 4 value
    heads one GPU of eight holds: the segment length the call chooses against
    the one-pass kernel."""
    w = workloads.get("ragged_prefill")
    x = workloads.make_inputs(w, DEV, seed=31)
    heads = {"q": 2, "k": 2, "v": 4, "g": 4, "beta": 4, "state": 4}
    x = {k: (v[:, :heads[k]].contiguous() if k in heads else v) for k, v in x.items()}
    o_s, s_s = _gpu("chunked", x, GatedDeltaRule(algo="tensor_split"))
    o_1, s_1 = _gpu("chunked", x, GatedDeltaRule(algo="tensor"))
    assert rel_err(o_s, o_1) < TOL_BF16_OUT and rel_err(s_s, s_1) < TOL_BF16_STATE


def test_split_state_in_place_and_repeatable():
    """state_out may be state_in, and a repeated call gives the same bits."""
    x = _rand_bf16(LENS, state=True, seed=14)
    rule = GatedDeltaRule(algo="tensor_split", split_chunks=2)
    o1, s1 = _gpu("chunked", x, rule)
    o2, s2 = _gpu("chunked", x, rule)
    assert (o1 == o2).all() and (s1 == s2).all()
    st = x["state"].clone()
    out, got = rule.chunked(x["q"], x["k"], x["v"], x["g"], x["beta"], st,
                            cu_seqlens=x["cu_seqlens"], state_out=st)
    torch.cuda.synchronize()
    assert got.data_ptr() == st.data_ptr()
    assert (_np(out) == o1).all() and (_np(st) == s1).all()


def test_release_scratch_and_run_again():
    """gdr_release_scratch returns the pool's unused memory; the next split
    call reserves it again and gives the same bits."""
    from bunsen_b200 import _lib

    x = _rand_bf16(LENS, state=True, seed=15)
    rule = GatedDeltaRule(algo="tensor_split", split_chunks=2)
    o1, s1 = _gpu("chunked", x, rule)
    assert _lib.load().gdr_release_scratch() == _lib.GDR_OK
    o2, s2 = _gpu("chunked", x, rule)
    assert (o1 == o2).all() and (s1 == s2).all()
