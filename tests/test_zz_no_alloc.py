"""gdr_mixed_noalloc: the continuous-batch launch for callers that cannot
allocate device memory (a budgeted serving loop, code inside another
framework's memory pool, a thread that must not take the allocator's locks).
Its work list lives in a fixed array inside the library instead of a caller
workspace. Checked through the C ABI against gdr_mixed on the same inputs, on
two calls in a row (the array keeps the first call's contents, which the
second must not see), and against its capacity limit.

This file is collected last on purpose: it must pass in a fresh process, where
its first call sets the array up, and after every other test."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from bunsen_b200 import _lib
from bunsen_b200.rule import GatedDeltaRule
from tests.conftest import TOL_BF16_OUT, TOL_BF16_STATE, rel_err

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _batch(lens, seed, hq=2, hv=4):
    gen = torch.Generator(device=DEV).manual_seed(seed)
    t = sum(lens)
    f = dict(device=DEV, generator=gen)
    unit = lambda a: a / a.norm(dim=-1, keepdim=True)  # noqa: E731
    n_slots = len(lens) + 2
    return {
        "q": unit(torch.randn(t, hq, 128, **f)).to(torch.bfloat16),
        "k": unit(torch.randn(t, hq, 128, **f)).to(torch.bfloat16),
        "v": torch.randn(t, hv, 128, **f).to(torch.bfloat16),
        "g": torch.log(torch.rand(t, hv, **f) * 0.099 + 0.9),
        "beta": torch.sigmoid(torch.randn(t, hv, **f)),
        "cu": torch.tensor(np.concatenate([[0], np.cumsum(lens)]), dtype=torch.int32, device=DEV),
        "pool": torch.randn(n_slots, hv, 128, 128, **f) * 0.1,
        "slots": torch.randperm(n_slots, generator=torch.Generator().manual_seed(seed))[
            :len(lens)].to(torch.int32).to(DEV),
    }


def _noalloc(x, pool, out):
    lib = _lib.load()
    p = GatedDeltaRule().params(x["q"], x["v"], x["cu"])
    return lib.gdr_mixed_noalloc(
        ctypes.byref(p), x["q"].data_ptr(), x["k"].data_ptr(), x["v"].data_ptr(),
        x["g"].data_ptr(), x["beta"].data_ptr(), pool.data_ptr(), x["slots"].data_ptr(),
        pool.shape[0], out.data_ptr(), x["cu"].data_ptr(),
        torch.cuda.current_stream().cuda_stream)


def test_noalloc_matches_mixed_on_two_calls_in_a_row():
    lib = _lib.load()
    # The second batch is smaller than the first, so stale work-list entries
    # from the first call sit past the second call's end.
    for seed, lens in ((31, [190, 1, 1, 70, 1, 0, 129, 1, 1, 64]), (32, [1, 65, 1])):
        x = _batch(lens, seed)
        pool_ref, pool_na = x["pool"].clone(), x["pool"].clone()
        out_ref = GatedDeltaRule().mixed(x["q"], x["k"], x["v"], x["g"], x["beta"], pool_ref,
                                         cu_seqlens=x["cu"], state_slots=x["slots"])
        out_na = torch.empty_like(out_ref)
        assert _noalloc(x, pool_na, out_na) == _lib.GDR_OK
        torch.cuda.synchronize()
        assert lib.gdr_device_error() == _lib.GDR_OK
        assert rel_err(out_na.float().cpu().numpy(), out_ref.float().cpu().numpy()) < TOL_BF16_OUT
        assert rel_err(pool_na.cpu().numpy(), pool_ref.cpu().numpy()) < TOL_BF16_STATE


def test_noalloc_rejects_more_sequences_than_it_holds():
    n = _lib.GDR_MIXED_NOALLOC_MAX_SEQS + 1
    x = _batch([1, 1], seed=33)
    x["cu"] = torch.arange(n + 1, dtype=torch.int32, device=DEV).clamp(max=2)
    out = torch.empty_like(x["v"])
    assert _noalloc(x, x["pool"], out) == _lib.GDR_ERR_CAPACITY
    assert b"GDR_MIXED_NOALLOC_MAX_SEQS" in _lib.load().gdr_status_string(_lib.GDR_ERR_CAPACITY)
