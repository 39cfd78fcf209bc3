"""Calls issued at the same time: on several streams of one host thread, and
from several host threads (ctypes releases the GIL for the call), as a
serving process issues them. Each result must equal the same call made alone
-- bit for bit: the split form's scratch comes from the library pool in
stream order, the host-buffer path shares the library's worker streams, and
the library's lazily made state is set up under a lock."""

from __future__ import annotations

import threading

import numpy as np
import pytest
import torch

from bunsen_b200 import _lib
from bunsen_b200.rule import GatedDeltaRule

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _batch(lens, seed, device=DEV):
    gen = torch.Generator(device=DEV).manual_seed(seed)
    t, hq, hv, d = sum(lens), 4, 8, 128
    x = {"q": torch.randn(t, hq, d, device=DEV, generator=gen, dtype=torch.bfloat16),
         "k": torch.randn(t, hq, d, device=DEV, generator=gen, dtype=torch.bfloat16),
         "v": torch.randn(t, hv, d, device=DEV, generator=gen, dtype=torch.bfloat16),
         "g": torch.log(torch.rand(t, hv, device=DEV, generator=gen) * 0.099 + 0.9),
         "beta": torch.sigmoid(torch.randn(t, hv, device=DEV, generator=gen)),
         "state": torch.randn(len(lens), hv, d, d, device=DEV, generator=gen) * 0.1,
         "cu_seqlens": torch.tensor(np.concatenate([[0], np.cumsum(lens)]), dtype=torch.int32,
                                    device=DEV)}
    return {k: v.to(device) for k, v in x.items()}


def _call(rule, x, form="chunked"):
    return getattr(rule, form)(x["q"], x["k"], x["v"], x["g"], x["beta"], x["state"],
                               cu_seqlens=x["cu_seqlens"])


# Long sequences at 8 value heads: GDR_ALGO_AUTO takes the split form (plan,
# two passes, scan, scratch from the pool); the others are single launches.
BATCHES = [([3000, 17, 2500, 64], "auto"), ([4000, 1, 300], "auto"),
           ([700, 1, 65, 129], "tensor"), ([1] * 40, "recurrent")]


def _alone():
    out = []
    for i, (lens, algo) in enumerate(BATCHES):
        x = _batch(lens, seed=i)
        form = "recurrent" if algo == "recurrent" else "chunked"
        rule = GatedDeltaRule(algo="auto" if algo == "recurrent" else algo)
        o, s = _call(rule, x, form)
        out.append((x, rule, form, o, s))
    torch.cuda.synchronize()
    return out


def test_calls_on_several_streams_at_once():
    ref = _alone()
    streams = [torch.cuda.Stream() for _ in ref]
    got = [None] * len(ref)
    for rep in range(3):
        for i, (x, rule, form, _, _) in enumerate(ref):
            streams[i].wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(streams[i]):
                got[i] = _call(rule, x, form)
        torch.cuda.synchronize()
        assert _lib.load().gdr_device_error() == _lib.GDR_OK
        for (x, rule, form, o, s), (o2, s2) in zip(ref, got):
            assert torch.equal(o, o2) and torch.equal(s, s2), (rep, form, rule.algo)


def test_calls_from_several_host_threads():
    ref = _alone()
    got = [None] * len(ref)
    errors = []

    def work(i):
        try:
            x, rule, form, _, _ = ref[i]
            s = torch.cuda.Stream()
            with torch.cuda.stream(s):
                for _ in range(3):
                    got[i] = _call(rule, x, form)
            s.synchronize()
        except Exception as e:  # noqa: BLE001 - reported below
            errors.append(e)

    threads = [threading.Thread(target=work, args=(i,)) for i in range(len(ref))]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=120)
    assert not errors, errors
    assert _lib.load().gdr_device_error() == _lib.GDR_OK
    for (x, rule, form, o, s), (o2, s2) in zip(ref, got):
        assert torch.equal(o, o2) and torch.equal(s, s2), (form, rule.algo)


def test_host_buffer_calls_from_several_threads():
    """gdr_chunked_host from three threads at once (the library's worker
    streams are shared): each equals the same call alone."""
    rule = GatedDeltaRule(algo="tensor")
    host = [{k: v.cpu().pin_memory() for k, v in _batch(lens, seed=10 + i).items()}
            for i, lens in enumerate(([900, 30, 2000], [64] * 20, [1500, 1]))]
    ref = [rule.chunked_host(h["q"], h["k"], h["v"], h["g"], h["beta"], h["state"],
                             cu_seqlens=h["cu_seqlens"]) for h in host]
    got = [None] * len(host)
    errors = []

    def work(i):
        try:
            h = host[i]
            for _ in range(2):
                got[i] = rule.chunked_host(h["q"], h["k"], h["v"], h["g"], h["beta"], h["state"],
                                           cu_seqlens=h["cu_seqlens"])
        except Exception as e:  # noqa: BLE001 - reported below
            errors.append(e)

    threads = [threading.Thread(target=work, args=(i,)) for i in range(len(host))]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=120)
    assert not errors, errors
    for (o, s), (o2, s2) in zip(ref, got):
        assert torch.equal(o, o2) and torch.equal(s, s2)
