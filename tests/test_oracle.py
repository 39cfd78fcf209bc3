"""The CPU oracle pinned against bunsen's own known answers and the
properties bunsen's tests hold its rule to (delta_rule.rs:449-661)."""

from __future__ import annotations

import numpy as np
import pytest

from oracle import oracle
from tests.conftest import rel_err

CASES = ["scalar", "parts", "t8", "t10", "t3", "t70", "t1", "t13"]


def _case(golden, name):
    d = golden["hf_cases"]
    return {k: d[f"{name}.{k}"] for k in ("q", "k", "v", "g", "beta", "s0")}, d


@pytest.mark.parametrize("toy", ["toy_layer0", "toy_untied_layer0"])
@pytest.mark.parametrize("form", ["chunked", "recurrent", "scalar_f64"])
def test_known_answer_layer0_core(golden, toy, form):
    """bunsen's fixture io.layer0_core (testdata/qwen3_5/toy*.safetensors):
    layer 0's delta-rule output of the toy Qwen3.5, 72 tokens across the
    64-position chunk boundary; q/k passed with their H_qk heads."""
    d = golden[toy]
    ratio = d["v"].shape[2] // int(d["n_key_heads"])
    q, k = d["q"][:, :, ::ratio], d["k"][:, :, ::ratio]
    assert np.array_equal(np.repeat(q, ratio, axis=2), d["q"])
    out, _ = getattr(oracle, form)(q, k, d["v"], d["g"], d["beta"], None)
    assert np.abs(out - d["core"]).max() < 2e-6


@pytest.mark.parametrize("name", CASES)
@pytest.mark.parametrize("initial", [False, True])
@pytest.mark.parametrize("norm", [True, False])
def test_scalar_and_recurrent_against_f64_rule(golden, name, initial, norm):
    """delta_rule.rs:449-495: the recurrent form against the scalar f64 rule
    (here also transformers' f64 loop), 1e-4, with/without state and norm."""
    x, d = _case(golden, name)
    tag = f"{name}.i{int(initial)}n{int(norm)}"
    st = x["s0"] if initial else None
    eps = 1e-6 if norm else None
    o64, s64 = oracle.scalar_f64(x["q"], x["k"], x["v"], x["g"], x["beta"], st, l2norm_eps=eps)
    assert np.abs(o64 - d[tag + ".out"]).max() < 1e-10
    assert np.abs(s64 - d[tag + ".state"]).max() < 1e-10
    o, s = oracle.recurrent(x["q"], x["k"], x["v"], x["g"], x["beta"], st, l2norm_eps=eps)
    assert rel_err(o, d[tag + ".out"]) < 1e-5 and rel_err(s, d[tag + ".state"]) < 1e-5


@pytest.mark.parametrize("t,chunk", [(8, 4), (10, 4), (3, 4), (70, 64), (1, 64)])
@pytest.mark.parametrize("initial", [False, True])
@pytest.mark.parametrize("norm", [True, False])
def test_chunked_is_recurrent(golden, t, chunk, initial, norm):
    """delta_rule.rs:549-599: chunks that divide the sequence, that do not,
    longer than it; bunsen holds the two forms to 1e-5."""
    x, _ = _case(golden, f"t{t}")
    st = x["s0"] if initial else None
    eps = 1e-6 if norm else None
    oc, sc = oracle.chunked(x["q"], x["k"], x["v"], x["g"], x["beta"], st, l2norm_eps=eps,
                            chunk_size=chunk)
    orr, sr = oracle.recurrent(x["q"], x["k"], x["v"], x["g"], x["beta"], st, l2norm_eps=eps)
    assert rel_err(oc, orr) < 1e-5 and rel_err(sc, sr) < 1e-5


@pytest.mark.parametrize("form,cuts", [("recurrent", [0, 3, 7]), ("recurrent", list(range(8))),
                                       ("chunked", [0, 5, 6, 13])])
def test_parts_agree_with_one_pass(golden, form, cuts):
    """delta_rule.rs:499-532 and :612-642: a run in parts, each from the
    state the last left (mid-chunk cuts, one-token parts), is one pass."""
    x, _ = _case(golden, "t13")
    fn = getattr(oracle, form)
    kw = {"chunk_size": 4} if form == "chunked" else {}
    cuts = [c for c in cuts if c <= 13] + ([13] if cuts[-1] < 13 else [])
    whole, whole_s = fn(x["q"], x["k"], x["v"], x["g"], x["beta"], None, **kw)
    state, parts = None, []
    for a, b in zip(cuts[:-1], cuts[1:]):
        sl = slice(a, b)
        y, state = fn(x["q"][:, sl], x["k"][:, sl], x["v"][:, sl], x["g"][:, sl],
                      x["beta"][:, sl], state, **kw)
        parts.append(y)
    assert rel_err(np.concatenate(parts, axis=1), whole) < 1e-5
    assert rel_err(state, whole_s) < 1e-5


def test_zero_beta_only_decays(golden):
    """delta_rule.rs:646-661: beta = 0 and g = 0 leave the state unchanged;
    beta = 0 alone leaves it the decayed state."""
    x, _ = _case(golden, "t3")
    z = np.zeros_like(x["g"])
    _, s = oracle.recurrent(x["q"], x["k"], x["v"], z, z, x["s0"])
    assert np.array_equal(s, x["s0"])
    _, s = oracle.chunked(x["q"], x["k"], x["v"], x["g"], z, x["s0"], chunk_size=4)
    decay = np.exp(x["g"].sum(axis=1))[:, :, None, None]
    assert rel_err(s, x["s0"] * decay) < 1e-6


def test_ragged_pack_is_independent_sequences(golden):
    """A packed batch (cu_seqlens) runs each sequence on its own."""
    x, _ = _case(golden, "t70")
    rng = np.random.default_rng(0)
    lens = [70, 1, 33, 0, 64, 5]
    tot = sum(lens)
    q = rng.standard_normal((tot, 3, 4)).astype(np.float32)
    k = rng.standard_normal((tot, 3, 4)).astype(np.float32)
    v = rng.standard_normal((tot, 3, 5)).astype(np.float32)
    g = rng.uniform(-1, 0, (tot, 3)).astype(np.float32)
    b = rng.uniform(0, 1, (tot, 3)).astype(np.float32)
    s0 = rng.standard_normal((len(lens), 3, 4, 5)).astype(np.float32)
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    for fn, kw in ((oracle.chunked, {"chunk_size": 16}), (oracle.recurrent, {})):
        o, s = fn(q, k, v, g, b, s0, cu_seqlens=cu, **kw)
        for i, (a, e) in enumerate(zip(cu[:-1], cu[1:])):
            oi, si = fn(q[None, a:e], k[None, a:e], v[None, a:e], g[None, a:e], b[None, a:e],
                        s0[i:i + 1], **kw)
            assert np.array_equal(o[a:e], oi[0]) and np.array_equal(s[i], si[0])


def test_grouped_heads_are_repeat_interleave(golden):
    """Value head h reads key head h // (H_v / H_qk): the same as repeating
    q and k with repeat_interleave first (ops/repeat.rs:51-66)."""
    rng = np.random.default_rng(1)
    q = rng.standard_normal((2, 9, 2, 4)).astype(np.float32)
    k = rng.standard_normal((2, 9, 2, 4)).astype(np.float32)
    v = rng.standard_normal((2, 9, 6, 3)).astype(np.float32)
    g = rng.uniform(-1, 0, (2, 9, 6)).astype(np.float32)
    b = rng.uniform(0, 1, (2, 9, 6)).astype(np.float32)
    o1, s1 = oracle.chunked(q, k, v, g, b, None, chunk_size=4)
    o2, s2 = oracle.chunked(np.repeat(q, 3, axis=2), np.repeat(k, 3, axis=2), v, g, b, None,
                            chunk_size=4)
    assert np.array_equal(o1, o2) and np.array_equal(s1, s2)


def test_zero_chunk_is_rejected():
    with pytest.raises(ValueError, match="at least one position"):
        oracle.chunked(*(np.zeros((1, 1, 1, 1), np.float32),) * 3, np.zeros((1, 1, 1), np.float32),
                       np.zeros((1, 1, 1), np.float32), None, chunk_size=0)
