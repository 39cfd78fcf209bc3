"""The numpy oracles of the layer's steps around the rule (oracle/layer.py),
pinned against transformers' Qwen3.5 layer 0 (tests/golden/*_layer0.npz, made
by tests/golden/make_golden.py) and against bunsen's own property tests
(causal_conv.rs:75-180, state.rs tests)."""

from __future__ import annotations

import numpy as np
import pytest

from oracle import layer

GOLDEN = ["toy", "toy_untied"]


@pytest.mark.parametrize("name", GOLDEN)
def test_conv_silu_split_reproduces_the_rule_inputs(golden, name):
    """silu(causal conv(in_proj_qkv x)) split into q, k, v is exactly what
    layer 0 handed its rule (q and k before repeat_interleave)."""
    d = golden[f"{name}_layer0"]
    y, _ = layer.causal_conv1d(d["conv_x"], d["conv_w"], activation=True)
    hk = int(d["n_key_heads"])
    q, k, v = d["q"][0], d["k"][0], d["v"][0]
    hv, dk, dv = v.shape[1], q.shape[2], v.shape[2]
    r = hv // hk
    scale = max(np.abs(q).max(), np.abs(v).max())
    assert np.abs(y[:, :hk * dk].reshape(-1, hk, dk) - q[:, ::r]).max() < 2e-6 * scale
    assert np.abs(y[:, hk * dk:2 * hk * dk].reshape(-1, hk, dk) - k[:, ::r]).max() < 2e-6 * scale
    assert np.abs(y[:, 2 * hk * dk:].reshape(-1, hv, dv) - v).max() < 2e-6 * scale


@pytest.mark.parametrize("name", GOLDEN)
def test_gates_reproduce_g_and_beta(golden, name):
    d = golden[f"{name}_layer0"]
    g, beta = layer.gates(d["a"], d["b"], d["a_log"], d["dt_bias"])
    assert np.abs(g - d["g"][0]).max() < 1e-6 * np.abs(d["g"]).max()
    assert np.abs(beta - d["beta"][0]).max() < 1e-6


@pytest.mark.parametrize("name", GOLDEN)
def test_gated_norm_reproduces_the_layer(golden, name):
    d = golden[f"{name}_layer0"]
    y = layer.gated_norm(d["norm_x"], d["norm_z"], d["norm_w"], float(d["norm_eps"]))
    assert np.abs(y - d["norm_out"]).max() < 1e-6 * np.abs(d["norm_out"]).max()


def test_conv_against_the_sum():
    """causal_conv.rs:75-115: each output written out as a sum over its
    channel's taps, zeros before the first input; the state is the last K - 1
    inputs."""
    rng = np.random.default_rng(1)
    b, t, c, k = 2, 5, 3, 4
    x = rng.standard_normal((b, t, c)).astype(np.float32)
    w = rng.standard_normal((c, k)).astype(np.float32)
    y, nxt = layer.causal_conv1d(x, w)
    for row in range(b):
        for pos in range(t):
            for ch in range(c):
                want = sum(w[ch, j] * x[row, pos - (k - 1) + j, ch]
                           for j in range(k) if pos - (k - 1) + j >= 0)
                assert abs(y[row, pos, ch] - want) < 1e-5
    assert np.array_equal(nxt, x[:, t - (k - 1):])


@pytest.mark.parametrize("cuts", [[0, 4, 9], list(range(10)), [0, 2, 7, 9]])
def test_conv_parts_agree_with_one_pass(cuts):
    """causal_conv.rs:117-160: run in parts, each from the state the last
    left (parts shorter than the kernel, and one position at a time), the
    convolution is the one-pass convolution."""
    rng = np.random.default_rng(3)
    b, t, c, k = 2, 9, 4, 4
    x = rng.standard_normal((b, t, c)).astype(np.float32)
    w = rng.standard_normal((c, k)).astype(np.float32)
    whole, whole_next = layer.causal_conv1d(x, w)
    state, parts = None, []
    for a, e in zip(cuts[:-1], cuts[1:]):
        y, state = layer.causal_conv1d(x[:, a:e], w, state)
        parts.append(y)
    assert np.allclose(np.concatenate(parts, axis=1), whole, atol=1e-5)
    assert np.allclose(state, whole_next)


def test_conv_packed_equals_per_sequence():
    rng = np.random.default_rng(4)
    lens = [5, 1, 0, 7, 2]
    c, k = 6, 3
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    x = rng.standard_normal((cu[-1], c)).astype(np.float32)
    w = rng.standard_normal((c, k)).astype(np.float32)
    s0 = rng.standard_normal((len(lens), k - 1, c)).astype(np.float32)
    y, nxt = layer.causal_conv1d(x, w, s0, cu_seqlens=cu)
    for s, (a, e) in enumerate(zip(cu[:-1], cu[1:])):
        ys, ns = layer.causal_conv1d(x[None, a:e], w, s0[s:s + 1])
        assert np.allclose(y[a:e], ys[0]) and np.allclose(nxt[s], ns[0])


def test_reorder_moves_rows():
    """state.rs reorder: row r becomes row sources[r] (beams branching)."""
    pool = np.arange(4 * 3 * 2, dtype=np.float32).reshape(4, 3, 2)
    got = layer.reorder(pool, [2, 2, 0, 3])
    assert np.array_equal(got[0], pool[2]) and np.array_equal(got[1], pool[2])
    assert np.array_equal(got[2], pool[0]) and np.array_equal(got[3], pool[3])
