"""The layer's steps around the rule on the GPU (causal conv + silu + split,
gates, gated norm, state reorder) against the numpy oracles of oracle/layer.py
and against transformers' Qwen3.5 layer 0 end to end.

Tolerances: 1e-4 (max |got - want| / max |want|) for f32 runs; 2e-2 for bf16
outputs, as for the rule."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from bunsen_b200 import _lib
from bunsen_b200.layer import causal_conv1d, gated_norm, state_reorder
from bunsen_b200.rule import GatedDeltaRule
from oracle import layer as olayer
from tests.conftest import TOL_BF16_OUT, TOL_BF16_STATE, TOL_F32, rel_err
from tests.test_gpu_rule import _np, _oracle, _rand_bf16

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _ok():
    torch.cuda.synchronize()
    assert _lib.load().gdr_device_error() == _lib.GDR_OK


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("taps", [2, 4, 7])
@pytest.mark.parametrize("with_state", [False, True])
@pytest.mark.parametrize("c", [200, 203])  # 16-byte vectors / one channel per thread
def test_conv_packed_against_oracle(dtype, taps, with_state, c):
    gen = torch.Generator(device=DEV).manual_seed(taps)
    lens = [300, 1, 0, 2, 131, 64, 3]
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]), dtype=torch.int32, device=DEV)
    x = torch.randn(sum(lens), c, device=DEV, generator=gen).to(dtype)
    w = (torch.randn(c, taps, device=DEV, generator=gen) * 0.5).to(dtype)
    s0 = (torch.randn(len(lens), taps - 1, c, device=DEV, generator=gen).to(dtype).float()
          if with_state else None)
    (q, k, v), nxt = causal_conv1d(x, w, s0, cu_seqlens=cu, silu=True, splits=(64, 128))
    _ok()
    want, want_next = olayer.causal_conv1d(_np(x), _np(w), _np(s0), cu_seqlens=_np(cu).astype(
        np.int32), activation=True)
    got = np.concatenate([_np(q), _np(k), _np(v)], axis=1)
    tol = TOL_F32 if dtype == torch.float32 else TOL_BF16_OUT
    assert rel_err(got, want) < tol
    assert np.array_equal(_np(nxt), want_next)  # the inputs themselves, exactly


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("silu", [True, False])
@pytest.mark.parametrize("splits", [(264, 528), (66, 132)])  # 8-channel threads / 2-channel
def test_conv_16bit_across_spans_and_column_blocks(dtype, silu, splits):
    """bf16 and f16 with positions past one CTA's 512 (windows whose history
    comes from x), sequences starting inside a window, 1032 channels (a second,
    mostly idle block of 1024) and state for every sequence."""
    gen = torch.Generator(device=DEV).manual_seed(17)
    lens = [700, 1, 0, 900, 5, 31, 17, 500]
    c, taps = 1032, 4
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]), dtype=torch.int32, device=DEV)
    x = torch.randn(sum(lens), c, device=DEV, generator=gen).to(dtype)
    w = (torch.randn(c, taps, device=DEV, generator=gen) * 0.5).to(dtype)
    s0 = torch.randn(len(lens), taps - 1, c, device=DEV, generator=gen).to(dtype).float()
    (q, k, v), nxt = causal_conv1d(x, w, s0, cu_seqlens=cu, silu=silu, splits=splits)
    _ok()
    want, want_next = olayer.causal_conv1d(_np(x), _np(w), _np(s0), cu_seqlens=_np(cu).astype(
        np.int32), activation=silu)
    got = np.concatenate([_np(q), _np(k), _np(v)], axis=1)
    assert rel_err(got, want) < (TOL_BF16_OUT if dtype == torch.bfloat16 else 2e-3)
    assert np.array_equal(_np(nxt), want_next)


def test_conv_dense_decode_steps_in_place():
    """One position at a time (the decode update) from the state the last
    step left, in place, is the one-pass convolution."""
    gen = torch.Generator(device=DEV).manual_seed(9)
    b, t, c, taps = 3, 9, 96, 4
    x = torch.randn(b, t, c, device=DEV, generator=gen)
    w = torch.randn(c, taps, device=DEV, generator=gen)
    whole, whole_next = causal_conv1d(x, w)
    st = torch.zeros(b, taps - 1, c, device=DEV)
    parts = []
    for i in range(t):
        y, _ = causal_conv1d(x[:, i:i + 1], w, st, state_out=st)
        parts.append(y)
    _ok()
    assert rel_err(_np(torch.cat(parts, 1)), _np(whole)) < TOL_F32
    assert torch.equal(st, whole_next)


@pytest.mark.parametrize("name", ["toy", "toy_untied"])
def test_layer_steps_reproduce_transformers_layer0(golden, name):
    """in_proj_qkv(x), the gate projections and z of the toy Qwen3.5's first
    layer through our conv + silu + split, gates, rule and gated norm (all on
    the GPU, f32) reproduce transformers' gated-norm output."""
    d = golden[f"{name}_layer0"]
    T = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(DEV)  # noqa: E731
    hk = int(d["n_key_heads"])
    hv, dk, dv = d["v"].shape[2], d["q"].shape[3], d["v"].shape[3]
    (q, k, v), _ = causal_conv1d(T(d["conv_x"])[None], T(d["conv_w"]), silu=True,
                                 splits=(hk * dk, 2 * hk * dk))
    q, k, v = q.reshape(1, -1, hk, dk), k.reshape(1, -1, hk, dk), v.reshape(1, -1, hv, dv)
    z = T(d["norm_z"]).reshape(1, -1, hv, dv)
    rule = GatedDeltaRule(chunk_size=int(d["chunk_size"]))
    out, _ = rule.chunked(q, k, v, None, None, None,
                          gates=(T(d["a"])[None], T(d["b"])[None], T(d["a_log"]), T(d["dt_bias"])),
                          norm=(z, T(d["norm_w"]), float(d["norm_eps"])))
    _ok()
    assert rel_err(_np(out).reshape(-1, dv), d["norm_out"]) < TOL_F32


@pytest.mark.parametrize("form", ["chunked", "recurrent"])
def test_gates_and_norm_bf16_d128_against_oracle(form):
    """bf16, d 128: the tensor-core prefill and the d-128 decode kernel with
    the layer's gates and gated norm, against the oracle rule on the oracle's
    gates followed by the oracle's norm."""
    lens = [200, 1, 70] if form == "chunked" else [1] * 6
    x = _rand_bf16(lens, state=True, seed=31)
    gen = torch.Generator(device=DEV).manual_seed(32)
    t = sum(lens)
    a = torch.randn(t, 4, device=DEV, generator=gen).bfloat16()
    b = torch.randn(t, 4, device=DEV, generator=gen).bfloat16()
    a_log = torch.log(torch.rand(4, device=DEV, generator=gen) * 0.5 + 0.05)
    dt_bias = torch.randn(4, device=DEV, generator=gen) * 0.1
    z = torch.randn(t, 4, 128, device=DEV, generator=gen).bfloat16()
    w = torch.rand(128, device=DEV, generator=gen) + 0.5
    out, st = getattr(GatedDeltaRule(), form)(
        x["q"], x["k"], x["v"], None, None, x["state"], cu_seqlens=x["cu_seqlens"],
        gates=(a, b, a_log, dt_bias), norm=(z, w, 1e-6))
    _ok()
    g, beta = olayer.gates(_np(a), _np(b), _np(a_log), _np(dt_bias), beta_dtype="bf16")
    y = dict(x, g=torch.from_numpy(g), beta=torch.from_numpy(beta))
    core, want_st = _oracle(form, y)
    core = _np(torch.from_numpy(core).bfloat16())  # the rule's output in q's dtype
    want = olayer.gated_norm(core, _np(z), _np(w), 1e-6)
    assert rel_err(_np(out), want) < TOL_BF16_OUT
    assert rel_err(_np(st), want_st) < TOL_BF16_STATE


def test_reorder_and_bad_source():
    gen = torch.Generator(device=DEV).manual_seed(5)
    pool = torch.randn(6, 4, 16, 16, device=DEV, generator=gen)
    conv = torch.randn(6, 3, 40, device=DEV, generator=gen)
    src = torch.tensor([5, 5, 0, 1, 2, 3], dtype=torch.int32, device=DEV)
    got = state_reorder(pool, src)
    got_c = state_reorder(conv, src)
    _ok()
    assert torch.equal(got, pool[src.long()]) and torch.equal(got_c, conv[src.long()])
    out = torch.zeros_like(pool)
    state_reorder(pool, torch.tensor([0, 9, 1, 2, 3, 4], dtype=torch.int32, device=DEV), out=out)
    torch.cuda.synchronize()
    assert _lib.load().gdr_device_error() == _lib.GDR_ERR_INVALID
    assert torch.count_nonzero(out[1]) == 0 and torch.equal(out[2], pool[1])


def test_gates_and_norm_on_the_split_path():
    """The split form with fused gates and norm: every segment kind (first,
    B and M runs, middle and last) stages the projections and normalises."""
    lens = [700, 64 * 5 + 3, 1, 1500]
    x = _rand_bf16(lens, state=True, seed=41)
    gen = torch.Generator(device=DEV).manual_seed(42)
    t = sum(lens)
    a = torch.randn(t, 4, device=DEV, generator=gen).bfloat16()
    b = torch.randn(t, 4, device=DEV, generator=gen).bfloat16()
    a_log = torch.log(torch.rand(4, device=DEV, generator=gen) * 0.2 + 0.01)
    dt_bias = torch.randn(4, device=DEV, generator=gen) * 0.1
    z = torch.randn(t, 4, 128, device=DEV, generator=gen).bfloat16()
    w = torch.rand(128, device=DEV, generator=gen) + 0.5
    out, st = GatedDeltaRule(algo="tensor_split", split_chunks=2).chunked(
        x["q"], x["k"], x["v"], None, None, x["state"], cu_seqlens=x["cu_seqlens"],
        gates=(a, b, a_log, dt_bias), norm=(z, w, 1e-6))
    _ok()
    g, beta = olayer.gates(_np(a), _np(b), _np(a_log), _np(dt_bias), beta_dtype="bf16")
    core, want_st = _oracle("chunked", dict(x, g=torch.from_numpy(g), beta=torch.from_numpy(beta)))
    want = olayer.gated_norm(_np(torch.from_numpy(core).bfloat16()), _np(z), _np(w), 1e-6)
    assert rel_err(_np(out), want) < TOL_BF16_OUT
    assert rel_err(_np(st), want_st) < TOL_BF16_STATE


@pytest.mark.parametrize("name", ["toy", "toy_untied"])
def test_layer0_one_position_at_a_time(golden, name):
    """The toy layer 0 as a decode: recurrent (gates fused into the generic
    recurrent kernel, the norm after it) reproduces transformers' output."""
    d = golden[f"{name}_layer0"]
    T = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(DEV)  # noqa: E731
    hk = int(d["n_key_heads"])
    hv, dk, dv = d["v"].shape[2], d["q"].shape[3], d["v"].shape[3]
    (q, k, v), _ = causal_conv1d(T(d["conv_x"])[None], T(d["conv_w"]), silu=True,
                                 splits=(hk * dk, 2 * hk * dk))
    q, k, v = q.reshape(1, -1, hk, dk), k.reshape(1, -1, hk, dk), v.reshape(1, -1, hv, dv)
    z = T(d["norm_z"]).reshape(1, -1, hv, dv)
    out, _ = GatedDeltaRule().recurrent(
        q, k, v, None, None, None,
        gates=(T(d["a"])[None], T(d["b"])[None], T(d["a_log"]), T(d["dt_bias"])),
        norm=(z, T(d["norm_w"]), float(d["norm_eps"])))
    _ok()
    assert rel_err(_np(out).reshape(-1, dv), d["norm_out"]) < TOL_F32


def test_mixed_batch_with_gates_and_norm_matches_separate_calls():
    """gdr_mixed_layer: the continuous batch with the layer's gates and norm
    equals the layer calls on its prefill segments and decode rows (the same
    fused kernels run both)."""
    from tests.test_gpu_mixed import _batch
    lens = [200, 1, 1, 70, 1]
    x = _batch(lens)
    t = sum(lens)
    gen = torch.Generator(device=DEV).manual_seed(51)
    hv = x["v"].shape[-2]
    a = torch.randn(t, hv, device=DEV, generator=gen).bfloat16()
    b = torch.randn(t, hv, device=DEV, generator=gen).bfloat16()
    a_log = torch.log(torch.rand(hv, device=DEV, generator=gen) * 0.3 + 0.01)
    dt_bias = torch.randn(hv, device=DEV, generator=gen) * 0.1
    z = torch.randn(t, hv, 128, device=DEV, generator=gen).bfloat16()
    w = torch.rand(128, device=DEV, generator=gen) + 0.5
    pool0 = x["pool"].clone()
    out = GatedDeltaRule().mixed(x["q"], x["k"], x["v"], None, None, x["pool"],
                                 cu_seqlens=x["cu_seqlens"], state_slots=x["slots"],
                                 gates=(a, b, a_log, dt_bias), norm=(z, w, 1e-6))
    _ok()
    g, beta = olayer.gates(_np(a), _np(b), _np(a_log), _np(dt_bias), beta_dtype="bf16")
    cu = _np(x["cu_seqlens"]).astype(np.int64)
    slots = _np(x["slots"]).astype(np.int64)
    from oracle import oracle
    for s_, (lo, hi) in enumerate(zip(cu[:-1], cu[1:])):
        if hi == lo:
            continue
        args = [_np(x[key][lo:hi])[None] for key in ("q", "k", "v")]
        st0 = _np(pool0[slots[s_]])[None]
        fn = oracle.recurrent if hi - lo == 1 else oracle.chunked
        core, st = fn(*args, g[lo:hi][None], beta[lo:hi][None], st0)
        want = olayer.gated_norm(_np(torch.from_numpy(core).bfloat16()), _np(z[lo:hi])[None],
                                 _np(w), 1e-6)
        assert rel_err(_np(out[lo:hi])[None], want) < TOL_BF16_OUT
        assert rel_err(_np(x["pool"][slots[s_]])[None], st) < TOL_BF16_STATE


def test_mixer_steps_in_parts_agree_with_one_pass():
    """gated_delta_net.rs:495-523 after the projections: the layer's conv,
    gates, rule and norm run in parts [0, 4), [4, 5), [5, 9) through the conv
    and recurrent states (the one-position part as a decode step) equal the
    one pass, outputs and final states (f32, within 1e-4)."""
    gen = torch.Generator(device=DEV).manual_seed(71)
    b, t, hk, hv, dk, dv, taps = 2, 9, 2, 4, 8, 8, 4
    c = 2 * hk * dk + hv * dv
    f = dict(device=DEV, generator=gen)
    mixed = torch.randn(b, t, c, **f)
    wconv = torch.randn(c, taps, **f) * 0.5
    a, bb = torch.randn(b, t, hv, **f), torch.randn(b, t, hv, **f)
    a_log, dt_bias = torch.randn(hv, **f) * 0.5, torch.randn(hv, **f) * 0.1
    z, nw = torch.randn(b, t, hv, dv, **f), torch.rand(dv, **f) + 0.5
    rule = GatedDeltaRule(chunk_size=4)

    def layer(sl, conv_state, rec_state):
        (q, k, v), conv_next = causal_conv1d(mixed[:, sl].contiguous(), wconv, conv_state,
                                             silu=True, splits=(hk * dk, 2 * hk * dk))
        n = q.shape[1]
        q, k, v = q.reshape(b, n, hk, dk), k.reshape(b, n, hk, dk), v.reshape(b, n, hv, dv)
        form = rule.recurrent if n == 1 else rule.chunked
        out, rec_next = form(q, k, v, None, None, rec_state,
                             gates=(a[:, sl].contiguous(), bb[:, sl].contiguous(), a_log,
                                    dt_bias),
                             norm=(z[:, sl].contiguous(), nw, 1e-6))
        return out, conv_next, rec_next

    whole, conv1, rec1 = layer(slice(0, t), None, None)
    conv_s, rec_s, parts = None, None, []
    for lo, hi in ((0, 4), (4, 5), (5, 9)):
        out, conv_s, rec_s = layer(slice(lo, hi), conv_s, rec_s)
        parts.append(out)
    _ok()
    assert rel_err(_np(torch.cat(parts, 1)), _np(whole)) < TOL_F32
    assert rel_err(_np(conv_s), _np(conv1)) < TOL_F32
    assert rel_err(_np(rec_s), _np(rec1)) < TOL_F32


def test_conv_silu_elementwise_over_the_negative_range():
    """The conv's bf16 silu element by element over x in [-20, 4] (a
    two-tap filter (0, 1) passes x through): within 1e-2 of f32 silu(x)
    relative to each element, the bf16 rounding of the result included."""
    x = torch.linspace(-20.0, 4.0, 4096, device=DEV).bfloat16().reshape(-1, 64)
    w = torch.zeros(64, 2, device=DEV, dtype=torch.bfloat16)
    w[:, 1] = 1.0
    y, _ = causal_conv1d(x[None], w, silu=True)
    _ok()
    xf = _np(x)
    want = xf / (1.0 + np.exp(-xf.astype(np.float64)))
    got = _np(y)[0]
    err = np.abs(got - want)
    assert np.all(err <= 1e-2 * np.abs(want)), float((err / np.maximum(np.abs(want), 1e-30)).max())


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("rows", [1, 2, 3, 5, 4099])
def test_gated_norm_16bit_128_rows_and_in_place(dtype, rows):
    """The standalone gated norm's 16-bit, 128-feature kernel (two rows per
    warp instruction, four per warp): row counts that leave a warp partly
    empty, element by element against the oracle (within the output type's
    rounding), and in place (out = x)."""
    gen = torch.Generator(device=DEV).manual_seed(rows)
    x = torch.randn(rows, 128, device=DEV, generator=gen).to(dtype)
    z = (torch.randn(rows, 128, device=DEV, generator=gen) * 3).to(dtype)
    w = torch.rand(128, device=DEV, generator=gen) + 0.5
    want = olayer.gated_norm(_np(x), _np(z), _np(w), 1e-6)
    y = gated_norm(x, z, w, 1e-6)
    _ok()
    err = np.abs(_np(y) - want)
    tol = 1e-2 if dtype == torch.bfloat16 else 2e-3
    assert np.all(err <= tol * np.abs(want) + 1e-6), float(err.max())
    y2 = gated_norm(x, z, w, 1e-6, out=x)
    _ok()
    assert y2.data_ptr() == x.data_ptr() and torch.equal(y2, y)


def test_fused_norm_elementwise_against_the_plain_prefill():
    """The tensor-core prefill's fused gated norm against the same kernel's
    plain output normalised on the host, element by element, with z over
    [-20, 4]: the fused silu(z) and the row norm within 1e-2 of each element."""
    x = _rand_bf16([200, 70], state=True, seed=61)
    t = 270
    gen = torch.Generator(device=DEV).manual_seed(62)
    z = (torch.rand(t, 4, 128, device=DEV, generator=gen) * 24.0 - 20.0).bfloat16()
    w = torch.rand(128, device=DEV, generator=gen) + 0.5
    rule = GatedDeltaRule(algo="tensor")
    plain, _ = rule.chunked(x["q"], x["k"], x["v"], x["g"], x["beta"], x["state"],
                            cu_seqlens=x["cu_seqlens"])
    fused, _ = rule.chunked(x["q"], x["k"], x["v"], x["g"], x["beta"], x["state"],
                            cu_seqlens=x["cu_seqlens"], norm=(z, w, 1e-6))
    _ok()
    want = olayer.gated_norm(_np(plain), _np(z), _np(w), 1e-6)
    err = np.abs(_np(fused) - want)
    assert np.all(err <= 1e-2 * np.abs(want) + 1e-6), float(err.max())
