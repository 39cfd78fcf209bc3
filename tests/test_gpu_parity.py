"""Parity of the bf16 / d 128 / chunk 64 paths with the CPU oracle where the
per-position factors matter, and at every benchmark configuration's full shape.

The tensor-core kernels feed raw q and k to the tensor cores and apply the
L2 norms (``delta_rule.rs:112-123``), eps inside the square root, and the
``1/sqrt(d_k)`` query scale (``:153``) as per-position factors afterwards.
With unit-norm q and k those factors are all about 1, so here q and k are
raw N(0, 1) vectors (norms near 11), the silu outputs of the layer's
convolution (``gated_delta_net.rs:396-420``), or, with ``qk_l2norm_eps =
None``, vectors of norms far from 1, through every path that reaches the
tensor cores: the one-pass kernel, the split form, the continuous batch and
the layer calls.

Tolerances (max |got - want| / max |want|): 2e-2 on outputs, 1e-2 on states
for bf16 inputs; the observed errors are printed (``pytest -s``)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from bunsen_b200 import _lib, workloads
from bunsen_b200.layer import causal_conv1d
from bunsen_b200.rule import GatedDeltaRule
from oracle import layer as olayer
from oracle import oracle
from tests.conftest import TOL_BF16_OUT, TOL_BF16_STATE, rel_err

pytestmark = pytest.mark.gpu
DEV = "cuda"

LENS = [64, 1, 65, 63, 0, 300, 128, 2, 700]


def _np(x):
    return None if x is None else workloads.to_numpy_f32(x)


def _ok():
    torch.cuda.synchronize()
    assert _lib.load().gdr_device_error() == _lib.GDR_OK


def _cu(lens):
    return torch.tensor(np.concatenate([[0], np.cumsum(lens)]), dtype=torch.int32, device=DEV)


def _inputs(lens, kind, hq=2, hv=4, seed=0, state=True):
    """q, k of the given kind; v ~ N(0, 1); beta = sigmoid(N(0, 1)); g =
    ln U(0.9, 0.999); states N(0, 0.01).
      raw     q, k ~ N(0, 1) (norms near sqrt(128))
      skewed  q ~ 3 N(0, 1); k = unit vector x U(0.4, 1.3) per position, so
              that the rule without the norm stays stable (beta |k|^2 < 2)"""
    gen = torch.Generator(device=DEV).manual_seed(seed)
    f = dict(device=DEV, generator=gen)
    t = sum(lens)
    if kind == "raw":
        q = torch.randn(t, hq, 128, **f)
        k = torch.randn(t, hq, 128, **f)
    elif kind == "skewed":
        q = 3.0 * torch.randn(t, hq, 128, **f)
        k = torch.randn(t, hq, 128, **f)
        k = k / k.norm(dim=-1, keepdim=True) * (0.4 + 0.9 * torch.rand(t, hq, 1, **f))
    else:
        raise KeyError(kind)
    x = {"q": q.bfloat16(), "k": k.bfloat16(), "v": torch.randn(t, hv, 128, **f).bfloat16(),
         "g": torch.log(torch.rand(t, hv, **f) * 0.099 + 0.9),
         "beta": torch.sigmoid(torch.randn(t, hv, **f)), "cu_seqlens": _cu(lens)}
    if state:
        x["state"] = torch.randn(len(lens), hv, 128, 128, **f) * 0.1
    return x


def _oracle(x, eps, form="chunked", g=None, beta=None):
    fn = oracle.chunked if form == "chunked" else oracle.recurrent
    cu = x.get("cu_seqlens")
    return fn(_np(x["q"]), _np(x["k"]), _np(x["v"]), _np(x["g"]) if g is None else g,
              _np(x["beta"]) if beta is None else beta, _np(x.get("state")), l2norm_eps=eps,
              cu_seqlens=None if cu is None else _np(cu).astype(np.int32))


def _check(name, o, s, wo, ws):
    eo, es = rel_err(o, wo), rel_err(s, ws)
    print(f"{name}: out {eo:.2e} state {es:.2e}")
    assert eo < TOL_BF16_OUT and es < TOL_BF16_STATE, (eo, es)


# -- q/k norms far from 1 through every tensor-core path ------------------------
CASES = [("raw", 1e-6), ("skewed", 1e-6), ("skewed", None)]


@pytest.mark.parametrize("kind,eps", CASES)
@pytest.mark.parametrize("algo,split", [("tensor", 0), ("tensor_split", 2), ("tensor_split", 1)])
def test_tensor_core_norm_factors_against_oracle(kind, eps, algo, split):
    x = _inputs(LENS, kind, seed=3)
    rule = GatedDeltaRule(qk_l2norm_eps=eps, algo=algo, split_chunks=split)
    o, s = rule.chunked(x["q"], x["k"], x["v"], x["g"], x["beta"], x["state"],
                        cu_seqlens=x["cu_seqlens"])
    _ok()
    wo, ws = _oracle(x, eps)
    _check(f"{algo}/{split} {kind} eps={eps}", _np(o), _np(s), wo, ws)


@pytest.mark.parametrize("kind,eps", CASES)
def test_tensor_core_dense_batch_norm_factors(kind, eps):
    x = _inputs([256, 256, 256], kind, seed=4, state=False)
    d = {k_: x[k_].reshape((3, 256) + x[k_].shape[1:]) for k_ in ("q", "k", "v", "g", "beta")}
    o, s = GatedDeltaRule(qk_l2norm_eps=eps, algo="tensor").chunked(
        d["q"], d["k"], d["v"], d["g"], d["beta"])
    _ok()
    wo, ws = oracle.chunked(*(_np(d[k_]) for k_ in ("q", "k", "v", "g", "beta")), None,
                            l2norm_eps=eps)
    _check(f"dense {kind} eps={eps}", _np(o), _np(s), wo, ws)


@pytest.mark.parametrize("kind,eps", CASES)
def test_mixed_norm_factors_against_oracle(kind, eps):
    """gdr_mixed: prefill segments through the persistent tensor-core kernel
    and decode rows through the d-128 recurrent code, states in a pool."""
    lens = [200, 1, 1, 64, 1, 0, 130, 1, 65, 1]
    x = _inputs(lens, kind, seed=5)
    pool = x["state"].clone()
    out = GatedDeltaRule(qk_l2norm_eps=eps).mixed(x["q"], x["k"], x["v"], x["g"], x["beta"],
                                                  pool, cu_seqlens=x["cu_seqlens"])
    _ok()
    f = {k_: _np(x[k_]) for k_ in ("q", "k", "v", "g", "beta", "state")}
    want_o = np.zeros(f["v"].shape, np.float32)
    want_s = f["state"].copy()
    cu = np.concatenate([[0], np.cumsum(lens)])
    for s_, (a, e) in enumerate(zip(cu[:-1], cu[1:])):
        if e == a:
            continue
        fn = oracle.chunked if e - a > 1 else oracle.recurrent
        o, st = fn(*(f[k_][None, a:e] for k_ in ("q", "k", "v", "g", "beta")),
                   f["state"][s_][None], l2norm_eps=eps)
        want_o[a:e], want_s[s_] = o[0], st[0]
    _check(f"mixed {kind} eps={eps}", _np(out), _np(pool), want_o, want_s)


@pytest.mark.parametrize("eps", [1e-6, None])
def test_recurrent_d128_norm_factors(eps):
    x = _inputs([1] * 12, "skewed", seed=6)
    d = {k_: x[k_][:, None] for k_ in ("q", "k", "v", "g", "beta")}
    o, s = GatedDeltaRule(qk_l2norm_eps=eps).recurrent(d["q"], d["k"], d["v"], d["g"],
                                                       d["beta"], x["state"])
    _ok()
    wo, ws = oracle.recurrent(*(_np(d[k_]) for k_ in ("q", "k", "v", "g", "beta")),
                              _np(x["state"]), l2norm_eps=eps)
    _check(f"recurrent eps={eps}", _np(o), _np(s), wo, ws)


# -- the layer as it runs: conv + silu + split feeding the rule ---------------------
def _layer_inputs(lens, hq=2, hv=4, seed=7):
    """q, k, v as the layer makes them (silu of the causal conv of a
    projection, split), the gate projections, z and the norm weight."""
    gen = torch.Generator(device=DEV).manual_seed(seed)
    f = dict(device=DEV, generator=gen)
    t = sum(lens)
    c = 2 * hq * 128 + hv * 128
    cu = _cu(lens)
    xin = torch.randn(t, c, **f).bfloat16()
    wconv = (torch.randn(c, 4, **f) * 0.5).bfloat16()
    (q, k, v), _ = causal_conv1d(xin, wconv, None, cu_seqlens=cu, silu=True,
                                 splits=(hq * 128, 2 * hq * 128))
    x = {"q": q.reshape(t, hq, 128), "k": k.reshape(t, hq, 128), "v": v.reshape(t, hv, 128),
         "cu_seqlens": cu, "state": torch.randn(len(lens), hv, 128, 128, **f) * 0.1,
         "a": torch.randn(t, hv, **f).bfloat16(), "b": torch.randn(t, hv, **f).bfloat16(),
         "a_log": torch.log(torch.rand(hv, **f) * 0.3 + 0.01),
         "dt_bias": torch.randn(hv, **f) * 0.1,
         "z": torch.randn(t, hv, 128, **f).bfloat16(), "w": torch.rand(128, **f) + 0.5}
    return x


def _layer_want(x, form="chunked"):
    g, beta = olayer.gates(_np(x["a"]), _np(x["b"]), _np(x["a_log"]), _np(x["dt_bias"]),
                           beta_dtype="bf16")
    y = dict(x, g=None, beta=None)
    core, st = _oracle(y, 1e-6, form=form, g=g, beta=beta)
    core = _np(torch.from_numpy(core).bfloat16())  # the rule's output in q's dtype
    return olayer.gated_norm(core, _np(x["z"]), _np(x["w"]), 1e-6), st


@pytest.mark.parametrize("algo,split", [("tensor", 0), ("tensor_split", 2)])
def test_layer_conv_outputs_through_tensor_core(algo, split):
    x = _layer_inputs(LENS)
    out, st = GatedDeltaRule(algo=algo, split_chunks=split).chunked(
        x["q"], x["k"], x["v"], None, None, x["state"], cu_seqlens=x["cu_seqlens"],
        gates=(x["a"], x["b"], x["a_log"], x["dt_bias"]), norm=(x["z"], x["w"], 1e-6))
    _ok()
    want, want_st = _layer_want(x)
    _check(f"layer {algo}/{split}", _np(out), _np(st), want, want_st)


def test_layer_conv_outputs_through_mixed():
    lens = [200, 1, 1, 64, 1, 130, 1]
    x = _layer_inputs(lens, seed=8)
    pool = x["state"].clone()
    out = GatedDeltaRule().mixed(x["q"], x["k"], x["v"], None, None, pool,
                                 cu_seqlens=x["cu_seqlens"],
                                 gates=(x["a"], x["b"], x["a_log"], x["dt_bias"]),
                                 norm=(x["z"], x["w"], 1e-6))
    _ok()
    g, beta = olayer.gates(_np(x["a"]), _np(x["b"]), _np(x["a_log"]), _np(x["dt_bias"]),
                           beta_dtype="bf16")
    f = {k_: _np(x[k_]) for k_ in ("q", "k", "v", "state", "z")}
    cu = np.concatenate([[0], np.cumsum(lens)])
    for s_, (a, e) in enumerate(zip(cu[:-1], cu[1:])):
        fn = oracle.chunked if e - a > 1 else oracle.recurrent
        core, st = fn(f["q"][None, a:e], f["k"][None, a:e], f["v"][None, a:e], g[None, a:e],
                      beta[None, a:e], f["state"][s_][None])
        core = _np(torch.from_numpy(core).bfloat16())
        want = olayer.gated_norm(core, f["z"][None, a:e], _np(x["w"]), 1e-6)
        _check(f"mixed layer seq {s_}", _np(out[a:e])[None], _np(pool[s_])[None], want, st)


def test_layer_conv_outputs_decode():
    x = _layer_inputs([1] * 10, seed=9)
    d = {k_: x[k_][:, None] for k_ in ("q", "k", "v", "a", "b", "z")}
    out, st = GatedDeltaRule().recurrent(d["q"], d["k"], d["v"], None, None, x["state"],
                                         gates=(d["a"], d["b"], x["a_log"], x["dt_bias"]),
                                         norm=(d["z"], x["w"], 1e-6))
    _ok()
    g, beta = olayer.gates(_np(d["a"]), _np(d["b"]), _np(x["a_log"]), _np(x["dt_bias"]),
                           beta_dtype="bf16")
    core, want_st = oracle.recurrent(_np(d["q"]), _np(d["k"]), _np(d["v"]), g, beta,
                                     _np(x["state"]))
    want = olayer.gated_norm(_np(torch.from_numpy(core).bfloat16()), _np(d["z"]), _np(x["w"]),
                             1e-6)
    _check("layer decode", _np(out), _np(st), want, want_st)


# -- every benchmark configuration at its full shape ---------------------------------
def test_config_dense_prefill_full_against_oracle():
    """8 x 4096 tokens, 16 q/k and 32 v heads, d 128, chunk 64, bf16, zero
    state, through the default (auto) path."""
    w = workloads.get("dense_prefill")
    x = workloads.make_inputs(w, DEV, seed=101)
    o, s = GatedDeltaRule().chunked(x["q"], x["k"], x["v"], x["g"], x["beta"])
    _ok()
    wo, ws = _oracle(x, 1e-6)
    _check("config dense 8x4096", _np(o), _np(s), wo, ws)


def test_config_dense_prefill_full_raw_qk():
    """The dense shape with raw N(0, 1) q and k instead of unit vectors."""
    w = workloads.get("dense_prefill")
    x = workloads.make_inputs(w, DEV, seed=102)
    gen = torch.Generator(device=DEV).manual_seed(103)
    x["q"] = torch.randn(x["q"].shape, device=DEV, generator=gen).bfloat16()
    x["k"] = torch.randn(x["k"].shape, device=DEV, generator=gen).bfloat16()
    o, s = GatedDeltaRule().chunked(x["q"], x["k"], x["v"], x["g"], x["beta"])
    _ok()
    wo, ws = _oracle(x, 1e-6)
    _check("config dense raw q/k", _np(o), _np(s), wo, ws)


@pytest.mark.parametrize("heads", [32, 4])
def test_config_ragged_prefill_full_against_oracle(heads):
    """131072 tokens in 64 lognormal sequences with f32 initial states,
    through the default (auto) path the benchmark times: all 32 value heads
    (one GPU) and the 4 value heads one GPU of eight holds, where the call
    splits the long sequences into segments."""
    w = workloads.get("ragged_prefill")
    x = workloads.make_inputs(w, DEV, seed=104)
    if heads != w.heads_v:
        hq = heads * w.heads_qk // w.heads_v
        cut = {"q": hq, "k": hq, "v": heads, "g": heads, "beta": heads, "state": heads}
        x = {k_: (v[:, :cut[k_]].contiguous() if k_ in cut else v) for k_, v in x.items()}
    rule = GatedDeltaRule()
    launches = rule.chunked_launches(x["q"], x["v"], x["cu_seqlens"])
    o, s = rule.chunked(x["q"], x["k"], x["v"], x["g"], x["beta"], x["state"],
                        cu_seqlens=x["cu_seqlens"])
    _ok()
    wo, ws = _oracle(x, 1e-6)
    _check(f"config ragged 131072 x {heads} heads ({launches} launches)", _np(o), _np(s), wo, ws)


def test_config_decode_full_64_steps_against_oracle():
    """256 rows x 1 token, 32 v / 16 q/k heads, d 128, bf16, f32 states
    [256, 32, 128, 128] updated in place for 64 consecutive steps; the oracle
    steps its own states. Every step's output and the final states are
    checked."""
    w = workloads.get("decode")
    x = workloads.make_inputs(w, DEV, seed=105)
    st = x["state"].clone()
    want_st = _np(x["state"])
    rule = GatedDeltaRule()
    worst = 0.0
    for i in range(64):
        y = workloads.make_inputs(w, DEV, seed=1000 + i) if i else x
        out, _ = rule.recurrent(y["q"], y["k"], y["v"], y["g"], y["beta"], st, state_out=st)
        torch.cuda.synchronize()
        wo, want_st = oracle.recurrent(_np(y["q"]), _np(y["k"]), _np(y["v"]), _np(y["g"]),
                                       _np(y["beta"]), want_st)
        worst = max(worst, rel_err(_np(out), wo))
        assert worst < TOL_BF16_OUT, (i, worst)
    _ok()
    _check("config decode 64 steps", np.zeros(1), _np(st), np.zeros(1), want_st)
    print(f"config decode: worst step output {worst:.2e}")


def test_config_mixed_full_against_oracle():
    """8 prefill segments x 2048 tokens continuing from states + 1024 decode
    rows with states, one gdr_mixed launch, states in place."""
    w = workloads.get("mixed")
    x = workloads.make_inputs(w, DEV, seed=107)
    pool = x["state"].clone()
    out = GatedDeltaRule().mixed(x["q"], x["k"], x["v"], x["g"], x["beta"], pool,
                                 cu_seqlens=x["cu_seqlens"])
    _ok()
    f = {k_: _np(x[k_]) for k_ in ("q", "k", "v", "g", "beta", "state")}
    n_pre = sum(1 for L in w.seqlens if L > 1)
    t_pre = sum(L for L in w.seqlens if L > 1)
    cu = np.concatenate([[0], np.cumsum(w.seqlens[:n_pre])]).astype(np.int32)
    o1, s1 = oracle.chunked(*(f[k_][:t_pre] for k_ in ("q", "k", "v", "g", "beta")),
                            f["state"][:n_pre], cu_seqlens=cu)
    o2, s2 = oracle.recurrent(*(f[k_][t_pre:, None] for k_ in ("q", "k", "v", "g", "beta")),
                              f["state"][n_pre:])
    got = _np(out)
    _check("config mixed prefill", got[:t_pre], _np(pool[:n_pre]), o1, s1)
    _check("config mixed decode", got[t_pre:], _np(pool[n_pre:]), o2[:, 0], s2)
