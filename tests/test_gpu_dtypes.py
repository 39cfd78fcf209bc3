"""Dtypes and shapes beyond the tensor-core kernels' bf16 / d 128 / chunk 64,
against the CPU oracle.

bunsen widens half-precision inputs to f32 and narrows the output back to
q's dtype (``burner/tensor/widening.rs:58-60``, ``delta_rule.rs:151-155``):
f16 runs compute in f32 here too, so they are held to f32 rounding plus the
f16 rounding of the output (2e-3 on outputs, 1e-4 on the f32 states). A
chunk above 64 or heads above 128 (up to 256) run on the recurrent kernel,
which bunsen's own tests hold to its chunked form at 1e-5
(``delta_rule.rs:549-608``): f32 runs at 1e-4, bf16 at 2e-2 / 1e-2."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from bunsen_b200 import _lib, workloads
from bunsen_b200.layer import causal_conv1d, gated_norm
from bunsen_b200.rule import GatedDeltaRule
from oracle import layer as olayer
from oracle import oracle
from tests.conftest import TOL_BF16_OUT, TOL_BF16_STATE, TOL_F32, rel_err

pytestmark = pytest.mark.gpu
DEV = "cuda"
TOL_F16_OUT = 2e-3


def _np(x):
    return None if x is None else workloads.to_numpy_f32(x)


def _ok():
    torch.cuda.synchronize()
    assert _lib.load().gdr_device_error() == _lib.GDR_OK


def _inputs(lens, dtype, hq=2, hv=4, dk=128, dv=128, seed=0, state=True):
    gen = torch.Generator(device=DEV).manual_seed(seed)
    f = dict(device=DEV, generator=gen)
    t = sum(lens)
    unit = lambda a: a / a.norm(dim=-1, keepdim=True)  # noqa: E731
    x = {"q": unit(torch.randn(t, hq, dk, **f)).to(dtype),
         "k": unit(torch.randn(t, hq, dk, **f)).to(dtype),
         "v": torch.randn(t, hv, dv, **f).to(dtype),
         "g": torch.log(torch.rand(t, hv, **f) * 0.099 + 0.9),
         "beta": torch.sigmoid(torch.randn(t, hv, **f)),
         "cu_seqlens": torch.tensor(np.concatenate([[0], np.cumsum(lens)]), dtype=torch.int32,
                                    device=DEV)}
    if state:
        x["state"] = torch.randn(len(lens), hv, dk, dv, **f) * 0.1
    return x


def _run(form, x, rule):
    o, s = getattr(rule, form)(x["q"], x["k"], x["v"], x["g"], x["beta"], x.get("state"),
                               cu_seqlens=x["cu_seqlens"])
    _ok()
    return _np(o), _np(s)


def _want(form, x, chunk=64, eps=1e-6):
    kw = {"chunk_size": chunk} if form == "chunked" else {}
    return getattr(oracle, form)(*(_np(x[k]) for k in ("q", "k", "v", "g", "beta")),
                                 _np(x.get("state")), l2norm_eps=eps,
                                 cu_seqlens=_np(x["cu_seqlens"]).astype(np.int32), **kw)


@pytest.mark.parametrize("form", ["chunked", "recurrent"])
@pytest.mark.parametrize("dk,dv", [(128, 128), (32, 32), (8, 12)])
def test_f16_against_oracle(form, dk, dv):
    lens = [70, 1, 64, 0, 130] if form == "chunked" else [3, 1, 2]
    x = _inputs(lens, torch.float16, dk=dk, dv=dv, seed=1)
    o, s = _run(form, x, GatedDeltaRule())
    wo, ws = _want(form, x)
    assert rel_err(o, wo) < TOL_F16_OUT and rel_err(s, ws) < TOL_F32, (rel_err(o, wo),
                                                                      rel_err(s, ws))


def test_f16_decode_rows_and_output_dtype():
    x = _inputs([1] * 16, torch.float16, seed=2)
    d = {k: x[k][:, None] for k in ("q", "k", "v", "g", "beta")}
    out, st = GatedDeltaRule().recurrent(d["q"], d["k"], d["v"], d["g"], d["beta"], x["state"])
    _ok()
    assert out.dtype == torch.float16 and st.dtype == torch.float32
    wo, ws = oracle.recurrent(*(_np(d[k]) for k in ("q", "k", "v", "g", "beta")),
                              _np(x["state"]))
    assert rel_err(_np(out), wo) < TOL_F16_OUT and rel_err(_np(st), ws) < TOL_F32


def test_f16_host_buffers():
    x = _inputs([300, 65, 1], torch.float16, seed=3)
    h = {k: v.cpu().pin_memory() for k, v in x.items()}
    out, st = GatedDeltaRule().chunked_host(h["q"], h["k"], h["v"], h["g"], h["beta"], h["state"],
                                           cu_seqlens=h["cu_seqlens"])
    wo, ws = _want("chunked", x)
    assert rel_err(_np(out), wo) < TOL_F16_OUT and rel_err(_np(st), ws) < TOL_F32


@pytest.mark.parametrize("chunk", [128, 96, 256])
def test_chunk_above_64_bf16_d128(chunk):
    x = _inputs([300, 1, 128, 129], torch.bfloat16, seed=4)
    rule = GatedDeltaRule(chunk_size=chunk)
    assert rule.chunked_launches(x["q"], x["v"], x["cu_seqlens"]) == 1
    o, s = _run("chunked", x, rule)
    wo, ws = _want("chunked", x, chunk=chunk)
    assert rel_err(o, wo) < TOL_BF16_OUT and rel_err(s, ws) < TOL_BF16_STATE


@pytest.mark.parametrize("chunk", [128, 100])
@pytest.mark.parametrize("eps", [1e-6, None])
def test_chunk_above_64_f32(chunk, eps):
    x = _inputs([257, 3, 128], torch.float32, dk=32, dv=48, seed=5)
    o, s = _run("chunked", x, GatedDeltaRule(chunk_size=chunk, qk_l2norm_eps=eps))
    wo, ws = _want("chunked", x, chunk=chunk, eps=eps)
    assert rel_err(o, wo) < TOL_F32 and rel_err(s, ws) < TOL_F32


@pytest.mark.parametrize("dk,dv", [(192, 192), (256, 128), (160, 256), (256, 256)])
def test_heads_above_128_chunked_f32(dk, dv):
    """Head sizes above 128 run on the recurrent kernel, whose CTAs split a
    state wider than their shared memory into column blocks."""
    x = _inputs([90, 1, 65], torch.float32, hq=1, hv=2, dk=dk, dv=dv, seed=6)
    for algo in ("auto", "cuda_core"):
        o, s = _run("chunked", x, GatedDeltaRule(algo=algo))
        wo, ws = _want("chunked", x)
        assert rel_err(o, wo) < TOL_F32 and rel_err(s, ws) < TOL_F32
    o, s = _run("recurrent", x, GatedDeltaRule())
    wo, ws = _want("recurrent", x)
    assert rel_err(o, wo) < TOL_F32 and rel_err(s, ws) < TOL_F32


def test_f16_layer_steps():
    """The layer's conv (+ silu, split), gates from f16 projections (beta
    rounded to f16), rule and gated norm, all f16, against the oracles."""
    gen = torch.Generator(device=DEV).manual_seed(7)
    f = dict(device=DEV, generator=gen)
    lens = [70, 1, 33]
    t, hq, hv, d = sum(lens), 2, 4, 64
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]), dtype=torch.int32, device=DEV)
    c = 2 * hq * d + hv * d
    xin = torch.randn(t, c, **f).half()
    wconv = (torch.randn(c, 4, **f) * 0.5).half()
    (q, k, v), _ = causal_conv1d(xin, wconv, None, cu_seqlens=cu, silu=True,
                                 splits=(hq * d, 2 * hq * d))
    _ok()
    want_conv, _ = olayer.causal_conv1d(_np(xin), _np(wconv), None,
                                        cu_seqlens=_np(cu).astype(np.int32), activation=True)
    got_conv = np.concatenate([_np(q), _np(k), _np(v)], axis=1)
    assert rel_err(got_conv, want_conv) < TOL_F16_OUT
    q, k, v = q.reshape(t, hq, d), k.reshape(t, hq, d), v.reshape(t, hv, d)
    a, b = torch.randn(t, hv, **f).half(), torch.randn(t, hv, **f).half()
    a_log = torch.log(torch.rand(hv, **f) * 0.3 + 0.01)
    dt_bias = torch.randn(hv, **f) * 0.1
    z = torch.randn(t, hv, d, **f).half()
    w = torch.rand(d, **f) + 0.5
    s0 = torch.randn(len(lens), hv, d, d, **f) * 0.1
    out, st = GatedDeltaRule().chunked(q, k, v, None, None, s0, cu_seqlens=cu,
                                       gates=(a, b, a_log, dt_bias), norm=(z, w, 1e-6))
    _ok()
    assert out.dtype == torch.float16
    g_, beta_ = olayer.gates(_np(a), _np(b), _np(a_log), _np(dt_bias))
    beta_ = torch.from_numpy(beta_).half().float().numpy()  # sigmoid in the projection's dtype
    core, want_st = oracle.chunked(_np(q), _np(k), _np(v), g_, beta_, _np(s0),
                                   cu_seqlens=_np(cu).astype(np.int32))
    core = _np(torch.from_numpy(core).half())  # the rule's output in q's dtype
    want = olayer.gated_norm(core, _np(z), _np(w), 1e-6)
    assert rel_err(_np(out), want) < TOL_F16_OUT and rel_err(_np(st), want_st) < TOL_F32
    # The gated norm on its own.
    y = gated_norm(torch.from_numpy(core).half().to(DEV), z, w, 1e-6)
    _ok()
    assert rel_err(_np(y), want) < TOL_F16_OUT


@pytest.mark.parametrize("eps", [1e-6, None])
@pytest.mark.parametrize("state", [False, True])
@pytest.mark.parametrize("algo", ["auto", "cuda_core"])
def test_f32_d128_chunked_against_oracle(eps, state, algo):
    """f32 at the production head size: the register-tiled f32 kernel, every
    padding case of a ragged pack, held to the oracle at 1e-4."""
    lens = [70, 1, 64, 0, 130, 200, 63]
    x = _inputs(lens, torch.float32, seed=8, state=state)
    if eps is None:  # keep the rule stable without the norm: k of norm below 1
        x["k"] = x["k"] * 0.9
    o, s = _run("chunked", x, GatedDeltaRule(qk_l2norm_eps=eps, algo=algo))
    wo, ws = _want("chunked", x, eps=eps)
    assert rel_err(o, wo) < TOL_F32 and rel_err(s, ws) < TOL_F32, (rel_err(o, wo), rel_err(s, ws))


def test_bf16_inputs_on_the_f32_kernel():
    """bf16 inputs through GDR_ALGO_CUDA_CORE compute in f32: states to 1e-4,
    outputs to their bf16 rounding."""
    x = _inputs([300, 65], torch.bfloat16, seed=9)
    o, s = _run("chunked", x, GatedDeltaRule(algo="cuda_core"))
    wo, ws = _want("chunked", x)
    assert rel_err(o, wo) < 1e-2 and rel_err(s, ws) < TOL_F32


TOL_F64 = 1e-10


@pytest.mark.parametrize("form", ["chunked", "recurrent"])
@pytest.mark.parametrize("dk,dv", [(8, 12), (128, 128), (256, 256)])
@pytest.mark.parametrize("eps", [1e-6, None])
def test_f64_against_the_scalar_f64_rule(form, dk, dv, eps):
    """f64 inputs compute in f64 (bunsen keeps f64 as its compute dtype, g,
    beta and the state included), held to the f64 scalar rule of bunsen's
    tests (delta_rule.rs:399-445) at 1e-10; a 256 x 256 state runs as column
    blocks."""
    lens = [70, 1, 0, 33]
    x = _inputs(lens, torch.float64, hq=1, hv=2, dk=dk, dv=dv, seed=10)
    x["g"], x["beta"], x["state"] = (x[n].double() for n in ("g", "beta", "state"))
    if eps is None:  # keep the rule stable without the norm
        x["k"] = x["k"] * 0.9
    rule = GatedDeltaRule(qk_l2norm_eps=eps)
    o, s = getattr(rule, form)(x["q"], x["k"], x["v"], x["g"], x["beta"], x["state"],
                               cu_seqlens=x["cu_seqlens"])
    _ok()
    assert o.dtype == torch.float64 and s.dtype == torch.float64
    wo, ws = oracle.scalar_f64(*(x[n].cpu().numpy() for n in ("q", "k", "v", "g", "beta")),
                               x["state"].cpu().numpy(), l2norm_eps=eps,
                               cu_seqlens=x["cu_seqlens"].cpu().numpy().astype(np.int32))
    assert rel_err(o.cpu().numpy(), wo) < TOL_F64 and rel_err(s.cpu().numpy(), ws) < TOL_F64


def test_f64_dense_batch_and_refusals():
    """A dense f64 batch through both forms (the chunk size changes nothing);
    f64 with the layer's gates or in a continuous batch is refused."""
    gen = torch.Generator(device=DEV).manual_seed(11)
    f = dict(device=DEV, generator=gen, dtype=torch.float64)
    b, t, h, d = 2, 37, 2, 16
    q, k, v = (torch.randn(b, t, h, d, **f) for _ in range(3))
    g = torch.log(torch.rand(b, t, h, **f) * 0.099 + 0.9)
    beta = torch.sigmoid(torch.randn(b, t, h, **f))
    s0 = torch.randn(b, h, d, d, **f) * 0.1
    o1, s1 = GatedDeltaRule(chunk_size=16).chunked(q, k, v, g, beta, s0)
    o2, s2 = GatedDeltaRule().recurrent(q, k, v, g, beta, s0)
    _ok()
    assert torch.equal(o1, o2) and torch.equal(s1, s2)
    wo, ws = oracle.scalar_f64(*(x.cpu().numpy() for x in (q, k, v, g, beta, s0)))
    assert rel_err(o1.cpu().numpy(), wo) < TOL_F64 and rel_err(s1.cpu().numpy(), ws) < TOL_F64
    with pytest.raises(TypeError):
        GatedDeltaRule().chunked(q, k, v, None, None, s0, gates=(g, beta, g[0, 0], g[0, 0]))
    cu = torch.tensor([0, t, 2 * t], dtype=torch.int32, device=DEV)
    pool = torch.zeros(2, h, d, d, device=DEV)
    with pytest.raises(TypeError):
        GatedDeltaRule().mixed(q.reshape(-1, h, d), k.reshape(-1, h, d), v.reshape(-1, h, d),
                               g.reshape(-1, h), beta.reshape(-1, h), pool, cu_seqlens=cu)
