"""The CUDA kernels against the CPU oracle, through the C ABI.

Tolerances (max |got - want| / max |want|): 1e-4 for f32 runs; 2e-2 on
outputs and 1e-2 on states for bf16 inputs (the oracle runs in f32 on the
same bf16-rounded values, as bunsen widens them, delta_rule.rs:151-155)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from bunsen_b200 import _lib, workloads
from bunsen_b200.rule import GatedDeltaRule
from oracle import oracle
from tests.conftest import TOL_BF16_OUT, TOL_BF16_STATE, TOL_F32, rel_err

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _np(x):
    return None if x is None else workloads.to_numpy_f32(x)


def _oracle(form, x, chunk=64, eps=1e-6, state="state"):
    kw = {"chunk_size": chunk} if form == "chunked" else {}
    cu = x.get("cu_seqlens")
    return getattr(oracle, form)(
        _np(x["q"]), _np(x["k"]), _np(x["v"]), _np(x["g"]), _np(x["beta"]),
        _np(x.get(state)), l2norm_eps=eps, cu_seqlens=None if cu is None else _np(cu).astype(
            np.int32), **kw)


def _gpu(form, x, rule, state="state"):
    fn = getattr(rule, form)
    out, st = fn(x["q"], x["k"], x["v"], x["g"], x["beta"], x.get(state),
                 cu_seqlens=x.get("cu_seqlens"))
    torch.cuda.synchronize()
    assert _lib.load().gdr_device_error() == _lib.GDR_OK
    return _np(out), _np(st)


def _to(x, dev=DEV):
    return {k: (v.to(dev) if isinstance(v, torch.Tensor) else v) for k, v in x.items()}


def _from_golden(golden, name, dtype=torch.float32):
    d = golden["hf_cases"]
    x = {k: torch.from_numpy(d[f"{name}.{k}"]) for k in ("q", "k", "v", "g", "beta")}
    x["state"] = torch.from_numpy(d[f"{name}.s0"])
    return _to(x)


# -- small shapes: the generic kernels, f32 ---------------------------------
@pytest.mark.parametrize("name", ["scalar", "parts", "t8", "t10", "t3", "t70", "t1", "t13"])
@pytest.mark.parametrize("initial", [False, True])
@pytest.mark.parametrize("eps", [1e-6, None])
def test_recurrent_small_f32(golden, name, initial, eps):
    x = _from_golden(golden, name)
    if not initial:
        x.pop("state")
    rule = GatedDeltaRule(qk_l2norm_eps=eps)
    o, s = _gpu("recurrent", x, rule)
    wo, ws = _oracle("recurrent", x, eps=eps)
    assert rel_err(o, wo) < TOL_F32 and rel_err(s, ws) < TOL_F32


@pytest.mark.parametrize("name,chunk", [("t8", 4), ("t10", 4), ("t3", 4), ("t70", 64), ("t1", 64),
                                        ("t13", 4), ("t70", 16)])
@pytest.mark.parametrize("initial", [False, True])
@pytest.mark.parametrize("eps", [1e-6, None])
def test_chunked_small_f32(golden, name, chunk, initial, eps):
    x = _from_golden(golden, name)
    if not initial:
        x.pop("state")
    rule = GatedDeltaRule(qk_l2norm_eps=eps, chunk_size=chunk)
    o, s = _gpu("chunked", x, rule)
    wo, ws = _oracle("chunked", x, chunk=chunk, eps=eps)
    assert rel_err(o, wo) < TOL_F32 and rel_err(s, ws) < TOL_F32
    ro, rs = _oracle("recurrent", x, eps=eps)
    assert rel_err(o, ro) < TOL_F32 and rel_err(s, rs) < TOL_F32


@pytest.mark.parametrize("toy", ["toy_layer0", "toy_untied_layer0"])
@pytest.mark.parametrize("form", ["chunked", "recurrent"])
def test_known_answer_layer0_core(golden, toy, form):
    """bunsen's io.layer0_core fixture through the GPU, q/k with H_qk heads."""
    d = golden[toy]
    ratio = d["v"].shape[2] // int(d["n_key_heads"])
    x = _to({"q": torch.from_numpy(np.ascontiguousarray(d["q"][:, :, ::ratio])),
             "k": torch.from_numpy(np.ascontiguousarray(d["k"][:, :, ::ratio])),
             "v": torch.from_numpy(d["v"]), "g": torch.from_numpy(d["g"]),
             "beta": torch.from_numpy(d["beta"])})
    o, _ = _gpu(form, x, GatedDeltaRule())
    assert rel_err(o, d["core"]) < TOL_F32


def test_fixture_f32_config():
    """The CPU-runnable fixture: B 2 x T 64, 4 heads, d 32, chunk 16, f32."""
    w = workloads.get("fixture_f32")
    x = workloads.make_inputs(w, DEV, seed=7)
    rule = GatedDeltaRule(chunk_size=w.chunk)
    for form in ("chunked", "recurrent"):
        o, s = _gpu(form, x, rule)
        wo, ws = _oracle(form, x, chunk=w.chunk)
        assert rel_err(o, wo) < TOL_F32 and rel_err(s, ws) < TOL_F32


# -- d = 128: the decode kernel --------------------------------------------
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("t", [1, 5])
def test_recurrent_d128(dtype, t):
    gen = torch.Generator(device=DEV).manual_seed(11)
    b, hq, hv = 6, 2, 4
    x = {"q": torch.randn(b, t, hq, 128, device=DEV, generator=gen).to(dtype),
         "k": torch.randn(b, t, hq, 128, device=DEV, generator=gen).to(dtype),
         "v": torch.randn(b, t, hv, 128, device=DEV, generator=gen).to(dtype),
         "g": -torch.rand(b, t, hv, device=DEV, generator=gen),
         "beta": torch.rand(b, t, hv, device=DEV, generator=gen),
         "state": torch.randn(b, hv, 128, 128, device=DEV, generator=gen) * 0.1}
    o, s = _gpu("recurrent", x, GatedDeltaRule())
    wo, ws = _oracle("recurrent", x)
    tol_o = TOL_F32 if dtype == torch.float32 else TOL_BF16_OUT
    assert rel_err(o, wo) < tol_o and rel_err(s, ws) < TOL_F32


def test_decode_workload_rows_against_oracle():
    """The decode benchmark's shape (256 rows, 32 v / 16 q-k heads, d 128,
    bf16, f32 states in place); 16 rows checked against the oracle."""
    w = workloads.get("decode")
    x = workloads.make_inputs(w, DEV, seed=3)
    st = x["state"].clone()
    out, st2 = GatedDeltaRule().recurrent(x["q"], x["k"], x["v"], x["g"], x["beta"], st,
                                          state_out=st)
    torch.cuda.synchronize()
    assert st2.data_ptr() == st.data_ptr()
    sub = {k: v[:16] for k, v in x.items()}
    wo, ws = _oracle("recurrent", sub)
    assert rel_err(_np(out[:16]), wo) < TOL_BF16_OUT
    assert rel_err(_np(st[:16]), ws) < TOL_F32


# -- bf16, d = 128, chunk 64: the tensor-core kernel -------------------------
def _rand_bf16(lens, hq=2, hv=4, state=True, seed=5, packed=True):
    gen = torch.Generator(device=DEV).manual_seed(seed)
    t = sum(lens)
    f = dict(device=DEV, generator=gen)
    unit = lambda a: a / a.norm(dim=-1, keepdim=True)  # noqa: E731
    x = {"q": unit(torch.randn(t, hq, 128, **f)).to(torch.bfloat16),
         "k": unit(torch.randn(t, hq, 128, **f)).to(torch.bfloat16),
         "v": torch.randn(t, hv, 128, **f).to(torch.bfloat16),
         "g": torch.log(torch.rand(t, hv, **f) * 0.099 + 0.9),
         "beta": torch.sigmoid(torch.randn(t, hv, **f))}
    if state:
        x["state"] = torch.randn(len(lens), hv, 128, 128, **f) * 0.1
    if packed:
        x["cu_seqlens"] = torch.tensor(np.concatenate([[0], np.cumsum(lens)]), dtype=torch.int32,
                                       device=DEV)
    else:
        for key in ("q", "k", "v", "g", "beta"):
            x[key] = x[key].reshape((len(lens), lens[0]) + x[key].shape[1:])
    return x


@pytest.mark.parametrize("lens,packed", [([256, 256], False), ([200, 200], False),
                                         ([64, 1, 65, 63, 0, 300, 128, 2], True)])
@pytest.mark.parametrize("state", [False, True])
def test_chunked_tensor_core_against_oracle(lens, packed, state):
    x = _rand_bf16(lens, state=state, packed=packed)
    o, s = _gpu("chunked", x, GatedDeltaRule(algo="tensor"))
    wo, ws = _oracle("chunked", x)
    assert rel_err(o, wo) < TOL_BF16_OUT, rel_err(o, wo)
    assert rel_err(s, ws) < TOL_BF16_STATE, rel_err(s, ws)


def test_chunked_tensor_core_long_sequence():
    """One 4096-token sequence per head (the dense benchmark's length)."""
    x = _rand_bf16([4096], hq=1, hv=2, state=True)
    o, s = _gpu("chunked", x, GatedDeltaRule(algo="tensor"))
    wo, ws = _oracle("chunked", x)
    assert rel_err(o, wo) < TOL_BF16_OUT and rel_err(s, ws) < TOL_BF16_STATE


def test_tensor_core_agrees_with_f32_kernel_at_full_dense_size():
    """The dense prefill benchmark's full shape: the tensor-core kernel against
    the f32 CUDA-core kernel (itself held to the oracle at 1e-4 above)."""
    w = workloads.get("dense_prefill")
    x = workloads.make_inputs(w, DEV, seed=21)
    o_tc, s_tc = _gpu("chunked", x, GatedDeltaRule(algo="tensor"))
    o_f, s_f = _gpu("chunked", x, GatedDeltaRule(algo="cuda_core"))
    assert rel_err(o_tc, o_f) < TOL_BF16_OUT and rel_err(s_tc, s_f) < TOL_BF16_STATE


def test_chunked_parts_agree_with_one_pass_tensor_core():
    """Prefill in parts (cut mid-chunk), each from the state the last left,
    is the one-pass prefill (delta_rule.rs:612-642), at d 128 / chunk 64."""
    x = _rand_bf16([500], hq=2, hv=4, state=True)
    rule = GatedDeltaRule(algo="tensor")
    whole, whole_s = _gpu("chunked", x, rule)
    st = x["state"]
    parts = []
    for a, b in ((0, 100), (100, 101), (101, 500)):
        y = {k: x[k][a:b] for k in ("q", "k", "v", "g", "beta")}
        y["cu_seqlens"] = torch.tensor([0, b - a], dtype=torch.int32, device=DEV)
        y["state"] = st
        o, s = rule.chunked(y["q"], y["k"], y["v"], y["g"], y["beta"], st,
                            cu_seqlens=y["cu_seqlens"])
        parts.append(_np(o))
        st = s
    torch.cuda.synchronize()
    assert rel_err(np.concatenate(parts), whole) < TOL_BF16_OUT
    assert rel_err(_np(st), whole_s) < TOL_BF16_STATE


def test_chunked_matches_recurrent_on_gpu_ragged():
    """A scaled ragged pack: chunked (tensor core) against recurrent (CUDA
    cores, f32 state), both on the GPU."""
    w = workloads.get("ragged_prefill", scale=0.125)
    x = workloads.make_inputs(w, DEV, seed=4)
    o_c, s_c = _gpu("chunked", x, GatedDeltaRule())
    o_r, s_r = _gpu("recurrent", x, GatedDeltaRule())
    assert rel_err(o_c, o_r) < TOL_BF16_OUT and rel_err(s_c, s_r) < TOL_BF16_STATE


def test_empty_batch_is_a_no_op():
    x = _rand_bf16([5], state=True)
    x["cu_seqlens"] = torch.zeros(1, dtype=torch.int32, device=DEV)
    out, st = GatedDeltaRule().chunked(x["q"][:0], x["k"][:0], x["v"][:0], x["g"][:0],
                                       x["beta"][:0], None, cu_seqlens=x["cu_seqlens"])
    torch.cuda.synchronize()
    assert out.shape == (0, 4, 128) and st.shape == (0, 4, 128, 128)


def test_zero_length_sequences_pass_the_state_through():
    """Sequences with no tokens return their state unchanged (zeros without
    one), on every path."""
    x = _rand_bf16([3], state=True)
    cu = torch.zeros(3, dtype=torch.int32, device=DEV)
    s0 = torch.randn(2, 4, 128, 128, device=DEV)
    e = {k: x[k][:0] for k in ("q", "k", "v", "g", "beta")}
    for form in ("chunked", "recurrent"):
        out, st = getattr(GatedDeltaRule(), form)(e["q"], e["k"], e["v"], e["g"], e["beta"], s0,
                                                  cu_seqlens=cu)
        torch.cuda.synchronize()
        assert out.shape == (0, 4, 128) and torch.equal(st, s0)
        _, st = getattr(GatedDeltaRule(), form)(e["q"], e["k"], e["v"], e["g"], e["beta"], None,
                                                cu_seqlens=cu)
        torch.cuda.synchronize()
        assert torch.count_nonzero(st) == 0
