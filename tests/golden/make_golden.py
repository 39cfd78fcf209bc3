#!/usr/bin/env python3
"""Generate the golden vectors the oracle is pinned against.

Run once where the bunsen sources are readable and ``transformers`` is
installed; commit the ``.npz`` files it writes next to this script. Nothing at
test time reads the reference.

    python tests/golden/make_golden.py <bunsen checkout>
    BUNSEN_SRC=<bunsen checkout> python tests/golden/make_golden.py

Two groups of vectors are written:

1. ``toy_layer0.npz`` and ``toy_untied_layer0.npz`` -- bunsen's own known-answer
   fixture. ``crates/public/bunsen/testdata/qwen3_5/{toy,toy_untied}.safetensors``
   store ``io.layer0_core``: the first decoder layer's delta-rule output
   ``[1, 72, H_v, d_v]`` of a tiny seeded Qwen3.5 (written by
   ``tools/gen_qwen3_5_toy_fixtures.py:200-214``). The rule's inputs are not
   stored, so the toy model is rebuilt here from its ``config.json`` with the
   installed ``transformers``, its weights loaded, and the arguments of layer 0's
   ``chunk_gated_delta_rule`` call captured (q, k already repeated to the value
   heads; ``modeling_qwen3_5.py`` ``Qwen3_5GatedDeltaNet.forward``). The
   captured call's own output must reproduce ``io.layer0_core``; the script
   asserts it before writing. Inputs are stored as float32 (the dtype the rule
   computes in); the golden output is the fixture's ``io.layer0_core`` itself.

2. ``hf_cases.npz`` -- seeded small cases on the shapes of bunsen's unit tests
   (``delta_rule.rs:452, 501, 554-555, 614``) run through ``transformers``'
   ``torch_recurrent_gated_delta_rule`` in float64: the same published rule
   bunsen's ``scalar_rule`` restates (``delta_rule.rs:396-445``), a second,
   independent anchor for the oracle's recurrent and chunked forms.
"""

from __future__ import annotations

import json
import pathlib

import numpy as np
import torch

# The toy fixtures' directory inside a bunsen checkout (set by main()).
FIXTURES = "crates/public/bunsen/testdata/qwen3_5"
REF = pathlib.Path(FIXTURES)
OUT = pathlib.Path(__file__).resolve().parent


def toy_vectors(name: str) -> dict[str, np.ndarray]:
    from safetensors.torch import load_file
    from transformers import Qwen3_5Config, Qwen3_5ForConditionalGeneration

    cfg = json.loads((REF / f"{name}.config.json").read_text())
    config = Qwen3_5Config(**{k: v for k, v in cfg.items() if k not in ("architectures",)})
    config._attn_implementation = "eager"
    config.text_config._attn_implementation = "eager"
    torch.manual_seed(0)
    model = Qwen3_5ForConditionalGeneration(config).to(torch.float64).eval()
    tensors = load_file(str(REF / f"{name}.safetensors"))
    io = {k[3:]: v for k, v in tensors.items() if k.startswith("io.")}
    tied = cfg["text_config"]["tie_word_embeddings"]
    weights = {
        k: v.to(torch.float64)
        for k, v in tensors.items()
        if not k.startswith(("io.", "mtp.")) and not (tied and k == "lm_head.weight")
    }
    missing, unexpected = model.load_state_dict(weights, strict=False)
    assert not unexpected, unexpected
    assert all(k == "lm_head.weight" for k in missing), missing
    if tied:
        model.tie_weights()

    lm = model.model.language_model
    mixer = lm.layers[0].linear_attn
    captured: dict[str, torch.Tensor] = {}
    # The layer's other steps around the rule (gated_delta_net.rs:396-440):
    # the short convolution's input, the gate projections, the gated norm.
    assert mixer.causal_conv1d_fn is None and mixer.conv1d.bias is None
    hooks = [
        mixer.conv1d.register_forward_hook(
            lambda m, i, o: captured.update(conv_x=i[0])),
        mixer.in_proj_a.register_forward_hook(lambda m, i, o: captured.update(a=o)),
        mixer.in_proj_b.register_forward_hook(lambda m, i, o: captured.update(b=o)),
        mixer.norm.register_forward_hook(
            lambda m, i, o: captured.update(norm_x=i[0], norm_z=i[1], norm_out=o)),
    ]
    inner = mixer.chunk_gated_delta_rule

    def spy(query, key, value, g, beta, **kw):
        out, state = inner(query, key, value, g=g, beta=beta, **kw)
        captured.update(q=query, k=key, v=value, g=g, beta=beta, out=out)
        captured["kw"] = kw
        return out, state

    mixer.chunk_gated_delta_rule = spy
    ids = io["input_ids"].to(torch.int64)
    with torch.no_grad():
        lm(input_ids=ids)
    for h in hooks:
        h.remove()
    kw = captured["kw"]
    assert kw.get("use_qk_l2norm_in_kernel") is True and kw.get("initial_state") is None
    core = io["layer0_core"].to(torch.float64)
    got = captured["out"].to(torch.float64)
    err = (got - core).abs().max().item()
    assert err < 1e-5, f"{name}: captured call reproduces io.layer0_core only to {err}"
    print(f"{name}: rule inputs captured; reproduce io.layer0_core to {err:.2e}")
    f32 = lambda x: x.detach().to(torch.float32).numpy()  # noqa: E731
    return {
        "q": f32(captured["q"]),
        "k": f32(captured["k"]),
        "v": f32(captured["v"]),
        "g": f32(captured["g"]),
        "beta": f32(captured["beta"]),
        "core": io["layer0_core"].numpy().astype(np.float32),
        "chunk_size": np.array(64, dtype=np.int64),
        "n_key_heads": np.array(cfg["text_config"]["linear_num_key_heads"], dtype=np.int64),
        # The steps around the rule: conv input [T, C] and kernel [C, K]
        # (its output, after silu and the q/k/v split, is q/k/v above, q and k
        # repeated to the value heads); the gate projections a, b [T, H_v] with
        # A_log and dt_bias [H_v] (giving g and beta above); the gated norm's
        # input [T * H_v, d_v], gate z, weight [d_v], epsilon and output.
        "conv_x": f32(captured["conv_x"][0].transpose(0, 1)),
        "conv_w": f32(mixer.conv1d.weight[:, 0, :]),
        "a": f32(captured["a"][0]),
        "b": f32(captured["b"][0]),
        "a_log": f32(mixer.A_log),
        "dt_bias": f32(mixer.dt_bias),
        "norm_x": f32(captured["norm_x"]),
        "norm_z": f32(captured["norm_z"]),
        "norm_w": f32(mixer.norm.weight),
        "norm_eps": np.array(mixer.norm.variance_epsilon, dtype=np.float64),
        "norm_out": f32(captured["norm_out"]),
    }


def hf_cases() -> dict[str, np.ndarray]:
    """transformers' recurrent rule in float64 on seeded inputs of bunsen's
    unit-test shapes, with and without an initial state and the L2 norm."""
    from transformers.models.qwen3_5.modeling_qwen3_5 import torch_recurrent_gated_delta_rule

    rng = np.random.default_rng(20240611)
    shapes = {
        "scalar": (2, 5, 3, 4, 6),
        "parts": (2, 7, 2, 4, 3),
        "t8": (2, 8, 3, 4, 5),
        "t10": (2, 10, 3, 4, 5),
        "t3": (2, 3, 3, 4, 5),
        "t70": (2, 70, 3, 4, 5),
        "t1": (2, 1, 3, 4, 5),
        "t13": (1, 13, 2, 4, 3),
    }
    out: dict[str, np.ndarray] = {}
    for name, (b, t, h, dk, dv) in shapes.items():
        q = rng.standard_normal((b, t, h, dk))
        k = rng.standard_normal((b, t, h, dk))
        v = rng.standard_normal((b, t, h, dv))
        g = rng.uniform(-1.0, 0.0, (b, t, h))
        beta = rng.uniform(0.0, 1.0, (b, t, h))
        s0 = rng.standard_normal((b, h, dk, dv))
        # The inputs are rounded to f32 first, so the f64 rule runs on exactly
        # the values an f32 implementation sees.
        q, k, v, g, beta, s0 = (x.astype(np.float32) for x in (q, k, v, g, beta, s0))
        for key, arr in (("q", q), ("k", k), ("v", v), ("g", g), ("beta", beta), ("s0", s0)):
            out[f"{name}.{key}"] = arr
        for initial in (False, True):
            for norm in (True, False):
                T = lambda x: torch.from_numpy(x).to(torch.float64)  # noqa: E731
                qq, kk = T(q), T(k)
                if norm:  # bunsen's form: x / sqrt(sum x^2 + eps), in f64
                    qq = qq / torch.sqrt((qq * qq).sum(-1, keepdim=True) + 1e-6)
                    kk = kk / torch.sqrt((kk * kk).sum(-1, keepdim=True) + 1e-6)
                o, s = _recurrent_f64(qq, kk, T(v), T(g), T(beta), T(s0) if initial else None)
                tag = f"{name}.i{int(initial)}n{int(norm)}"
                out[f"{tag}.out"] = o.numpy()
                out[f"{tag}.state"] = s.numpy()
        # transformers' function itself, once per case, as a cross-check of
        # the f64 loop above (it normalises with rsqrt and runs in f32).
        o_hf, s_hf = torch_recurrent_gated_delta_rule(
            torch.from_numpy(q), torch.from_numpy(k), torch.from_numpy(v), torch.from_numpy(g),
            torch.from_numpy(beta), torch.from_numpy(s0), True, use_qk_l2norm_in_kernel=True)
        ref_o = out[f"{name}.i1n1.out"]
        assert np.abs(o_hf.numpy() - ref_o).max() < 1e-4 * max(1.0, np.abs(ref_o).max())
    return out


def _recurrent_f64(q, k, v, g, beta, s0):
    """The per-position rule in f64: decay, read at the key, correct, read at
    the query (``delta_rule.rs:195-206``), q scaled by 1/sqrt(d_k)."""
    b, t, h, dk = q.shape
    dv = v.shape[-1]
    s = torch.zeros(b, h, dk, dv, dtype=torch.float64) if s0 is None else s0.clone()
    q = q / dk**0.5
    out = torch.zeros(b, t, h, dv, dtype=torch.float64)
    for i in range(t):
        s = s * g[:, i].exp()[..., None, None]
        read = torch.einsum("bhk,bhkv->bhv", k[:, i], s)
        delta = (v[:, i] - read) * beta[:, i][..., None]
        s = s + torch.einsum("bhk,bhv->bhkv", k[:, i], delta)
        out[:, i] = torch.einsum("bhk,bhkv->bhv", q[:, i], s)
    return out, s


def main() -> None:
    torch.set_grad_enabled(False)
    for name in ("toy", "toy_untied"):
        np.savez_compressed(OUT / f"{name}_layer0.npz", **toy_vectors(name))
    np.savez_compressed(OUT / "hf_cases.npz", **hf_cases())
    print("wrote", sorted(p.name for p in OUT.glob("*.npz")))


if __name__ == "__main__":
    import os
    import sys

    src = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("BUNSEN_SRC")
    if not src:
        sys.exit("usage: make_golden.py <bunsen checkout> (or set BUNSEN_SRC)")
    REF = pathlib.Path(src) / FIXTURES
    main()
