"""The C ABI without a GPU: the library loads, exports every function
include/gdr.h declares, lays out gdr_params as the header does, and rejects
bad arguments (bunsen's panics, delta_rule.rs:135-150, :233) before touching
the device."""

from __future__ import annotations

import ctypes
import re
import subprocess

import pytest

from bunsen_b200 import _lib
from tests.conftest import ROOT

HEADER = ROOT / "include" / "gdr.h"


def declared() -> list[str]:
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(gdr_[a-z_0-9]+)\s*\(", text)))


def test_library_exports_every_declared_function():
    lib = _lib.load()
    names = declared()
    assert {"gdr_recurrent", "gdr_chunked", "gdr_mixed"} <= set(names)
    for name in names:
        assert hasattr(lib, name), name
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r" T (gdr_\w+)", out))
    assert set(names) <= exported


def test_params_layout_matches_header(tmp_path):
    src = tmp_path / "layout.c"
    src.write_text(
        '#include <stdio.h>\n#include <stddef.h>\n#include "gdr.h"\n'
        "int main(void) { printf(\"%zu" + " %zu" * len(_lib.GdrParams._fields_)
        + "\\n\", sizeof(gdr_params)"
        + "".join(f", offsetof(gdr_params, {f})" for f, _ in _lib.GdrParams._fields_)
        + "); return 0; }\n")
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-I", str(ROOT / "include"), "-o", str(exe), str(src)], check=True)
    got = [int(x) for x in subprocess.run([str(exe)], capture_output=True, text=True,
                                          check=True).stdout.split()]
    want = [ctypes.sizeof(_lib.GdrParams)] + [getattr(_lib.GdrParams, f).offset
                                              for f, _ in _lib.GdrParams._fields_]
    assert got == want


def test_binding_version_matches_the_header():
    """The bindings' ABI_VERSION is include/gdr.h's GDR_ABI_VERSION (build()
    checks the loaded library against it)."""
    text = HEADER.read_text()
    assert int(re.search(r"#define GDR_ABI_VERSION (\d+)", text).group(1)) == _lib.ABI_VERSION


def test_abi_version_and_status_strings():
    lib = _lib.load()
    assert lib.gdr_abi_version() == _lib.ABI_VERSION == 3
    for s in range(5):
        assert lib.gdr_status_string(s)
    assert lib.gdr_status_string(99) == b"unknown status"


def _params(**kw):
    base = dict(batch=1, seq_len=4, n_seqs=0, heads_qk=2, heads_v=4, d_k=8, d_v=8, chunk_size=4,
                use_l2norm=1, l2norm_eps=1e-6, dtype=_lib.GDR_DTYPE_F32, algo=0)
    base.update(kw)
    return _lib.GdrParams(**base)


@pytest.mark.parametrize("fn", ["gdr_recurrent", "gdr_chunked"])
@pytest.mark.parametrize("bad", [dict(heads_v=3), dict(heads_qk=0), dict(d_k=0), dict(dtype=7),
                                 dict(batch=-1), dict(use_l2norm=1, l2norm_eps=-1.0)])
def test_invalid_arguments_are_rejected_before_launch(fn, bad):
    lib = _lib.load()
    p = _params(**bad)
    dummy = ctypes.c_void_p(16)  # never dereferenced: the checks come first
    st = getattr(lib, fn)(ctypes.byref(p), dummy, dummy, dummy, dummy, dummy, None, dummy, dummy,
                          None, None)
    assert st == _lib.GDR_ERR_INVALID


def test_null_pointers_and_zero_chunk_are_rejected():
    lib = _lib.load()
    d = ctypes.c_void_p(16)
    assert lib.gdr_chunked(None, d, d, d, d, d, None, d, d, None, None) == _lib.GDR_ERR_INVALID
    p = _params()
    assert lib.gdr_chunked(ctypes.byref(p), None, d, d, d, d, None, d, d, None,
                           None) == _lib.GDR_ERR_INVALID
    p = _params(chunk_size=0)
    assert lib.gdr_chunked(ctypes.byref(p), d, d, d, d, d, None, d, d, None,
                           None) == _lib.GDR_ERR_INVALID


def test_tensor_path_needs_its_shapes():
    """The tensor-core kernel serves bf16, d_k = d_v = 128, chunk 64 only;
    asking it for anything else is GDR_ERR_UNSUPPORTED, not a fallback."""
    lib = _lib.load()
    d = ctypes.c_void_p(16)
    p = _params(algo=_lib.GDR_ALGO_TENSOR)
    assert lib.gdr_chunked(ctypes.byref(p), d, d, d, d, d, None, d, d, None,
                           None) == _lib.GDR_ERR_UNSUPPORTED


def test_split_path_needs_its_shapes_and_a_valid_length():
    lib = _lib.load()
    d = ctypes.c_void_p(16)
    p = _params(algo=_lib.GDR_ALGO_TENSOR_SPLIT)
    assert lib.gdr_chunked(ctypes.byref(p), d, d, d, d, d, None, d, d, None,
                           None) == _lib.GDR_ERR_UNSUPPORTED
    p = _params(split_chunks=-1)
    assert lib.gdr_chunked(ctypes.byref(p), d, d, d, d, d, None, d, d, None,
                           None) == _lib.GDR_ERR_INVALID


def test_chunked_launch_counts():
    """gdr_chunked_launches reports the kernels a call runs, without running
    anything: one for a single-pass kernel, four for the split form (plan,
    pass A, scan, pass B), none for an empty batch, -1 for a rejected call."""
    lib = _lib.load()
    n = lambda p, packed=1: lib.gdr_chunked_launches(ctypes.byref(p), packed)  # noqa: E731
    tc = dict(d_k=128, d_v=128, chunk_size=64, dtype=_lib.GDR_DTYPE_BF16, n_seqs=64,
              seq_len=131072)
    assert n(_params(**tc, algo=_lib.GDR_ALGO_TENSOR)) == 1
    assert n(_params(**tc, algo=_lib.GDR_ALGO_TENSOR_SPLIT)) == 4
    assert n(_params(**tc, algo=_lib.GDR_ALGO_AUTO)) == 4  # a 131072-token pack may split
    assert n(_params(**dict(tc, seq_len=64, n_seqs=1), algo=_lib.GDR_ALGO_AUTO)) == 1
    assert n(_params(**dict(tc, n_seqs=0), algo=_lib.GDR_ALGO_AUTO)) == 0
    assert n(_params(**dict(tc, seq_len=0), algo=_lib.GDR_ALGO_AUTO)) == 1  # state passes through
    assert n(_params(), 0) == 1  # dense f32, d 8: the CUDA-core kernel
    assert n(_params(chunk_size=0)) == -1
    assert n(_params(algo=9)) == -1


def test_dtype_and_shape_routes():
    """f16 runs and the shapes the f32 chunked kernel does not take still
    have a kernel: f16 computes in f32 on the CUDA cores (bunsen widens half
    types to f32), a chunk above 64 or heads up to 256 run the recurrent
    kernel (the same rule); only the tensor-core algorithms refuse them, and
    heads above 256 have no kernel."""
    lib = _lib.load()
    n = lambda p, packed=1: lib.gdr_chunked_launches(ctypes.byref(p), packed)  # noqa: E731
    tc = dict(d_k=128, d_v=128, chunk_size=64, n_seqs=4, seq_len=256)
    f16 = dict(tc, dtype=_lib.GDR_DTYPE_F16)
    assert n(_params(**f16)) == 1
    assert n(_params(**f16, algo=_lib.GDR_ALGO_CUDA_CORE)) == 1
    assert n(_params(**f16, algo=_lib.GDR_ALGO_TENSOR)) == -1
    assert n(_params(**dict(tc, dtype=_lib.GDR_DTYPE_BF16, chunk_size=128))) == 1
    assert n(_params(**dict(tc, dtype=_lib.GDR_DTYPE_BF16, chunk_size=128),
                     algo=_lib.GDR_ALGO_TENSOR)) == -1
    assert n(_params(**dict(tc, d_k=192, d_v=256))) == 1
    assert n(_params(**dict(tc, d_k=192, d_v=256), algo=_lib.GDR_ALGO_CUDA_CORE)) == 1
    assert n(_params(**dict(tc, d_k=257))) == -1
    d = ctypes.c_void_p(16)
    # gdr_mixed is tensor-core only: an f16 batch is refused before any launch.
    p = _params(**dict(f16, n_seqs=1, seq_len=4))
    cu = ctypes.c_void_p(16)
    ws = ctypes.c_void_p(16)
    assert lib.gdr_mixed(ctypes.byref(p), d, d, d, d, d, d, None, 1, d, cu, ws, 1 << 20,
                         None) == _lib.GDR_ERR_UNSUPPORTED


def test_f64_entry_points_check_before_any_launch():
    """The f64 forms take only GDR_DTYPE_F64 (and the other entry points never
    take it), refuse a zero chunk like bunsen (delta_rule.rs:233) and heads
    above 256; all before any CUDA call."""
    lib = _lib.load()
    d = ctypes.c_void_p(16)
    args = lambda p: (ctypes.byref(p), d, d, d, d, d, None, d, d, None, None)  # noqa: E731
    f64 = dict(batch=2, seq_len=8, d_k=32, d_v=32, dtype=_lib.GDR_DTYPE_F64)
    for fn in (lib.gdr_recurrent_f64, lib.gdr_chunked_f64):
        assert fn(*args(_params(**dict(f64, dtype=_lib.GDR_DTYPE_F32)))) == _lib.GDR_ERR_INVALID
        assert fn(*args(_params(**dict(f64, d_v=257)))) == _lib.GDR_ERR_UNSUPPORTED
        assert fn(*args(_params(**dict(f64, heads_v=3)))) == _lib.GDR_ERR_INVALID
    assert lib.gdr_chunked_f64(*args(_params(**dict(f64, chunk_size=0)))) == _lib.GDR_ERR_INVALID
    for fn in (lib.gdr_recurrent, lib.gdr_chunked):
        assert fn(*args(_params(**f64))) == _lib.GDR_ERR_INVALID
    assert lib.gdr_chunked_launches(ctypes.byref(_params(**f64)), 0) == -1


def test_host_call_rejects_malformed_offsets_before_any_copy():
    """gdr_chunked_host reads cu_seqlens on the host: offsets that do not start
    at 0, decrease, or miss T_total are GDR_ERR_INVALID before any CUDA call."""
    lib = _lib.load()
    buf = (ctypes.c_uint8 * 4096)()
    d = ctypes.cast(buf, ctypes.c_void_p)
    for cu in ([0, 5, 3, 8], [1, 3, 5, 8], [0, 3, 5, 7]):
        arr = (ctypes.c_int32 * 4)(*cu)
        p = _params(n_seqs=3, seq_len=8, batch=0)
        assert lib.gdr_chunked_host(ctypes.byref(p), d, d, d, d, d, None, d, d,
                                    ctypes.cast(arr, ctypes.c_void_p), None) == _lib.GDR_ERR_INVALID


def test_layer_entry_points_reject_bad_arguments_before_any_launch():
    """The layer steps' entry points check shapes and options on the host and
    answer GDR_ERR_INVALID (or UNSUPPORTED) before touching the device."""
    lib = _lib.load()
    d = ctypes.c_void_p(16)
    conv = lambda **kw: lib.gdr_causal_conv1d(  # noqa: E731
        ctypes.byref(_lib.GdrConvParams(**dict(dict(batch=1, seq_len=4, channels=8, taps=4,
                                                     split0=8, split1=8, dtype=0), **kw))),
        d, d, None, d, d, d, None, None, None)
    assert conv(taps=1) == _lib.GDR_ERR_INVALID          # causal_conv.rs:47
    assert conv(taps=9) == _lib.GDR_ERR_UNSUPPORTED
    assert conv(split0=9, split1=9) == _lib.GDR_ERR_INVALID
    assert conv(split0=6, split1=4) == _lib.GDR_ERR_INVALID
    assert conv(dtype=5) == _lib.GDR_ERR_INVALID
    assert conv(channels=0) == _lib.GDR_ERR_INVALID
    norm = lib.gdr_gated_norm
    assert norm(4, 0, d, d, d, 1e-6, 0, d, None) == _lib.GDR_ERR_INVALID
    assert norm(4, 8, d, d, d, -1.0, 0, d, None) == _lib.GDR_ERR_INVALID
    assert norm(4, 8, d, d, d, 1e-6, 3, d, None) == _lib.GDR_ERR_INVALID
    assert norm(0, 8, None, None, None, 1e-6, 0, None, None) == _lib.GDR_OK  # nothing to do
    buf = (ctypes.c_uint8 * 256)()
    base = ctypes.cast(buf, ctypes.c_void_p).value
    reorder = lib.gdr_state_reorder
    assert reorder(base, base + 32, d, 4, 4, 16, None) == _lib.GDR_ERR_INVALID  # overlap
    assert reorder(base, base + 128, d, 4, 4, 6, None) == _lib.GDR_ERR_INVALID  # not words
    assert reorder(base, base + 128, d, 0, 4, 16, None) == _lib.GDR_OK         # no rows
    p = _params()
    io = _lib.GdrLayerIO(gate_a=16, gate_b=16, a_log=16, dt_bias=16, gate_dtype=0)
    assert lib.gdr_chunked_layer(ctypes.byref(p), d, d, d, d, None, ctypes.byref(io), None, d,
                                 d, None, None) == _lib.GDR_ERR_INVALID  # g given with gates
    io = _lib.GdrLayerIO(gate_a=16, gate_b=16, a_log=16, dt_bias=16, gate_dtype=7)
    assert lib.gdr_recurrent_layer(ctypes.byref(p), d, d, d, None, None, ctypes.byref(io), None,
                                   d, d, None, None) == _lib.GDR_ERR_INVALID
    io = _lib.GdrLayerIO(norm_z=16, norm_weight=16, norm_eps=-1.0)
    assert lib.gdr_chunked_layer(ctypes.byref(p), d, d, d, d, d, ctypes.byref(io), None, d, d,
                                 None, None) == _lib.GDR_ERR_INVALID
