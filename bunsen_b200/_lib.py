"""ctypes binding of ``libgdr.so`` (the C ABI of ``include/gdr.h``).

The library is built in-tree by ``python -m bunsen_b200.build``. Loading never
falls back to anything: a missing or unloadable library raises.
"""

from __future__ import annotations

import ctypes
import pathlib

PKG = pathlib.Path(__file__).resolve().parent
LIB_PATH = PKG / "libgdr.so"

GDR_OK, GDR_ERR_INVALID, GDR_ERR_UNSUPPORTED, GDR_ERR_CUDA, GDR_ERR_TIMEOUT = range(5)
GDR_ERR_CAPACITY = 5
GDR_MIXED_NOALLOC_MAX_SEQS = 16384
GDR_DTYPE_F32, GDR_DTYPE_BF16, GDR_DTYPE_F16, GDR_DTYPE_F64 = 0, 1, 2, 3
ABI_VERSION = 3  # GDR_ABI_VERSION of include/gdr.h these bindings follow
GDR_ALGO_AUTO, GDR_ALGO_CUDA_CORE, GDR_ALGO_TENSOR, GDR_ALGO_TENSOR_SPLIT = 0, 1, 2, 3

# Every function include/gdr.h declares, with its ctypes signature.
_vp, _i32, _sz = ctypes.c_void_p, ctypes.c_int32, ctypes.c_size_t


class GdrParams(ctypes.Structure):
    """``struct gdr_params`` of include/gdr.h."""

    _fields_ = [
        ("batch", ctypes.c_int32),
        ("seq_len", ctypes.c_int32),
        ("n_seqs", ctypes.c_int32),
        ("heads_qk", ctypes.c_int32),
        ("heads_v", ctypes.c_int32),
        ("d_k", ctypes.c_int32),
        ("d_v", ctypes.c_int32),
        ("chunk_size", ctypes.c_int32),
        ("use_l2norm", ctypes.c_int32),
        ("l2norm_eps", ctypes.c_double),
        ("dtype", ctypes.c_int32),
        ("algo", ctypes.c_int32),
        ("split_chunks", ctypes.c_int32),
    ]


class GdrConvParams(ctypes.Structure):
    """``struct gdr_conv_params`` of include/gdr.h."""

    _fields_ = [(name, ctypes.c_int32) for name in (
        "batch", "seq_len", "n_seqs", "channels", "taps", "split0", "split1", "silu", "dtype")]


class GdrLayerIO(ctypes.Structure):
    """``struct gdr_layer_io`` of include/gdr.h."""

    _fields_ = [
        ("gate_a", ctypes.c_void_p),
        ("gate_b", ctypes.c_void_p),
        ("a_log", ctypes.c_void_p),
        ("dt_bias", ctypes.c_void_p),
        ("gate_dtype", ctypes.c_int32),
        ("norm_z", ctypes.c_void_p),
        ("norm_weight", ctypes.c_void_p),
        ("norm_eps", ctypes.c_double),
    ]


_RULE_ARGS = [ctypes.POINTER(GdrParams), _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp]
_LAYER_ARGS = [ctypes.POINTER(GdrParams), _vp, _vp, _vp, _vp, _vp, ctypes.POINTER(GdrLayerIO),
               _vp, _vp, _vp, _vp, _vp]
SIGNATURES = {
    "gdr_recurrent": (_i32, _RULE_ARGS),
    "gdr_chunked": (_i32, _RULE_ARGS),
    "gdr_recurrent_f64": (_i32, _RULE_ARGS),
    "gdr_chunked_f64": (_i32, _RULE_ARGS),
    "gdr_chunked_launches": (_i32, [ctypes.POINTER(GdrParams), _i32]),
    "gdr_chunked_host": (_i32, _RULE_ARGS),
    "gdr_chunked_layer": (_i32, _LAYER_ARGS),
    "gdr_recurrent_layer": (_i32, _LAYER_ARGS),
    "gdr_mixed_layer": (_i32, [ctypes.POINTER(GdrParams), _vp, _vp, _vp, _vp, _vp,
                               ctypes.POINTER(GdrLayerIO), _vp, _vp, _i32, _vp, _vp, _vp, _sz,
                               _vp]),
    "gdr_causal_conv1d": (_i32, [ctypes.POINTER(GdrConvParams), _vp, _vp, _vp, _vp, _vp, _vp,
                                 _vp, _vp, _vp]),
    "gdr_state_reorder": (_i32, [_vp, _vp, _vp, _i32, _i32, _sz, _vp]),
    "gdr_gated_norm": (_i32, [ctypes.c_int64, _i32, _vp, _vp, _vp, ctypes.c_double, _i32, _vp,
                              _vp]),
    "gdr_mixed_workspace_size": (_sz, [ctypes.POINTER(GdrParams)]),
    "gdr_mixed": (_i32, [ctypes.POINTER(GdrParams), _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i32,
                         _vp, _vp, _vp, _sz, _vp]),
    "gdr_mixed_noalloc": (_i32, [ctypes.POINTER(GdrParams), _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                                 _i32, _vp, _vp, _vp]),
    "gdr_selftest_wait_timeout": (_i32, [ctypes.c_int64, _vp]),
    "gdr_release_scratch": (_i32, []),
    "gdr_device_error": (_i32, []),
    "gdr_status_string": (ctypes.c_char_p, [_i32]),
    "gdr_abi_version": (_i32, []),
}

_lib: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    """The loaded library, with its signatures declared."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH} is not built; run `python -m bunsen_b200.build` (needs nvcc)")
        lib = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


class GdrError(RuntimeError):
    """A non-OK status from libgdr."""

    def __init__(self, fn: str, status: int):
        msg = load().gdr_status_string(status).decode()
        super().__init__(f"{fn}: {msg} (status {status})")
        self.status = status


def check(fn: str, status: int) -> None:
    if status != GDR_OK:
        if status == GDR_ERR_INVALID:
            raise ValueError(f"{fn}: {load().gdr_status_string(status).decode()}")
        raise GdrError(fn, status)
