"""ctypes front end of the CPU oracle -- TEST INFRASTRUCTURE ONLY.

Loads ``oracle/libgdr_oracle.so`` (``make -C oracle``), the C++ restatement of
bunsen's ``GatedDeltaRule`` (``crates/public/bunsen/src/ops/transformers/
linear_attention/delta_rule.rs``), and runs it on numpy arrays. Only the tests,
the smoke check and the benchmark's CPU-baseline leg import this module; the
product package never does.

Argument order and meaning follow the Rust operator (``delta_rule.rs:182-190``):
``q, k, v, g, beta, state`` with

* dense inputs ``q, k [B, T, H_qk, d_k]``, ``v [B, T, H_v, d_v]``,
  ``g, beta [B, T, H_v]``, ``state [B, H_v, d_k, d_v]`` or ``None``; or
* packed inputs ``[T_total, H, .]`` with ``cu_seqlens`` (``n_seqs + 1`` int32
  offsets) and ``state [n_seqs, H_v, d_k, d_v]``.

``H_qk`` may divide ``H_v``: value head ``h`` reads key head ``h // (H_v //
H_qk)``, which is what ``repeat_interleave`` before bunsen's rule produces
(``ops/repeat.rs:51-66``, ``gated_delta_net.rs:404-419``). ``l2norm_eps=None``
is bunsen's ``qk_l2norm_eps: None``.
"""

from __future__ import annotations

import ctypes
import pathlib
import subprocess

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
LIB = HERE / "libgdr_oracle.so"


class _Batch(ctypes.Structure):
    _fields_ = [
        ("n_seqs", ctypes.c_int32),
        ("cu_seqlens", ctypes.POINTER(ctypes.c_int32)),
        ("heads_qk", ctypes.c_int32),
        ("heads_v", ctypes.c_int32),
        ("d_k", ctypes.c_int32),
        ("d_v", ctypes.c_int32),
        ("chunk_size", ctypes.c_int32),
        ("l2norm_eps", ctypes.c_double),
        ("threads", ctypes.c_int32),
    ]


_lib = None


def build() -> None:
    """Compile the oracle library (a no-op when it is up to date)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB.exists():
            build()
        _lib = ctypes.CDLL(str(LIB))
        for name in ("gdr_oracle_recurrent", "gdr_oracle_chunked", "gdr_oracle_scalar_f64"):
            getattr(_lib, name).restype = ctypes.c_int
        _lib.gdr_oracle_max_threads.restype = ctypes.c_int
    return _lib


def max_threads() -> int:
    return int(lib().gdr_oracle_max_threads())


def _pack(q, k, v, g, beta, state, cu_seqlens):
    """Dense [B, T, ...] inputs as the packed [B*T, ...] form with offsets."""
    if cu_seqlens is None:
        b, t = q.shape[:2]
        cu = np.arange(b + 1, dtype=np.int32) * t
        flat = [x.reshape((b * t,) + x.shape[2:]) for x in (q, k, v, g, beta)]
        return flat, cu, (b, t)
    return [q, k, v, g, beta], np.ascontiguousarray(cu_seqlens, dtype=np.int32), None


def _run(fn: str, dtype, q, k, v, g, beta, state, l2norm_eps, chunk_size, cu_seqlens, threads,
         out=None, state_out=None):
    (q, k, v, g, beta), cu, dense = _pack(q, k, v, g, beta, state, cu_seqlens)
    q, k, v, g, beta = (np.ascontiguousarray(x, dtype=dtype) for x in (q, k, v, g, beta))
    t_total, h_qk, d_k = q.shape
    h_v, d_v = v.shape[1:]
    n = len(cu) - 1
    assert k.shape == q.shape and v.shape[0] == t_total and g.shape == beta.shape == (t_total, h_v)
    assert int(cu[-1]) == t_total
    # Output buffers may be the caller's (reused between timed runs, so that
    # first-touch page faults of fresh buffers are not timed).
    if out is None:
        out = np.zeros((t_total, h_v, d_v), dtype=dtype)
    if state_out is None:
        state_out = np.zeros((n, h_v, d_k, d_v), dtype=dtype)
    assert out.shape == (t_total, h_v, d_v) and out.dtype == dtype and out.flags.c_contiguous
    assert state_out.shape == (n, h_v, d_k, d_v) and state_out.dtype == dtype
    assert state_out.flags.c_contiguous
    st_out = state_out
    st_in = None
    if state is not None:
        st_in = np.ascontiguousarray(state, dtype=dtype).reshape(n, h_v, d_k, d_v)
    batch = _Batch(
        n, cu.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), h_qk, h_v, d_k, d_v,
        int(chunk_size), -1.0 if l2norm_eps is None else float(l2norm_eps), int(threads))
    ptr = lambda x: None if x is None else x.ctypes.data_as(ctypes.c_void_p)  # noqa: E731
    rc = getattr(lib(), fn)(ctypes.byref(batch), ptr(q), ptr(k), ptr(v), ptr(g), ptr(beta),
                            ptr(st_in), ptr(out), ptr(st_out))
    if rc != 0:
        raise ValueError(f"{fn}: invalid arguments (status {rc})")
    if dense is not None:
        out = out.reshape(dense + out.shape[1:])
    return out, st_out


def recurrent(q, k, v, g, beta, state=None, *, l2norm_eps=1e-6, cu_seqlens=None, threads=0,
              out=None, state_out=None):
    """``GatedDeltaRule::recurrent`` in f32 (``delta_rule.rs:182-209``);
    ``out`` / ``state_out``: packed f32 buffers to write into."""
    return _run("gdr_oracle_recurrent", np.float32, q, k, v, g, beta, state, l2norm_eps, 1,
                cu_seqlens, threads, out, state_out)


def chunked(q, k, v, g, beta, state=None, *, chunk_size=64, l2norm_eps=1e-6, cu_seqlens=None,
            threads=0, out=None, state_out=None):
    """``GatedDeltaRule::chunked`` in f32 (``delta_rule.rs:223-310``);
    ``out`` / ``state_out``: packed f32 buffers to write into."""
    if chunk_size <= 0:
        raise ValueError("a chunk of at least one position")
    return _run("gdr_oracle_chunked", np.float32, q, k, v, g, beta, state, l2norm_eps,
                chunk_size, cu_seqlens, threads, out, state_out)


def scalar_f64(q, k, v, g, beta, state=None, *, l2norm_eps=1e-6, cu_seqlens=None, threads=0):
    """The scalar rule in f64 that bunsen's tests hold the recurrent form to
    (``delta_rule.rs:399-445``)."""
    return _run("gdr_oracle_scalar_f64", np.float64, q, k, v, g, beta, state, l2norm_eps, 1,
                cu_seqlens, threads)

