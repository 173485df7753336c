"""ctypes loader for the CPU oracle (TEST INFRASTRUCTURE ONLY).

The oracle restates the reference's attention procs in C (attn_oracle.c); tests, the smoke
check and the benchmark's CPU-baseline leg call it as the checker.  The product library never
uses it.  Parity is unpinned: the reference (Nim) cannot be built on these machines and ships
no golden vectors for this path.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "liboracle.so")


def build() -> str:
    srcs = [os.path.join(HERE, f) for f in ("attn_oracle.c", "attn_ops_oracle.c", "attn_oracle.h",
                                            os.path.join("..", "include", "tl_host.h"))]
    if not os.path.exists(LIB) or os.path.getmtime(LIB) < max(os.path.getmtime(f) for f in srcs):
        subprocess.run(["make", "-s", "-C", HERE, "liboracle.so"], check=True)
    return LIB


def _load():
    build()
    lib = C.CDLL(LIB)
    P, I, F = C.c_void_p, C.c_int, C.c_float
    sig = {
        "ora_rope_single": [P, I, I, I, F, I],
        "ora_rope_at_pos": [P, I, I, I, F, I, I],
        "ora_store_kv_range": [P, P, I, I, P, P, I, I],
        "ora_attention_full_ctx": [P, P, P, I, I, I, I, P],
        "ora_linear_ggml_col": [P, P, I, I, I, P],
        "ora_attention_full": [P, P, P, P, I, I, I, I, I, P],
        "ora_attention_cached": [P, P, P, I, I, I, I, I, P],
        "ora_decode_step": [P, P, P, P, P, I, I, I, I, I, I, F, P],
        "ora_prefill_step": [P, P, P, P, P, I, I, I, I, I, I, F, P],
    }
    for name, args in sig.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = None
    lib.ora_rope_theta.argtypes = [I, I, F]
    lib.ora_rope_theta.restype = F
    lib.ora_attn_ops_create.argtypes = [I, I, I]
    lib.ora_attn_ops_create.restype = P
    lib.ora_attn_ops_destroy.argtypes = [P]
    lib.ora_attn_ops_destroy.restype = None
    return lib


_lib = None


def lib():
    global _lib
    if _lib is None:
        _lib = _load()
    return _lib


def _p(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data_as(C.c_void_p)


def rope_single(x: np.ndarray, nHead, headDim, ropeDim, base) -> np.ndarray:
    y = np.array(x, np.float32, copy=True, order="C")
    lib().ora_rope_single(_p(y), nHead, headDim, ropeDim, base, y.shape[1])
    return y


def rope_at_pos(x: np.ndarray, nHead, headDim, ropeDim, base, pos) -> np.ndarray:
    y = np.array(x, np.float32, copy=True, order="C")
    lib().ora_rope_at_pos(_p(y), nHead, headDim, ropeDim, base, pos, y.shape[1])
    return y


def store_kv_range(kc: np.ndarray, vc: np.ndarray, startPos, k: np.ndarray, v: np.ndarray):
    k = np.ascontiguousarray(k, np.float32)
    v = np.ascontiguousarray(v, np.float32)
    lib().ora_store_kv_range(_p(kc), _p(vc), kc.shape[1], startPos, _p(k), _p(v), k.shape[0], k.shape[1])


def attention_full_ctx(q, k, v, nHead, nHeadKv, headDim) -> np.ndarray:
    q, k, v = (np.ascontiguousarray(a, np.float32) for a in (q, k, v))
    ctx = np.empty((nHead * headDim, q.shape[1]), np.float32)
    lib().ora_attention_full_ctx(_p(q), _p(k), _p(v), q.shape[1], nHead, nHeadKv, headDim, _p(ctx))
    return ctx


def linear_ggml_col(x, w) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    in_dim, out_dim = w.shape
    out = np.empty((out_dim, x.shape[1]), np.float32)
    lib().ora_linear_ggml_col(_p(x), _p(w), in_dim, out_dim, x.shape[1], _p(out))
    return out


def attention_cached(q, kc, vc, curLen, nHead, nHeadKv, headDim) -> np.ndarray:
    q = np.ascontiguousarray(q, np.float32)
    kc = np.ascontiguousarray(kc, np.float32)
    vc = np.ascontiguousarray(vc, np.float32)
    ctx = np.empty((nHead * headDim, 1), np.float32)
    lib().ora_attention_cached(_p(q), _p(kc), _p(vc), kc.shape[1], curLen, nHead, nHeadKv, headDim, _p(ctx))
    return ctx


def rope_theta(i, ropeDim, base) -> float:
    return lib().ora_rope_theta(i, ropeDim, base)


def decode_step(q, k, v, kc, vc, pos, nHead, nHeadKv, headDim, ropeDim, base) -> np.ndarray:
    """src/forward.nim:314-317 for one sequence: RoPE q,k at pos, store at pos, attend pos+1.
    q and k are copied; kc, vc ([nHeadKv*headDim, cacheCols]) are written in place."""
    q = np.array(q, np.float32, copy=True, order="C")
    k = np.array(k, np.float32, copy=True, order="C")
    v = np.ascontiguousarray(v, np.float32)
    ctx = np.empty((nHead * headDim, 1), np.float32)
    lib().ora_decode_step(_p(q), _p(k), _p(v), _p(kc), _p(vc), kc.shape[1], pos, nHead, nHeadKv,
                          headDim, ropeDim, base, _p(ctx))
    return ctx
