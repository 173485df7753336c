"""Python mirror of tinylama's attention procs (src/forward.nim), running on libtlattn.so.

Same names, argument meaning and error behaviour as the Nim procs they replace, so that a test
reads like the reference's forward pass:

    cache = initKvCache(hp, maxLen)                       # forward.nim:94
    applyRopeSingle(q, hp.nHead, headDim, ropeDim, base)  # forward.nim:108
    storeKVRange(cache, layer, 0, k, v)                   # forward.nim:232
    out = attentionFull(q, k, v, wo, nHead, nHeadKv, headDim)   # forward.nim:141
    ctx = attentionCached(q, cache, layer, curLen, nHead, nHeadKv, headDim)  # forward.nim:179

Tensors are float32 numpy arrays in the reference's ggml column layout [rows, cols]
(src/tensor.nim:11-26).  Every computation runs in the CUDA library; the only host math here is
the wo projection of attentionFull (linearGGMLCol, forward.nim:177), which belongs to the
caller's linear layers and is outside the attention path.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from . import _lib
from ._lib import check, lib


def _fp(a: np.ndarray):
    return a.ctypes.data_as(C.c_void_p)


def _f32(a, writable: bool = False) -> np.ndarray:
    arr = np.ascontiguousarray(a, dtype=np.float32)
    if writable and arr is not a:
        raise ValueError("in-place argument must be a contiguous float32 array")
    return arr


@dataclass
class HParams:
    """The HParams fields the attention path reads (src/model.nim:18-29)."""
    nEmb: int
    nHead: int
    nHeadKv: int
    nLayer: int
    ropeDim: int = 0
    ropeFreqBase: float = 10000.0
    arch: str = "llama"


class KvCache:
    """KvCache (src/forward.nim:85-92) backed by the library's device cache.

    ``curLen``, ``maxLen``, ``nHeadKv`` and ``headDim`` are the reference's public fields.
    ``k[layer]`` / ``v[layer]`` return host copies in the reference layout
    [nHeadKv*headDim, maxLen] (the bench's cloneCache reads them, bench_tinylama.nim:18-32).
    """

    def __init__(self, hp: HParams, maxLen: int, kv_dtype: int = _lib.TL_KV_F32,
                 max_batch: int = 1, device: int = 0):
        if hp.nHead <= 0:
            raise ValueError("KV cache requires llama-style head_count")
        self.hp = hp
        self.maxLen = maxLen
        self.nHeadKv = hp.nHeadKv
        self.headDim = hp.nEmb // hp.nHead
        self.nLayer = hp.nLayer
        self.ropeDim = hp.ropeDim if hp.ropeDim > 0 else self.headDim
        self.kv_dtype = kv_dtype
        self.max_batch = max_batch
        h = C.c_void_p()
        check(lib.tl_attn_create(C.byref(h), hp.nLayer, hp.nHead, hp.nHeadKv, self.headDim,
                                 self.ropeDim, float(hp.ropeFreqBase), maxLen, max_batch,
                                 kv_dtype, device))
        self.handle = h
        self.k = _LayerView(self, 0)
        self.v = _LayerView(self, 1)

    # curLen of slot 0 (the reference cache holds one sequence)
    @property
    def curLen(self) -> int:
        return self.get_len(0)

    @curLen.setter
    def curLen(self, value: int) -> None:
        self.set_len(0, value)

    def get_len(self, slot: int) -> int:
        n = C.c_int()
        check(lib.tl_kv_get_len(self.handle, slot, C.byref(n)))
        return n.value

    def set_len(self, slot: int, value: int) -> None:
        check(lib.tl_kv_set_len(self.handle, slot, int(value)))

    def read(self, layer: int, slot: int = 0) -> tuple[np.ndarray, np.ndarray]:
        kvDim = self.nHeadKv * self.headDim
        k = np.empty((kvDim, self.maxLen), np.float32)
        v = np.empty((kvDim, self.maxLen), np.float32)
        check(lib.tl_kv_read(self.handle, layer, slot, _fp(k), _fp(v)))
        return k, v

    def reset(self) -> None:
        check(lib.tl_kv_reset(self.handle))

    def close(self) -> None:
        if self.handle:
            lib.tl_attn_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class _LayerView:
    def __init__(self, cache: KvCache, which: int):
        self.cache, self.which = cache, which

    def __getitem__(self, layer: int) -> np.ndarray:
        return self.cache.read(layer)[self.which]

    def __len__(self) -> int:
        return self.cache.nLayer


def initKvCache(hp: HParams, maxLen: int, **kw) -> KvCache:
    """initKvCache (src/forward.nim:94-106)."""
    return KvCache(hp, maxLen, **kw)


def cloneCache(src: KvCache) -> KvCache:
    """cloneCache (bench/bench_tinylama.nim:18-32): deep copy of contents and lengths."""
    dst = KvCache(src.hp, src.maxLen, kv_dtype=src.kv_dtype, max_batch=src.max_batch)
    check(lib.tl_kv_clone(dst.handle, src.handle))
    return dst


def _any_handle(cache: KvCache | None) -> C.c_void_p:
    if cache is not None:
        return cache.handle
    return _scratch_handle()


_SCRATCH = {}


def _scratch_handle() -> C.c_void_p:
    """A minimal handle used for calls that need a device and a stream but no cache."""
    h = _SCRATCH.get("h")
    if h is None:
        h = C.c_void_p()
        check(lib.tl_attn_create(C.byref(h), 1, 1, 1, 64, 64, 10000.0, 32, 1, 0, 0))
        _SCRATCH["h"] = h
    return h


def applyRopeSingle(x: np.ndarray, nHead: int, headDim: int, ropeDim: int, base: float,
                    cache: KvCache | None = None) -> None:
    """applyRopeSingle (src/forward.nim:108-123): in place on x = [nHead*headDim, seqLen]."""
    _f32(x, writable=True)
    check(lib.tl_rope_single_host(_any_handle(cache), _fp(x), nHead, headDim, ropeDim,
                                  float(base), x.shape[1]))


def applyRopeAtPos(x: np.ndarray, nHead: int, headDim: int, ropeDim: int, base: float, pos: int,
                   cache: KvCache | None = None) -> None:
    """applyRopeAtPos (src/forward.nim:125-139): rotates column 0 of x at position pos."""
    _f32(x, writable=True)
    check(lib.tl_rope_at_pos_host(_any_handle(cache), _fp(x), nHead, headDim, ropeDim,
                                  float(base), int(pos), x.shape[1]))


def storeKVRange(cache: KvCache, layer: int, startPos: int, k: np.ndarray, v: np.ndarray,
                 slot: int = 0) -> None:
    """storeKVRange (src/forward.nim:232-241)."""
    k = _f32(k)
    v = _f32(v)
    if k.shape != v.shape or k.shape[0] != cache.nHeadKv * cache.headDim:
        raise ValueError("storeKVRange: k/v shape mismatch")
    check(lib.tl_kv_store_host(cache.handle, layer, slot, int(startPos), _fp(k), _fp(v),
                               k.shape[1]))


def attentionFullCtx(q: np.ndarray, k: np.ndarray, v: np.ndarray, nHead: int, nHeadKv: int,
                     headDim: int, cache: KvCache | None = None) -> np.ndarray:
    """The attention part of attentionFull (src/forward.nim:141-176), ctx = [nHead*headDim, S]."""
    q, k, v = _f32(q), _f32(k), _f32(v)
    S = q.shape[1]
    ctx = np.empty((nHead * headDim, S), np.float32)
    check(lib.tl_attention_full_host(_any_handle(cache), _fp(q), _fp(k), _fp(v), S, nHead,
                                     nHeadKv, headDim, _fp(ctx)))
    return ctx


def linearGGMLCol(x: np.ndarray, w: np.ndarray) -> np.ndarray:
    """linearGGMLCol (src/forward.nim:40-83): the caller's wo projection, outside the path.
    w has shape [in, out] and is laid out row-major as rows=out, cols=in."""
    in_dim, out_dim = w.shape
    wmat = np.asarray(w, np.float32).reshape(out_dim, in_dim)
    return (wmat @ np.asarray(x, np.float32)).astype(np.float32)


def attentionFull(q, k, v, wo, nHead: int, nHeadKv: int, headDim: int,
                  cache: KvCache | None = None) -> np.ndarray:
    """attentionFull (src/forward.nim:141-177): GPU attention, then the caller's wo."""
    return linearGGMLCol(attentionFullCtx(q, k, v, nHead, nHeadKv, headDim, cache), wo)


def attentionCached(q: np.ndarray, cache: KvCache, layer: int, curLen: int, nHead: int,
                    nHeadKv: int, headDim: int, slot: int = 0) -> np.ndarray:
    """attentionCached (src/forward.nim:179-211) over cache.k[layer], cache.v[layer]."""
    q = _f32(q)
    ctx = np.empty((nHead * headDim, 1), np.float32)
    check(lib.tl_attention_cached_host(cache.handle, layer, slot, _fp(q), int(curLen), nHead,
                                       nHeadKv, headDim, _fp(ctx)))
    return ctx


def decodeLayer(cache: KvCache, layer: int, q: np.ndarray, k: np.ndarray, v: np.ndarray,
                pos: int, slot: int = 0) -> np.ndarray:
    """The attention block of forwardDecode (src/forward.nim:314-317) in one call."""
    q, k, v = _f32(q), _f32(k), _f32(v)
    ctx = np.empty((cache.hp.nHead * cache.headDim, 1), np.float32)
    check(lib.tl_decode_layer_host(cache.handle, layer, slot, _fp(q), _fp(k), _fp(v), int(pos),
                                   _fp(ctx)))
    return ctx


def prefillLayer(cache: KvCache, layer: int, q: np.ndarray, k: np.ndarray, v: np.ndarray,
                 slot: int = 0) -> np.ndarray:
    """The attention block of forwardPrefill (src/forward.nim:271-274) in one call."""
    q, k, v = _f32(q), _f32(k), _f32(v)
    S = q.shape[1]
    ctx = np.empty((cache.hp.nHead * cache.headDim, S), np.float32)
    check(lib.tl_prefill_layer_host(cache.handle, layer, slot, _fp(q), _fp(k), _fp(v), S,
                                    _fp(ctx)))
    return ctx


def prefillLayerAt(cache: KvCache, layer: int, startPos: int, q: np.ndarray, k: np.ndarray,
                   v: np.ndarray, slot: int = 0) -> np.ndarray:
    """The attention blocks of S successive forwardDecode steps from pos = startPos
    (src/forward.nim:314-317 for pos = startPos .. startPos+S-1: the reference's multi-turn
    path feeds a later prompt this way, src/tinylama.nim:70-73) in one call: q, k, v are
    [.., S] columns, token t is rotated at startPos + t, stored there, and attends positions
    0..startPos+t.  The caller advances curLen to startPos + S."""
    q, k, v = _f32(q), _f32(k), _f32(v)
    S = q.shape[1]
    ctx = np.empty((cache.hp.nHead * cache.headDim, S), np.float32)
    check(lib.tl_prefill_layer_at_host(cache.handle, layer, slot, int(startPos), _fp(q), _fp(k), _fp(v),
                                       S, _fp(ctx)))
    return ctx


def forwardDecodeCheck(cache: KvCache) -> None:
    """The guard at the top of forwardDecode (src/forward.nim:290-291)."""
    if cache.curLen >= cache.maxLen:
        raise ValueError("KV cache full")
