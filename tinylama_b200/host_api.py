"""ctypes binding of libtlhost.so (include/tl_host.h): tinylama's host forward pass with the
attention procs behind a table, filled here with the B200 path (libtlattn.so)."""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libtlhost.so")
if not os.path.exists(LIB_PATH):
    raise ImportError(f"{LIB_PATH} is not built; run `python -m tinylama_b200.build`")

_P, _I, _L, _F = C.c_void_p, C.c_int, C.c_long, C.c_float


class HParams(C.Structure):
    _fields_ = [("nVocab", _I), ("nCtx", _I), ("nEmb", _I), ("nLayer", _I), ("nFfn", _I),
                ("nHead", _I), ("nHeadKv", _I), ("ropeDim", _I), ("ropeFreqBase", _F), ("rmsEps", _F)]


lib = C.CDLL(LIB_PATH)
lib.tlh_model_load.restype = _P
lib.tlh_model_load.argtypes = [C.c_char_p, _I, C.c_char_p, _I]
lib.tlh_model_open.restype = _P
lib.tlh_model_open.argtypes = [C.c_char_p, C.c_char_p, _I]
lib.tlh_model_free.argtypes = [_P]
lib.tlh_model_free.restype = None
lib.tlh_model_hparams.argtypes = [_P, C.POINTER(HParams)]
lib.tlh_model_hparams.restype = _I
lib.tlh_model_tensor.argtypes = [_P, C.c_char_p, _P, _L, C.POINTER(_L)]
lib.tlh_model_tensor.restype = _I
lib.tlh_generate.argtypes = [_P, _P, _P, _I, _I, _P, _P, _P, _L]
lib.tlh_generate.restype = _L
lib.tlh_session_init.argtypes = [_P, _I]
lib.tlh_session_init.restype = _I
lib.tlh_run_prompt.argtypes = [_P, _P, _P, _I, _I, _I, _P, _P, _P, _L]
lib.tlh_run_prompt.restype = _L
lib.tlh_model_to_gpu.argtypes = [_P, _P]
lib.tlh_model_to_gpu.restype = _I
lib.tlh_gpu_attn_ops_create.argtypes = [_I, _I, _I, _I, _I, _F, _I]
lib.tlh_gpu_attn_ops_create.restype = _P
lib.tlh_gpu_attn_ops_destroy.argtypes = [_P]
lib.tlh_gpu_attn_ops_destroy.restype = None
lib.tlh_last_error.restype = C.c_char_p


class Model:
    """loadModel (src/model.nim:105-114) with every tensor dequantised up front, or with
    mapped=True the file mapped without a float32 copy (for to_gpu only)."""

    def __init__(self, path: str, nthreads: int = 1, mapped: bool = False):
        err = C.create_string_buffer(512)
        if mapped:
            self.h = lib.tlh_model_open(path.encode(), err, 512)
        else:
            self.h = lib.tlh_model_load(path.encode(), nthreads, err, 512)
        if not self.h:
            raise ValueError(err.value.decode())
        self.hp = HParams()
        lib.tlh_model_hparams(self.h, C.byref(self.hp))

    def tensor(self, name: str) -> np.ndarray:
        n = C.c_long()
        if lib.tlh_model_tensor(self.h, name.encode(), None, 0, C.byref(n)) != 0:
            raise KeyError(name)
        out = np.empty(n.value, np.float32)
        lib.tlh_model_tensor(self.h, name.encode(), out.ctypes.data_as(C.c_void_p), n.value, C.byref(n))
        return out

    def generate(self, ops, prompt, n_new: int, dump: bool = True):
        """runPrompt (src/tinylama.nim:49-69): greedy ids, top-2 logit gaps and (optionally) every
        attention output in call order."""
        hp = self.hp
        prompt = np.ascontiguousarray(prompt, np.int32)
        ids = np.zeros(n_new, np.int32)
        gaps = np.zeros(n_new, np.float32)
        hd = hp.nEmb // hp.nHead
        cap = hp.nLayer * hp.nHead * hd * (len(prompt) + n_new) if dump else 0
        buf = np.zeros(max(cap, 1), np.float32)
        n = lib.tlh_generate(self.h, ops, prompt.ctypes.data_as(C.c_void_p), len(prompt), n_new,
                             ids.ctypes.data_as(C.c_void_p), gaps.ctypes.data_as(C.c_void_p),
                             buf.ctypes.data_as(C.c_void_p) if dump else None, cap)
        if n < 0:
            raise RuntimeError(lib.tlh_last_error().decode())
        return ids, gaps, buf[:n] if dump else None

    @staticmethod
    def session_init(ops, n_new: int) -> None:
        """initKvCache(max(32, nNew + 32)) of the REPL (src/tinylama.nim:47): the cache that
        the following run_prompt calls share."""
        if lib.tlh_session_init(ops, n_new) != 0:
            raise RuntimeError(lib.tlh_last_error().decode())

    def run_prompt(self, ops, prompt, n_new: int, chunked: bool = False, dump: bool = True):
        """runPrompt (src/tinylama.nim:49-86) for one REPL line on the session's cache: the
        first line is prefilled, a later one is fed through forwardDecode token by token, or
        with chunked=True in one pass at positions curLen.. (tables with prefill_at).  Returns
        greedy ids, top-2 gaps and the attention outputs in call order."""
        hp = self.hp
        prompt = np.ascontiguousarray(prompt, np.int32)
        ids = np.zeros(n_new, np.int32)
        gaps = np.zeros(n_new, np.float32)
        hd = hp.nEmb // hp.nHead
        cap = hp.nLayer * hp.nHead * hd * (len(prompt) + n_new) if dump else 0
        buf = np.zeros(max(cap, 1), np.float32)
        n = lib.tlh_run_prompt(self.h, ops, prompt.ctypes.data_as(C.c_void_p), len(prompt), n_new,
                               1 if chunked else 0, ids.ctypes.data_as(C.c_void_p),
                               gaps.ctypes.data_as(C.c_void_p),
                               buf.ctypes.data_as(C.c_void_p) if dump else None, cap)
        if n < 0:
            msg = lib.tlh_last_error().decode()
            raise (ValueError if "KV cache full" in msg else RuntimeError)(msg)
        return ids, gaps, buf[:n] if dump else None

    def to_gpu(self, max_len: int, device: int = 0) -> "GpuModel":
        """The whole forward pass on the B200 (include/tl_model.h) with this model's weights:
        Q2_K tensors as stored in the file, the others as loaded float32."""
        return GpuModel(self, max_len, device)

    def close(self):
        if self.h:
            lib.tlh_model_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def gpu_attn_ops(hp: HParams, device: int = 0):
    """The reference's attention procs on the B200 (libtlattn.so), as a tlh_attn_ops table."""
    hd = hp.nEmb // hp.nHead
    return lib.tlh_gpu_attn_ops_create(hp.nLayer, hp.nHead, hp.nHeadKv, hd, hp.ropeDim or hd,
                                       hp.ropeFreqBase, device)


def free_gpu_attn_ops(ops) -> None:
    lib.tlh_gpu_attn_ops_destroy(ops)


class TlModelConfig(C.Structure):
    _fields_ = [("nVocab", _I), ("nEmb", _I), ("nLayer", _I), ("nFfn", _I), ("nHead", _I), ("nHeadKv", _I),
                ("ropeDim", _I), ("ropeFreqBase", _F), ("rmsEps", _F), ("maxLen", _I)]


class GpuModel:
    """tl_model (include/tl_model.h): weights resident on the GPU, a greedy generation with one
    CUDA graph replay per decode step."""

    def __init__(self, model: Model, max_len: int, device: int = 0):
        from tinylama_b200 import _lib
        self._l = _lib
        hp = model.hp
        cfg = TlModelConfig(hp.nVocab, hp.nEmb, hp.nLayer, hp.nFfn, hp.nHead, hp.nHeadKv, hp.ropeDim,
                            hp.ropeFreqBase, hp.rmsEps, max_len)
        self.hp = hp
        self.h = C.c_void_p()
        _lib.check(_lib.lib.tl_model_create(C.byref(self.h), C.byref(cfg), device))
        if lib.tlh_model_to_gpu(model.h, self.h) != 0:
            msg = lib.tlh_last_error().decode()
            self.close()
            raise RuntimeError(msg)

    def generate(self, prompt, n_new: int):
        """runPrompt on the device: greedy ids and top-2 logit gaps."""
        prompt = np.ascontiguousarray(prompt, np.int32)
        ids = np.zeros(n_new, np.int32)
        gaps = np.zeros(n_new, np.float32)
        self._l.check(self._l.lib.tl_model_generate(self.h, prompt.ctypes.data_as(C.c_void_p), len(prompt), n_new,
                                                    ids.ctypes.data_as(C.c_void_p), gaps.ctypes.data_as(C.c_void_p)))
        return ids, gaps

    def last_logits(self) -> np.ndarray:
        out = np.empty(self.hp.nVocab, np.float32)
        self._l.check(self._l.lib.tl_model_last_logits(self.h, out.ctypes.data_as(C.c_void_p)))
        return out

    def last_timing(self) -> tuple[float, float]:
        a, b = C.c_float(), C.c_float()
        self._l.check(self._l.lib.tl_model_last_timing(self.h, C.byref(a), C.byref(b)))
        return a.value, b.value

    def close(self):
        if self.h:
            self._l.lib.tl_model_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
