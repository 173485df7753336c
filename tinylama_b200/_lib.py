"""ctypes binding of libtlattn.so (the C ABI in include/tl_attn.h).

This is the same binding a Nim host writes with {.importc, dynlib.}: plain pointers, sizes
and int status codes.  The library must have been built (``python -m tinylama_b200.build``);
there is no fallback implementation, so a missing library is an ImportError.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libtlattn.so")

TL_KV_F32 = 0
TL_KV_BF16 = 1

TL_OK = 0
TL_ERR_INVALID = -1
TL_ERR_CUDA = -2
TL_ERR_KV_FULL = -3
TL_ERR_RANGE = -4
TL_ERR_DEVICE = -5
TL_ERR_NCCL = -6
TL_ERR_NOMEM = -7
TL_ERR_UNSUPPORTED = -8

_P = C.c_void_p
_I = C.c_int
_F = C.c_float
_FP = C.POINTER(C.c_float)
_IP = C.POINTER(C.c_int)

# name -> (restype, argtypes); must match include/tl_attn.h
SIGNATURES = {
    "tl_last_error": (C.c_char_p, []),
    "tl_version": (_I, []),
    "tl_attn_create": (_I, [C.POINTER(_P), _I, _I, _I, _I, _I, _F, _I, _I, _I, _I]),
    "tl_attn_destroy": (None, [_P]),
    "tl_kv_get_len": (_I, [_P, _I, _IP]),
    "tl_kv_set_len": (_I, [_P, _I, _I]),
    "tl_kv_reset": (_I, [_P]),
    "tl_kv_clone": (_I, [_P, _P]),
    "tl_kv_read": (_I, [_P, _I, _I, _P, _P]),
    "tl_rope_single_host": (_I, [_P, _P, _I, _I, _I, _F, _I]),
    "tl_rope_at_pos_host": (_I, [_P, _P, _I, _I, _I, _F, _I, _I]),
    "tl_kv_store_host": (_I, [_P, _I, _I, _I, _P, _P, _I]),
    "tl_attention_full_host": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _P]),
    "tl_attention_cached_host": (_I, [_P, _I, _I, _P, _I, _I, _I, _I, _P]),
    "tl_decode_layer_host": (_I, [_P, _I, _I, _P, _P, _P, _I, _P]),
    "tl_prefill_layer_host": (_I, [_P, _I, _I, _P, _P, _P, _I, _P]),
    "tl_prefill_layer_at_host": (_I, [_P, _I, _I, _I, _P, _P, _P, _I, _P]),
    "tl_decode_batch_host": (_I, [_P, _I, _I, _I, _P, _P, _P, _P, _P]),
    "tl_decode_step": (_I, [_P, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P]),
    "tl_decode_attention": (_I, [_P, _I, _I, _I, _P, _P, _P, _P, _P]),
    "tl_prefill_step": (_I, [_P, _I, _I, _I, _I, _P, _P, _P, _P, _P]),
    "tl_prefill_step_f32": (_I, [_P, _I, _I, _I, _I, _P, _P, _P, _P, _P]),
    "tl_prefill_step_at": (_I, [_P, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P]),
    "tl_kv_store": (_I, [_P, _I, _I, _I, _P, _P, _I, _P]),
    "tl_check_device": (_I, [_P, _P]),
    "tl_decode_attention_noalloc": (_I, [_P, _P, _P, _I, _I, _I, _I, _I, _I, _P, _P, _P, _P]),
    "tl_dist_unique_id": (_I, [_P]),
    "tl_dist_init": (_I, [_P, _P, _I, _I]),
    "tl_dist_resync": (_I, [_P]),
    "tl_decode_attention_dist": (_I, [_P, _I, _I, _I, _P, _P, _P, _P, _P]),
    "tl_dist_finalize": (None, [_P]),
    # include/tl_model.h
    "tl_model_create": (_I, [_P, _P, _I]),
    "tl_model_destroy": (None, [_P]),
    "tl_model_set_tensor": (_I, [_P, C.c_char_p, _I, _P, C.c_longlong, C.c_longlong]),
    "tl_model_generate": (_I, [_P, _P, _I, _I, _P, _P]),
    "tl_model_last_logits": (_I, [_P, _P]),
    "tl_model_last_timing": (_I, [_P, _P, _P]),
}

if not os.path.exists(LIB_PATH):
    raise ImportError(
        f"{LIB_PATH} is not built; run `python -m tinylama_b200.build` (nvcc, sm_100a). "
        "The attention path has no CPU fallback.")

lib = C.CDLL(LIB_PATH)
for _name, (_res, _args) in SIGNATURES.items():
    _fn = getattr(lib, _name)
    _fn.restype = _res
    _fn.argtypes = _args


class TlError(RuntimeError):
    """A C-ABI call failed; .code is the TL_ERR_* status."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"[{code}] {msg}")
        self.code = code


class TlValueError(TlError, ValueError):
    """Argument errors, raised as ValueError like the reference's ValueError/IndexDefect."""


def check(rc: int) -> None:
    if rc == TL_OK:
        return
    msg = lib.tl_last_error().decode("utf-8", "replace")
    if rc in (TL_ERR_INVALID, TL_ERR_KV_FULL, TL_ERR_RANGE, TL_ERR_UNSUPPORTED):
        raise TlValueError(rc, msg)
    raise TlError(rc, msg)


def exported_symbols() -> list[str]:
    return list(SIGNATURES)
