"""The C-ABI library without a GPU: it loads, and it exports every function include/tl_attn.h
and include/tl_model.h declare (no compute calls)."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADERS = [os.path.join(ROOT, "include", h) for h in ("tl_attn.h", "tl_model.h")]
LIB = os.path.join(ROOT, "tinylama_b200", "libtlattn.so")


def declared_functions():
    names = set()
    for header in HEADERS:
        text = re.sub(r"/\*.*?\*/", "", open(header).read(), flags=re.S)
        names.update(re.findall(r"\b(tl_[a-z0-9_]+)\s*\(", text))
    return sorted(names)


@pytest.fixture(scope="module")
def built_lib():
    if not os.path.exists(LIB):
        from tinylama_b200 import build
        build.build()
    return ctypes.CDLL(LIB)


def test_header_declares_the_reference_procs():
    fns = declared_functions()
    for name in ("tl_attn_create", "tl_rope_single_host", "tl_rope_at_pos_host", "tl_kv_store_host",
                 "tl_attention_full_host", "tl_attention_cached_host", "tl_kv_clone"):
        assert name in fns


def test_library_exports_every_declared_symbol(built_lib):
    missing = [f for f in declared_functions() if not hasattr(built_lib, f)]
    assert not missing, missing


def test_binding_table_matches_header(built_lib):
    from tinylama_b200 import _lib
    assert sorted(_lib.SIGNATURES) == declared_functions()


def test_version_and_error_string_need_no_gpu(built_lib):
    built_lib.tl_version.restype = ctypes.c_int
    assert built_lib.tl_version() == 1
    built_lib.tl_last_error.restype = ctypes.c_char_p
    assert built_lib.tl_last_error() == b""


def test_create_fails_cleanly_without_gpu_or_with_bad_shape(built_lib):
    from tinylama_b200 import _lib
    h = ctypes.c_void_p()
    # nHead not divisible by nHeadKv: rejected before any device call, with the reference's text
    rc = _lib.lib.tl_attn_create(ctypes.byref(h), 1, 6, 4, 64, 64, 10000.0, 16, 1, 0, 0)
    assert rc == _lib.TL_ERR_INVALID
    assert b"GQA requires head_count divisible by head_count_kv" in _lib.lib.tl_last_error()
    rc = _lib.lib.tl_attn_create(ctypes.byref(h), 1, 32, 4, 96, 96, 10000.0, 16, 1, 0, 0)
    assert rc == _lib.TL_ERR_UNSUPPORTED


def test_model_create_checks_shapes_before_any_device_call(built_lib):
    """tl_model_create refuses bad hyper-parameters with the reference's messages before it
    touches a GPU (so these run here, without one)."""
    from tinylama_b200 import _lib
    from tinylama_b200.host_api import TlModelConfig
    h = ctypes.c_void_p()
    bad_gqa = TlModelConfig(512, 256, 2, 512, 6, 4, 64, 10000.0, 1e-5, 32)
    assert _lib.lib.tl_model_create(ctypes.byref(h), ctypes.byref(bad_gqa), 0) == _lib.TL_ERR_INVALID
    assert b"GQA requires head_count divisible by head_count_kv" in _lib.lib.tl_last_error()
    odd_ffn = TlModelConfig(512, 256, 2, 500, 4, 2, 64, 10000.0, 1e-5, 32)
    assert _lib.lib.tl_model_create(ctypes.byref(h), ctypes.byref(odd_ffn), 0) == _lib.TL_ERR_UNSUPPORTED
    zero = TlModelConfig(512, 256, 0, 512, 4, 2, 64, 10000.0, 1e-5, 32)
    assert _lib.lib.tl_model_create(ctypes.byref(h), ctypes.byref(zero), 0) == _lib.TL_ERR_INVALID
    assert not h.value
