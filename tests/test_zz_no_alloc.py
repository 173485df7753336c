"""The allocation-free decode entry point (tl_decode_attention_noalloc) against the handle-based
one (tl_decode_attention), through the C ABI, on a B200.

It exists for callers that cannot call cudaMalloc -- a host whose allocator owns all device
memory, a loop that must not pay an allocation's latency -- and
keeps its scratch in a fixed array inside the library.  Two calls in a row must both match the
handle-based result, which shows the shared scratch is cleared between calls.  This file is
collected last so that a stop-at-first-failure run has run every other test before it."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


RAGGED = [1900, 37, 1024, 1, 700, 1333]  # several sequences need multiple chunks


@pytest.mark.parametrize("kvd,Hq,Hkv,D,lens,maxLen", [
    (0, 32, 8, 128, RAGGED, 2048),     # f32, G = 4: tensor-core kernel (tf32 split)
    (1, 32, 8, 128, RAGGED, 2048),     # bf16: tensor-core kernel
    (0, 32, 32, 128, RAGGED, 2048),    # f32, G = 1: CUDA-core kernel
    # 64 x 8192 positions at 64/8/128: at the usual chunk of 1024 the partials (4096 units x
    # 1040 floats) exceed the scratch, so the call raises the chunk length until they fit
    (1, 64, 8, 128, [8192] * 64, 8192),
])
def test_noalloc_matches_handle_decode(cuda_lib, kvd, Hq, Hkv, D, lens, maxLen):
    import torch
    _lib = cuda_lib
    torch.cuda.set_device(0)
    B = len(lens)
    g = torch.Generator(device="cuda").manual_seed(123 + kvd)
    kt = torch.randn(B, maxLen, Hkv * D, device="cuda", generator=g)
    vt = torch.randn(B, maxLen, Hkv * D, device="cuda", generator=g)
    q = torch.randn(B, Hq * D, device="cuda", generator=g)
    p = lambda t: C.c_void_p(t.data_ptr())

    # handle-based reference: same K/V stored through tl_kv_store
    h = C.c_void_p()
    _lib.check(_lib.lib.tl_attn_create(C.byref(h), 1, Hq, Hkv, D, D, 10000.0, maxLen, B, kvd, 0))
    try:
        for b in range(B):
            _lib.check(_lib.lib.tl_kv_store(h, 0, b, 0, p(kt[b]), p(vt[b]), maxLen, None))
        pos = np.array([L - 1 for L in lens], np.int32)
        dpos = torch.from_numpy(pos).cuda()
        ref = torch.empty(B, Hq * D, device="cuda")
        _lib.check(_lib.lib.tl_decode_attention(h, 0, 0, B, p(dpos), pos.ctypes.data_as(C.c_void_p),
                                                p(q), p(ref), None))
        _lib.check(_lib.lib.tl_check_device(h, None))
    finally:
        _lib.lib.tl_attn_destroy(h)

    # the caller's own cache, head-major [B][Hkv][maxLen][D]
    dt = torch.float32 if kvd == 0 else torch.bfloat16
    kc = kt.view(B, maxLen, Hkv, D).permute(0, 2, 1, 3).contiguous().to(dt)
    vc = vt.view(B, maxLen, Hkv, D).permute(0, 2, 1, 3).contiguous().to(dt)
    stream = torch.cuda.current_stream()
    for call in range(2):
        out = torch.full((B, Hq * D), float("nan"), device="cuda")
        _lib.check(_lib.lib.tl_decode_attention_noalloc(
            p(q), p(kc), p(vc), kvd, Hq, Hkv, D, maxLen, B, p(dpos), pos.ctypes.data_as(C.c_void_p),
            p(out), C.c_void_p(stream.cuda_stream)))
        torch.cuda.synchronize()
        assert torch.isfinite(out).all(), call
        # same kernel, possibly a different chunk length: equal up to fp32 summation order
        assert torch.allclose(out, ref, rtol=1e-4, atol=1e-5), (call, (out - ref).abs().max().item())


def test_noalloc_rejects_sizes_beyond_its_scratch(cuda_lib):
    import torch
    _lib = cuda_lib
    torch.cuda.set_device(0)
    q = torch.zeros(8, device="cuda")
    pos = np.zeros(1, np.int32)
    dpos = torch.zeros(1, dtype=torch.int32, device="cuda")
    p = lambda t: C.c_void_p(t.data_ptr())
    # 4097 sequences x 16 kv-heads = 65552 (sequence, kv-head) pairs > 65536
    nseq = 4097
    posn = np.zeros(nseq, np.int32)
    rc = _lib.lib.tl_decode_attention_noalloc(p(q), p(q), p(q), 0, 16, 16, 64, 1, nseq, p(dpos),
                                              posn.ctypes.data_as(C.c_void_p), p(q), None)
    assert rc == _lib.TL_ERR_INVALID
    assert b"exceeds the no-alloc scratch limit" in _lib.lib.tl_last_error()
    rc = _lib.lib.tl_decode_attention_noalloc(p(q), p(q), p(q), 0, 32, 8, 128, 4, 1, p(dpos),
                                              np.array([4], np.int32).ctypes.data_as(C.c_void_p), p(q), None)
    assert rc == _lib.TL_ERR_KV_FULL
    # 40000 sequences x 1 kv-head fit the pairs limit but not the decode kernel's shared memory
    # (8 bytes per sequence): refused before any launch
    nseq = 40000
    posn = np.zeros(nseq, np.int32)
    rc = _lib.lib.tl_decode_attention_noalloc(p(q), p(q), p(q), 0, 1, 1, 128, 1, nseq, p(dpos),
                                              posn.ctypes.data_as(C.c_void_p), p(q), None)
    assert rc == _lib.TL_ERR_INVALID
    assert b"shared memory" in _lib.lib.tl_last_error()


def test_noalloc_refusal_on_the_device_gives_nan(cuda_lib):
    """A position past maxLen given only on the device (pos_host is in range) is caught by the
    kernel's bounds check; with no handle to report it through, the output is set to NaN.  The
    next good call gives finite output again."""
    import torch
    _lib = cuda_lib
    torch.cuda.set_device(0)
    B, Hq, Hkv, D, maxLen = 2, 32, 8, 128, 512
    g = torch.Generator(device="cuda").manual_seed(9)
    kc = torch.randn(B, Hkv, maxLen, D, device="cuda", generator=g).to(torch.bfloat16)
    vc = torch.randn(B, Hkv, maxLen, D, device="cuda", generator=g).to(torch.bfloat16)
    q = torch.randn(B, Hq * D, device="cuda", generator=g)
    p = lambda t: C.c_void_p(t.data_ptr())
    pos = np.array([100, 300], np.int32)
    bad = torch.tensor([100, 5000], dtype=torch.int32, device="cuda")
    good = torch.from_numpy(pos).cuda()
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    out = torch.zeros(B, Hq * D, device="cuda")
    _lib.check(_lib.lib.tl_decode_attention_noalloc(p(q), p(kc), p(vc), 1, Hq, Hkv, D, maxLen, B, p(bad),
                                                    pos.ctypes.data_as(C.c_void_p), p(out), stream))
    torch.cuda.synchronize()
    assert torch.isnan(out).all()
    _lib.check(_lib.lib.tl_decode_attention_noalloc(p(q), p(kc), p(vc), 1, Hq, Hkv, D, maxLen, B, p(good),
                                                    pos.ctypes.data_as(C.c_void_p), p(out), stream))
    torch.cuda.synchronize()
    assert torch.isfinite(out).all()
