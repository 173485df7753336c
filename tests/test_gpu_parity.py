"""Parity of the CUDA path (through the C ABI) against the oracle, on a B200.

Host-tier tests call the Python mirror of the Nim procs (tinylama_b200.forward_attn), which
binds libtlattn.so the way the Nim host would.  Device-tier tests drive the batched entry
points with device buffers.  Tolerances: max rel err <= 1e-3 for the fp32 cache, <= 2e-2 for
the bf16 cache (tests/helpers.py)."""
import ctypes as C

import numpy as np
import pytest

from oracle import oracle as ora
from tests import numpy_ref
from tests.helpers import (TOL_BF16, TOL_F32, bf16_round, check_rope, max_rel_err, normwise_err,
                           parity, randn)

pytestmark = pytest.mark.gpu

TINY = dict(nEmb=2048, nHead=32, nHeadKv=4, nLayer=2, ropeFreqBase=10000.0)


@pytest.fixture(scope="module")
def fa(cuda_lib):
    from tinylama_b200 import forward_attn
    return forward_attn


def hp(fa, **kw):
    d = dict(TINY)
    d.update(kw)
    return fa.HParams(**d)


# ---- RoPE ---------------------------------------------------------------------------------

def test_apply_rope_single(fa):
    rng = np.random.default_rng(10)
    x = randn(rng, 32 * 64, 8)
    y = x.copy()
    fa.applyRopeSingle(y, 32, 64, 64, 10000.0)
    check_rope(y, ora.rope_single(x, 32, 64, 64, 10000.0))


@pytest.mark.parametrize("pos,base", [(0, 10000.0), (37, 10000.0), (4095, 10000.0), (131071, 500000.0)])
def test_apply_rope_at_pos(fa, pos, base):
    rng = np.random.default_rng(pos)
    x = randn(rng, 8 * 128, 3)
    y = x.copy()
    fa.applyRopeAtPos(y, 8, 128, 128, base, pos)
    ref = ora.rope_at_pos(x, 8, 128, 128, base, pos)
    # column 0 rotated, other columns untouched; the angles are the same float32 products, so
    # only a last-bit difference between glibc's and the device's cos/sin can remain
    assert np.array_equal(y[:, 1:], x[:, 1:])
    check_rope(y, ref)


def test_rope_partial_ropedim(fa):
    rng = np.random.default_rng(11)
    x = randn(rng, 4 * 64, 5)
    y = x.copy()
    fa.applyRopeSingle(y, 4, 64, 32, 10000.0)
    check_rope(y, ora.rope_single(x, 4, 64, 32, 10000.0))
    assert np.array_equal(y.reshape(4, 64, 5)[:, 32:], x.reshape(4, 64, 5)[:, 32:])


# ---- storeKVRange / KvCache ---------------------------------------------------------------

@pytest.mark.parametrize("kvd", [0, 1])
def test_store_kv_range_and_read_back(fa, kvd):
    rng = np.random.default_rng(12)
    cache = fa.initKvCache(hp(fa), 40, kv_dtype=kvd)
    k, v = randn(rng, 256, 9), randn(rng, 256, 9)
    fa.storeKVRange(cache, 1, 5, k, v)
    kc, vc = cache.k[1], cache.v[1]
    expect_k = k if kvd == 0 else bf16_round(k)
    expect_v = v if kvd == 0 else bf16_round(v)
    assert np.array_equal(kc[:, 5:14], expect_k) and np.array_equal(vc[:, 5:14], expect_v)
    assert not kc[:, :5].any() and not kc[:, 14:].any()
    assert not cache.k[0].any()


def test_store_kv_range_overflow_is_refused(fa):
    cache = fa.initKvCache(hp(fa), 16)
    k = np.zeros((256, 4), np.float32)
    with pytest.raises(ValueError, match="exceed maxLen"):
        fa.storeKVRange(cache, 0, 14, k, k)
    with pytest.raises(ValueError, match="layer"):
        fa.storeKVRange(cache, 2, 0, k, k)


def test_clone_cache_deep_copies(fa):
    rng = np.random.default_rng(13)
    cache = fa.initKvCache(hp(fa), 24)
    k, v = randn(rng, 256, 6), randn(rng, 256, 6)
    fa.storeKVRange(cache, 0, 0, k, v)
    cache.curLen = 6
    cl = fa.cloneCache(cache)
    assert cl.curLen == 6
    assert np.array_equal(cl.k[0], cache.k[0])
    fa.storeKVRange(cache, 0, 0, v, k)
    assert np.array_equal(cl.k[0][:, :6], k)


# ---- attentionCached (decode) -------------------------------------------------------------

def _fill_cache(fa, rng, cache, layer, L, slot=0):
    kvDim = cache.nHeadKv * cache.headDim
    k, v = randn(rng, kvDim, L), randn(rng, kvDim, L)
    fa.storeKVRange(cache, layer, 0, k, v, slot=slot)
    kc = np.zeros((kvDim, cache.maxLen), np.float32)
    vc = np.zeros((kvDim, cache.maxLen), np.float32)
    kc[:, :L], vc[:, :L] = k, v
    if cache.kv_dtype == 1:
        kc, vc = bf16_round(kc), bf16_round(vc)
    return kc, vc


@pytest.mark.parametrize("Hq,Hkv,D,L,kvd", [
    (32, 4, 64, 1, 0), (32, 4, 64, 31, 0), (32, 4, 64, 33, 0), (32, 4, 64, 128, 0),
    (32, 4, 64, 512, 0), (32, 4, 64, 2048, 0), (32, 4, 64, 2048, 1),
    (32, 32, 128, 257, 0), (32, 32, 128, 4096, 1), (32, 8, 128, 1000, 0), (32, 8, 128, 8191, 1),
    (16, 8, 64, 100, 0), (8, 8, 64, 70, 1),
])
def test_attention_cached_matches_oracle(fa, Hq, Hkv, D, L, kvd):
    rng = np.random.default_rng(L * 7 + Hkv)
    h = fa.HParams(nEmb=Hq * D, nHead=Hq, nHeadKv=Hkv, nLayer=1)
    cache = fa.initKvCache(h, L + 3, kv_dtype=kvd)
    kc, vc = _fill_cache(fa, rng, cache, 0, L)
    q = randn(rng, Hq * D, 1)
    ctx = fa.attentionCached(q, cache, 0, L, Hq, Hkv, D)
    ref = ora.attention_cached(q, kc, vc, L, Hq, Hkv, D)
    # a bf16 cache is compared with the oracle fed the same bf16-rounded K/V, under the bf16-KV
    # bound (the tensor-core kernel rounds q and p into bf16 hi/lo parts)
    exact = numpy_ref.attention(q, kc, vc, Hq, Hkv, D, np.array([L - 1]), L) if L >= 1024 else None
    err, allowed = parity(ctx, ref, exact, TOL_F32 if kvd == 0 else TOL_BF16)
    assert err <= allowed, (err, allowed)


def test_attention_cached_bad_args(fa):
    cache = fa.initKvCache(hp(fa), 16)
    q = np.zeros((2048, 1), np.float32)
    with pytest.raises(ValueError):
        fa.attentionCached(q, cache, 0, 17, 32, 4, 64)
    with pytest.raises(ValueError):
        fa.attentionCached(q, cache, 0, 0, 32, 4, 64)
    with pytest.raises(ValueError, match="does not match"):
        fa.attentionCached(q, cache, 0, 4, 32, 8, 64)


@pytest.mark.parametrize("kvd", [0, 1])
def test_decode_layer_matches_oracle_step(fa, kvd):
    """forwardDecode's attention block: RoPE q,k at pos, store, attend pos+1 columns."""
    rng = np.random.default_rng(14 + kvd)
    cache = fa.initKvCache(hp(fa), 64, kv_dtype=kvd)
    L = 40
    kc, vc = _fill_cache(fa, rng, cache, 1, L)
    q, k, v = randn(rng, 2048, 1), randn(rng, 256, 1), randn(rng, 256, 1)
    ctx = fa.decodeLayer(cache, 1, q, k, v, L)
    qr = ora.rope_at_pos(q, 32, 64, 64, 10000.0, L)
    kr = ora.rope_at_pos(k, 4, 64, 64, 10000.0, L)
    kc[:, L:L + 1] = kr if kvd == 0 else bf16_round(kr)
    vc[:, L:L + 1] = v if kvd == 0 else bf16_round(v)
    ref = ora.attention_cached(qr, kc, vc, L + 1, 32, 4, 64)
    assert max_rel_err(ctx, ref) <= (TOL_F32 if kvd == 0 else TOL_BF16)
    if kvd == 0:
        check_rope(cache.k[1][:, L:L + 1], kc[:, L:L + 1])
    else:
        assert np.max(np.abs(cache.k[1][:, L:L + 1] - kc[:, L:L + 1])) <= 2 ** -7 * np.max(np.abs(kc[:, L:L + 1]))


def test_decode_kv_full(fa):
    cache = fa.initKvCache(hp(fa), 8)
    z = np.zeros((2048, 1), np.float32)
    with pytest.raises(ValueError, match="KV cache full"):
        fa.decodeLayer(cache, 0, z, z[:256], z[:256], 8)
    cache.curLen = 8
    with pytest.raises(ValueError, match="KV cache full"):
        fa.forwardDecodeCheck(cache)


# ---- attentionFull (prefill) --------------------------------------------------------------

@pytest.mark.parametrize("Hq,Hkv,D,S", [(32, 4, 64, 1), (32, 4, 64, 8), (32, 4, 64, 70), (32, 8, 64, 200),
                                        (32, 32, 128, 65), (32, 8, 128, 129)])
def test_attention_full_matches_oracle(fa, Hq, Hkv, D, S):
    rng = np.random.default_rng(S + Hkv)
    q, k, v = randn(rng, Hq * D, S), randn(rng, Hkv * D, S), randn(rng, Hkv * D, S)
    ctx = fa.attentionFullCtx(q, k, v, Hq, Hkv, D)
    ref = ora.attention_full_ctx(q, k, v, Hq, Hkv, D)
    assert max_rel_err(ctx, ref) <= TOL_F32, max_rel_err(ctx, ref)


def test_attention_full_with_wo(fa):
    rng = np.random.default_rng(15)
    q, k, v = randn(rng, 2048, 8), randn(rng, 256, 8), randn(rng, 256, 8)
    wo = randn(rng, 2048, 2048) * np.float32(0.02)
    out = fa.attentionFull(q, k, v, wo, 32, 4, 64)
    ref = ora.linear_ggml_col(ora.attention_full_ctx(q, k, v, 32, 4, 64), wo)
    assert max_rel_err(out, ref) <= TOL_F32


@pytest.mark.parametrize("S,kvd", [(8, 0), (100, 0), (8, 1), (300, 1)])
def test_prefill_layer_matches_oracle_step(fa, S, kvd):
    """forwardPrefill's attention block: RoPE q,k over 0..S-1, store at 0, attentionFull."""
    rng = np.random.default_rng(S + 100 * kvd)
    cache = fa.initKvCache(hp(fa), S + 4, kv_dtype=kvd)
    q, k, v = randn(rng, 2048, S), randn(rng, 256, S), randn(rng, 256, S)
    ctx = fa.prefillLayer(cache, 0, q, k, v)
    qr = ora.rope_single(q, 32, 64, 64, 10000.0)
    kr = ora.rope_single(k, 4, 64, 64, 10000.0)
    ref = ora.attention_full_ctx(qr, kr, v, 32, 4, 64)
    if kvd == 0:
        assert max_rel_err(ctx, ref) <= TOL_F32
        check_rope(cache.k[0][:, :S], kr)
    else:
        # bf16 tensor-core path: Q, K, V and P are bf16, so entries near zero carry an absolute
        # error of a few 1e-3; the bound is normwise against the fp32 oracle, and tighter
        # against the oracle fed the same bf16-rounded inputs
        assert normwise_err(ctx, ref) <= TOL_BF16, normwise_err(ctx, ref)
        ref_b = ora.attention_full_ctx(bf16_round(qr), bf16_round(kr), bf16_round(v), 32, 4, 64)
        assert normwise_err(ctx, ref_b) <= 5e-3, normwise_err(ctx, ref_b)


def _decode_steps_ref(q, k, v, kc, vc, start, Hq, Hkv, D, base, kvd):
    """The reference's way through a later prompt: one forwardDecode attention block per token
    (src/forward.nim:314-317 at pos = start + t).  kc, vc are written in place; returns the ctx
    columns, and for a bf16 cache also the ctx with q rounded to bf16 as the tensor cores see it."""
    out, out_b = [], []
    for t in range(q.shape[1]):
        pos = start + t
        qr = ora.rope_at_pos(q[:, t:t + 1], Hq, D, D, base, pos)
        kr = ora.rope_at_pos(k[:, t:t + 1], Hkv, D, D, base, pos)
        kc[:, pos:pos + 1] = kr if kvd == 0 else bf16_round(kr)
        vc[:, pos:pos + 1] = v[:, t:t + 1] if kvd == 0 else bf16_round(v[:, t:t + 1])
        out.append(ora.attention_cached(qr, kc, vc, pos + 1, Hq, Hkv, D))
        if kvd == 1:
            out_b.append(ora.attention_cached(bf16_round(qr), kc, vc, pos + 1, Hq, Hkv, D))
    return np.concatenate(out, axis=1), (np.concatenate(out_b, axis=1) if out_b else None)


@pytest.mark.parametrize("kvd", [0, 1])
def test_prefill_layer_at_matches_decode_steps(fa, kvd):
    """A prompt fed in chunks through prefillLayerAt (the first at position 0, each next one at
    startPos = curLen) against the reference's multi-turn path, which feeds every token through
    forwardDecode (src/tinylama.nim:70-73).  Chunk boundaries fall inside the 128-key tiles; a
    bf16 cache with head_dim 64 runs the tcgen05 kernel with its key range shifted by startPos."""
    rng = np.random.default_rng(77 + kvd)
    chunks = [130, 77, 200, 1]
    total = sum(chunks)
    cache = fa.initKvCache(hp(fa), total + 5, kv_dtype=kvd)
    kc = np.zeros((256, total + 5), np.float32)
    vc = np.zeros((256, total + 5), np.float32)
    start = 0
    for S in chunks:
        q, k, v = randn(rng, 2048, S), randn(rng, 256, S), randn(rng, 256, S)
        ctx = fa.prefillLayerAt(cache, 0, start, q, k, v)
        ref, ref_b = _decode_steps_ref(q, k, v, kc, vc, start, 32, 4, 64, 10000.0, kvd)
        if kvd == 0:
            assert max_rel_err(ctx, ref) <= TOL_F32, (start, max_rel_err(ctx, ref))
        else:
            assert normwise_err(ctx, ref) <= TOL_BF16, (start, normwise_err(ctx, ref))
            assert normwise_err(ctx, ref_b) <= 5e-3, (start, normwise_err(ctx, ref_b))
        start += S
    z = np.zeros((2048, 6), np.float32)
    with pytest.raises(ValueError, match="exceeds the KV cache"):
        fa.prefillLayerAt(cache, 0, start, z, z[:256], z[:256])


def test_prefill_overflow_is_refused(fa):
    cache = fa.initKvCache(hp(fa), 8)
    z = np.zeros((2048, 9), np.float32)
    with pytest.raises(ValueError, match="exceeds the KV cache"):
        fa.prefillLayer(cache, 0, z, z[:256], z[:256])
