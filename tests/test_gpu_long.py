"""The hot-path branches that only the benchmark's full sizes reach, against the oracle, on a B200.

* The tcgen05 prefill's persistent schedule (src/forward.nim:141-176, batched): the grid holds
  one CTA per SM and a work tile is 256 query rows of one (sequence, q-head), so a CTA walks a
  second and later tile only when there are more than 148 tiles.  8 sequences of 512 tokens at
  32 q-heads are 512 tiles (every CTA takes three or four, heaviest first); 2048 and 8192
  tokens are the prefill configuration's own sizes (2048 and 8192 tiles), checked on sampled
  (sequence, head) pairs.
* The decode kernel's cluster mode for long sequences of equal length that fill the GPU
  (attentionCached, src/forward.nim:179-211): one cluster of 8 CTAs per (sequence, kv-head),
  each CTA streaming a chunk of 1024 positions (8192-token context) or 16384 positions (the
  131072-token split-KV configuration on one GPU), merged through distributed shared memory;
  at 131072 tokens also through the split-KV exchange with one rank, the single-GPU point of
  the multi-GPU workload.

bf16 figures.  Every bf16 check prints the floored elementwise error against the oracle on the
unrounded float32 inputs, the same against the oracle fed the bf16-rounded operands, the
normwise error, and the floored error that rounding the operands to bf16 causes by itself."""
import ctypes as C

import numpy as np
import pytest

from oracle import oracle as ora
from tests import numpy_ref
from tests.helpers import TOL_BF16, bf16_round, max_rel_err, normwise_err, parity, randn

pytestmark = pytest.mark.gpu

BASE = 10000.0


@pytest.fixture(scope="module")
def env(cuda_lib):
    import torch
    return torch, cuda_lib


def ptr(t):
    return C.c_void_p(t.data_ptr())


def create(_lib, Hq, Hkv, D, maxLen, maxBatch, kvd, base=BASE):
    h = C.c_void_p()
    _lib.check(_lib.lib.tl_attn_create(C.byref(h), 1, Hq, Hkv, D, D, base, maxLen, maxBatch, kvd, 0))
    return h


def bf16_figures(got, ref_unrounded, ref_rounded):
    return {"floored_vs_fp32": max_rel_err(got, ref_unrounded),
            "floored_vs_rounded_operands": max_rel_err(got, ref_rounded),
            "normwise_vs_fp32": normwise_err(got, ref_unrounded),
            "rounding_alone_floored": max_rel_err(ref_rounded, ref_unrounded)}


def _prefill(env, B, S, seed):
    """tl_prefill_step (RoPE + bf16 cache write + tcgen05 attention) on B seeded sequences of S
    tokens, 32 q / 8 kv heads, head_dim 64.  Returns the inputs and the output (host arrays)."""
    torch, _lib = env
    Hq, Hkv, D = 32, 8, 64
    rng = np.random.default_rng(seed)
    q, k, v = randn(rng, B, S, Hq * D), randn(rng, B, S, Hkv * D), randn(rng, B, S, Hkv * D)
    h = create(_lib, Hq, Hkv, D, S, B, 1)
    try:
        dq, dk, dv = (torch.from_numpy(a).cuda() for a in (q, k, v))
        out = torch.empty(B, S, Hq * D, device="cuda")
        _lib.check(_lib.lib.tl_prefill_step(h, 0, 0, B, S, ptr(dq), ptr(dk), ptr(dv), ptr(out), None))
        _lib.check(_lib.lib.tl_check_device(h, None))
        got = out.cpu().numpy()
        # a second call on the same handle overwrites the cache with the same values and must
        # give the same result (barrier phases and the tile counter start over)
        dq, dk = (torch.from_numpy(a).cuda() for a in (q, k))
        out2 = torch.empty_like(out)
        _lib.check(_lib.lib.tl_prefill_step(h, 0, 0, B, S, ptr(dq), ptr(dk), ptr(dv), ptr(out2), None))
        _lib.check(_lib.lib.tl_check_device(h, None))
        assert torch.equal(out, out2)
    finally:
        _lib.lib.tl_attn_destroy(h)
    return q, k, v, got


def _check_heads(q, k, v, got, pairs, S, rounded_too=True):
    """Oracle per (sequence, q-head): RoPE over positions 0..S-1 (applyRopeSingle), then
    attentionFull's ctx for that head alone (nHead = nHeadKv = 1 on the head's rows)."""
    Hq, Hkv, D = 32, 8, 64
    G = Hq // Hkv
    worst = {}
    for b, hd in pairs:
        g = hd // G
        qh = ora.rope_single(np.ascontiguousarray(q[b, :, hd * D:(hd + 1) * D].T), 1, D, D, BASE)
        kh = ora.rope_single(np.ascontiguousarray(k[b, :, g * D:(g + 1) * D].T), 1, D, D, BASE)
        vh = np.ascontiguousarray(v[b, :, g * D:(g + 1) * D].T)
        ref = ora.attention_full_ctx(qh, kh, vh, 1, 1, D)
        gh = np.ascontiguousarray(got[b, :, hd * D:(hd + 1) * D].T)
        nw = normwise_err(gh, ref)
        assert nw <= TOL_BF16, (b, hd, nw)
        fig = {"normwise_vs_fp32": nw, "floored_vs_fp32": max_rel_err(gh, ref)}
        if rounded_too:
            ref_b = ora.attention_full_ctx(bf16_round(qh), bf16_round(kh), bf16_round(vh), 1, 1, D)
            nb = normwise_err(gh, ref_b)
            assert nb <= 5e-3, (b, hd, nb)
            fig.update(bf16_figures(gh, ref, ref_b))
        for key, val in fig.items():
            worst[key] = max(worst.get(key, 0.0), val)
    return worst


def test_prefill_persistent_tiles_512(env):
    """8 x 512 tokens: 512 work tiles over 148 CTAs, every sequence and head checked."""
    B, S = 8, 512
    q, k, v, got = _prefill(env, B, S, 512)
    worst = _check_heads(q, k, v, got, [(b, hd) for b in range(B) for hd in range(32)], S)
    print(f"\nprefill 8x512 bf16 (all heads): " + ", ".join(f"{k} {v:.2e}" for k, v in worst.items()))


def test_prefill_persistent_tiles_2048(env):
    """8 x 2048 tokens (the prefill configuration): 2048 tiles; sampled heads."""
    B, S = 8, 2048
    q, k, v, got = _prefill(env, B, S, 2048)
    pairs = [(0, 0), (2, 9), (3, 13), (5, 22), (7, 31)]
    worst = _check_heads(q, k, v, got, pairs, S)
    print(f"\nprefill 8x2048 bf16 (5 heads): " + ", ".join(f"{k} {v:.2e}" for k, v in worst.items()))


def test_prefill_persistent_tiles_8192(env):
    """8 x 8192 tokens (the prefill configuration's largest size): 8192 tiles; the first and
    the last (sequence, head), where the heavy-first order starts and ends."""
    B, S = 8, 8192
    q, k, v, got = _prefill(env, B, S, 8192)
    worst = _check_heads(q, k, v, got, [(0, 0)], S, rounded_too=True)
    worst2 = _check_heads(q, k, v, got, [(7, 31)], S, rounded_too=False)
    for key, val in worst2.items():
        worst[key] = max(worst.get(key, 0.0), val)
    print(f"\nprefill 8x8192 bf16 (2 heads): " + ", ".join(f"{k} {v:.2e}" for k, v in worst.items()))


def _decode_uniform(env, B, L, seed, keep, dist=False):
    """B sequences of L cached positions (32 q / 8 kv heads, head_dim 128, bf16 cache, theta
    5e5), one query at position L-1 each.  The cached keys are N(0,1) without RoPE (the
    attention does not depend on how they were made; RoPE has its own tests).  Returns q, the
    K/V of the sequences in `keep` in the reference layout, and the device output(s)."""
    torch, _lib = env
    Hq, Hkv, D = 32, 8, 128
    h = create(_lib, Hq, Hkv, D, L, B, 1, base=500000.0)
    seqs = []
    try:
        rng = np.random.default_rng(seed)
        for b in range(B):
            kb = rng.standard_normal((L, Hkv * D), dtype=np.float32)
            vb = rng.standard_normal((L, Hkv * D), dtype=np.float32)
            kk, vv = torch.from_numpy(kb).cuda(), torch.from_numpy(vb).cuda()
            _lib.check(_lib.lib.tl_kv_store(h, 0, b, 0, ptr(kk), ptr(vv), L, None))
            torch.cuda.synchronize()
            del kk, vv
            seqs.append((np.ascontiguousarray(kb.T), np.ascontiguousarray(vb.T)) if b in keep else None)
            del kb, vb
        q = randn(rng, B, Hq * D)
        pos = np.full(B, L - 1, np.int32)
        dq, dpos = torch.from_numpy(q).cuda(), torch.from_numpy(pos).cuda()
        out = torch.empty(B, Hq * D, device="cuda")
        f = pos.ctypes.data_as(C.c_void_p)
        _lib.check(_lib.lib.tl_decode_attention(h, 0, 0, B, ptr(dpos), f, ptr(dq), ptr(out), None))
        _lib.check(_lib.lib.tl_check_device(h, None))
        outs = {"local": out.cpu().numpy()}
        if dist:
            uid = C.create_string_buffer(128)
            _lib.check(_lib.lib.tl_dist_unique_id(uid))
            _lib.check(_lib.lib.tl_dist_init(h, uid, 1, 0))
            o2 = torch.empty_like(out)
            for _ in range(2):  # both halves of the exchange buffer
                _lib.check(_lib.lib.tl_decode_attention_dist(h, 0, 0, B, ptr(dpos), f, ptr(dq), ptr(o2), None))
            _lib.check(_lib.lib.tl_check_device(h, None))
            outs["split-KV exchange, one rank"] = o2.cpu().numpy()
    finally:
        _lib.lib.tl_attn_destroy(h)
    return q, seqs, outs


def _check_decode(q, seqs, outs, L, check):
    Hq, Hkv, D = 32, 8, 128
    worst = {}
    for b in check:
        kc, vc = seqs[b]
        qb = q[b].reshape(-1, 1)
        kr, vr = bf16_round(kc), bf16_round(vc)
        ref_b = ora.attention_cached(qb, kr, vr, L, Hq, Hkv, D)  # the stored (bf16) K/V
        ref = ora.attention_cached(qb, kc, vc, L, Hq, Hkv, D)   # unrounded float32 K/V
        exact_b = numpy_ref.attention(qb, kr, vr, Hq, Hkv, D, np.array([L - 1]), L)
        exact = numpy_ref.attention(qb, kc, vc, Hq, Hkv, D, np.array([L - 1]), L)
        for name, o in outs.items():
            got = o[b].reshape(-1, 1)
            # against the oracle on the stored K/V, with the oracle's own float32 drift over
            # L positions (its distance from float64) added to the bound
            err, allowed = parity(got, ref_b, exact_b, TOL_BF16)
            assert err <= allowed, (name, b, err, allowed)
            # against the unrounded inputs: the kernel adds at most the bf16 bound to what the
            # bf16 storage of K/V costs by itself (and to the oracle's own drift)
            fig = bf16_figures(got, ref, ref_b)
            alone = max_rel_err(exact_b, exact)
            assert fig["floored_vs_fp32"] <= alone + TOL_BF16 + max_rel_err(ref, exact), (name, b, fig, alone)
            fig["oracle_drift_floored"] = max_rel_err(ref_b, exact_b)
            for key, val in fig.items():
                worst[(name, key)] = max(worst.get((name, key), 0.0), val)
    return worst


def test_decode_cluster_long_chunks_8192(env):
    """4 x 8192 positions, 32/8/128 bf16: 32 (sequence, kv-head) clusters of 8 CTAs fill 256 of
    the 296 resident CTAs, each CTA 1024 positions -- the cluster branch for long chunks."""
    L = 8192
    q, seqs, outs = _decode_uniform(env, 4, L, 81, keep=range(4))
    worst = _check_decode(q, seqs, outs, L, range(4))
    print("\ndecode 4x8192 bf16: " + ", ".join(f"{n}/{k} {v:.2e}" for (n, k), v in worst.items()))


def test_decode_cluster_long_chunks_131072(env):
    """4 x 131072 positions (the split-KV configuration on one GPU): chunks of 16384 positions
    per CTA, through tl_decode_attention and through the split-KV exchange with one rank."""
    L = 131072
    q, seqs, outs = _decode_uniform(env, 4, L, 131, keep=[0, 3], dist=True)
    worst = _check_decode(q, seqs, outs, L, [0, 3])
    print("\ndecode 4x131072 bf16: " + ", ".join(f"{n}/{k} {v:.2e}" for (n, k), v in worst.items()))
