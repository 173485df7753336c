"""Device-tier (batched, token-major) entry points against the oracle, on a B200: the
configurations of the batched decode (independent sequences of ragged length, 32 q = 32 kv
heads, head_dim 128), long-context split-KV (32 q / 8 kv heads, theta 5e5) and the batched
prefill (32 q / 8 kv heads, head_dim 64), at sizes the oracle finishes in seconds."""
import ctypes as C
import os

import numpy as np
import pytest

from oracle import oracle as ora
from tests import numpy_ref
from tests.helpers import TOL_BF16, TOL_F32, bf16_round, max_rel_err, normwise_err, parity, randn

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def env(cuda_lib):
    import torch
    from tinylama_b200 import _lib
    return torch, _lib


def create(_lib, nLayer, Hq, Hkv, D, maxLen, maxBatch, kvd, base=10000.0):
    h = C.c_void_p()
    _lib.check(_lib.lib.tl_attn_create(C.byref(h), nLayer, Hq, Hkv, D, D, base, maxLen, maxBatch, kvd, 0))
    return h


def ptr(t):
    return C.c_void_p(t.data_ptr())


def fill_cache(torch, _lib, h, layer, lens, Hkv, D, rng, base, kvd):
    """Write seeded K/V for every slot via tl_kv_store_host; return oracle-layout caches."""
    caches = []
    for b, L in enumerate(lens):
        k = randn(rng, Hkv * D, L)
        v = randn(rng, Hkv * D, L)
        kr = ora.rope_single(k, Hkv, D, D, base)  # cached keys carry their RoPE
        _lib.check(_lib.lib.tl_kv_store_host(h, layer, b, 0, kr.ctypes.data_as(C.c_void_p),
                                             v.ctypes.data_as(C.c_void_p), L))
        if kvd == 1:
            kr, v = bf16_round(kr), bf16_round(v)
        caches.append((kr, v))
    return caches


@pytest.mark.parametrize("kvd", [0, 1])
@pytest.mark.parametrize("Hq,Hkv,D,lens", [
    (32, 32, 128, [256, 1000, 4095, 300, 2049, 31, 1]),  # ragged batch, head_dim 128
    (32, 4, 64, [128, 512, 2048]),                       # TinyLlama GQA 8:1
    (32, 8, 128, [5000, 77]),                            # GQA 4:1, multi-chunk
])
def test_decode_step_batched(env, kvd, Hq, Hkv, D, lens):
    torch, _lib = env
    rng = np.random.default_rng(sum(lens) + kvd)
    base = 10000.0
    B = len(lens)
    maxLen = max(lens) + 2
    h = create(_lib, 2, Hq, Hkv, D, maxLen, B, kvd, base)
    try:
        caches = fill_cache(torch, _lib, h, 1, lens, Hkv, D, rng, base, kvd)
        q = randn(rng, B, Hq * D)
        k = randn(rng, B, Hkv * D)
        v = randn(rng, B, Hkv * D)
        pos = np.array(lens, np.int32)  # new token at position L, attends L+1 positions
        dq, dk, dv = (torch.from_numpy(a).cuda() for a in (q, k, v))
        dpos = torch.from_numpy(pos).cuda()
        out = torch.empty(B, Hq * D, device="cuda")
        _lib.check(_lib.lib.tl_decode_step(h, 1, 0, B, ptr(dpos), pos.ctypes.data_as(C.c_void_p),
                                           ptr(dq), ptr(dk), ptr(dv), ptr(out), None))
        _lib.check(_lib.lib.tl_check_device(h, None))
        got = out.cpu().numpy()
        for b, L in enumerate(lens):
            qr = ora.rope_at_pos(q[b].reshape(-1, 1), Hq, D, D, base, L)
            kr = ora.rope_at_pos(k[b].reshape(-1, 1), Hkv, D, D, base, L)
            kc = np.zeros((Hkv * D, L + 1), np.float32)
            vc = np.zeros((Hkv * D, L + 1), np.float32)
            kc[:, :L], vc[:, :L] = caches[b]
            kc[:, L:] = kr if kvd == 0 else bf16_round(kr)
            vc[:, L:] = v[b].reshape(-1, 1) if kvd == 0 else bf16_round(v[b].reshape(-1, 1))
            ref = ora.attention_cached(qr, kc, vc, L + 1, Hq, Hkv, D)
            exact = numpy_ref.attention(qr, kc, vc, Hq, Hkv, D, np.array([L]), L + 1) if L >= 1024 else None
            # bf16 cache: the tensor-core kernel (bf16 hi/lo q and p, fp32 accumulate) is held to
            # the bf16-KV bound against the oracle fed the same bf16-rounded K/V
            err, allowed = parity(got[b].reshape(-1, 1), ref, exact, TOL_F32 if kvd == 0 else TOL_BF16)
            assert err <= allowed, (b, L, err, allowed)
        # repeated calls give identical results (counters are reset by the merging CTA)
        out2 = torch.empty_like(out)
        dq2, dk2 = (torch.from_numpy(a).cuda() for a in (q, k))
        _lib.check(_lib.lib.tl_decode_step(h, 1, 0, B, ptr(dpos), None, ptr(dq2), ptr(dk2), ptr(dv),
                                           ptr(out2), None))
        _lib.check(_lib.lib.tl_check_device(h, None))
        assert torch.allclose(out2, out, rtol=1e-5, atol=1e-6)
    finally:
        _lib.lib.tl_attn_destroy(h)


@pytest.mark.parametrize("parts", [None, "2", "4"])
def test_decode_batch_host_matches_device_tier(env, parts):
    """tl_decode_batch_host (host buffers) against tl_decode_step on device copies of the same
    inputs.  TL_HOST_PARTS forces the number of parts the host call cuts the batch into (copies
    of one part overlap the attention of another); the default keeps one part at this size."""
    torch, _lib = env
    rng = np.random.default_rng(21)
    lens = [700, 33, 1500, 256]
    B, Hq, Hkv, D = 4, 32, 32, 128
    h = create(_lib, 1, Hq, Hkv, D, 2048, B, 0)
    old = os.environ.pop("TL_HOST_PARTS", None)
    if parts is not None:
        os.environ["TL_HOST_PARTS"] = parts
    try:
        fill_cache(torch, _lib, h, 0, lens, Hkv, D, rng, 10000.0, 0)
        q, k, v = randn(rng, B, Hq * D), randn(rng, B, Hkv * D), randn(rng, B, Hkv * D)
        pos = np.array(lens, np.int32)
        out = np.empty((B, Hq * D), np.float32)
        f = lambda a: a.ctypes.data_as(C.c_void_p)
        _lib.check(_lib.lib.tl_decode_batch_host(h, 0, 0, B, f(pos), f(q), f(k), f(v), f(out)))
        for b, L in enumerate(lens):
            assert out[b].any()
        # same inputs through the device tier
        dq, dk, dv = (torch.from_numpy(a).cuda() for a in (q, k, v))
        dpos = torch.from_numpy(pos).cuda()
        o2 = torch.empty(B, Hq * D, device="cuda")
        _lib.check(_lib.lib.tl_decode_step(h, 0, 0, B, ptr(dpos), f(pos), ptr(dq), ptr(dk), ptr(dv), ptr(o2), None))
        _lib.check(_lib.lib.tl_check_device(h, None))
        # a part is planned alone (its own chunk length): the sums may differ in order
        assert np.allclose(o2.cpu().numpy(), out, rtol=1e-4, atol=1e-5)
    finally:
        _lib.lib.tl_attn_destroy(h)
        os.environ.pop("TL_HOST_PARTS", None)
        if old is not None:
            os.environ["TL_HOST_PARTS"] = old


def test_device_error_word_reports_bad_position(env):
    """A position past maxLen given only on the device is caught by the kernel's bounds check
    (no write happens) and reported through tl_check_device."""
    torch, _lib = env
    h = create(_lib, 1, 32, 4, 64, 16, 1, 0)
    try:
        dpos = torch.tensor([16], dtype=torch.int32, device="cuda")
        q = torch.zeros(1, 2048, device="cuda")
        k = torch.zeros(1, 256, device="cuda")
        out = torch.empty(1, 2048, device="cuda")
        rc = _lib.lib.tl_decode_step(h, 0, 0, 1, ptr(dpos), None, ptr(q), ptr(k), ptr(k), ptr(out), None)
        if rc == _lib.TL_OK:
            rc = _lib.lib.tl_check_device(h, None)
        assert rc == _lib.TL_ERR_DEVICE
        assert b"position-out-of-range" in _lib.lib.tl_last_error()
        # the handle stays usable
        dpos.fill_(3)
        _lib.check(_lib.lib.tl_decode_attention(h, 0, 0, 1, ptr(dpos), None, ptr(q), ptr(out), None))
        _lib.check(_lib.lib.tl_check_device(h, None))
    finally:
        _lib.lib.tl_attn_destroy(h)


def test_unaligned_q_is_refused_before_any_launch(env):
    """The decode kernels read q in 16-byte vectors: a q 4 bytes past a 16-byte boundary is
    refused on the host with TL_ERR_INVALID (no kernel runs, nothing faults), for the step, the
    attention-only call and the no-alloc entry point; the handle stays usable."""
    torch, _lib = env
    h = create(_lib, 1, 32, 4, 64, 16, 1, 0)
    try:
        pos = np.array([3], np.int32)
        dpos = torch.from_numpy(pos).cuda()
        f = pos.ctypes.data_as(C.c_void_p)
        qbuf = torch.zeros(1, 2048 + 4, device="cuda")
        k = torch.zeros(1, 256, device="cuda")
        out = torch.empty(1, 2048, device="cuda")
        bad = C.c_void_p(qbuf.data_ptr() + 4)
        rc = _lib.lib.tl_decode_step(h, 0, 0, 1, ptr(dpos), f, bad, ptr(k), ptr(k), ptr(out), None)
        assert rc == _lib.TL_ERR_INVALID and b"16-byte aligned" in _lib.lib.tl_last_error()
        rc = _lib.lib.tl_decode_attention(h, 0, 0, 1, ptr(dpos), f, bad, ptr(out), None)
        assert rc == _lib.TL_ERR_INVALID and b"16-byte aligned" in _lib.lib.tl_last_error()
        kc = torch.zeros(16, 256, device="cuda")
        rc = _lib.lib.tl_decode_attention_noalloc(bad, ptr(kc), ptr(kc), 0, 32, 4, 64, 16, 1, ptr(dpos), f,
                                                  ptr(out), None)
        assert rc == _lib.TL_ERR_INVALID and b"16-byte aligned" in _lib.lib.tl_last_error()
        q = qbuf[:, :2048].contiguous()
        _lib.check(_lib.lib.tl_decode_attention(h, 0, 0, 1, ptr(dpos), f, ptr(q), ptr(out), None))
        _lib.check(_lib.lib.tl_check_device(h, None))
    finally:
        _lib.lib.tl_attn_destroy(h)


@pytest.mark.parametrize("kvd,S", [(0, 64), (0, 200), (1, 128), (1, 300)])
def test_prefill_step_batched(env, kvd, S):
    torch, _lib = env
    rng = np.random.default_rng(S + kvd)
    B, Hq, Hkv, D = 2, 32, 8, 64
    h = create(_lib, 1, Hq, Hkv, D, S, B, kvd)
    try:
        q, k, v = randn(rng, B, S, Hq * D), randn(rng, B, S, Hkv * D), randn(rng, B, S, Hkv * D)
        dq, dk, dv = (torch.from_numpy(a).cuda() for a in (q, k, v))
        out = torch.empty(B, S, Hq * D, device="cuda")
        _lib.check(_lib.lib.tl_prefill_step(h, 0, 0, B, S, ptr(dq), ptr(dk), ptr(dv), ptr(out), None))
        _lib.check(_lib.lib.tl_check_device(h, None))
        got = out.cpu().numpy()
        tol = TOL_F32 if kvd == 0 else TOL_BF16
        for b in range(B):
            qc = np.ascontiguousarray(q[b].T)
            kc = np.ascontiguousarray(k[b].T)
            vc = np.ascontiguousarray(v[b].T)
            qr = ora.rope_single(qc, Hq, D, D, 10000.0)
            kr = ora.rope_single(kc, Hkv, D, D, 10000.0)
            ref = ora.attention_full_ctx(qr, kr, vc, Hq, Hkv, D)
            g = np.ascontiguousarray(got[b].T)
            if kvd == 0:
                err = max_rel_err(g, ref)
                assert err <= TOL_F32, (b, err)
            else:
                # bf16 tensor-core path (see test_prefill_layer_matches_oracle_step)
                assert normwise_err(g, ref) <= TOL_BF16, (b, normwise_err(g, ref))
                ref_b = ora.attention_full_ctx(bf16_round(qr), bf16_round(kr), bf16_round(vc), Hq, Hkv, D)
                assert normwise_err(g, ref_b) <= 5e-3, (b, normwise_err(g, ref_b))
    finally:
        _lib.lib.tl_attn_destroy(h)


@pytest.mark.parametrize("kvd", [0, 1])
def test_prefill_step_at_continues_prefixes(env, kvd):
    """tl_prefill_step_at: three sequences continue cached prefixes of 0, 300 and 1000 tokens
    with 150 new tokens each (the prefill shape: 32 q / 8 kv heads, head_dim 64).  Each token is
    checked against the reference's per-token path: RoPE at its position, store, attend every
    position up to it (src/forward.nim:314-317)."""
    torch, _lib = env
    rng = np.random.default_rng(500 + kvd)
    prefix = [0, 300, 1000]
    B, Hq, Hkv, D, S, base = 3, 32, 8, 64, 150, 10000.0
    maxLen = max(prefix) + S
    h = create(_lib, 1, Hq, Hkv, D, maxLen, B, kvd, base)
    try:
        caches = []
        for b, P in enumerate(prefix):
            kc = np.zeros((Hkv * D, maxLen), np.float32)
            vc = np.zeros((Hkv * D, maxLen), np.float32)
            if P > 0:
                k = randn(rng, Hkv * D, P)
                v = randn(rng, Hkv * D, P)
                kr = ora.rope_single(k, Hkv, D, D, base)
                _lib.check(_lib.lib.tl_kv_store_host(h, 0, b, 0, kr.ctypes.data_as(C.c_void_p),
                                                     v.ctypes.data_as(C.c_void_p), P))
                kc[:, :P] = kr if kvd == 0 else bf16_round(kr)
                vc[:, :P] = v if kvd == 0 else bf16_round(v)
            caches.append((kc, vc))
        q, k, v = randn(rng, B, S, Hq * D), randn(rng, B, S, Hkv * D), randn(rng, B, S, Hkv * D)
        dq, dk, dv = (torch.from_numpy(a).cuda() for a in (q, k, v))
        pos0 = np.array(prefix, np.int32)
        dpos0 = torch.from_numpy(pos0).cuda()
        out = torch.empty(B, S, Hq * D, device="cuda")
        _lib.check(_lib.lib.tl_prefill_step_at(h, 0, 0, B, S, ptr(dpos0), pos0.ctypes.data_as(C.c_void_p),
                                               ptr(dq), ptr(dk), ptr(dv), ptr(out), None))
        _lib.check(_lib.lib.tl_check_device(h, None))
        got = out.cpu().numpy()
        for b, P in enumerate(prefix):
            kc, vc = caches[b]
            out_ref, out_b = [], []
            for t in range(S):
                pos = P + t
                qr = ora.rope_at_pos(q[b, t].reshape(-1, 1), Hq, D, D, base, pos)
                kr = ora.rope_at_pos(k[b, t].reshape(-1, 1), Hkv, D, D, base, pos)
                kc[:, pos:pos + 1] = kr if kvd == 0 else bf16_round(kr)
                vc[:, pos:pos + 1] = v[b, t].reshape(-1, 1) if kvd == 0 else bf16_round(v[b, t].reshape(-1, 1))
                out_ref.append(ora.attention_cached(qr, kc, vc, pos + 1, Hq, Hkv, D))
                if kvd == 1:
                    out_b.append(ora.attention_cached(bf16_round(qr), kc, vc, pos + 1, Hq, Hkv, D))
            ref = np.concatenate(out_ref, axis=1)
            g = np.ascontiguousarray(got[b].T)
            if kvd == 0:
                assert max_rel_err(g, ref) <= TOL_F32, (b, max_rel_err(g, ref))
            else:
                assert normwise_err(g, ref) <= TOL_BF16, (b, normwise_err(g, ref))
                ref_b = np.concatenate(out_b, axis=1)
                assert normwise_err(g, ref_b) <= 5e-3, (b, normwise_err(g, ref_b))
        # a start past maxLen - S is refused before any launch
        bad = np.array([0, 300, maxLen - S + 1], np.int32)
        rc = _lib.lib.tl_prefill_step_at(h, 0, 0, B, S, ptr(dpos0), bad.ctypes.data_as(C.c_void_p),
                                         ptr(dq), ptr(dk), ptr(dv), ptr(out), None)
        assert rc != 0 and b"exceeds the KV cache" in _lib.lib.tl_last_error()
    finally:
        _lib.lib.tl_attn_destroy(h)


@pytest.mark.parametrize("cluster", ["1", "0"])
@pytest.mark.parametrize("exchange", ["peer", "nccl"])
def test_dist_single_rank_matches_local(env, exchange, cluster):
    """tl_decode_attention_dist with one rank must reproduce the single-GPU result.  "peer" is
    the fused exchange (the decode kernel stores its (o, m, l) into the gather buffer, raises
    the epoch flag, waits for it and merges); "nccl" is the fallback (local partials, NCCL
    all-gather, merge launch), chosen by TL_DIST_NCCL=1 at tl_dist_init.  Three calls in a row
    use both halves of the exchange buffer.  TL_DECODE_CLUSTER=0 keeps the decode kernel off
    cluster mode (one cluster per (sequence, kv-head), which these sizes otherwise select)."""
    torch, _lib = env
    rng = np.random.default_rng(31)
    lens = [3000, 129, 1]
    B, Hq, Hkv, D = 3, 32, 8, 128
    old = os.environ.pop("TL_DIST_NCCL", None)
    old_cl = os.environ.pop("TL_DECODE_CLUSTER", None)
    os.environ["TL_DECODE_CLUSTER"] = cluster
    if exchange == "nccl":
        os.environ["TL_DIST_NCCL"] = "1"
    h = create(_lib, 1, Hq, Hkv, D, 4096, B, 1, 500000.0)
    try:
        fill_cache(torch, _lib, h, 0, lens, Hkv, D, rng, 500000.0, 1)
        uid = C.create_string_buffer(128)
        _lib.check(_lib.lib.tl_dist_unique_id(uid))
        _lib.check(_lib.lib.tl_dist_init(h, uid, 1, 0))
        pos = np.array([L - 1 for L in lens], np.int32)
        dpos = torch.from_numpy(pos).cuda()
        f = pos.ctypes.data_as(C.c_void_p)
        for _ in range(3):
            q = torch.from_numpy(randn(rng, B, Hq * D)).cuda()
            o1 = torch.empty(B, Hq * D, device="cuda")
            o2 = torch.empty(B, Hq * D, device="cuda")
            _lib.check(_lib.lib.tl_decode_attention(h, 0, 0, B, ptr(dpos), f, ptr(q), ptr(o1), None))
            _lib.check(_lib.lib.tl_decode_attention_dist(h, 0, 0, B, ptr(dpos), f, ptr(q), ptr(o2), None))
            _lib.check(_lib.lib.tl_check_device(h, None))
            assert torch.allclose(o1, o2, rtol=1e-4, atol=1e-5)
    finally:
        _lib.lib.tl_attn_destroy(h)
        os.environ.pop("TL_DIST_NCCL", None)
        if old is not None:
            os.environ["TL_DIST_NCCL"] = old
        os.environ.pop("TL_DECODE_CLUSTER", None)
        if old_cl is not None:
            os.environ["TL_DECODE_CLUSTER"] = old_cl


@pytest.mark.parametrize("kvd,Hq,Hkv,D,lens", [
    (0, 32, 4, 64, [2048]),           # TinyLlama batch 1: 8 CTAs of 256 positions per kv head
    (0, 32, 4, 64, [1]),
    (0, 32, 4, 64, [1, 100, 700]),    # chunks past a short sequence's end are empty
    (1, 32, 4, 64, [2048]),
    (1, 32, 8, 128, [1000, 3]),
    (0, 32, 8, 128, [4000]),
    (1, 8, 8, 64, [70, 511]),
])
def test_decode_cluster_mode_matches_queue_mode(env, kvd, Hq, Hkv, D, lens):
    """Few short sequences run in cluster mode (one thread-block cluster per (sequence,
    kv-head), merged through distributed shared memory); TL_DECODE_CLUSTER=0 sends the same
    call through the unit queue and the global merge.  Both against the oracle and each other."""
    torch, _lib = env
    rng = np.random.default_rng(sum(lens) * 3 + kvd)
    base = 10000.0
    B = len(lens)
    h = create(_lib, 1, Hq, Hkv, D, max(lens) + 1, B, kvd, base)
    old = os.environ.pop("TL_DECODE_CLUSTER", None)
    try:
        caches = fill_cache(torch, _lib, h, 0, lens, Hkv, D, rng, base, kvd)
        q = randn(rng, B, Hq * D)
        pos = np.array([L - 1 for L in lens], np.int32)
        dq = torch.from_numpy(q).cuda()
        dpos = torch.from_numpy(pos).cuda()
        f = pos.ctypes.data_as(C.c_void_p)
        outs = []
        for mode in ("1", "0"):
            os.environ["TL_DECODE_CLUSTER"] = mode
            o = torch.empty(B, Hq * D, device="cuda")
            for _ in range(2):  # a second call reuses the barriers and counters
                _lib.check(_lib.lib.tl_decode_attention(h, 0, 0, B, ptr(dpos), f, ptr(dq), ptr(o), None))
            _lib.check(_lib.lib.tl_check_device(h, None))
            outs.append(o.cpu().numpy())
        for b, L in enumerate(lens):
            kc, vc = caches[b]
            qb = q[b].reshape(-1, 1)
            ref = ora.attention_cached(qb, kc, vc, L, Hq, Hkv, D)
            exact = numpy_ref.attention(qb, kc, vc, Hq, Hkv, D, np.array([L - 1]), L) if L >= 1024 else None
            for got in outs:
                err, allowed = parity(got[b].reshape(-1, 1), ref, exact, TOL_F32 if kvd == 0 else TOL_BF16)
                assert err <= allowed, (b, L, err, allowed)
        # the two modes sum in a different order (chunk boundaries, merge tree): f32 results
        # agree to the f32 bound, bf16 ones (same hi/lo rounding of q and p) to 1e-3
        assert max_rel_err(outs[0], outs[1]) < (TOL_F32 if kvd == 0 else 1e-3)
    finally:
        _lib.lib.tl_attn_destroy(h)
        os.environ.pop("TL_DECODE_CLUSTER", None)
        if old is not None:
            os.environ["TL_DECODE_CLUSTER"] = old


@pytest.mark.parametrize("kvd,Hq,Hkv,D,ropeDim,lens", [
    (0, 32, 4, 64, 64, [128]),               # TinyLlama batch 1 (f32 cache, tf32 tensor-core path)
    (0, 32, 4, 64, 64, [2048]),
    (0, 32, 4, 64, 32, [64, 257]),           # partial rotary; new rows at tile boundaries
    (1, 32, 8, 128, 128, [100, 700, 1]),     # bf16 cache, head_dim 128, a one-position sequence
    (1, 8, 8, 64, 64, [255, 256]),           # G = 1
])
def test_decode_step_fused_equals_two_launches(env, kvd, Hq, Hkv, D, ropeDim, lens):
    """In cluster mode tl_decode_step runs as one launch: the decode kernel rotates q and the new
    k at the step's position and writes k and v into the cache itself.  TL_DECODE_FUSE=0 runs
    the RoPE/append kernel first, as before.  Both must give the same bits: the output, q and k
    rotated in place, and the cache (the new row and everything else)."""
    torch, _lib = env
    rng = np.random.default_rng(sum(lens) + D + ropeDim)
    base = 10000.0
    B = len(lens)
    maxLen = max(lens) + 3
    pos = np.array(lens, np.int32)  # the new token sits at position L
    q, k, v = randn(rng, B, Hq * D), randn(rng, B, Hkv * D), randn(rng, B, Hkv * D)
    kc0, vc0 = randn(rng, B, maxLen, Hkv * D), randn(rng, B, maxLen, Hkv * D)
    results = []
    old = os.environ.pop("TL_DECODE_FUSE", None)
    try:
        for mode in ("1", "0"):
            os.environ["TL_DECODE_FUSE"] = mode
            h = C.c_void_p()
            _lib.check(_lib.lib.tl_attn_create(C.byref(h), 1, Hq, Hkv, D, ropeDim, base, maxLen, B, kvd, 0))
            try:
                for b in range(B):
                    kk, vv = torch.from_numpy(kc0[b]).cuda(), torch.from_numpy(vc0[b]).cuda()
                    _lib.check(_lib.lib.tl_kv_store(h, 0, b, 0, ptr(kk), ptr(vv), maxLen, None))
                dq, dk, dv = (torch.from_numpy(a.copy()).cuda() for a in (q, k, v))
                dpos = torch.from_numpy(pos).cuda()
                out = torch.empty(B, Hq * D, device="cuda")
                _lib.check(_lib.lib.tl_decode_step(h, 0, 0, B, ptr(dpos), pos.ctypes.data_as(C.c_void_p),
                                                   ptr(dq), ptr(dk), ptr(dv), ptr(out), None))
                _lib.check(_lib.lib.tl_check_device(h, None))
                caches = []
                for b in range(B):
                    kr = np.empty((Hkv * D, maxLen), np.float32)
                    vr = np.empty((Hkv * D, maxLen), np.float32)
                    _lib.check(_lib.lib.tl_kv_read(h, 0, b, kr.ctypes.data_as(C.c_void_p), vr.ctypes.data_as(C.c_void_p)))
                    caches.append((kr, vr))
                results.append((out.cpu().numpy(), dq.cpu().numpy(), dk.cpu().numpy(), caches))
            finally:
                _lib.lib.tl_attn_destroy(h)
    finally:
        os.environ.pop("TL_DECODE_FUSE", None)
        if old is not None:
            os.environ["TL_DECODE_FUSE"] = old
    (o1, q1, k1, c1), (o0, q0, k0, c0) = results
    assert np.array_equal(q1, q0) and np.array_equal(k1, k0)
    for b in range(B):
        assert np.array_equal(c1[b][0], c0[b][0]) and np.array_equal(c1[b][1], c0[b][1]), b
    assert np.array_equal(o1, o0), float(np.max(np.abs(o1 - o0)))
    # and the rotation is the reference's (applyRopeAtPos, src/forward.nim:125-139): within 2
    # ulps of the row's magnitude.  At one position a pair whose cos/sin differ from glibc's in
    # the last bit moves that pair in every head, so the bit-identical share is lower than over
    # many positions (1 pair in 32 is 3 %).
    from tests.helpers import rope_agrees
    for b, L in enumerate(lens):
        for got, x, H in ((q1[b], q[b], Hq), (k1[b], k[b], Hkv)):
            same, ulps = rope_agrees(got.reshape(-1, 1), ora.rope_at_pos(x.reshape(-1, 1), H, D, ropeDim, base, L))
            assert ulps <= 2 and same >= 0.9, (b, L, same, ulps)
