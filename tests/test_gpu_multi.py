"""Split-KV decode across 2, 4 and 8 GPUs (tl_decode_attention_dist: the decode kernel stores each
(sequence, head) result into every rank's buffer over NVLink as epoch-tagged words and merges them
as they arrive) against the single-GPU decode over the whole context, on B200s; each count runs
when the box has that many GPUs.  One process per GPU, spawned; the NCCL id (used once, to
exchange the IPC handles) is created in the parent.  Three calls in a row with different
queries exercise both halves of the double-buffered exchange and the epoch tags, and with 4 or 8
ranks the shorter sequence leaves the last ranks' slices empty."""
import ctypes as C
import multiprocessing as mp
import os
import sys

import numpy as np
import pytest

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _ngpus() -> int:
    import torch
    return torch.cuda.device_count()


def _worker(rank, nranks, uid, kvd, L, out_q):
    sys.path.insert(0, ROOT)
    import torch
    from tinylama_b200 import _lib
    torch.cuda.set_device(rank)
    B, Hq, Hkv, D = 2, 32, 8, 128
    sl = L // nranks
    rng = np.random.default_rng(7 + kvd)
    k = rng.standard_normal((B, L, Hkv * D), dtype=np.float32)
    v = rng.standard_normal((B, L, Hkv * D), dtype=np.float32)
    qs = [rng.standard_normal((B, Hq * D), dtype=np.float32) for _ in range(3)]
    lens = [L - 1, L // 2 - 3]  # the second sequence ends in the first half of the ranks' slices
    p = lambda t: C.c_void_p(t.data_ptr())
    h = C.c_void_p()
    _lib.check(_lib.lib.tl_attn_create(C.byref(h), 1, Hq, Hkv, D, D, 500000.0, sl, B, kvd, rank))
    try:
        for b in range(B):
            kk = torch.from_numpy(np.ascontiguousarray(k[b, rank * sl:(rank + 1) * sl])).cuda()
            vv = torch.from_numpy(np.ascontiguousarray(v[b, rank * sl:(rank + 1) * sl])).cuda()
            _lib.check(_lib.lib.tl_kv_store(h, 0, b, 0, p(kk), p(vv), sl, None))
        _lib.check(_lib.lib.tl_dist_init(h, C.create_string_buffer(uid, 128), nranks, rank))
        pos = np.array(lens, np.int32)
        dpos = torch.from_numpy(pos).cuda()
        dqs = [torch.from_numpy(q).cuda() for q in qs]
        outs = [torch.empty(B, Hq * D, device="cuda") for _ in qs]
        for dq, out in zip(dqs, outs):  # back to back, no host synchronisation in between
            _lib.check(_lib.lib.tl_decode_attention_dist(h, 0, 0, B, p(dpos), pos.ctypes.data_as(C.c_void_p),
                                                         p(dq), p(out), None))
        _lib.check(_lib.lib.tl_check_device(h, None))
        got = [out.cpu().numpy() for out in outs]
        ref = None
        if rank == 0:  # whole context on one GPU
            h1 = C.c_void_p()
            _lib.check(_lib.lib.tl_attn_create(C.byref(h1), 1, Hq, Hkv, D, D, 500000.0, L, B, kvd, rank))
            for b in range(B):
                kk = torch.from_numpy(np.ascontiguousarray(k[b])).cuda()
                vv = torch.from_numpy(np.ascontiguousarray(v[b])).cuda()
                _lib.check(_lib.lib.tl_kv_store(h1, 0, b, 0, p(kk), p(vv), L, None))
            ref = []
            for dq in dqs:
                o1 = torch.empty(B, Hq * D, device="cuda")
                _lib.check(_lib.lib.tl_decode_attention(h1, 0, 0, B, p(dpos), pos.ctypes.data_as(C.c_void_p),
                                                        p(dq), p(o1), None))
                _lib.check(_lib.lib.tl_check_device(h1, None))
                ref.append(o1.cpu().numpy())
            _lib.lib.tl_attn_destroy(h1)
        out_q.put((rank, got, ref, None))
    except Exception as e:  # report, never hang the parent
        out_q.put((rank, None, None, repr(e)))
    finally:
        _lib.lib.tl_attn_destroy(h)


@pytest.mark.parametrize("cluster", ["1", "0"])
@pytest.mark.parametrize("nranks", [2, 4, 8])
@pytest.mark.parametrize("kvd", [0, 1])
def test_splitkv_gpus_match_one(cuda_lib, kvd, nranks, cluster):
    """Split-KV over nranks GPUs against the whole context on one.  At these sizes the decode
    kernel runs in cluster mode (one cluster per (sequence, kv-head)); TL_DECODE_CLUSTER=0
    runs the unit queue instead."""
    if _ngpus() < nranks:
        pytest.skip(f"needs {nranks} GPUs")
    _lib = cuda_lib
    uid = C.create_string_buffer(128)
    _lib.check(_lib.lib.tl_dist_unique_id(uid))
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    # spawned children take the parent's environment: set it for them, then put it back
    saved = {k: os.environ.get(k) for k in ("NCCL_NVLS_ENABLE", "TL_DECODE_CLUSTER")}
    os.environ.update(NCCL_NVLS_ENABLE="0", TL_DECODE_CLUSTER=cluster)
    procs = [ctx.Process(target=_worker, args=(r, nranks, uid.raw, kvd, 8192, q)) for r in range(nranks)]
    try:
        for pr in procs:
            pr.start()
    finally:
        for k, v in saved.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v
    results = {}
    try:
        for _ in range(nranks):
            rank, got, ref, err = q.get(timeout=180)
            assert err is None, (rank, err)
            results[rank] = (got, ref)
    finally:
        for pr in procs:
            pr.join(timeout=60)
            if pr.is_alive():
                pr.kill()
    refs = results[0][1]
    for rank in range(nranks):
        for i, (got, ref) in enumerate(zip(results[rank][0], refs)):
            assert np.allclose(got, ref, rtol=1e-4, atol=1e-5), (rank, i, float(np.max(np.abs(got - ref))))


def _skip_worker(rank, nranks, uid, out_q):
    """Rank 1 skips the second of four split-KV calls.  Rank 0's second call must end with the
    timeout bit of the device error word after TL_DIST_WAIT_MS; after tl_dist_resync on both
    ranks, calls three and four (both halves of the exchange buffer, one of them holding rank
    0's unread values of the failed call) must give the single-GPU result again."""
    sys.path.insert(0, ROOT)
    import torch
    from tinylama_b200 import _lib
    torch.cuda.set_device(rank)
    B, Hq, Hkv, D, L = 2, 32, 8, 128, 4096
    sl = L // nranks
    rng = np.random.default_rng(17)
    k = rng.standard_normal((B, L, Hkv * D), dtype=np.float32)
    v = rng.standard_normal((B, L, Hkv * D), dtype=np.float32)
    qs = [rng.standard_normal((B, Hq * D), dtype=np.float32) for _ in range(4)]
    lens = [L - 1, L // 2 + 5]
    p = lambda t: C.c_void_p(t.data_ptr())
    h = C.c_void_p()
    _lib.check(_lib.lib.tl_attn_create(C.byref(h), 1, Hq, Hkv, D, D, 500000.0, sl, B, 1, rank))
    res = {}
    try:
        for b in range(B):
            kk = torch.from_numpy(np.ascontiguousarray(k[b, rank * sl:(rank + 1) * sl])).cuda()
            vv = torch.from_numpy(np.ascontiguousarray(v[b, rank * sl:(rank + 1) * sl])).cuda()
            _lib.check(_lib.lib.tl_kv_store(h, 0, b, 0, p(kk), p(vv), sl, None))
        _lib.check(_lib.lib.tl_dist_init(h, C.create_string_buffer(uid, 128), nranks, rank))
        pos = np.array(lens, np.int32)
        dpos = torch.from_numpy(pos).cuda()
        f = pos.ctypes.data_as(C.c_void_p)
        outs = []
        for i, qh in enumerate(qs):
            if i == 2:  # both ranks recover before the third call
                _lib.check(_lib.lib.tl_dist_resync(h))
            dq = torch.from_numpy(qh).cuda()
            o = torch.zeros(B, Hq * D, device="cuda")
            if i == 1 and rank == 1:
                outs.append(None)
                continue
            _lib.check(_lib.lib.tl_decode_attention_dist(h, 0, 0, B, p(dpos), f, p(dq), p(o), None))
            rc = _lib.lib.tl_check_device(h, None)
            res[i] = (rc, _lib.lib.tl_last_error().decode() if rc else "")
            outs.append(o.cpu().numpy())
        ref = None
        if rank == 0:
            h1 = C.c_void_p()
            _lib.check(_lib.lib.tl_attn_create(C.byref(h1), 1, Hq, Hkv, D, D, 500000.0, L, B, 1, rank))
            for b in range(B):
                kk = torch.from_numpy(np.ascontiguousarray(k[b])).cuda()
                vv = torch.from_numpy(np.ascontiguousarray(v[b])).cuda()
                _lib.check(_lib.lib.tl_kv_store(h1, 0, b, 0, p(kk), p(vv), L, None))
            ref = []
            for qh in qs:
                o1 = torch.empty(B, Hq * D, device="cuda")
                _lib.check(_lib.lib.tl_decode_attention(h1, 0, 0, B, p(dpos), f, p(torch.from_numpy(qh).cuda()),
                                                        p(o1), None))
                _lib.check(_lib.lib.tl_check_device(h1, None))
                ref.append(o1.cpu().numpy())
            _lib.lib.tl_attn_destroy(h1)
        out_q.put((rank, res, outs, ref, None))
    except Exception as e:  # report, never hang the parent
        out_q.put((rank, None, None, None, repr(e)))
    finally:
        _lib.lib.tl_attn_destroy(h)


def test_splitkv_rank_skips_a_call_then_resyncs(cuda_lib):
    if _ngpus() < 2:
        pytest.skip("needs 2 GPUs")
    _lib = cuda_lib
    uid = C.create_string_buffer(128)
    _lib.check(_lib.lib.tl_dist_unique_id(uid))
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    saved = {k: os.environ.get(k) for k in ("NCCL_NVLS_ENABLE", "TL_DIST_WAIT_MS")}
    os.environ.update(NCCL_NVLS_ENABLE="0", TL_DIST_WAIT_MS="300")
    procs = [ctx.Process(target=_skip_worker, args=(r, 2, uid.raw, q)) for r in range(2)]
    try:
        for pr in procs:
            pr.start()
    finally:
        for k, v in saved.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v
    results = {}
    try:
        for _ in range(2):
            rank, res, outs, ref, err = q.get(timeout=180)
            assert err is None, (rank, err)
            results[rank] = (res, outs, ref)
    finally:
        for pr in procs:
            pr.join(timeout=60)
            if pr.is_alive():
                pr.kill()
    res0, outs0, refs = results[0]
    res1, outs1, _ = results[1]
    assert res0[0][0] == 0 and res1[0][0] == 0
    assert res0[1][0] == _lib.TL_ERR_DEVICE and "wait-timeout" in res0[1][1], res0[1]
    for i in (0, 2, 3):
        assert res0[i][0] == 0 and res1[i][0] == 0, (i, res0.get(i), res1.get(i))
        for outs in (outs0, outs1):
            assert np.allclose(outs[i], refs[i], rtol=1e-4, atol=1e-5), (i, float(np.max(np.abs(outs[i] - refs[i]))))
