"""The split-KV partition and the (m, l, o) merge across two ranks on the CPU (gloo): each rank
attends its slice of the context with the same log2-domain partials the GPU kernels write, the
partials are all-gathered, merged, and compared with the oracle over the whole context."""
import os
import socket

import numpy as np
import pytest

from oracle import oracle as ora

LOG2E = 1.4426950408889634


def local_partial(q, k, v, Hq, Hkv, D, lo, hi):
    """(o, m, l) over positions [lo, hi) per q-head, m and l in the log2 domain, o un-normalised."""
    G = Hq // Hkv
    out = np.zeros((Hq, D + 2), np.float64)
    for h in range(Hq):
        g = h // G
        if hi <= lo:
            out[h, D] = -np.inf
            continue
        s = (k[g * D:(g + 1) * D, lo:hi].T.astype(np.float64) @ q[h * D:(h + 1) * D, 0]) * (LOG2E / np.sqrt(D))
        m = s.max()
        p = np.exp2(s - m)
        out[h, :D] = v[g * D:(g + 1) * D, lo:hi].astype(np.float64) @ p
        out[h, D], out[h, D + 1] = m, p.sum()
    return out


def merge(parts, D):
    M = np.max([p[:, D] for p in parts], axis=0)
    w = [np.where(np.isneginf(p[:, D]), 0.0, np.exp2(p[:, D] - M)) for p in parts]
    L = sum(p[:, D + 1] * wi for p, wi in zip(parts, w))
    O = sum(p[:, :D] * wi[:, None] for p, wi in zip(parts, w))
    return O / L[:, None]


def _rank(rank, world, port, ctx_len, result_path):
    import torch
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    Hq, Hkv, D = 8, 2, 64
    rng = np.random.default_rng(3)
    k = rng.standard_normal((Hkv * D, ctx_len), dtype=np.float32)
    v = rng.standard_normal((Hkv * D, ctx_len), dtype=np.float32)
    q = rng.standard_normal((Hq * D, 1), dtype=np.float32)
    sl = (ctx_len + world - 1) // world
    lo, hi = rank * sl, min(ctx_len, (rank + 1) * sl)
    mine = torch.from_numpy(local_partial(q, k, v, Hq, Hkv, D, lo, hi))
    gathered = [torch.zeros_like(mine) for _ in range(world)]
    dist.all_gather(gathered, mine)
    ctx = merge([t.numpy() for t in gathered], D)
    if rank == 0:
        ref = ora.attention_cached(q, k, v, ctx_len, Hq, Hkv, D).reshape(Hq, D)
        np.save(result_path, np.stack([ctx, ref]))
    dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("ctx_len", [1000, 3])
def test_splitkv_merge_two_gloo_ranks(tmp_path, ctx_len):
    import torch.multiprocessing as tmp
    path = str(tmp_path / "res.npy")
    tmp.spawn(_rank, args=(2, _free_port(), ctx_len, path), nprocs=2, join=True)
    ctx, ref = np.load(path)
    assert np.max(np.abs(ctx - ref)) / np.max(np.abs(ref)) < 1e-5


def _rank_never_exchanges(rank, world, port, result_path):
    """Rank 1 joins the group but never takes part in the exchange of partials.  Rank 0's
    exchange must end with an error once the group's timeout has passed, not wait for ever --
    the host-side counterpart of the bounded waits in the split-KV kernel."""
    import datetime
    import time

    import torch
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=3))
    Hq, Hkv, D, ctx_len = 8, 2, 64, 64
    rng = np.random.default_rng(3)
    k = rng.standard_normal((Hkv * D, ctx_len), dtype=np.float32)
    v = rng.standard_normal((Hkv * D, ctx_len), dtype=np.float32)
    q = rng.standard_normal((Hq * D, 1), dtype=np.float32)
    if rank == 1:
        time.sleep(8)  # alive, but never exchanges; leaves after rank 0 has given up
        return
    mine = torch.from_numpy(local_partial(q, k, v, Hq, Hkv, D, 0, ctx_len // 2))
    gathered = [torch.zeros_like(mine) for _ in range(world)]
    t0 = time.perf_counter()
    try:
        dist.all_gather(gathered, mine)
        outcome = "completed"
    except RuntimeError as e:
        outcome = "error: " + str(e).splitlines()[0][:200]
    np.save(result_path, np.array([outcome, f"{time.perf_counter() - t0:.2f}"]))


def test_splitkv_exchange_ends_in_an_error_when_a_rank_never_joins(tmp_path):
    import time

    import torch.multiprocessing as tmp
    path = str(tmp_path / "res.npy")
    t0 = time.perf_counter()
    tmp.spawn(_rank_never_exchanges, args=(2, _free_port(), path), nprocs=2, join=True)
    outcome, waited = np.load(path)
    assert outcome.startswith("error"), outcome
    assert float(waited) < 30.0 and time.perf_counter() - t0 < 120.0
