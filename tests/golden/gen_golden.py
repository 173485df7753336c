"""Generate the golden fixtures in tests/golden/ from the C oracle (oracle/attn_oracle.c).

The reference (Nim) cannot run on these machines and ships no golden vectors for this path,
so these fixtures pin the oracle against itself across changes (and against the numpy
restatement in tests/numpy_ref.py); they are not outputs of the reference.  Inputs are seeded
N(0,1) float32 at TinyLlama shapes (32 q-heads, 4 kv-heads, head_dim 64, rope theta 1e4) and
at Llama-3 long-context RoPE (theta 5e5, positions up to 131071).

    python tests/golden/gen_golden.py      # rewrites tests/golden/attn_small.npz
"""
from __future__ import annotations

import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
from oracle import oracle as ora  # noqa: E402

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "attn_small.npz")


def make() -> dict[str, np.ndarray]:
    rng = np.random.default_rng(20261201)
    f = {}
    Hq, Hkv, D, base = 32, 4, 64, 10000.0
    # applyRopeSingle on q and k, S = 8
    S = 8
    f["rope_single_q_in"] = rng.standard_normal((Hq * D, S)).astype(np.float32)
    f["rope_single_q_out"] = ora.rope_single(f["rope_single_q_in"], Hq, D, D, base)
    # applyRopeAtPos at three positions, including long-context ones
    for name, pos, b in (("p37", 37, 10000.0), ("p4095", 4095, 10000.0), ("p131071", 131071, 500000.0)):
        x = rng.standard_normal((Hkv * D, 1)).astype(np.float32)
        f[f"rope_at_{name}_in"] = x
        f[f"rope_at_{name}_out"] = ora.rope_at_pos(x, Hkv, D, D, b, pos)
    # attentionFull ctx over S = 8 fresh projections
    q = rng.standard_normal((Hq * D, S)).astype(np.float32)
    k = rng.standard_normal((Hkv * D, S)).astype(np.float32)
    v = rng.standard_normal((Hkv * D, S)).astype(np.float32)
    f["full_q"], f["full_k"], f["full_v"] = q, k, v
    f["full_ctx"] = ora.attention_full_ctx(q, k, v, Hq, Hkv, D)
    # attentionCached over a 24-column cache of maxLen 32
    maxLen, L = 32, 24
    kc = np.zeros((Hkv * D, maxLen), np.float32)
    vc = np.zeros((Hkv * D, maxLen), np.float32)
    kn = rng.standard_normal((Hkv * D, L)).astype(np.float32)
    vn = rng.standard_normal((Hkv * D, L)).astype(np.float32)
    ora.store_kv_range(kc, vc, 0, kn, vn)
    qd = rng.standard_normal((Hq * D, 1)).astype(np.float32)
    f["cached_k"], f["cached_v"], f["cached_q"] = kc, vc, qd
    f["cached_ctx"] = ora.attention_cached(qd, kc, vc, L, Hq, Hkv, D)
    return f


def main() -> None:
    f = make()
    np.savez_compressed(OUT, **f)
    print(OUT, sum(a.nbytes for a in f.values()), "bytes")


if __name__ == "__main__":
    main()
