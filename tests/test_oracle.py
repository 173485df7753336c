"""The oracle (C restatement of src/forward.nim's attention procs) checked on the CPU:
analytic known answers, an independent numpy restatement, and the committed golden fixtures."""
import os

import numpy as np
import pytest

from oracle import oracle as ora
from tests.helpers import max_rel_err, randn
from tests import numpy_ref

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "attn_small.npz")


def test_rope_position_zero_is_identity():
    rng = np.random.default_rng(0)
    x = randn(rng, 4 * 64, 1)
    assert np.array_equal(ora.rope_at_pos(x, 4, 64, 64, 10000.0, 0), x)


def test_rope_single_column_p_uses_position_p():
    # applyRopeSingle rotates column p at position p (forward.nim:112-117)
    rng = np.random.default_rng(1)
    x = randn(rng, 2 * 64, 5)
    y = ora.rope_single(x, 2, 64, 64, 10000.0)
    for p in range(5):
        col = np.ascontiguousarray(x[:, p:p + 1])
        assert np.array_equal(y[:, p:p + 1], ora.rope_at_pos(col, 2, 64, 64, 10000.0, p))


def test_rope_preserves_pair_norms_and_skips_unrotated_dims():
    rng = np.random.default_rng(2)
    x = randn(rng, 3 * 64, 1)
    y = ora.rope_at_pos(x, 3, 64, 32, 10000.0, 1234)  # ropeDim 32 < headDim 64
    for h in range(3):
        for i in range(16):
            a = x[h * 64 + 2 * i:h * 64 + 2 * i + 2, 0].astype(np.float64)
            b = y[h * 64 + 2 * i:h * 64 + 2 * i + 2, 0].astype(np.float64)
            assert abs(np.hypot(*a) - np.hypot(*b)) < 1e-5 * max(1.0, np.hypot(*a))
        assert np.array_equal(y[h * 64 + 32:h * 64 + 64], x[h * 64 + 32:h * 64 + 64])


def test_rope_theta_is_float32_powf():
    th = np.float32(1.0) / np.float32(10000.0)
    for i in (0, 1, 7, 31):
        expect = np.float32(np.power(np.float64(th), np.float64(np.float32(2 * i) / np.float32(64))))
        assert abs(ora.rope_theta(i, 64, 10000.0) - expect) <= np.spacing(expect)


def test_rope_matches_numpy_restatement():
    rng = np.random.default_rng(3)
    x = randn(rng, 4 * 64, 16)
    y = ora.rope_single(x, 4, 64, 64, 10000.0)
    r = numpy_ref.rope_cols(x, 4, 64, 64, 10000.0, np.arange(16))
    assert np.max(np.abs(y - r)) < 1e-5


def test_store_kv_range_layout():
    rng = np.random.default_rng(4)
    kc = np.zeros((8, 10), np.float32)
    vc = np.zeros((8, 10), np.float32)
    k, v = randn(rng, 8, 3), randn(rng, 8, 3)
    ora.store_kv_range(kc, vc, 4, k, v)
    assert np.array_equal(kc[:, 4:7], k) and np.array_equal(vc[:, 4:7], v)
    assert not kc[:, :4].any() and not kc[:, 7:].any()


def test_attention_cached_single_position_returns_v():
    rng = np.random.default_rng(5)
    Hq, Hkv, D = 8, 2, 64
    kc, vc = randn(rng, Hkv * D, 16), randn(rng, Hkv * D, 16)
    q = randn(rng, Hq * D, 1)
    ctx = ora.attention_cached(q, kc, vc, 1, Hq, Hkv, D)
    for h in range(Hq):
        kvh = h // (Hq // Hkv)
        assert np.array_equal(ctx[h * D:(h + 1) * D, 0], vc[kvh * D:(kvh + 1) * D, 0])


def test_attention_cached_equal_keys_average_v():
    rng = np.random.default_rng(6)
    Hq, Hkv, D, L = 4, 4, 64, 7
    kc = np.tile(randn(rng, Hkv * D, 1), (1, L))
    vc = randn(rng, Hkv * D, L)
    ctx = ora.attention_cached(randn(rng, Hq * D, 1), kc, vc, L, Hq, Hkv, D)
    assert np.max(np.abs(ctx[:, 0] - vc.mean(axis=1))) < 1e-5


@pytest.mark.parametrize("Hq,Hkv,D,L", [(32, 4, 64, 128), (32, 32, 128, 300), (32, 8, 128, 77)])
def test_attention_cached_matches_numpy(Hq, Hkv, D, L):
    rng = np.random.default_rng(Hq + Hkv + D + L)
    kc, vc = randn(rng, Hkv * D, L + 5), randn(rng, Hkv * D, L + 5)
    q = randn(rng, Hq * D, 1)
    ctx = ora.attention_cached(q, kc, vc, L, Hq, Hkv, D)
    r = numpy_ref.attention(q, kc, vc, Hq, Hkv, D, np.array([L - 1]), L)
    assert max_rel_err(ctx, r) < 5e-4  # float32 sequential sums vs float64


@pytest.mark.parametrize("Hq,Hkv,D,S", [(32, 4, 64, 8), (32, 8, 64, 33), (4, 4, 128, 20)])
def test_attention_full_matches_numpy(Hq, Hkv, D, S):
    rng = np.random.default_rng(S)
    q, k, v = randn(rng, Hq * D, S), randn(rng, Hkv * D, S), randn(rng, Hkv * D, S)
    ctx = ora.attention_full_ctx(q, k, v, Hq, Hkv, D)
    r = numpy_ref.attention(q, k, v, Hq, Hkv, D, np.arange(S), S)
    assert max_rel_err(ctx, r) < 5e-4  # float32 sequential sums vs float64


def test_attention_full_with_wo_is_linear_of_ctx():
    rng = np.random.default_rng(7)
    Hq, Hkv, D, S, nEmb = 4, 2, 64, 5, 96
    q, k, v = randn(rng, Hq * D, S), randn(rng, Hkv * D, S), randn(rng, Hkv * D, S)
    wo = randn(rng, Hq * D, nEmb)
    out = ora.linear_ggml_col(ora.attention_full_ctx(q, k, v, Hq, Hkv, D), wo)
    ref = wo.reshape(nEmb, Hq * D).astype(np.float64) @ numpy_ref.attention(q, k, v, Hq, Hkv, D, np.arange(S), S)
    assert max_rel_err(out, ref) < 1e-3


def test_golden_fixtures_reproduce():
    g = np.load(GOLDEN)
    Hq, Hkv, D = 32, 4, 64
    assert np.array_equal(ora.rope_single(g["rope_single_q_in"], Hq, D, D, 10000.0), g["rope_single_q_out"])
    for name, pos, b in (("p37", 37, 10000.0), ("p4095", 4095, 10000.0), ("p131071", 131071, 500000.0)):
        assert np.array_equal(ora.rope_at_pos(g[f"rope_at_{name}_in"], Hkv, D, D, b, pos), g[f"rope_at_{name}_out"])
    assert np.array_equal(ora.attention_full_ctx(g["full_q"], g["full_k"], g["full_v"], Hq, Hkv, D), g["full_ctx"])
    assert np.array_equal(ora.attention_cached(g["cached_q"], g["cached_k"], g["cached_v"], 24, Hq, Hkv, D),
                          g["cached_ctx"])
    # and the fixtures agree with the independent restatement
    r = numpy_ref.attention(g["full_q"], g["full_k"], g["full_v"], Hq, Hkv, D, np.arange(8), 8)
    assert max_rel_err(g["full_ctx"], r) < 1e-4


def test_attention_cached_ignores_columns_past_curlen():
    """attentionCached reads columns j < curLen only (src/forward.nim:191-205): what the cache
    holds past them cannot change ctx."""
    rng = np.random.default_rng(12)
    Hq, Hkv, D, L, cap = 8, 2, 64, 40, 64
    kc, vc = randn(rng, Hkv * D, cap), randn(rng, Hkv * D, cap)
    q = randn(rng, Hq * D, 1)
    a = ora.attention_cached(q, kc, vc, L, Hq, Hkv, D)
    kc[:, L:] = 1e4
    vc[:, L:] = np.nan
    b = ora.attention_cached(q, kc, vc, L, Hq, Hkv, D)
    assert np.array_equal(a, b)


@pytest.mark.parametrize("Hq,Hkv,D,S", [(32, 4, 64, 9), (8, 8, 128, 5)])
def test_prefill_equals_one_decode_step_per_token(Hq, Hkv, D, S):
    """forwardPrefill's attention block over S tokens (RoPE over 0..S-1, store, attentionFull)
    against S forwardDecode blocks (RoPE at t, store at t, attentionCached over t+1 columns):
    the two procs do the same float32 arithmetic per query, so the columns agree exactly.  This
    is the equivalence the REPL path relies on when it feeds a later line in one pass."""
    rng = np.random.default_rng(S * 3 + D)
    base = 10000.0
    q, k, v = randn(rng, Hq * D, S), randn(rng, Hkv * D, S), randn(rng, Hkv * D, S)
    qr = ora.rope_single(q, Hq, D, D, base)
    kr = ora.rope_single(k, Hkv, D, D, base)
    full = ora.attention_full_ctx(qr, kr, v, Hq, Hkv, D)
    kc = np.zeros((Hkv * D, S), np.float32)
    vc = np.zeros((Hkv * D, S), np.float32)
    steps = [ora.decode_step(q[:, t:t + 1], k[:, t:t + 1], v[:, t:t + 1], kc, vc, t, Hq, Hkv, D, D, base)
             for t in range(S)]
    assert np.array_equal(kc, kr) and np.array_equal(vc, v)
    assert np.array_equal(np.concatenate(steps, axis=1), full)
