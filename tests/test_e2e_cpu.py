"""The end-to-end harness on the CPU: the synthetic GGUF writer and its Q2_K quantiser against
the reference's dequantiser, the C++ loader (libtlhost.so), and the C++ forward pass with the
oracle's attention procs against an independent numpy forward, on a small llama model."""
import ctypes as C
import os

import numpy as np
import pytest

from oracle import gguf_synth, oracle as ora
from tests.e2e_numpy import NumpyModel

SMALL = dict(nLayer=2, nEmb=256, nHead=4, nHeadKv=2, nFfn=512, nVocab=512)


@pytest.fixture(scope="module")
def small_model(tmp_path_factory):
    keep = {}
    path = str(tmp_path_factory.mktemp("gguf") / "small.gguf")
    gguf_synth.write_model(path, seed=7, keep=keep, **SMALL)
    return path, keep


def test_q2k_quantiser_round_trip():
    rng = np.random.default_rng(0)
    x = rng.standard_normal(256 * 64, dtype=np.float32) * np.float32(0.02)
    raw = gguf_synth.quantize_q2k(x)
    assert len(raw) == 64 * 84
    y = gguf_synth.dequantize_q2k(raw, x.size)
    # per 16-value sub-block the grid step is <= (max-min)/3 plus the 4-bit scale rounding
    err = np.abs(y - x).reshape(-1, 16).max(axis=1)
    rng16 = (x.reshape(-1, 16).max(axis=1) - np.minimum(x.reshape(-1, 16).min(axis=1), 0))
    assert np.all(err <= rng16 * 0.75 + 1e-6)
    assert float(np.sqrt(np.mean((y - x) ** 2))) < 0.5 * 0.02


def test_loader_matches_reference_dequant(small_model):
    from tinylama_b200.host_api import Model
    path, keep = small_model
    m = Model(path, nthreads=2)
    hp = m.hp
    assert (hp.nVocab, hp.nEmb, hp.nLayer, hp.nFfn, hp.nHead, hp.nHeadKv, hp.ropeDim) == (512, 256, 2, 512, 4, 2, 64)
    assert abs(hp.ropeFreqBase - 10000.0) < 1e-3 and abs(hp.rmsEps - 1e-5) < 1e-9
    for name in ("blk.0.attn_q.weight", "blk.1.ffn_down.weight", "output.weight", "token_embd.weight"):
        ne, typ, raw = keep[name]
        n = int(np.prod(ne))
        expect = np.frombuffer(raw, np.float32) if typ == 0 else gguf_synth.dequantize_q2k(raw, n)
        assert np.array_equal(m.tensor(name), expect), name
    m.close()


def _numpy_model(keep, seed_hp):
    t = {}
    for name, (ne, typ, raw) in keep.items():
        n = int(np.prod(ne))
        a = np.frombuffer(raw, np.float32) if typ == 0 else gguf_synth.dequantize_q2k(raw, n)
        t[name] = a.reshape(ne[::-1]) if len(ne) == 2 else a
    return NumpyModel(t, seed_hp)


def test_forward_with_oracle_attention_matches_numpy(small_model):
    from tinylama_b200.host_api import Model
    path, keep = small_model
    m = Model(path, nthreads=2)
    ops = ora.lib().ora_attn_ops_create(m.hp.nLayer, m.hp.nHeadKv, m.hp.nEmb // m.hp.nHead)
    try:
        prompt = np.random.default_rng(1).integers(3, 512, size=8).astype(np.int32)
        ids, gaps, dump = m.generate(ops, prompt, 6)
        ids2, _, dump2 = m.generate(ops, prompt, 6)
        assert np.array_equal(ids, ids2) and np.array_equal(dump, dump2)  # deterministic
        npm = _numpy_model(keep, dict(nLayer=2, nEmb=256, nHead=4, nHeadKv=2, base=10000.0, eps=1e-5))
        nids, ngaps, ndump = npm.generate(prompt, 6, 38)
        ref = np.concatenate([d.reshape(-1) for d in ndump])
        assert ref.size == dump.size
        assert np.max(np.abs(dump - ref)) <= 1e-3 * np.max(np.abs(ref))
        for j in range(6):  # ids agree wherever the top-2 gap is not a float32 near-tie
            if ngaps[j] > 1e-3:
                assert ids[j] == nids[j], (j, ids, nids, ngaps)
            else:
                break
    finally:
        ora.lib().ora_attn_ops_destroy(ops)
        m.close()


def test_forward_errors_follow_the_reference(small_model):
    from tinylama_b200 import host_api
    with pytest.raises(ValueError, match="cannot open"):
        host_api.Model("/nonexistent/model.gguf")
