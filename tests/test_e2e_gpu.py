"""End-to-end TinyLlama-architecture greedy decode with the attention on the B200.

A llama GGUF is synthesised from a seed, with the TinyLlama-1.1B shapes:
* 22 layers, dim 2048, 32 q-heads and 4 kv-heads, head_dim 64;
* ffn 5632, vocab 32000, rope theta 1e4, rms eps 1e-5;
* N(0, 0.02) weights quantised to Q2_K;
* float32 RMSNorm weights of 1.0 and a float32 token embedding.

The C++ host forward pass (libtlhost.so) then runs the reference's runPrompt twice: once with
the B200 attention procs (libtlattn.so) and once with the oracle's.  The prompt is 8 random ids
in [3, 32000) followed by 16 greedy tokens, batch 1.

The generated ids must be identical.  Every attention output (each layer of the prefill and of
each decode step) is compared.  Its inputs come from the run's own earlier layers, so it carries
the upstream differences too; the bound on it is normwise.
"""
import os

import numpy as np
import pytest

from oracle import gguf_synth, oracle as ora
from tests.helpers import max_rel_err, normwise_err

pytestmark = pytest.mark.gpu

TINYLLAMA = dict(nLayer=22, nEmb=2048, nHead=32, nHeadKv=4, nFfn=5632, nVocab=32000)
SEED = 20261201


@pytest.fixture(scope="module")
def tinyllama(tmp_path_factory, cuda_lib):
    from tinylama_b200.host_api import Model
    path = str(tmp_path_factory.mktemp("gguf") / "tinyllama_synth.gguf")
    gguf_synth.write_model(path, seed=SEED, **TINYLLAMA)
    m = Model(path, nthreads=os.cpu_count() or 1)
    yield m
    m.close()


def _chunks(hp, n_prompt, n_new):
    hd = hp.nEmb // hp.nHead
    sizes = [hp.nHead * hd * n_prompt] * hp.nLayer + [hp.nHead * hd] * (hp.nLayer * (n_new - 1))
    return sizes


def test_tinyllama_greedy_ids_identical(tinyllama):
    from tinylama_b200 import host_api
    m = tinyllama
    prompt = np.random.default_rng(SEED).integers(3, 32000, size=8).astype(np.int32)
    ops_o = ora.lib().ora_attn_ops_create(m.hp.nLayer, m.hp.nHeadKv, m.hp.nEmb // m.hp.nHead)
    ops_g = host_api.gpu_attn_ops(m.hp)
    try:
        ids_o, gaps_o, dump_o = m.generate(ops_o, prompt, 16)
        ids_g, gaps_g, dump_g = m.generate(ops_g, prompt, 16)
    finally:
        ora.lib().ora_attn_ops_destroy(ops_o)
        host_api.free_gpu_attn_ops(ops_g)
    worst_norm, worst_floor, off = 0.0, 0.0, 0
    for size in _chunks(m.hp, 8, 16):
        a, b = dump_g[off:off + size], dump_o[off:off + size]
        worst_norm = max(worst_norm, normwise_err(a, b))
        worst_floor = max(worst_floor, max_rel_err(a, b))
        off += size
    assert off == dump_o.size == dump_g.size
    print(f"\nids {ids_g.tolist()}\nmin top-2 gap {gaps_o.min():.4f}; per-layer attention: "
          f"normwise {worst_norm:.2e}, floored elementwise {worst_floor:.2e}")
    assert worst_norm <= 1e-3, worst_norm
    assert np.array_equal(ids_g, ids_o), (ids_g, ids_o, gaps_o)


def test_tinyllama_repl_lines_chunked(tinyllama):
    """The REPL (src/tinylama.nim:45-100): three lines on one cache.  The reference feeds a later
    line token by token through forwardDecode (:70-73); the B200 table also takes it in one
    pass at positions curLen.. (prefill_at = tl_prefill_layer_at_host).  Ids of all three runs
    (oracle per token, B200 per token, B200 chunked) must be identical, and the chunked run's
    attention outputs, reordered per token, agree with the oracle's."""
    from tinylama_b200 import host_api
    m = tinyllama
    hp = m.hp
    width = hp.nHead * (hp.nEmb // hp.nHead)
    rng = np.random.default_rng(SEED + 1)
    lines = [rng.integers(3, 32000, size=n).astype(np.int32) for n in (8, 5, 6)]
    n_new = 4
    ops_o = ora.lib().ora_attn_ops_create(hp.nLayer, hp.nHeadKv, hp.nEmb // hp.nHead)
    ops_g = host_api.gpu_attn_ops(hp)
    runs = {}
    try:
        for name, ops, chunked in (("oracle", ops_o, False), ("b200", ops_g, False), ("b200_chunked", ops_g, True)):
            m.session_init(ops, n_new)
            runs[name] = [m.run_prompt(ops, line, n_new, chunked=chunked) for line in lines]
    finally:
        ora.lib().ora_attn_ops_destroy(ops_o)
        host_api.free_gpu_attn_ops(ops_g)
    worst = 0.0
    for li, line in enumerate(lines):
        ids_o, gaps_o, dump_o = runs["oracle"][li]
        for name in ("b200", "b200_chunked"):
            assert np.array_equal(runs[name][li][0], ids_o), (name, li, runs[name][li][0], ids_o, gaps_o)
        dump_c = runs["b200_chunked"][li][2]
        if li > 0:
            S = len(line)
            head = dump_c[:hp.nLayer * width * S].reshape(hp.nLayer, width, S).transpose(2, 0, 1).reshape(-1)
            dump_c = np.concatenate([head, dump_c[hp.nLayer * width * S:]])
        assert dump_c.size == dump_o.size
        # per layer: the first line's prefill outputs [width, S], then one column per token
        sizes = ([width * len(line)] * hp.nLayer if li == 0 else []) + \
            [width] * ((dump_o.size - (hp.nLayer * width * len(line) if li == 0 else 0)) // width)
        off = 0
        for size in sizes:
            worst = max(worst, normwise_err(dump_c[off:off + size], dump_o[off:off + size]))
            off += size
        assert off == dump_o.size
    print(f"\nREPL ids {[r[0].tolist() for r in runs['oracle']]}; chunked attention normwise {worst:.2e}")
    assert worst <= 1e-3, worst


def test_tinyllama_whole_model_on_gpu(tinyllama):
    """The whole forward pass on the B200 (tl_model.h: Q2_K weights resident in HBM, the decode
    steps replayed from a CUDA graph) against the reference-equivalent pipeline (C++ host
    linears in float32, the oracle's attention): the same 8-token prompt and 16 greedy ids."""
    import time
    m = tinyllama
    prompt = np.random.default_rng(SEED).integers(3, 32000, size=8).astype(np.int32)
    ops_o = ora.lib().ora_attn_ops_create(m.hp.nLayer, m.hp.nHeadKv, m.hp.nEmb // m.hp.nHead)
    try:
        t0 = time.perf_counter()
        ids_o, gaps_o, _ = m.generate(ops_o, prompt, 16, dump=False)
        cpu_s = time.perf_counter() - t0
    finally:
        ora.lib().ora_attn_ops_destroy(ops_o)
    g = m.to_gpu(max_len=48)
    try:
        ids_g, gaps_g = g.generate(prompt, 16)
        ids_g2, _ = g.generate(prompt, 16)
        pre_ms, dec_ms = g.last_timing()
    finally:
        g.close()
    print(f"\nwhole model on the GPU: ids {ids_g.tolist()}; prefill {pre_ms:.3f} ms, "
          f"{dec_ms / 15 * 1e3:.1f} us per decode step; CPU pipeline {cpu_s:.2f} s for 24 tokens; "
          f"largest gap difference {float(np.max(np.abs(gaps_g - gaps_o))):.2e}")
    assert np.array_equal(ids_g, ids_g2)
    assert np.array_equal(ids_g, ids_o), (ids_g, ids_o, gaps_o)
    assert float(np.max(np.abs(gaps_g - gaps_o))) <= 1e-2 * max(1.0, float(np.max(np.abs(gaps_o))))
