"""The whole forward pass on the B200 (include/tl_model.h) on a small synthetic llama model:
greedy ids and top-2 logit gaps against the independent numpy forward (float64 linears over the
reference's dequantised weights), and the errors the reference raises."""
import numpy as np
import pytest

from oracle import gguf_synth
from tests.e2e_numpy import NumpyModel

pytestmark = pytest.mark.gpu

SMALL = dict(nLayer=2, nEmb=256, nHead=4, nHeadKv=2, nFfn=512, nVocab=512)


@pytest.fixture(scope="module")
def small(tmp_path_factory, cuda_lib):
    from tinylama_b200.host_api import Model
    keep = {}
    path = str(tmp_path_factory.mktemp("gguf") / "small.gguf")
    gguf_synth.write_model(path, seed=7, keep=keep, **SMALL)
    t = {}
    for name, (ne, typ, raw) in keep.items():
        n = int(np.prod(ne))
        a = np.frombuffer(raw, np.float32) if typ == 0 else gguf_synth.dequantize_q2k(raw, n)
        t[name] = a.reshape(ne[::-1]) if len(ne) == 2 else a
    npm = NumpyModel(t, dict(nLayer=2, nEmb=256, nHead=4, nHeadKv=2, base=10000.0, eps=1e-5))
    m = Model(path, nthreads=2)
    yield m, npm
    m.close()


@pytest.mark.parametrize("n_prompt,n_new", [(8, 6), (1, 4), (5, 1)])
def test_generate_matches_numpy(small, n_prompt, n_new):
    """runPrompt on the device: prompt of 1 to 8 tokens (the prefill runs its matrix products 4
    tokens at a time), the first decode step eagerly, the others from the captured graph."""
    m, npm = small
    prompt = np.random.default_rng(n_prompt).integers(3, 512, size=n_prompt).astype(np.int32)
    g = m.to_gpu(max_len=max(32, n_new + 32))
    try:
        ids, gaps = g.generate(prompt, n_new)
        ids2, gaps2 = g.generate(prompt, n_new)  # the cached graph, the same answer
    finally:
        g.close()
    nids, ngaps, _ = npm.generate(prompt, n_new, max(32, n_new + 32))
    assert np.array_equal(ids, ids2) and np.array_equal(gaps, gaps2)
    for j in range(n_new):
        if ngaps[j] > 1e-3:  # not a float32 near-tie
            assert ids[j] == nids[j], (j, ids, nids, ngaps)
            assert abs(gaps[j] - ngaps[j]) <= 1e-3 * max(1.0, abs(ngaps[j])), (j, gaps, ngaps)
        else:
            break


def test_mapped_file_uploads_the_same_model(small, tmp_path):
    """Weights uploaded straight from the mapped GGUF (no float32 copy on the host) give the
    same greedy ids and gaps as those from the loaded model."""
    from tinylama_b200.host_api import Model
    m, _ = small
    path = str(tmp_path / "small.gguf")
    gguf_synth.write_model(path, seed=7, **SMALL)
    prompt = np.random.default_rng(4).integers(3, 512, size=6).astype(np.int32)
    mm = Model(path, mapped=True)
    g1, g2 = m.to_gpu(max_len=32), mm.to_gpu(max_len=32)
    try:
        ids1, gaps1 = g1.generate(prompt, 5)
        ids2, gaps2 = g2.generate(prompt, 5)
    finally:
        g1.close()
        g2.close()
        mm.close()
    assert np.array_equal(ids1, ids2) and np.array_equal(gaps1, gaps2)


def test_logits_match_numpy(small):
    """The logits of the prefill's last token against the numpy forward."""
    m, npm = small
    prompt = np.random.default_rng(11).integers(3, 512, size=7).astype(np.int32)
    g = m.to_gpu(max_len=32)
    try:
        g.generate(prompt, 1)
        got = g.last_logits()
    finally:
        g.close()
    kvDim = 2 * 64
    kc = [np.zeros((kvDim, 32), np.float32) for _ in range(2)]
    vc = [np.zeros((kvDim, 32), np.float32) for _ in range(2)]
    ref = npm.forward(list(prompt), kc, vc, 0, [])[:, -1]
    err = float(np.max(np.abs(got - ref)) / np.max(np.abs(ref)))
    assert err <= 1e-4, err


def test_partial_rotary_matches_numpy(tmp_path, cuda_lib):
    """ropeDim < headDim (llama.rope.dimension_count = 32 of 64): the decode step's fused
    q/k/v + RoPE rotates only the first 32 dims of each head, as applyRopeAtPos does."""
    from tinylama_b200.host_api import Model
    keep = {}
    path = str(tmp_path / "rope32.gguf")
    gguf_synth.write_model(path, seed=9, keep=keep, ropeDim=32, **SMALL)
    t = {}
    for name, (ne, typ, raw) in keep.items():
        n = int(np.prod(ne))
        a = np.frombuffer(raw, np.float32) if typ == 0 else gguf_synth.dequantize_q2k(raw, n)
        t[name] = a.reshape(ne[::-1]) if len(ne) == 2 else a
    npm = NumpyModel(t, dict(nLayer=2, nEmb=256, nHead=4, nHeadKv=2, base=10000.0, eps=1e-5, ropeDim=32))
    m = Model(path, nthreads=2)
    assert m.hp.ropeDim == 32
    prompt = np.random.default_rng(5).integers(3, 512, size=5).astype(np.int32)
    g = m.to_gpu(max_len=32)
    try:
        ids, gaps = g.generate(prompt, 6)
    finally:
        g.close()
        m.close()
    nids, ngaps, _ = npm.generate(prompt, 6, 32)
    for j in range(6):
        if ngaps[j] > 1e-3:
            assert ids[j] == nids[j], (j, ids, nids, ngaps)
            assert abs(gaps[j] - ngaps[j]) <= 1e-3 * max(1.0, abs(ngaps[j])), (j, gaps, ngaps)
        else:
            break


def test_float32_matrices_take_the_generic_kernel(tmp_path, cuda_lib):
    """A model whose wo, ffn_down and output matrices are float32 (as a loader hands over any
    type other than Q2_K): those products run in the generic kernel, the others in the Q2_K
    one, and the result still matches numpy."""
    from tinylama_b200.host_api import Model
    keep = {}
    path = str(tmp_path / "mixed.gguf")
    gguf_synth.write_model(path, seed=13, keep=keep, f32=("attn_output.weight", "ffn_down.weight", "output.weight"),
                           **SMALL)
    t = {}
    for name, (ne, typ, raw) in keep.items():
        n = int(np.prod(ne))
        a = np.frombuffer(raw, np.float32) if typ == 0 else gguf_synth.dequantize_q2k(raw, n)
        t[name] = a.reshape(ne[::-1]) if len(ne) == 2 else a
    npm = NumpyModel(t, dict(nLayer=2, nEmb=256, nHead=4, nHeadKv=2, base=10000.0, eps=1e-5))
    m = Model(path, nthreads=2)
    prompt = np.random.default_rng(6).integers(3, 512, size=6).astype(np.int32)
    g = m.to_gpu(max_len=32)
    try:
        ids, gaps = g.generate(prompt, 5)
    finally:
        g.close()
        m.close()
    nids, ngaps, _ = npm.generate(prompt, 5, 32)
    for j in range(5):
        if ngaps[j] > 1e-3:
            assert ids[j] == nids[j], (j, ids, nids, ngaps)
            assert abs(gaps[j] - ngaps[j]) <= 1e-3 * max(1.0, abs(ngaps[j])), (j, gaps, ngaps)
        else:
            break


def test_errors_follow_the_reference(small):
    m, _ = small
    g = m.to_gpu(max_len=10)
    try:
        prompt = np.arange(3, 11, dtype=np.int32)
        with pytest.raises(ValueError, match="KV cache full"):
            g.generate(prompt, 4)  # 8 + 3 positions > 10
        with pytest.raises(ValueError, match="out of range"):
            g.generate(np.array([3, 512], np.int32), 1)
        ids, _ = g.generate(prompt, 3)  # 8 + 2 = 10 fits
        assert ids.shape == (3,)
    finally:
        g.close()
