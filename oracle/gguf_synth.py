"""Synthetic GGUF model files for the end-to-end tests (TEST INFRASTRUCTURE ONLY).

Writes a llama-architecture GGUF v3 file from a seed.  The weight matrices are N(0, sigma)
quantised to Q2_K, the RMSNorm weights are float32 ones, and the token embedding is float32
N(0, sigma).  The file holds exactly what the reference's reader and loader accept
(src/gguf_loader.nim:194-237, src/model.nim:50-103).

Q2_K has no quantiser in the reference.  The one here is written from the reference's
dequantiser (src/quant.nim:49-87), which computes y = d*sc*q - dmin*m.  In a 256-element block,
sub-block `is` (0..15) holds elements 16*is .. 16*is+15.  Its 4-bit scale and min share
scales[is].  The 2-bit code of element 16*is + l sits in qs[32*(is//8) + 16*(is%2) + l] at bit
2*((is%8)//2).  d and dmin are float16.

For each sub-block, the quantiser takes min = min(x, 0) and scale = (max - min) / 3.  The
block's d and dmin are the largest scale and |min| divided by 15.  The codes are rounded
to nearest.  It is a valid Q2_K encoding of the data, not a search for the best one.
"""
from __future__ import annotations

import struct

import numpy as np

QK_K = 256
Q2K_BLOCK = 84
ALIGN = 32

GGUF_U32, GGUF_F32, GGUF_STR = 4, 6, 8
GGML_F32, GGML_Q2K = 0, 10


def quantize_q2k(x: np.ndarray) -> bytes:
    """x: float32 array whose size is a multiple of 256 (row-major rows of ne0 % 256 == 0)."""
    xb = np.ascontiguousarray(x, np.float32).reshape(-1, 16, 16)  # (blocks, sub-block, l)
    nb = xb.shape[0]
    mn = np.minimum(xb.min(axis=2), 0.0)
    mx = xb.max(axis=2)
    scale = (mx - mn) / 3.0
    mneg = -mn
    d = (scale.max(axis=1) / 15.0).astype(np.float16)
    dmin = (mneg.max(axis=1) / 15.0).astype(np.float16)
    d32 = d.astype(np.float32)[:, None]
    m32 = dmin.astype(np.float32)[:, None]
    with np.errstate(divide="ignore", invalid="ignore"):
        sc = np.where(d32 > 0, np.rint(scale / d32), 0).clip(0, 15).astype(np.uint8)
        mq = np.where(m32 > 0, np.rint(mneg / m32), 0).clip(0, 15).astype(np.uint8)
        step = (d32 * sc)[:, :, None]
        off = (m32 * mq)[:, :, None]
        q = np.where(step > 0, np.rint((xb + off) / step), 0).clip(0, 3).astype(np.uint8)
    scales = (sc | (mq << 4)).astype(np.uint8)                      # (nb, 16)
    # qs[32n + 16*half + l] |= q << (2j), is = 8n + 2j + half
    q5 = q.reshape(nb, 2, 4, 2, 16)                                    # (nb, n, j, half, l)
    shifts = (np.arange(4, dtype=np.uint8) * 2)[None, None, :, None, None]
    qs = np.bitwise_or.reduce(q5 << shifts, axis=2).reshape(nb, 64)   # (n, half, l) order
    out = np.empty((nb, Q2K_BLOCK), np.uint8)
    out[:, 0:16] = scales
    out[:, 16:80] = qs
    out[:, 80:82] = d.view(np.uint8).reshape(nb, 2)
    out[:, 82:84] = dmin.view(np.uint8).reshape(nb, 2)
    return out.tobytes()


def dequantize_q2k(raw: bytes, n: int) -> np.ndarray:
    """numpy restatement of the reference's dequantRowQ2K, for checking the quantiser."""
    b = np.frombuffer(raw, np.uint8).reshape(-1, Q2K_BLOCK)
    nb = b.shape[0]
    sc = b[:, 0:16]
    qs = b[:, 16:80].reshape(nb, 2, 2, 16)                             # (n, half, l)
    d = b[:, 80:82].copy().view(np.float16).astype(np.float32)
    dmin = b[:, 82:84].copy().view(np.float16).astype(np.float32)
    q = np.stack([(qs >> (2 * j)) & 3 for j in range(4)], axis=2)     # (nb, n, j, half, l)
    q = q.reshape(nb, 16, 16).astype(np.float32)
    dl = d * (sc & 0xF).astype(np.float32)
    ml = dmin * (sc >> 4).astype(np.float32)
    return (dl[:, :, None] * q - ml[:, :, None]).reshape(-1)[:n]


def _kv_bytes(key: str, typ: int, val) -> bytes:
    kb = key.encode()
    out = struct.pack("<Q", len(kb)) + kb + struct.pack("<I", typ)
    if typ == GGUF_U32:
        out += struct.pack("<I", int(val))
    elif typ == GGUF_F32:
        out += struct.pack("<f", float(val))
    elif typ == GGUF_STR:
        vb = val.encode()
        out += struct.pack("<Q", len(vb)) + vb
    return out


def tensor_plan(nLayer, nEmb, nHead, nHeadKv, nFfn, nVocab, f32: tuple = ()):
    """(name, ne, ggml type) of every tensor, in file order.  Matrices whose name ends with one
    of the suffixes in `f32` are stored as float32 instead of Q2_K."""
    kvDim = nHeadKv * (nEmb // nHead)
    plan = [("token_embd.weight", (nEmb, nVocab), GGML_F32)]
    for i in range(nLayer):
        p = f"blk.{i}."
        plan += [
            (p + "attn_norm.weight", (nEmb,), GGML_F32),
            (p + "attn_q.weight", (nEmb, nEmb), GGML_Q2K),
            (p + "attn_k.weight", (nEmb, kvDim), GGML_Q2K),
            (p + "attn_v.weight", (nEmb, kvDim), GGML_Q2K),
            (p + "attn_output.weight", (nEmb, nEmb), GGML_Q2K),
            (p + "ffn_norm.weight", (nEmb,), GGML_F32),
            (p + "ffn_gate.weight", (nEmb, nFfn), GGML_Q2K),
            (p + "ffn_up.weight", (nEmb, nFfn), GGML_Q2K),
            (p + "ffn_down.weight", (nFfn, nEmb), GGML_Q2K),
        ]
    plan += [("output_norm.weight", (nEmb,), GGML_F32), ("output.weight", (nEmb, nVocab), GGML_Q2K)]
    return [(n, ne, GGML_F32 if any(n.endswith(sfx) for sfx in f32) else t) for n, ne, t in plan]


def _nbytes(ne, typ) -> int:
    n = int(np.prod(ne))
    return n * 4 if typ == GGML_F32 else n // QK_K * Q2K_BLOCK


def write_model(path: str, seed: int = 0, nLayer: int = 22, nEmb: int = 2048, nHead: int = 32,
                nHeadKv: int = 4, nFfn: int = 5632, nVocab: int = 32000, ropeBase: float = 10000.0,
                rmsEps: float = 1e-5, sigma: float = 0.02, nCtx: int = 2048, keep: dict | None = None,
                ropeDim: int = 0, f32: tuple = ()) -> str:
    """Write the synthetic model; tensors are generated and quantised one at a time.  When `keep`
    is a dict it receives every tensor's stored bytes (small models only)."""
    rng = np.random.default_rng(seed)
    kvs = [
        ("general.architecture", GGUF_STR, "llama"),
        ("general.alignment", GGUF_U32, ALIGN),
        ("llama.vocab_size", GGUF_U32, nVocab),
        ("llama.context_length", GGUF_U32, nCtx),
        ("llama.embedding_length", GGUF_U32, nEmb),
        ("llama.block_count", GGUF_U32, nLayer),
        ("llama.feed_forward_length", GGUF_U32, nFfn),
        ("llama.attention.head_count", GGUF_U32, nHead),
        ("llama.attention.head_count_kv", GGUF_U32, nHeadKv),
        ("llama.rope.dimension_count", GGUF_U32, ropeDim if ropeDim > 0 else nEmb // nHead),
        ("llama.rope.freq_base", GGUF_F32, ropeBase),
        ("llama.attention.layer_norm_rms_epsilon", GGUF_F32, rmsEps),
    ]
    plan = tensor_plan(nLayer, nEmb, nHead, nHeadKv, nFfn, nVocab, f32)
    header = b"GGUF" + struct.pack("<IQQ", 3, len(plan), len(kvs))
    header += b"".join(_kv_bytes(*kv) for kv in kvs)
    offset = 0
    infos = b""
    offsets = []
    for name, ne, typ in plan:
        nb = name.encode()
        infos += struct.pack("<Q", len(nb)) + nb + struct.pack("<I", len(ne))
        infos += b"".join(struct.pack("<Q", x) for x in ne) + struct.pack("<iQ", typ, offset)
        offsets.append(offset)
        offset += _nbytes(ne, typ)
        offset = (offset + ALIGN - 1) // ALIGN * ALIGN
    with open(path, "wb") as f:
        f.write(header + infos)
        pad = (-f.tell()) % ALIGN
        f.write(b"\0" * pad)
        base = f.tell()
        for (name, ne, typ), off in zip(plan, offsets):
            f.seek(base + off)
            n = int(np.prod(ne))
            if name.endswith("norm.weight"):
                data = np.ones(n, np.float32).tobytes()
            else:
                w = rng.standard_normal(n, dtype=np.float32) * np.float32(sigma)
                data = w.tobytes() if typ == GGML_F32 else quantize_q2k(w)
            if keep is not None:
                keep[name] = (ne, typ, data)
            f.write(data)
    return path
