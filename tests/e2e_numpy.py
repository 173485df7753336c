"""An independent numpy float32 restatement of tinylama's forward pass (src/forward.nim:243-329),
used to check the C++ host forward pass on small models.  Summation order differs from the
reference's sequential loops, so results agree to float32 rounding, not bit for bit."""
from __future__ import annotations

import numpy as np

from tests import numpy_ref


class NumpyModel:
    def __init__(self, tensors: dict, hp: dict):
        self.t = tensors  # name -> float32 array shaped like the reference Tensor data [ne1, ne0]
        self.hp = hp

    def lin(self, x, name):  # linearGGMLCol: x [in, S], w rows = out, cols = in
        w = self.t[name]
        return (w.astype(np.float64) @ x.astype(np.float64)).astype(np.float32)

    def rms(self, x, name):
        w = self.t[name].reshape(-1)
        ss = (x.astype(np.float64) ** 2).mean(axis=0)
        inv = 1.0 / np.sqrt(ss + self.hp["eps"])
        return (x * inv[None, :] * w[:, None]).astype(np.float32)

    def forward(self, tokens, kc, vc, pos0, dump):
        hp = self.hp
        nH, nKv, nEmb = hp["nHead"], hp["nHeadKv"], hp["nEmb"]
        hd = nEmb // nH
        emb = self.t["token_embd.weight"]  # [nVocab, nEmb]
        x = emb[np.array(tokens)].T.astype(np.float32)  # [nEmb, S]
        S = len(tokens)
        positions = np.arange(pos0, pos0 + S)
        for layer in range(hp["nLayer"]):
            p = f"blk.{layer}."
            xn = self.rms(x, p + "attn_norm.weight")
            q = self.lin(xn, p + "attn_q.weight")
            k = self.lin(xn, p + "attn_k.weight")
            v = self.lin(xn, p + "attn_v.weight")
            rd = hp.get("ropeDim", hd)  # partial rotary: the first ropeDim dims of a head
            q = numpy_ref.rope_cols(q, nH, hd, rd, hp["base"], positions).astype(np.float32)
            k = numpy_ref.rope_cols(k, nKv, hd, rd, hp["base"], positions).astype(np.float32)
            kc[layer][:, pos0:pos0 + S] = k
            vc[layer][:, pos0:pos0 + S] = v
            ctx = numpy_ref.attention(q, kc[layer], vc[layer], nH, nKv, hd, positions, pos0 + S).astype(np.float32)
            dump.append(ctx)
            x = x + self.lin(ctx, p + "attn_output.weight")
            xn2 = self.rms(x, p + "ffn_norm.weight")
            g = self.lin(xn2, p + "ffn_gate.weight")
            u = self.lin(xn2, p + "ffn_up.weight")
            act = (g / (1.0 + np.exp(-g.astype(np.float64)))).astype(np.float32) * u
            x = x + self.lin(act, p + "ffn_down.weight")
        xf = self.rms(x, "output_norm.weight")
        return self.lin(xf, "output.weight")

    def generate(self, prompt, n_new, max_len):
        hp = self.hp
        kvDim = hp["nHeadKv"] * (hp["nEmb"] // hp["nHead"])
        kc = [np.zeros((kvDim, max_len), np.float32) for _ in range(hp["nLayer"])]
        vc = [np.zeros((kvDim, max_len), np.float32) for _ in range(hp["nLayer"])]
        dump, ids, gaps = [], [], []
        logits = self.forward(list(prompt), kc, vc, 0, dump)
        pos = len(prompt)
        for j in range(n_new):
            col = logits[:, -1]
            order = np.argsort(col)
            ids.append(int(order[-1]))
            gaps.append(float(col[order[-1]] - col[order[-2]]))
            if j == n_new - 1:
                break
            logits = self.forward([ids[-1]], kc, vc, pos, dump)
            pos += 1
        return np.array(ids), np.array(gaps), dump

    def repl(self, lines, n_new, max_len):
        """The REPL of src/tinylama.nim:45-100 over several lines on one cache: the first line is
        prefilled; a later line's tokens go in at positions curLen.. (one forwardDecode each in
        the reference; the same attention in one numpy pass here).  Each line then decodes
        n_new - 1 greedy tokens; the last greedy id of a line is never fed back."""
        hp = self.hp
        kvDim = hp["nHeadKv"] * (hp["nEmb"] // hp["nHead"])
        kc = [np.zeros((kvDim, max_len), np.float32) for _ in range(hp["nLayer"])]
        vc = [np.zeros((kvDim, max_len), np.float32) for _ in range(hp["nLayer"])]
        out, pos = [], 0
        for line in lines:
            dump, ids, gaps = [], [], []
            logits = self.forward(list(line), kc, vc, pos, dump)
            pos += len(line)
            for j in range(n_new):
                col = logits[:, -1]
                order = np.argsort(col)
                ids.append(int(order[-1]))
                gaps.append(float(col[order[-1]] - col[order[-2]]))
                if j == n_new - 1:
                    break
                logits = self.forward([ids[-1]], kc, vc, pos, dump)
                pos += 1
            out.append((np.array(ids), np.array(gaps), dump))
        return out
