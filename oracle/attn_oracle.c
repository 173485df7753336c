/*
 * attn_oracle.c -- CPU restatement of tinylama's attention path (TEST INFRASTRUCTURE ONLY).
 *
 * This file is the oracle: the checker that the CUDA path in tinylama_b200/ is compared
 * against.  Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg load it.
 * The product library (libtlattn.so) never links or calls it.
 *
 * PARITY UNPINNED: the reference is Nim and no Nim compiler exists on either machine, and
 * the reference ships no golden vectors or known-answer tests for this path
 * (tests/tester.nim only compiles the CLI).  This restatement is therefore checked against
 * an independent numpy restatement and against analytic known answers (tests/), not
 * against outputs of the reference itself.
 *
 * Every function restates one proc of src/forward.nim with the same index arithmetic, the
 * same loop order (hence the same float32 summation order), float32 accumulators and the
 * same libm calls Nim's std/math emits for float32: pow -> powf, sqrt -> sqrtf,
 * exp -> expf, cos -> cosf, sin -> sinf.  Build with -O2 -ffp-contract=off and no
 * fast-math, which is what `nim c -d:release` hands to gcc on x86-64.
 *
 * Layout is the reference's "ggml column layout": a [rows, cols] tensor stores element
 * (r, c) at r*cols + c (src/tensor.nim:11-26, src/forward.nim:16,41).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "attn_oracle.h"

/* src/forward.nim:108-123 applyRopeSingle: x is [nHead*headDim, seqLen]; position = column. */
void ora_rope_single(float *x, int nHead, int headDim, int ropeDim, float base, int seqLen) {
    for (int h = 0; h < nHead; ++h) {
        const int hOffset = h * headDim;
        for (int p = 0; p < seqLen; ++p) {
            for (int i = 0; i < ropeDim / 2; ++i) {
                const int64_t idx0 = (int64_t)(hOffset + 2 * i) * seqLen + p;
                const int64_t idx1 = (int64_t)(hOffset + 2 * i + 1) * seqLen + p;
                const float theta = powf(1.0f / base, (float)(2 * i) / (float)ropeDim);
                const float angle = (float)p * theta;
                const float c = cosf(angle);
                const float s = sinf(angle);
                const float v0 = x[idx0];
                const float v1 = x[idx1];
                x[idx0] = v0 * c - v1 * s;
                x[idx1] = v0 * s + v1 * c;
            }
        }
    }
}

/* src/forward.nim:125-139 applyRopeAtPos: rotates column 0 of x ([nHead*headDim, seqLen])
 * at the explicit position `pos`. */
void ora_rope_at_pos(float *x, int nHead, int headDim, int ropeDim, float base, int pos,
                     int seqLen) {
    for (int h = 0; h < nHead; ++h) {
        const int hOffset = h * headDim;
        for (int i = 0; i < ropeDim / 2; ++i) {
            const int64_t idx0 = (int64_t)(hOffset + 2 * i) * seqLen;
            const int64_t idx1 = (int64_t)(hOffset + 2 * i + 1) * seqLen;
            const float theta = powf(1.0f / base, (float)(2 * i) / (float)ropeDim);
            const float angle = (float)pos * theta;
            const float c = cosf(angle);
            const float s = sinf(angle);
            const float v0 = x[idx0];
            const float v1 = x[idx1];
            x[idx0] = v0 * c - v1 * s;
            x[idx1] = v0 * s + v1 * c;
        }
    }
}

/* src/forward.nim:232-241 storeKVRange: copies k,v ([rows, cols]) into the per-layer caches
 * ([rows, cacheCols]) at column startPos.  Like the reference it does not check
 * startPos + cols <= cacheCols; the caller must. */
void ora_store_kv_range(float *kCache, float *vCache, int cacheCols, int startPos,
                        const float *k, const float *v, int rows, int cols) {
    for (int r = 0; r < rows; ++r) {
        const int64_t src = (int64_t)r * cols;
        const int64_t dst = (int64_t)r * cacheCols + startPos;
        for (int c = 0; c < cols; ++c) {
            kCache[dst + c] = k[src + c];
            vCache[dst + c] = v[src + c];
        }
    }
}

/* src/forward.nim:141-176 attentionFull, up to (not including) the wo projection at :177.
 * q: [nHead*headDim, seqLen], k,v: [nHeadKv*headDim, seqLen], ctx: [nHead*headDim, seqLen]. */
void ora_attention_full_ctx(const float *q, const float *k, const float *v, int seqLen,
                            int nHead, int nHeadKv, int headDim, float *ctx) {
    const int group = nHead / nHeadKv;
    float *scores = (float *)malloc(sizeof(float) * (size_t)(seqLen > 0 ? seqLen : 1));
    for (int h = 0; h < nHead; ++h) {
        const int kvh = h / group;
        const int hOff = h * headDim;
        for (int i = 0; i < seqLen; ++i) {
            const int n = i + 1;
            for (int j = 0; j < n; ++j) {
                float dot = 0.0f;
                for (int d = 0; d < headDim; ++d) {
                    const int64_t qIdx = (int64_t)(hOff + d) * seqLen + i;
                    const int64_t kIdx = (int64_t)(kvh * headDim + d) * seqLen + j;
                    dot += q[qIdx] * k[kIdx];
                }
                scores[j] = dot / sqrtf((float)headDim);
            }
            float maxv = scores[0];
            for (int j = 1; j < n; ++j)
                if (scores[j] > maxv) maxv = scores[j];
            float sum = 0.0f;
            for (int j = 0; j < n; ++j) {
                scores[j] = expf(scores[j] - maxv);
                sum += scores[j];
            }
            const float inv = 1.0f / sum;
            for (int j = 0; j < n; ++j) scores[j] *= inv;
            for (int d = 0; d < headDim; ++d) {
                float acc = 0.0f;
                for (int j = 0; j < n; ++j) {
                    const int64_t vIdx = (int64_t)(kvh * headDim + d) * seqLen + j;
                    acc += scores[j] * v[vIdx];
                }
                ctx[(int64_t)(hOff + d) * seqLen + i] = acc;
            }
        }
    }
    free(scores);
}

/* src/forward.nim:40-83 linearGGMLCol (scalar branch :75-83): x [in, seq], w laid out as
 * rows=out, cols=in; out [out, seq]. */
void ora_linear_ggml_col(const float *x, const float *w, int inDim, int outDim, int seqLen,
                         float *out) {
    for (int o = 0; o < outDim; ++o) {
        const int64_t wRow = (int64_t)o * inDim;
        const int64_t outRow = (int64_t)o * seqLen;
        for (int s = 0; s < seqLen; ++s) {
            float acc = 0.0f;
            for (int kk = 0; kk < inDim; ++kk) acc += w[wRow + kk] * x[(int64_t)kk * seqLen + s];
            out[outRow + s] = acc;
        }
    }
}

/* src/forward.nim:141-177 attentionFull including the wo projection. wo is [in=nHead*headDim,
 * out=nEmb] in the reference's shape convention; out is [nEmb, seqLen]. */
void ora_attention_full(const float *q, const float *k, const float *v, const float *wo,
                        int nEmb, int seqLen, int nHead, int nHeadKv, int headDim,
                        float *out) {
    const int64_t n = (int64_t)nHead * headDim * seqLen;
    float *ctx = (float *)malloc(sizeof(float) * (size_t)(n > 0 ? n : 1));
    ora_attention_full_ctx(q, k, v, seqLen, nHead, nHeadKv, headDim, ctx);
    ora_linear_ggml_col(ctx, wo, nHead * headDim, nEmb, seqLen, out);
    free(ctx);
}

/* src/forward.nim:179-211 attentionCached: q is [nHead*headDim, 1], caches are
 * [nHeadKv*headDim, cacheCols]; attends over columns 0..curLen-1; ctx is [nHead*headDim]. */
void ora_attention_cached(const float *q, const float *kCache, const float *vCache,
                          int cacheCols, int curLen, int nHead, int nHeadKv, int headDim,
                          float *ctx) {
    const int group = nHead / nHeadKv;
    float *scores = (float *)malloc(sizeof(float) * (size_t)(curLen > 0 ? curLen : 1));
    for (int h = 0; h < nHead; ++h) {
        const int kvh = h / group;
        const int hOff = h * headDim;
        for (int j = 0; j < curLen; ++j) {
            float dot = 0.0f;
            for (int d = 0; d < headDim; ++d) {
                const int64_t kIdx = (int64_t)(kvh * headDim + d) * cacheCols + j;
                dot += q[hOff + d] * kCache[kIdx];
            }
            scores[j] = dot / sqrtf((float)headDim);
        }
        float maxv = scores[0];
        for (int j = 1; j < curLen; ++j)
            if (scores[j] > maxv) maxv = scores[j];
        float sum = 0.0f;
        for (int j = 0; j < curLen; ++j) {
            scores[j] = expf(scores[j] - maxv);
            sum += scores[j];
        }
        const float inv = 1.0f / sum;
        for (int j = 0; j < curLen; ++j) scores[j] *= inv;
        for (int d = 0; d < headDim; ++d) {
            float acc = 0.0f;
            for (int j = 0; j < curLen; ++j) {
                const int64_t vIdx = (int64_t)(kvh * headDim + d) * cacheCols + j;
                acc += scores[j] * vCache[vIdx];
            }
            ctx[hOff + d] = acc;
        }
    }
    free(scores);
}

/* One full decode-attention step of src/forward.nim:314-317 for one sequence and one layer:
 * applyRopeAtPos(q), applyRopeAtPos(k), storeKVRange(pos), attentionCached(pos+1).
 * q ([nHead*headDim]) and k are rotated in place. */
void ora_decode_step(float *q, float *k, const float *v, float *kCache, float *vCache,
                     int cacheCols, int pos, int nHead, int nHeadKv, int headDim, int ropeDim,
                     float base, float *ctx) {
    ora_rope_at_pos(q, nHead, headDim, ropeDim, base, pos, 1);
    ora_rope_at_pos(k, nHeadKv, headDim, ropeDim, base, pos, 1);
    ora_store_kv_range(kCache, vCache, cacheCols, pos, k, v, nHeadKv * headDim, 1);
    ora_attention_cached(q, kCache, vCache, cacheCols, pos + 1, nHead, nHeadKv, headDim, ctx);
}

/* One full prefill-attention pass of src/forward.nim:271-274 for one sequence and one layer
 * (ctx only): applyRopeSingle(q), applyRopeSingle(k), storeKVRange(0), attentionFull ctx. */
void ora_prefill_step(float *q, float *k, const float *v, float *kCache, float *vCache,
                      int cacheCols, int seqLen, int nHead, int nHeadKv, int headDim,
                      int ropeDim, float base, float *ctx) {
    ora_rope_single(q, nHead, headDim, ropeDim, base, seqLen);
    ora_rope_single(k, nHeadKv, headDim, ropeDim, base, seqLen);
    ora_store_kv_range(kCache, vCache, cacheCols, 0, k, v, nHeadKv * headDim, seqLen);
    ora_attention_full_ctx(q, k, v, seqLen, nHead, nHeadKv, headDim, ctx);
}

/* The float32 RoPE frequency of pair i exactly as src/forward.nim:116 computes it. */
float ora_rope_theta(int i, int ropeDim, float base) {
    return powf(1.0f / base, (float)(2 * i) / (float)ropeDim);
}
