// tl_host.cpp -- tinylama's host forward pass (C++), with attention through tlh_attn_ops.
//
// Restates, in the reference's own float32 arithmetic and loop orders, everything around the
// attention path that an end-to-end run needs:
//   GGUF v2/v3 parsing            src/gguf_loader.nim:194-237
//   HParams / tensor loading      src/model.nim:50-123
//   halfToFloat, Q2_K/Q3_K/Q6_K   src/quant.nim:28-186
//   embedding, linearGGMLCol,     src/forward.nim:15-83, 213-230
//   ffn, linearOut, rmsnormCols,  src/tensor.nim:40-56, 97-113
//   silu/mul/add
//   forwardPrefill/forwardDecode  src/forward.nim:243-329
//   argmaxLast, runPrompt         src/infer_core.nim:6-32, src/tinylama.nim:47-69
// The attention procs are not restated here: they are the table's (the B200 path in
// libtlattn.so for tlh_gpu_attn_ops_create).  Build with -ffp-contract=off so that float32
// products and sums round as the reference's do.
#include "../../include/tl_host.h"

#include <fcntl.h>
#include <math.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <atomic>
#include <cstdint>
#include <map>
#include <string>
#include <thread>
#include <vector>

#include "../../include/tl_attn.h"
#include "../../include/tl_model.h"

namespace {

thread_local std::string g_err;

int fail(int code, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_err = buf;
    return code;
}

// ---- thread pool for the "Malebolgia" build: fixed chunks of output rows ------------------
template <typename F>
void parallel_chunks(int n, int chunk, int nthreads, F &&fn) {
    if (nthreads <= 1 || n <= chunk) {
        for (int s = 0; s < n; s += chunk) fn(s, std::min(s + chunk, n));
        return;
    }
    std::atomic<int> next{0};
    std::vector<std::thread> ts;
    for (int t = 0; t < nthreads; ++t)
        ts.emplace_back([&] {
            for (;;) {
                const int s = next.fetch_add(chunk);
                if (s >= n) break;
                fn(s, std::min(s + chunk, n));
            }
        });
    for (auto &t : ts) t.join();
}

// ---- float32 tensor in the reference's layout ----------------------------------------------
struct Tensor {
    std::vector<float> data;
    std::vector<int64_t> shape;  // shape[0] = ne0 (innermost), shape[1] = ne1
    Tensor() = default;
    Tensor(int64_t a, int64_t b) : data((size_t)(a * b), 0.f), shape{a, b} {}
};

// ---- GGUF ------------------------------------------------------------------------------------
struct TensorInfo {
    std::string name;
    uint32_t nDims = 0;
    uint64_t ne[4] = {1, 1, 1, 1};
    int32_t type = 0;
    uint64_t offset = 0;
};

struct Reader {
    const uint8_t *p;
    size_t size, pos = 0;
    bool ok = true;
    template <typename T>
    T get() {
        T v{};
        if (pos + sizeof(T) > size) { ok = false; return v; }
        memcpy(&v, p + pos, sizeof(T));
        pos += sizeof(T);
        return v;
    }
    std::string str() {
        const uint64_t n = get<uint64_t>();
        if (!ok || pos + n > size) { ok = false; return {}; }
        std::string s((const char *)p + pos, (size_t)n);
        pos += n;
        return s;
    }
};

enum GType { U8 = 0, I8, U16, I16, U32, I32, F32, BOOL, STR, ARR, U64, I64, F64 };

size_t scalar_size(uint32_t t) {
    switch (t) {
        case U8: case I8: case BOOL: return 1;
        case U16: case I16: return 2;
        case U32: case I32: case F32: return 4;
        case U64: case I64: case F64: return 8;
        default: return 0;
    }
}

struct KvVal {
    uint32_t type = 0;
    uint64_t u = 0;
    double f = 0;
    std::string s;
    uint64_t arrN = 0;
};

constexpr int QK_K = 256;
constexpr int BLOCK_Q2K = 2 + 2 + QK_K / 16 + QK_K / 4;   // 84
constexpr int BLOCK_Q3K = 2 + QK_K / 4 + QK_K / 8 + 12;   // 110
constexpr int BLOCK_Q6K = 2 + QK_K / 16 + 3 * QK_K / 4;   // 210

// src/quant.nim:28-47
float half_to_float(uint16_t h) {
    const uint32_t s = (h >> 15) & 1, e = (h >> 10) & 0x1F, f = h & 0x3FF;
    if (e == 0) {
        if (f == 0) return s ? -0.0f : 0.0f;
        return (s ? -1.0f : 1.0f) * powf(2.0f, -14.0f) * ((float)f / 1024.0f);
    }
    if (e == 31) return f == 0 ? (s ? -INFINITY : INFINITY) : NAN;
    const int ex = (int)e - 15;
    const float mant = 1.0f + (float)f / 1024.0f;
    return (s ? -1.0f : 1.0f) * mant * powf(2.0f, (float)ex);
}

// src/quant.nim:49-87
void dequant_q2k(const uint8_t *src, float *dst, int k) {
    int out = 0;
    for (int b = 0, off = 0; b < k / QK_K; ++b, off += BLOCK_Q2K) {
        const uint8_t *scales = src + off, *qs = src + off + QK_K / 16;
        uint16_t dr, mr;
        memcpy(&dr, src + off + QK_K / 16 + QK_K / 4, 2);
        memcpy(&mr, src + off + QK_K / 16 + QK_K / 4 + 2, 2);
        const float d = half_to_float(dr), dmin = half_to_float(mr);
        int is = 0, q = 0;
        for (int n = 0; n < 2; ++n) {
            int shift = 0;
            for (int j = 0; j < 4; ++j) {
                uint8_t sc = scales[is++];
                float dl = d * (float)(sc & 0x0F), ml = dmin * (float)(sc >> 4);
                for (int l = 0; l < 16; ++l) dst[out++] = dl * (float)((qs[q + l] >> shift) & 3) - ml;
                sc = scales[is++];
                dl = d * (float)(sc & 0x0F);
                ml = dmin * (float)(sc >> 4);
                for (int l = 0; l < 16; ++l) dst[out++] = dl * (float)((qs[q + 16 + l] >> shift) & 3) - ml;
                shift += 2;
            }
            q += 32;
        }
    }
}

// src/quant.nim:89-150
void dequant_q3k(const uint8_t *src, float *dst, int k) {
    int out = 0;
    for (int b = 0, off = 0; b < k / QK_K; ++b, off += BLOCK_Q3K) {
        const uint8_t *hmask = src + off, *qs = src + off + QK_K / 8;
        uint8_t sb[12];
        memcpy(sb, src + off + QK_K / 8 + QK_K / 4, 12);
        uint16_t dr;
        memcpy(&dr, src + off + QK_K / 8 + QK_K / 4 + 12, 2);
        const float dAll = half_to_float(dr);
        uint32_t aux[4];
        for (int i = 0; i < 3; ++i)
            aux[i] = (uint32_t)sb[4 * i] | ((uint32_t)sb[4 * i + 1] << 8) | ((uint32_t)sb[4 * i + 2] << 16) |
                     ((uint32_t)sb[4 * i + 3] << 24);
        const uint32_t km1 = 0x03030303u, km2 = 0x0f0f0f0fu, tmp = aux[2];
        aux[2] = ((aux[0] >> 4) & km2) | (((tmp >> 4) & km1) << 4);
        aux[3] = ((aux[1] >> 4) & km2) | (((tmp >> 6) & km1) << 4);
        aux[0] = (aux[0] & km2) | (((tmp >> 0) & km1) << 4);
        aux[1] = (aux[1] & km2) | (((tmp >> 2) & km1) << 4);
        int8_t scales[16];
        for (int i = 0; i < 4; ++i)
            for (int j = 0; j < 4; ++j) scales[4 * i + j] = (int8_t)((aux[i] >> (8 * j)) & 0xFF);
        int si = 0, q = 0;
        uint8_t m = 1;
        for (int n = 0; n < 2; ++n) {
            int shift = 0;
            for (int j = 0; j < 4; ++j) {
                const float dl = dAll * (float)(scales[si++] - 32);
                for (int l = 0; l < 16; ++l) {
                    const int qv = (qs[q + l] >> shift) & 3, hm = (hmask[l] & m) ? 0 : 4;
                    dst[out++] = dl * (float)(qv - hm);
                }
                const float dl2 = dAll * (float)(scales[si++] - 32);
                for (int l = 0; l < 16; ++l) {
                    const int qv = (qs[q + 16 + l] >> shift) & 3, hm = (hmask[16 + l] & m) ? 0 : 4;
                    dst[out++] = dl2 * (float)(qv - hm);
                }
                shift += 2;
                m = (uint8_t)(m << 1);
            }
            q += 32;
        }
    }
}

// src/quant.nim:152-186
void dequant_q6k(const uint8_t *src, float *dst, int k) {
    int out = 0;
    for (int b = 0, off = 0; b < k / QK_K; ++b, off += BLOCK_Q6K) {
        const uint8_t *ql = src + off, *qh = src + off + QK_K / 2;
        const int8_t *sc = (const int8_t *)(src + off + QK_K / 2 + QK_K / 4);
        uint16_t dr;
        memcpy(&dr, src + off + QK_K / 2 + QK_K / 4 + QK_K / 16, 2);
        const float d = half_to_float(dr);
        int qlo = 0, qho = 0, so = 0;
        for (int n = 0; n < 2; ++n) {
            for (int l = 0; l < 32; ++l) {
                const int is = l / 16;
                const int q1 = (int8_t)((ql[qlo + l] & 0xF) | (((qh[qho + l] >> 0) & 3) << 4)) - 32;
                const int q2 = (int8_t)((ql[qlo + l + 32] & 0xF) | (((qh[qho + l] >> 2) & 3) << 4)) - 32;
                const int q3 = (int8_t)((ql[qlo + l] >> 4) | (((qh[qho + l] >> 4) & 3) << 4)) - 32;
                const int q4 = (int8_t)((ql[qlo + l + 32] >> 4) | (((qh[qho + l] >> 6) & 3) << 4)) - 32;
                dst[out + l] = d * (float)sc[so + is] * (float)q1;
                dst[out + l + 32] = d * (float)sc[so + is + 2] * (float)q2;
                dst[out + l + 64] = d * (float)sc[so + is + 4] * (float)q3;
                dst[out + l + 96] = d * (float)sc[so + is + 6] * (float)q4;
            }
            out += 128;
            qlo += 64;
            qho += 32;
            so += 8;
        }
    }
}

}  // namespace

struct tlh_model {
    tlh_hparams hp{};
    std::string arch;
    std::map<std::string, Tensor> w;
    // the Q2_K tensors as stored in the file, for the GPU model (which keeps them quantised)
    struct Raw {
        int64_t ne0 = 0, ne1 = 0;
        std::vector<uint8_t> bytes;
    };
    std::map<std::string, Raw> q2k;
    // tlh_model_open: the file mapped read-only and each tensor's place in it, no float32 copy
    struct View {
        int32_t type = 0;
        int64_t ne0 = 0, rows = 0, rowBytes = 0;
        std::vector<int64_t> shape;
        const uint8_t *src = nullptr;
    };
    std::map<std::string, View> views;
    void *map = nullptr;
    size_t mapSize = 0;
    int nthreads = 1;
    ~tlh_model();
};

namespace {

int load_file(const char *path, std::vector<uint8_t> &buf) {
    FILE *f = fopen(path, "rb");
    if (!f) return fail(-1, "cannot open %s", path);
    fseek(f, 0, SEEK_END);
    const long n = ftell(f);
    fseek(f, 0, SEEK_SET);
    buf.resize((size_t)n);
    const size_t got = fread(buf.data(), 1, (size_t)n, f);
    fclose(f);
    if (got != (size_t)n) return fail(-1, "short read on %s", path);
    return 0;
}

// ---- forward-pass building blocks (src/forward.nim, src/tensor.nim) --------------------------

// embeddingLookup (src/forward.nim:15-38) -> [nEmb, seq]
Tensor embedding_lookup(const Tensor &w, const std::vector<int32_t> &tokens, int nVocab, int nEmb) {
    Tensor r(nEmb, (int64_t)tokens.size());
    const int64_t S = (int64_t)tokens.size();
    const int64_t a0 = w.shape[0], a1 = w.shape[1];
    const int64_t rowSize = (a0 == nVocab && a1 == nEmb) ? a1 : a0;
    for (int64_t i = 0; i < S; ++i) {
        const int64_t row = (int64_t)tokens[i] * rowSize;
        for (int e = 0; e < nEmb; ++e) r.data[(size_t)(e * S + i)] = w.data[(size_t)(row + e)];
    }
    return r;
}

// linearGGMLCol (src/forward.nim:40-83): x [in, seq], w rows = out, cols = in -> [out, seq].
// The per-row loop is the same in the scalar and the chunked (Malebolgia) build.
Tensor linear(const Tensor &x, const Tensor &w, int nthreads) {
    const int64_t in = x.shape[0], S = x.shape[1], out = w.shape[1];
    Tensor r(out, S);
    const int chunk = out >= 64 ? 32 : (int)out;
    parallel_chunks((int)out, chunk, nthreads, [&](int s, int e) {
        for (int o = s; o < e; ++o) {
            const float *wr = w.data.data() + (size_t)o * in;
            for (int64_t t = 0; t < S; ++t) {
                float acc = 0.0f;
                for (int64_t k = 0; k < in; ++k) acc += wr[k] * x.data[(size_t)(k * S + t)];
                r.data[(size_t)(o * S + t)] = acc;
            }
        }
    });
    return r;
}

// rmsnormCols (src/tensor.nim:97-113)
Tensor rmsnorm_cols(const Tensor &x, const Tensor &wt, float eps) {
    const int64_t dim = x.shape[0], S = x.shape[1];
    Tensor r(dim, S);
    for (int64_t s = 0; s < S; ++s) {
        float ss = 0.0f;
        for (int64_t i = 0; i < dim; ++i) {
            const float v = x.data[(size_t)(i * S + s)];
            ss += v * v;
        }
        const float inv = 1.0f / sqrtf(ss / (float)dim + eps);
        for (int64_t i = 0; i < dim; ++i)
            r.data[(size_t)(i * S + s)] = x.data[(size_t)(i * S + s)] * inv * wt.data[(size_t)i];
    }
    return r;
}

void add_inplace(Tensor &a, const Tensor &b) {  // add (src/tensor.nim:40-44)
    for (size_t i = 0; i < a.data.size(); ++i) a.data[i] = a.data[i] + b.data[i];
}

// ffn (src/forward.nim:213-217) with silu and mul (src/tensor.nim:46-56)
Tensor ffn(const Tensor &x, const Tensor &wg, const Tensor &wu, const Tensor &wd, int nthreads) {
    Tensor g = linear(x, wg, nthreads);
    const Tensor u = linear(x, wu, nthreads);
    for (size_t i = 0; i < g.data.size(); ++i) {
        const float v = g.data[i];
        g.data[i] = (v / (1.0f + expf(-v))) * u.data[i];
    }
    return linear(g, wd, nthreads);
}

// argmaxLast (src/infer_core.nim:6-32) on [nVocab, seq]; also the best-minus-second gap
int32_t argmax_last(const Tensor &logits, int nVocab, float *gap) {
    const int64_t S = logits.shape[1], col = S - 1;
    int best = 0;
    float bv = logits.data[(size_t)col], second = -INFINITY;
    for (int i = 1; i < nVocab; ++i) {
        const float v = logits.data[(size_t)(i * S + col)];
        if (v > bv) {
            second = bv;
            bv = v;
            best = i;
        } else if (v > second) {
            second = v;
        }
    }
    if (gap) *gap = bv - second;
    return best;
}

const Tensor *tensor_or(const tlh_model *m, const char *a, const char *b) {
    auto it = m->w.find(a);
    if (it != m->w.end()) return &it->second;
    it = m->w.find(b);
    return it != m->w.end() ? &it->second : nullptr;
}

const Tensor *tensor(const tlh_model *m, const std::string &name) {
    auto it = m->w.find(name);
    return it != m->w.end() ? &it->second : nullptr;
}

struct Dump {
    float *buf;
    long cap, n = 0;
    void put(const Tensor &t) {
        if (!buf) { n += (long)t.data.size(); return; }
        for (float v : t.data) {
            if (n < cap) buf[n] = v;
            ++n;
        }
    }
};

enum class Pass { Prefill, Decode, Continue };

// forwardPrefill (src/forward.nim:243-284) / forwardDecode (:286-329).  Continue: the tokens sit
// at positions curLen.. and attend the cache (ops->prefill_at): what feeding them one by one
// through forwardDecode computes, in one pass; logits of every column, the last one used.
int forward(tlh_model *m, tlh_attn_ops *ops, const std::vector<int32_t> &tokens, Pass mode, Tensor &logits,
            Dump &dump) {
    const bool prefill = mode == Pass::Prefill;
    const tlh_hparams &hp = m->hp;
    if (!m->arch.empty() && m->arch != "llama") return fail(-1, "unsupported architecture: %s", m->arch.c_str());
    if (hp.nHeadKv != 0 && hp.nHead % hp.nHeadKv != 0)
        return fail(-1, "GQA requires head_count divisible by head_count_kv");
    if (!prefill && ops->curLen >= ops->maxLen) return fail(-3, "KV cache full");
    if (mode == Pass::Continue && !ops->prefill_at) return fail(-1, "attention table has no prefill_at");
    if (mode == Pass::Continue && (long)ops->curLen + (long)tokens.size() > ops->maxLen)
        return fail(-3, "KV cache full");
    const int headDim = hp.nEmb / hp.nHead;
    const int ropeDim = hp.ropeDim > 0 ? hp.ropeDim : headDim;
    const int S = (int)tokens.size();
    const Tensor *emb = tensor_or(m, "tok_embeddings.weight", "token_embd.weight");
    if (!emb) return fail(-1, "missing tensor: token_embd.weight");
    Tensor x = embedding_lookup(*emb, tokens, hp.nVocab, hp.nEmb);
    const int pos = ops->curLen;
    if (prefill) ops->curLen = S;
    int rc = 0;
    for (int layer = 0; layer < hp.nLayer; ++layer) {
        const std::string p = "blk." + std::to_string(layer) + ".";
        const Tensor *an = tensor(m, p + "attn_norm.weight"), *fn = tensor(m, p + "ffn_norm.weight"),
                     *wq = tensor(m, p + "attn_q.weight"), *wk = tensor(m, p + "attn_k.weight"),
                     *wv = tensor(m, p + "attn_v.weight"), *wo = tensor(m, p + "attn_output.weight"),
                     *wg = tensor(m, p + "ffn_gate.weight"), *wu = tensor(m, p + "ffn_up.weight"),
                     *wd = tensor(m, p + "ffn_down.weight");
        if (!an || !fn || !wq || !wk || !wv || !wo || !wg || !wu || !wd)
            return fail(-1, "missing tensor in layer %d", layer);
        const Tensor xn = rmsnorm_cols(x, *an, hp.rmsEps);
        Tensor q = linear(xn, *wq, m->nthreads);
        Tensor k = linear(xn, *wk, m->nthreads);
        const Tensor v = linear(xn, *wv, m->nthreads);
        Tensor ctx(hp.nHead * headDim, S);
        if (mode == Pass::Continue) {
            if ((rc = ops->prefill_at(ops->ctx, layer, pos, q.data.data(), k.data.data(), v.data.data(), S,
                                      ctx.data.data())))
                return rc;
        } else if (prefill) {
            if ((rc = ops->rope_single(ops->ctx, q.data.data(), hp.nHead, headDim, ropeDim, hp.ropeFreqBase, S)) ||
                (rc = ops->rope_single(ops->ctx, k.data.data(), hp.nHeadKv, headDim, ropeDim, hp.ropeFreqBase, S)) ||
                (rc = ops->store_kv(ops->ctx, layer, 0, k.data.data(), v.data.data(), (int)k.shape[0], S)) ||
                (rc = ops->attention_full(ops->ctx, q.data.data(), k.data.data(), v.data.data(), S, hp.nHead,
                                          hp.nHeadKv, headDim, ctx.data.data())))
                return rc;
        } else {
            if ((rc = ops->rope_at_pos(ops->ctx, q.data.data(), hp.nHead, headDim, ropeDim, hp.ropeFreqBase, pos, 1)) ||
                (rc = ops->rope_at_pos(ops->ctx, k.data.data(), hp.nHeadKv, headDim, ropeDim, hp.ropeFreqBase, pos, 1)) ||
                (rc = ops->store_kv(ops->ctx, layer, pos, k.data.data(), v.data.data(), (int)k.shape[0], 1)) ||
                (rc = ops->attention_cached(ops->ctx, layer, q.data.data(), pos + 1, hp.nHead, hp.nHeadKv, headDim,
                                            ctx.data.data())))
                return rc;
        }
        dump.put(ctx);
        add_inplace(x, linear(ctx, *wo, m->nthreads));
        const Tensor xn2 = rmsnorm_cols(x, *fn, hp.rmsEps);
        add_inplace(x, ffn(xn2, *wg, *wu, *wd, m->nthreads));
    }
    if (mode == Pass::Decode) ops->curLen = pos + 1;
    if (mode == Pass::Continue) ops->curLen = pos + S;
    const Tensor *nw = tensor_or(m, "norm.weight", "output_norm.weight");
    const Tensor *ow = tensor(m, "output.weight");
    if (!nw || !ow) return fail(-1, "missing output tensors");
    const Tensor xf = rmsnorm_cols(x, *nw, hp.rmsEps);
    if (ow->shape[0] == hp.nEmb && ow->shape[1] == hp.nVocab) {
        logits = linear(xf, *ow, m->nthreads);  // linearOut (src/forward.nim:219-230)
    } else if (ow->shape[0] == hp.nVocab && ow->shape[1] == hp.nEmb) {
        Tensor t = *ow;
        t.shape = {hp.nEmb, hp.nVocab};
        logits = linear(xf, t, m->nthreads);
    } else {
        return fail(-1, "output weight shape mismatch");
    }
    return 0;
}

// ---- the attention procs on the B200 ------------------------------------------------------------
struct GpuOps {
    tlh_attn_ops ops{};
    tl_attn *h = nullptr;      // cache of the current prompt
    tl_attn *scratch = nullptr;
    int nLayer, nHead, nHeadKv, headDim, ropeDim, device;
    float base;
};

int g_init(void *c, int maxLen) {
    GpuOps *g = (GpuOps *)c;
    if (g->h) tl_attn_destroy(g->h);
    g->h = nullptr;
    int rc = tl_attn_create(&g->h, g->nLayer, g->nHead, g->nHeadKv, g->headDim, g->ropeDim, g->base, maxLen, 1,
                            TL_KV_F32, g->device);
    if (rc) return fail(rc, "%s", tl_last_error());
    g->ops.curLen = 0;
    g->ops.maxLen = maxLen;
    return 0;
}
int g_rope_single(void *c, float *x, int nH, int d, int rd, float base, int S) {
    GpuOps *g = (GpuOps *)c;
    const int rc = tl_rope_single_host(g->h, x, nH, d, rd, base, S);
    return rc ? fail(rc, "%s", tl_last_error()) : 0;
}
int g_rope_at_pos(void *c, float *x, int nH, int d, int rd, float base, int pos, int S) {
    GpuOps *g = (GpuOps *)c;
    const int rc = tl_rope_at_pos_host(g->h, x, nH, d, rd, base, pos, S);
    return rc ? fail(rc, "%s", tl_last_error()) : 0;
}
int g_store(void *c, int layer, int start, const float *k, const float *v, int rows, int cols) {
    GpuOps *g = (GpuOps *)c;
    (void)rows;
    const int rc = tl_kv_store_host(g->h, layer, 0, start, k, v, cols);
    return rc ? fail(rc, "%s", tl_last_error()) : 0;
}
int g_full(void *c, const float *q, const float *k, const float *v, int S, int nH, int nKv, int d, float *out) {
    GpuOps *g = (GpuOps *)c;
    const int rc = tl_attention_full_host(g->h, q, k, v, S, nH, nKv, d, out);
    return rc ? fail(rc, "%s", tl_last_error()) : 0;
}
int g_cached(void *c, int layer, const float *q, int curLen, int nH, int nKv, int d, float *out) {
    GpuOps *g = (GpuOps *)c;
    const int rc = tl_attention_cached_host(g->h, layer, 0, q, curLen, nH, nKv, d, out);
    return rc ? fail(rc, "%s", tl_last_error()) : 0;
}

int g_prefill_at(void *c, int layer, int start, const float *q, const float *k, const float *v, int S, float *out) {
    GpuOps *g = (GpuOps *)c;
    const int rc = tl_prefill_layer_at_host(g->h, layer, 0, start, q, k, v, S, out);
    return rc ? fail(rc, "%s", tl_last_error()) : 0;
}

}  // namespace

extern "C" {

const char *tlh_last_error(void) { return g_err.c_str(); }

}  // extern "C"

tlh_model::~tlh_model() {
    if (map) munmap(map, mapSize);
}

namespace {

// float32 of a mapped tensor, row by row (getTensor's dequantisation, model.nim:116-123).
void dequant_view(const tlh_model::View &v, float *dst) {
    for (int64_t r = 0; r < v.rows; ++r) {
        const uint8_t *sp = v.src + (size_t)r * v.rowBytes;
        float *d = dst + (size_t)r * v.ne0;
        switch (v.type) {
            case 0: memcpy(d, sp, (size_t)v.ne0 * 4); break;
            case 1:
                for (int64_t c = 0; c < v.ne0; ++c) {
                    uint16_t hv;
                    memcpy(&hv, sp + 2 * c, 2);
                    d[c] = half_to_float(hv);
                }
                break;
            case 10: dequant_q2k(sp, d, (int)v.ne0); break;
            case 11: dequant_q3k(sp, d, (int)v.ne0); break;
            case 14: dequant_q6k(sp, d, (int)v.ne0); break;
            default: break;
        }
    }
}

// Parse a GGUF image (gguf_loader.nim:194-237, model.nim:50-103).  mapped: keep views of the
// tensors in the image (which the caller keeps alive); otherwise dequantise every tensor to
// float32 (model.nim:116-123) and keep the Q2_K ones as stored too.
tlh_model *parse_gguf(const uint8_t *data, size_t size, bool mapped, int nthreads, char *err, int errlen) {
    auto bad = [&](const char *msg) -> tlh_model * {
        if (err && errlen > 0) snprintf(err, (size_t)errlen, "%s", msg);
        g_err = msg;
        return nullptr;
    };
    struct {
        const uint8_t *p;
        size_t n;
        const uint8_t *data() const { return p; }
        size_t size() const { return n; }
    } buf{data, size};
    Reader r{buf.data(), buf.size()};
    if (buf.size() < 4 || memcmp(buf.data(), "GGUF", 4) != 0) return bad("GGUF: invalid magic");
    r.pos = 4;
    const uint32_t version = r.get<uint32_t>();
    if (version < 2) return bad("GGUF: version 1 is not supported");
    const uint64_t nTensors = r.get<uint64_t>(), nKv = r.get<uint64_t>();
    uint32_t alignment = 32;
    std::map<std::string, KvVal> kv;
    for (uint64_t i = 0; i < nKv && r.ok; ++i) {
        const std::string key = r.str();
        KvVal val;
        val.type = r.get<uint32_t>();
        if (val.type == STR) {
            val.s = r.str();
        } else if (val.type == ARR) {
            const uint32_t et = r.get<uint32_t>();
            val.arrN = r.get<uint64_t>();
            if (et == STR) {
                for (uint64_t j = 0; j < val.arrN && r.ok; ++j) r.str();
            } else {
                const size_t es = scalar_size(et);
                if (!es) return bad("GGUF: invalid array elem type");
                r.pos += (size_t)(es * val.arrN);
                if (r.pos > r.size) r.ok = false;
            }
        } else {
            const size_t es = scalar_size(val.type);
            if (!es) return bad("GGUF: invalid value type");
            if (val.type == F32) val.f = r.get<float>();
            else if (val.type == F64) val.f = r.get<double>();
            else {
                uint64_t u = 0;
                if (r.pos + es > r.size) r.ok = false;
                else memcpy(&u, r.p + r.pos, es);
                r.pos += es;
                val.u = u;
            }
        }
        if (key == "general.alignment" && val.type == U32) alignment = (uint32_t)val.u;
        kv[key] = val;
    }
    std::vector<TensorInfo> infos((size_t)nTensors);
    for (auto &ti : infos) {
        ti.name = r.str();
        ti.nDims = r.get<uint32_t>();
        if (ti.nDims > 4) return bad("GGUF: invalid tensor dims");
        for (uint32_t d = 0; d < ti.nDims; ++d) ti.ne[d] = r.get<uint64_t>();
        ti.type = r.get<int32_t>();
        ti.offset = r.get<uint64_t>();
    }
    if (!r.ok) return bad("GGUF: truncated file");
    const uint64_t dataOffset = (r.pos + alignment - 1) / alignment * alignment;

    tlh_model *m = new tlh_model();
    m->nthreads = nthreads < 1 ? 1 : nthreads;
    auto u32 = [&](const char *k, int &dst) {
        auto it = kv.find(k);
        if (it != kv.end() && it->second.type == U32) dst = (int)it->second.u;
    };
    auto f32 = [&](const char *k, float &dst) {
        auto it = kv.find(k);
        if (it != kv.end() && it->second.type == F32) dst = (float)it->second.f;
    };
    auto it = kv.find("general.architecture");
    if (it != kv.end() && it->second.type == STR) m->arch = it->second.s;
    u32("llama.vocab_size", m->hp.nVocab);
    u32("llama.context_length", m->hp.nCtx);
    u32("llama.embedding_length", m->hp.nEmb);
    u32("llama.block_count", m->hp.nLayer);
    u32("llama.feed_forward_length", m->hp.nFfn);
    u32("llama.attention.head_count", m->hp.nHead);
    u32("llama.attention.head_count_kv", m->hp.nHeadKv);
    u32("llama.rope.dimension_count", m->hp.ropeDim);
    f32("llama.rope.freq_base", m->hp.ropeFreqBase);
    f32("llama.attention.layer_norm_rms_epsilon", m->hp.rmsEps);
    if (m->hp.nVocab == 0) {
        auto t = kv.find("tokenizer.ggml.tokens");
        if (t != kv.end() && t->second.type == ARR) m->hp.nVocab = (int)t->second.arrN;
    }
    for (const auto &ti : infos) {
        const int64_t ne0 = (int64_t)ti.ne[0], count = (int64_t)(ti.ne[0] * ti.ne[1] * ti.ne[2] * ti.ne[3]);
        const int64_t rows = ne0 > 0 ? count / ne0 : 0;
        Tensor t;
        t.shape.assign(ti.ne, ti.ne + std::max<uint32_t>(ti.nDims, 1));
        const uint8_t *src = buf.data() + dataOffset + ti.offset;
        int64_t rowBytes = 0;
        void (*deq)(const uint8_t *, float *, int) = nullptr;
        switch (ti.type) {
            case 0: rowBytes = ne0 * 4; break;
            case 1: rowBytes = ne0 * 2; break;
            case 10: rowBytes = ne0 / QK_K * BLOCK_Q2K; deq = dequant_q2k; break;
            case 11: rowBytes = ne0 / QK_K * BLOCK_Q3K; deq = dequant_q3k; break;
            case 14: rowBytes = ne0 / QK_K * BLOCK_Q6K; deq = dequant_q6k; break;
            default: delete m; return bad(("unsupported ggml type for " + ti.name).c_str());
        }
        if (deq && ne0 % QK_K != 0) { delete m; return bad("k-quant row size must be multiple of 256"); }
        if (dataOffset + ti.offset + (uint64_t)(rowBytes * rows) > buf.size()) {
            delete m;
            return bad("GGUF: tensor data offset out of range");
        }
        if (mapped) {
            tlh_model::View &v = m->views[ti.name];
            v.type = ti.type;
            v.ne0 = ne0;
            v.rows = rows;
            v.rowBytes = rowBytes;
            v.shape = t.shape;
            v.src = src;
            continue;
        }
        t.data.resize((size_t)count);
        parallel_chunks((int)rows, 64, m->nthreads, [&](int s, int e) {
            for (int rr = s; rr < e; ++rr) {
                float *dst = t.data.data() + (size_t)rr * ne0;
                const uint8_t *sp = src + (size_t)rr * rowBytes;
                if (ti.type == 0) {
                    memcpy(dst, sp, (size_t)ne0 * 4);
                } else if (ti.type == 1) {
                    for (int64_t c = 0; c < ne0; ++c) {
                        uint16_t hv;
                        memcpy(&hv, sp + 2 * c, 2);
                        dst[c] = half_to_float(hv);
                    }
                } else {
                    deq(sp, dst, (int)ne0);
                }
            }
        });
        if (ti.type == 10) {
            tlh_model::Raw &r = m->q2k[ti.name];
            r.ne0 = ne0;
            r.ne1 = rows;
            r.bytes.assign(src, src + (size_t)(rowBytes * rows));
        }
        m->w[ti.name] = std::move(t);
    }
    return m;
}

}  // namespace

extern "C" {

tlh_model *tlh_model_load(const char *path, int nthreads, char *err, int errlen) {
    std::vector<uint8_t> buf;
    if (load_file(path, buf)) {
        if (err && errlen > 0) snprintf(err, (size_t)errlen, "%s", g_err.c_str());
        return nullptr;
    }
    return parse_gguf(buf.data(), buf.size(), false, nthreads, err, errlen);
}

tlh_model *tlh_model_open(const char *path, char *err, int errlen) {
    const int fd = open(path, O_RDONLY);
    if (fd < 0) {
        fail(-1, "cannot open %s", path);
        if (err && errlen > 0) snprintf(err, (size_t)errlen, "%s", g_err.c_str());
        return nullptr;
    }
    struct stat st;
    void *p = MAP_FAILED;
    if (fstat(fd, &st) == 0 && st.st_size > 0) p = mmap(nullptr, (size_t)st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (p == MAP_FAILED) {
        fail(-1, "cannot map %s", path);
        if (err && errlen > 0) snprintf(err, (size_t)errlen, "%s", g_err.c_str());
        return nullptr;
    }
    tlh_model *m = parse_gguf(static_cast<const uint8_t *>(p), (size_t)st.st_size, true, 1, err, errlen);
    if (!m) {
        munmap(p, (size_t)st.st_size);
        return nullptr;
    }
    m->map = p;
    m->mapSize = (size_t)st.st_size;
    return m;
}

void tlh_model_free(tlh_model *m) { delete m; }

int tlh_model_hparams(const tlh_model *m, tlh_hparams *out) {
    if (!m || !out) return fail(-1, "NULL argument");
    *out = m->hp;
    return 0;
}

int tlh_model_tensor(const tlh_model *m, const char *name, float *out, long cap, long *n) {
    if (!m || !name) return fail(-1, "NULL argument");
    if (m->map) {
        auto v = m->views.find(name);
        if (v == m->views.end()) return fail(-1, "missing tensor: %s", name);
        const size_t count = (size_t)(v->second.ne0 * v->second.rows);
        if (n) *n = (long)count;
        if (out) {
            std::vector<float> tmp(count);
            dequant_view(v->second, tmp.data());
            memcpy(out, tmp.data(), sizeof(float) * std::min<size_t>((size_t)cap, count));
        }
        return 0;
    }
    auto it = m->w.find(name);
    if (it == m->w.end()) return fail(-1, "missing tensor: %s", name);
    if (n) *n = (long)it->second.data.size();
    if (out) memcpy(out, it->second.data.data(), sizeof(float) * std::min<size_t>((size_t)cap, it->second.data.size()));
    return 0;
}

long tlh_generate(tlh_model *m, tlh_attn_ops *ops, const int32_t *prompt, int nPrompt, int nNew, int32_t *outIds,
                  float *gaps, float *attnOut, long attnCap) {
    if (!m || !ops || !prompt || nPrompt <= 0 || nNew <= 0 || !outIds) return fail(-1, "bad argument");
    if (m->map) return fail(-1, "a model opened with tlh_model_open has no float32 weights; the CPU forward pass needs tlh_model_load");
    int rc = ops->init_cache(ops->ctx, std::max(32, nNew + 32));  // src/tinylama.nim:47
    if (rc) return rc;
    Dump dump{attnOut, attnCap};
    std::vector<int32_t> toks(prompt, prompt + nPrompt);
    Tensor logits;
    if ((rc = forward(m, ops, toks, Pass::Prefill, logits, dump))) return rc;
    int32_t next = argmax_last(logits, m->hp.nVocab, gaps ? &gaps[0] : nullptr);
    outIds[0] = next;
    for (int j = 1; j < nNew; ++j) {
        if ((rc = forward(m, ops, std::vector<int32_t>{next}, Pass::Decode, logits, dump))) return rc;
        next = argmax_last(logits, m->hp.nVocab, gaps ? &gaps[j] : nullptr);
        outIds[j] = next;
    }
    return dump.n;
}

int tlh_session_init(tlh_attn_ops *ops, int nNew) {
    if (!ops || nNew <= 0) return fail(-1, "bad argument");
    return ops->init_cache(ops->ctx, std::max(32, nNew + 32));  // src/tinylama.nim:47
}

long tlh_run_prompt(tlh_model *m, tlh_attn_ops *ops, const int32_t *prompt, int nPrompt, int nNew, int chunked,
                    int32_t *outIds, float *gaps, float *attnOut, long attnCap) {
    if (!m || !ops || !prompt || nPrompt <= 0 || nNew <= 0 || !outIds) return fail(-1, "bad argument");
    if (m->map) return fail(-1, "a model opened with tlh_model_open has no float32 weights; the CPU forward pass needs tlh_model_load");
    Dump dump{attnOut, attnCap};
    std::vector<int32_t> toks(prompt, prompt + nPrompt);
    Tensor logits;
    int rc = 0;
    if (ops->curLen == 0) {
        // the first line: forwardPrefill over its tokens (src/tinylama.nim:53-55)
        if ((rc = forward(m, ops, toks, Pass::Prefill, logits, dump))) return rc;
    } else if (chunked && ops->prefill_at) {
        if ((rc = forward(m, ops, toks, Pass::Continue, logits, dump))) return rc;
    } else {
        // a later line: one forwardDecode per token (src/tinylama.nim:70-73)
        for (int32_t t : toks)
            if ((rc = forward(m, ops, std::vector<int32_t>{t}, Pass::Decode, logits, dump))) return rc;
    }
    int32_t next = argmax_last(logits, m->hp.nVocab, gaps ? &gaps[0] : nullptr);
    outIds[0] = next;
    for (int j = 1; j < nNew; ++j) {
        if ((rc = forward(m, ops, std::vector<int32_t>{next}, Pass::Decode, logits, dump))) return rc;
        next = argmax_last(logits, m->hp.nVocab, gaps ? &gaps[j] : nullptr);
        outIds[j] = next;
    }
    return dump.n;
}

int tlh_model_to_gpu(const tlh_model *m, tl_model *g) {
    if (!m || !g) return fail(-1, "bad argument");
    if (m->map) {
        // straight from the mapped file: Q2_K and float32 tensors as stored, the others
        // dequantised one tensor at a time
        for (const auto &kv : m->views) {
            const tlh_model::View &v = kv.second;
            int rc;
            if (v.type == 10 || v.type == 0) {
                rc = tl_model_set_tensor(g, kv.first.c_str(), v.type == 10 ? TL_GGML_Q2_K : TL_GGML_F32, v.src, v.ne0,
                                         v.rows);
            } else {
                std::vector<float> tmp((size_t)(v.ne0 * v.rows));
                dequant_view(v, tmp.data());
                rc = tl_model_set_tensor(g, kv.first.c_str(), TL_GGML_F32, tmp.data(), v.ne0, v.rows);
            }
            if (rc) return fail(rc, "%s", tl_last_error());
        }
        return 0;
    }
    for (const auto &kv : m->w) {
        const Tensor &t = kv.second;
        const int64_t ne0 = t.shape.empty() ? 1 : t.shape[0];
        const int64_t ne1 = ne0 > 0 ? (int64_t)t.data.size() / ne0 : 0;
        auto q = m->q2k.find(kv.first);
        const int rc = q != m->q2k.end()
                           ? tl_model_set_tensor(g, kv.first.c_str(), TL_GGML_Q2_K, q->second.bytes.data(), ne0, ne1)
                           : tl_model_set_tensor(g, kv.first.c_str(), TL_GGML_F32, t.data.data(), ne0, ne1);
        if (rc) return fail(rc, "%s", tl_last_error());
    }
    return 0;
}

tlh_attn_ops *tlh_gpu_attn_ops_create(int nLayer, int nHead, int nHeadKv, int headDim, int ropeDim, float base,
                                      int device) {
    GpuOps *g = new GpuOps();
    g->nLayer = nLayer;
    g->nHead = nHead;
    g->nHeadKv = nHeadKv;
    g->headDim = headDim;
    g->ropeDim = ropeDim > 0 ? ropeDim : headDim;
    g->base = base;
    g->device = device;
    g->ops.ctx = g;
    g->ops.init_cache = g_init;
    g->ops.rope_single = g_rope_single;
    g->ops.rope_at_pos = g_rope_at_pos;
    g->ops.store_kv = g_store;
    g->ops.attention_full = g_full;
    g->ops.attention_cached = g_cached;
    g->ops.prefill_at = g_prefill_at;
    return &g->ops;  // ops is the first member: the pointer is also the GpuOps*
}

void tlh_gpu_attn_ops_destroy(tlh_attn_ops *ops) {
    if (!ops) return;
    GpuOps *g = (GpuOps *)ops->ctx;
    if (g->h) tl_attn_destroy(g->h);
    delete g;
}

}  // extern "C"
