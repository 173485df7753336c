// tl_attn_api.cu -- the C ABI of libtlattn.so (declared in include/tl_attn.h).
//
// Host-side runtime around the kernels: handle and KV-cache ownership, argument validation
// with the reference's error messages, the split-KV schedule, host<->device staging for the
// host tier, and the device error word.  No CPU fallback exists anywhere in this library: if
// a shape has no kernel the call fails with TL_ERR_UNSUPPORTED.
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <string>
#include <vector>

#include "common.cuh"
#include "internal.h"

using namespace tl;

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

#define TL_CUDA(call)                                                                         \
    do {                                                                                      \
        cudaError_t e_ = (call);                                                              \
        if (e_ != cudaSuccess)                                                                \
            return fail(e_ == cudaErrorMemoryAllocation ? TL_ERR_NOMEM : TL_ERR_CUDA,         \
                        "%s failed: %s", #call, cudaGetErrorString(e_));                      \
    } while (0)

#define TL_TRY(expr)            \
    do {                        \
        int r_ = (expr);        \
        if (r_ != TL_OK) return r_; \
    } while (0)

// Makes the handle's device current for the scope and restores the caller's device.
struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

size_t esize(int dtype) { return dtype == TL_KV_BF16 ? 2 : 4; }

bool supported_group(int g) { return g == 1 || g == 2 || g == 4 || g == 8; }

int check_shape(int nHead, int nHeadKv, int headDim) {
    if (nHead <= 0 || nHeadKv <= 0)
        return fail(TL_ERR_INVALID, "KV cache requires llama-style head_count");
    if (nHead % nHeadKv != 0)
        return fail(TL_ERR_INVALID, "GQA requires head_count divisible by head_count_kv");
    if (headDim != 64 && headDim != 128)
        return fail(TL_ERR_UNSUPPORTED, "headDim %d: kernels are built for 64 and 128", headDim);
    if (!supported_group(nHead / nHeadKv))
        return fail(TL_ERR_UNSUPPORTED, "GQA group %d: kernels are built for 1, 2, 4 and 8",
                    nHead / nHeadKv);
    return TL_OK;
}

int check_handle_shape(const tl_attn *h, int nHead, int nHeadKv, int headDim) {
    if (nHead != h->nHead || nHeadKv != h->nHeadKv || headDim != h->headDim)
        return fail(TL_ERR_INVALID,
                    "shape (%d,%d,%d) does not match the cache's (nHead %d, nHeadKv %d, headDim %d)",
                    nHead, nHeadKv, headDim, h->nHead, h->nHeadKv, h->headDim);
    return TL_OK;
}

int check_layer_slot(const tl_attn *h, int layer, int slot, int nseq = 1) {
    if (layer < 0 || layer >= h->nLayer)
        return fail(TL_ERR_INVALID, "layer %d out of range [0, %d)", layer, h->nLayer);
    if (nseq < 1 || slot < 0 || slot + nseq > h->maxBatch)
        return fail(TL_ERR_INVALID, "slots [%d, %d) out of range [0, %d)", slot, slot + nseq,
                    h->maxBatch);
    return TL_OK;
}

int ensure_io(tl_attn *h, size_t floats) {
    if (floats <= h->ioCap) return TL_OK;
    if (h->dIo) cudaFree(h->dIo);
    h->dIo = nullptr;
    h->ioCap = 0;
    size_t cap = std::max<size_t>(floats, 1 << 16);
    TL_CUDA(cudaMalloc(&h->dIo, cap * sizeof(float)));
    h->ioCap = cap;
    return TL_OK;
}

int ensure_partial(tl_attn *h, size_t floats) {
    if (floats <= h->partialCap) return TL_OK;
    if (h->dPartial) {
        // the old buffer may still be in use by queued work on any stream of this device
        TL_CUDA(cudaDeviceSynchronize());
        cudaFree(h->dPartial);
    }
    h->dPartial = nullptr;
    h->partialCap = 0;
    size_t cap = std::max<size_t>(floats + floats / 4, 1 << 16);
    TL_CUDA(cudaMalloc(&h->dPartial, cap * sizeof(float)));
    h->partialCap = cap;
    return TL_OK;
}

int ensure_qb(tl_attn *h, size_t bytes) {
    if (bytes <= h->qbCap) return TL_OK;
    if (h->dQb) {
        TL_CUDA(cudaDeviceSynchronize());
        cudaFree(h->dQb);
    }
    h->dQb = nullptr;
    h->qbCap = 0;
    TL_CUDA(cudaMalloc(&h->dQb, bytes));
    h->qbCap = bytes;
    return TL_OK;
}

cudaStream_t pick(const tl_attn *h, void *stream) {
    return stream ? reinterpret_cast<cudaStream_t>(stream) : h->stream;
}

// Split-KV schedule: chunk length and CTA count for one decode launch.
struct Plan {
    int chunk, ctas;
    size_t partial_floats;
    int cluster;  // > 0: cluster mode (one cluster of this many CTAs per (sequence, kv-head))
};

// Cluster mode: one thread-block cluster of up to 8 CTAs per (sequence, kv-head), CTA r of a
// cluster taking chunk r, merged through distributed shared memory -- no schedule, no unit
// queue, no global partials.  It needs every cluster resident at once (grid <= the resident
// CTAs) and is chosen for
//   * few short sequences (chunks of at most 512 positions: batch-1 decode, latency-bound), or
//   * sequences of about equal length (mean >= 3/4 of the longest) whose clusters fill at least
//     3/4 of the resident CTAs: every CTA then streams the same share, and there is no tail of
//     unevenly finished units or chunk merge to wait for.
// With the cross-GPU exchange the clusters must also be co-resident by the occupancy API's
// count, since every CTA waits for the other ranks' values of its pair after its own chunk.
// TL_DECODE_CLUSTER=0 in the environment of a call turns cluster mode off (read on every call).
bool cluster_mode_allowed() {
    const char *e = getenv("TL_DECODE_CLUSTER");
    return !(e && e[0] == '0');
}

bool plan_cluster(const tl_attn *h, int nseq, int nmax, long long tot, int ctas, bool exchange, Plan *p) {
    const int G = h->nHead / h->nHeadKv;
    if (!cluster_mode_allowed() || !decode_mma_covers(h->headDim, G, h->kvDtype) || nmax < 1) return false;
    constexpr int kTarget = 256, kShortChunk = 512, kMaxCl = 8, kTile = 64;
    const int cl = std::max(1, std::min(kMaxCl, (nmax + kTarget - 1) / kTarget));
    long long chunk = (nmax + cl - 1) / cl;
    chunk = std::max<long long>(kTile, (chunk + kTile - 1) / kTile * kTile);
    const long long grid = (long long)nseq * h->nHeadKv * cl;
    if (grid > ctas || chunk > INT32_MAX / 2) return false;
    const bool short_seqs = chunk <= kShortChunk;
    const bool uniform = tot * 4 >= (long long)nseq * nmax * 3;
    const bool fills = grid * 4 >= (long long)ctas * 3;
    if (!short_seqs && !(uniform && fills)) return false;
    if (exchange && grid / cl > decode_mma_cluster_capacity(h->headDim, G, h->kvDtype, cl)) return false;
    if (short_seqs && !exchange) {
        // few short sequences are latency-bound: spread each over up to 16 CTAs of 128 positions
        // (two tiles, both in flight at once) when that many fit; clusters of more than 8 (a
        // non-portable size) only where the device can hold one
        constexpr int kShortTarget = 128, kShortMaxCl = 16;
        int cl2 = std::min(kShortMaxCl, std::max(cl, (nmax + kShortTarget - 1) / kShortTarget));
        if (cl2 > kMaxCl && decode_mma_cluster_capacity(h->headDim, G, h->kvDtype, cl2) < 1) cl2 = kMaxCl;
        if (cl2 > cl) {
            long long chunk2 = (nmax + cl2 - 1) / cl2;
            chunk2 = std::max<long long>(kTile, (chunk2 + kTile - 1) / kTile * kTile);
            const long long grid2 = (long long)nseq * h->nHeadKv * cl2;
            if (grid2 <= ctas) {
                p->chunk = (int)chunk2;
                p->ctas = (int)grid2;
                p->partial_floats = 0;
                p->cluster = cl2;
                return true;
            }
        }
    }
    p->chunk = (int)chunk;
    p->ctas = (int)grid;
    p->partial_floats = 0;
    p->cluster = cl;
    return true;
}

Plan plan_decode(const tl_attn *h, int nseq, const int *pos_host, int pos_offset, int slice,
                 bool cluster_ok = false, bool exchange = false) {
    const int G = h->nHead / h->nHeadKv;
    const int occ = decode_ctas_per_sm(h->headDim, G, h->kvDtype, nseq);
    const int ctas = h->numSms * occ;
    long long tot = 0;
    int nmax = 0;
    std::vector<int> ns(nseq);
    for (int b = 0; b < nseq; ++b) {
        int n = slice;
        if (pos_host) {
            n = pos_host[b] + 1 - pos_offset;
            n = std::max(0, std::min(n, slice));
        }
        ns[b] = n;
        tot += n;
        nmax = std::max(nmax, n);
    }
    Plan p{};
    if (cluster_ok && plan_cluster(h, nseq, nmax, tot, ctas, exchange, &p)) return p;
    // Chunk length: about `upc` units per CTA, at most 4096 positions.  A unit has a fixed cost
    // (its q, the merge of the consumer warps and, when a sequence has several chunks, a partial
    // written and merged again) that outweighs the tail of unevenly finished units: at 256
    // sequences of L ~ U[256, 4096], 4 units per CTA of at most 1024 positions gave 0.66 of the
    // HBM peak on the bf16 GQA shape (32/4/64) and one unit per CTA of at most 4096 gave 0.88;
    // the f32 caches (two CTAs per SM, twice the bytes per position) do best with about three.
    const int upc = h->kvDtype == TL_KV_BF16 ? 1 : 3;
    long long want = (tot * h->nHeadKv + (long long)ctas * upc - 1) / ((long long)ctas * upc);
    int chunk = (int)std::min<long long>(4096, std::max<long long>(32, want));
    chunk = (chunk + 31) / 32 * 32;
    // at most 64 chunks per sequence: the last CTA of a sequence merges all of them
    const int min_chunk = ((nmax + 63) / 64 + 31) / 32 * 32;
    chunk = std::max(chunk, min_chunk);
    long long units = 0;
    bool multi = false;
    for (int b = 0; b < nseq; ++b) {
        const int nch = ns[b] <= 0 ? 1 : (ns[b] + chunk - 1) / chunk;
        multi |= nch > 1;
        units += (long long)nch * h->nHeadKv;
    }
    p.chunk = chunk;
    p.ctas = (int)std::max<long long>(1, std::min<long long>(units, ctas));
    p.partial_floats = multi ? decode_partial_floats((int)units, G, h->headDim) : 0;
    return p;
}

// A decode step (RoPE, append, attention) may run as one launch: when the plan picks cluster
// mode, the tensor-core kernel rotates q and the new k itself and writes k and v into the cache
// (DecodeArgs::Fuse).  TL_DECODE_FUSE=0 in a call's environment keeps the two launches.
bool fuse_allowed() {
    const char *e = getenv("TL_DECODE_FUSE");
    return !(e && e[0] == '0');
}

// rope (optional): the RoPE/append launch of a decode step, fused into the decode launch when
// the plan allows it, otherwise launched before it.
int run_decode(tl_attn *h, int layer, int slot0, int nseq, const int *pos_dev, const int *pos_host,
               const float *q, float *out, cudaStream_t s, int pos_offset, float *lse_out,
               const DecodeArgs::Peer *px = nullptr, const RopeAppendArgs *rope = nullptr) {
    // the decode kernels read a head's q in 16-byte vectors: an unaligned q is refused here
    // rather than faulting on the device
    if ((reinterpret_cast<uintptr_t>(q) & 15u) != 0) return fail(TL_ERR_INVALID, "q must be 16-byte aligned");
    Plan p = plan_decode(h, nseq, pos_host, pos_offset, h->maxLen, true, px != nullptr);
    TL_TRY(ensure_partial(h, std::max<size_t>(p.partial_floats, 1)));
    const RopeTab tab = make_rope_tab(h->ropeDim, h->ropeBase);
    const bool fused = rope && p.cluster > 0 && !px && !lse_out && pos_offset == 0 && fuse_allowed();
    if (rope && !fused) TL_CUDA(launch_rope_append(*rope, tab, s));
    DecodeArgs a{};
    a.q = q;
    a.out = out;
    a.pos = pos_dev;
    a.nseq = nseq;
    a.nHead = h->nHead;
    a.nHeadKv = h->nHeadKv;
    a.headDim = h->headDim;
    a.layer = layer;
    a.slot0 = slot0;
    a.pos_offset = pos_offset;
    a.chunk = p.chunk;
    a.kv = h->kv;
    a.partial = h->dPartial;
    a.partial_cap = h->partialCap;
    a.counter = h->dCounter + (size_t)slot0 * h->nHeadKv;
    a.work = h->dCounter + (size_t)h->maxBatch * h->nHeadKv;
    a.err = h->dErr;
    a.lse_out = lse_out;
    if (px) a.px = *px;
    a.cluster = p.cluster;
    if (fused) {
        a.fz.q = rope->q.ptr;
        a.fz.k = rope->k.ptr;
        a.fz.v = rope->v.ptr;
        a.fz.tab = tab;
    }
    cudaError_t e = launch_decode(a, p.ctas, s);
    if (e == cudaErrorNotSupported && p.cluster > 0) {
        // the tensor-core kernel could not be set up: plan again for the CUDA-core kernel
        if (fused) {
            a.fz = DecodeArgs::Fuse{};
            TL_CUDA(launch_rope_append(*rope, tab, s));
        }
        p = plan_decode(h, nseq, pos_host, pos_offset, h->maxLen);
        TL_TRY(ensure_partial(h, std::max<size_t>(p.partial_floats, 1)));
        a.chunk = p.chunk;
        a.partial = h->dPartial;
        a.partial_cap = h->partialCap;
        a.cluster = 0;
        e = launch_decode(a, p.ctas, s);
    }
    if (e == cudaErrorNotSupported) return fail(TL_ERR_UNSUPPORTED, "decode: shape not covered");
    TL_CUDA(e);
    return TL_OK;
}

RopeAppendArgs rope_args(tl_attn *h) {
    RopeAppendArgs a{};
    a.kv = h->kv;
    a.err = h->dErr;
    return a;
}

// Synchronise the stream, then read and clear the device error word.
int finish(tl_attn *h, cudaStream_t s) {
    unsigned word = 0;
    TL_CUDA(cudaMemcpyAsync(&word, h->dErr, sizeof word, cudaMemcpyDeviceToHost, s));
    TL_CUDA(cudaStreamSynchronize(s));
    if (word) {
        cudaMemsetAsync(h->dErr, 0, sizeof(unsigned), s);
        cudaMemsetAsync(h->dCounter, 0, sizeof(unsigned) * ((size_t)h->maxBatch * h->nHeadKv + 2), s);
        cudaStreamSynchronize(s);
        std::string bits;
        if (word & TL_DEVERR_POS_RANGE) bits += " position-out-of-range";
        if (word & TL_DEVERR_TIMEOUT) bits += " wait-timeout";
        if (word & TL_DEVERR_BAD_ARG) bits += " bad-argument";
        return fail(TL_ERR_DEVICE, "device error word 0x%x:%s", word, bits.c_str());
    }
    return TL_OK;
}

HeadView col_view(float *p, int H, int D, int S) {
    // reference column layout [H*D, S]: (h, d, token t) at (h*D + d)*S + t
    HeadView v{p, 0, 1, (int64_t)D * S, (int64_t)S};
    (void)H;
    return v;
}

HeadView tok_view(float *p, int H, int D, int S) {
    // token-major [B][S][H*D]
    HeadView v{p, (int64_t)S * H * D, (int64_t)H * D, (int64_t)D, 1};
    return v;
}

// q_rotated: the fp32 q view holds the rotated q (the RoPE kernel wrote it back); without it
// only the tensor-core path, which reads the bf16 copy, can run.
int prefill_attention(tl_attn *h, int layer, int slot0, int nseq, int S, HeadView q, HeadView out,
                      bool qb_ready, bool force_f32, cudaStream_t s, const int *pos0_dev = nullptr,
                      bool q_rotated = true) {
    PrefillArgs a{};
    a.q = q;
    a.out = out;
    a.kf.ptr = nullptr;
    a.vf.ptr = nullptr;
    a.pos0 = pos0_dev;
    a.nseq = nseq;
    a.ntok = S;
    a.nHead = h->nHead;
    a.nHeadKv = h->nHeadKv;
    a.headDim = h->headDim;
    a.layer = layer;
    a.slot0 = slot0;
    a.kv = h->kv;
    a.qb = h->dQb;
    a.err = h->dErr;
    if (!force_f32 && qb_ready) {
        cudaError_t e = launch_prefill_tc(a, s);
        if (e == cudaSuccess) return TL_OK;
        if (e != cudaErrorNotSupported) TL_CUDA(e);
        if (!q_rotated)
            return fail(TL_ERR_UNSUPPORTED, "prefill: the tensor-core kernel could not be set up for this shape");
    }
    cudaError_t e = launch_prefill_f32(a, s);
    if (e == cudaErrorNotSupported) return fail(TL_ERR_UNSUPPORTED, "prefill: shape not covered");
    TL_CUDA(e);
    return TL_OK;
}

bool tc_prefill_eligible(const tl_attn *h) { return h->kvDtype == TL_KV_BF16 && h->headDim == 64; }

int ensure_copy_streams(tl_attn *h) {
    if (h->cpIn) return TL_OK;
    TL_CUDA(cudaStreamCreateWithFlags(&h->cpOut, cudaStreamNonBlocking));
    for (int j = 0; j < 4; ++j) {
        TL_CUDA(cudaEventCreateWithFlags(&h->evIn[j], cudaEventDisableTiming));
        TL_CUDA(cudaEventCreateWithFlags(&h->evOut[j], cudaEventDisableTiming));
    }
    TL_CUDA(cudaEventCreateWithFlags(&h->evDone, cudaEventDisableTiming));
    TL_CUDA(cudaStreamCreateWithFlags(&h->cpIn, cudaStreamNonBlocking));  // last: marks the set complete
    return TL_OK;
}

// Split a batch into `parts` runs of consecutive sequences by their KV bytes (the attention
// time of a part follows its K/V bytes).  cut[j] .. cut[j+1] is part j.  Two parts are equal.
// Four parts take 1/8, 3/8, 3/8 and 1/8: only the copy in of the first part and the copy out of
// the last one are not hidden behind attention, so those two parts are the small ones.
int split_by_kv(const int *pos, int nseq, int parts, int *cut) {
    long long tot = 0;
    for (int b = 0; b < nseq; ++b) tot += pos[b] + 1;
    static const int kEnd4[4] = {1, 4, 7, 8};  // cumulative eighths
    auto reached = [&](long long acc, int j) {
        return parts == 4 ? acc * 8 >= tot * kEnd4[j - 1] : acc * parts >= tot * j;
    };
    int j = 1;
    long long acc = 0;
    cut[0] = 0;
    for (int b = 0; b < nseq && j < parts; ++b) {
        acc += pos[b] + 1;
        while (j < parts && reached(acc, j)) cut[j++] = b + 1;
    }
    while (j < parts) cut[j++] = nseq;
    cut[parts] = nseq;
    // drop empty parts
    int n = 0;
    for (int i = 0; i < parts; ++i)
        if (cut[i + 1] > cut[i]) cut[++n] = cut[i + 1];
    return n;
}

// The copies and launches of tl_decode_batch_host; on an error return, work may still be
// queued on the three streams.
int decode_batch_host_impl(tl_attn *h, int layer, int slot0, int nseq, const int *pos, const float *q,
                           const float *k, const float *v, float *out, long long kv_rows) {
    const int Dq = h->nHead * h->headDim, Dk = h->nHeadKv * h->headDim;
    const size_t nq = (size_t)nseq * Dq, nk = (size_t)nseq * Dk;
    TL_TRY(ensure_io(h, 2 * nq + 2 * nk));
    TL_TRY(ensure_copy_streams(h));
    float *dq = h->dIo, *dk = dq + nq, *dv = dk + nk, *dout = dv + nk;
    // Parts: the batch is cut into up to 4 runs of sequences; the copies in of part j+1 and out
    // of part j-1 (one copy stream each way) overlap the attention of part j on the handle's
    // stream.  Few K/V bytes (attention shorter than ~50 us at HBM speed) keep one part: there
    // the extra launches would cost more than the overlap saves.
    const double kv_bytes = (double)kv_rows * Dk * 2 * (h->kvDtype == TL_KV_F32 ? 4 : 2);
    int parts = kv_bytes >= 1.2e9 ? 4 : kv_bytes >= 3e8 ? 2 : 1;
    if (const char *e = getenv("TL_HOST_PARTS")) parts = std::max(1, std::min(4, atoi(e)));  // override
    parts = std::min(parts, nseq);
    int cut[5];
    parts = split_by_kv(pos, nseq, parts, cut);
    // the in-stream starts after whatever the handle's stream has queued (the cache writes)
    TL_CUDA(cudaEventRecord(h->evDone, h->stream));
    TL_CUDA(cudaStreamWaitEvent(h->cpIn, h->evDone, 0));
    TL_CUDA(cudaMemcpyAsync(h->dPos, pos, sizeof(int) * nseq, cudaMemcpyHostToDevice, h->cpIn));
    for (int j = 0; j < parts; ++j) {
        const size_t b0 = cut[j], nb = cut[j + 1] - cut[j];
        TL_CUDA(cudaMemcpyAsync(dq + b0 * Dq, q + b0 * Dq, nb * Dq * 4, cudaMemcpyHostToDevice, h->cpIn));
        TL_CUDA(cudaMemcpyAsync(dk + b0 * Dk, k + b0 * Dk, nb * Dk * 4, cudaMemcpyHostToDevice, h->cpIn));
        TL_CUDA(cudaMemcpyAsync(dv + b0 * Dk, v + b0 * Dk, nb * Dk * 4, cudaMemcpyHostToDevice, h->cpIn));
        TL_CUDA(cudaEventRecord(h->evIn[j], h->cpIn));
    }
    for (int j = 0; j < parts; ++j) {
        const int b0 = cut[j], nb = cut[j + 1] - cut[j];
        TL_CUDA(cudaStreamWaitEvent(h->stream, h->evIn[j], 0));
        TL_TRY(tl_decode_step(h, layer, slot0 + b0, nb, h->dPos + b0, pos + b0, dq + (size_t)b0 * Dq,
                              dk + (size_t)b0 * Dk, dv + (size_t)b0 * Dk, dout + (size_t)b0 * Dq, h->stream));
        TL_CUDA(cudaEventRecord(h->evOut[j], h->stream));
    }
    for (int j = 0; j < parts; ++j) {
        const size_t b0 = cut[j], nb = cut[j + 1] - cut[j];
        TL_CUDA(cudaStreamWaitEvent(h->cpOut, h->evOut[j], 0));
        TL_CUDA(cudaMemcpyAsync(out + b0 * Dq, dout + b0 * Dq, nb * Dq * 4, cudaMemcpyDeviceToHost, h->cpOut));
    }
    TL_CUDA(cudaEventRecord(h->evDone, h->cpOut));
    TL_CUDA(cudaStreamWaitEvent(h->stream, h->evDone, 0));
    return TL_OK;
}

}  // namespace

extern "C" {

const char *tl_last_error(void) { return g_err.c_str(); }
int tl_version(void) { return TL_ATTN_VERSION; }

int tl_attn_create(tl_attn **out, int nLayer, int nHead, int nHeadKv, int headDim, int ropeDim,
                   float ropeBase, int maxLen, int maxBatch, int kvDtype, int device) {
    if (!out) return fail(TL_ERR_INVALID, "out is NULL");
    *out = nullptr;
    TL_TRY(check_shape(nHead, nHeadKv, headDim));
    if (ropeDim == 0) ropeDim = headDim;
    if (ropeDim < 0 || ropeDim > headDim || (ropeDim & 1))
        return fail(TL_ERR_INVALID, "ropeDim %d must be even and <= headDim %d", ropeDim, headDim);
    if (nLayer <= 0 || maxLen <= 0 || maxBatch <= 0)
        return fail(TL_ERR_INVALID, "nLayer, maxLen and maxBatch must be positive");
    if (kvDtype != TL_KV_F32 && kvDtype != TL_KV_BF16)
        return fail(TL_ERR_INVALID, "kvDtype %d is neither TL_KV_F32 nor TL_KV_BF16", kvDtype);
    int ndev = 0;
    TL_CUDA(cudaGetDeviceCount(&ndev));
    if (device < 0 || device >= ndev)
        return fail(TL_ERR_INVALID, "device %d out of range [0, %d)", device, ndev);
    DeviceGuard g(device);
    tl_attn *h = new tl_attn();
    h->device = device;
    h->nLayer = nLayer;
    h->nHead = nHead;
    h->nHeadKv = nHeadKv;
    h->headDim = headDim;
    h->ropeDim = ropeDim;
    h->ropeBase = ropeBase;
    h->maxLen = maxLen;
    h->maxBatch = maxBatch;
    h->kvDtype = kvDtype;
    h->curLen.assign(maxBatch, 0);
    auto cleanup = [&](int code) {
        tl_attn_destroy(h);
        return code;
    };
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, device) != cudaSuccess)
        return cleanup(fail(TL_ERR_CUDA, "cudaGetDeviceProperties failed"));
    if (prop.major != 10)
        return cleanup(fail(TL_ERR_UNSUPPORTED, "device %d is sm_%d%d; this library is built for sm_100a",
                            device, prop.major, prop.minor));
    h->numSms = prop.multiProcessorCount;
    const size_t elems = (size_t)nLayer * maxBatch * nHeadKv * (size_t)maxLen * headDim;
    const size_t bytes = elems * esize(kvDtype);
    h->kv.nLayer = nLayer;
    h->kv.maxBatch = maxBatch;
    h->kv.nHeadKv = nHeadKv;
    h->kv.maxLen = maxLen;
    h->kv.headDim = headDim;
    h->kv.dtype = kvDtype;
    cudaError_t e;
    if ((e = cudaMalloc(&h->kv.k, bytes)) != cudaSuccess ||
        (e = cudaMalloc(&h->kv.v, bytes)) != cudaSuccess)
        return cleanup(fail(TL_ERR_NOMEM, "KV cache allocation of 2 x %zu bytes failed: %s", bytes,
                            cudaGetErrorString(e)));
    if ((e = cudaMemset(h->kv.k, 0, bytes)) != cudaSuccess ||
        (e = cudaMemset(h->kv.v, 0, bytes)) != cudaSuccess ||
        (e = cudaMalloc(&h->dPos, sizeof(int) * (size_t)maxBatch)) != cudaSuccess ||
        (e = cudaMalloc(&h->dErr, sizeof(unsigned) * 4)) != cudaSuccess ||
        (e = cudaMemset(h->dErr, 0, sizeof(unsigned) * 4)) != cudaSuccess ||
        (e = cudaMalloc(&h->dCounter, sizeof(unsigned) * ((size_t)maxBatch * nHeadKv + 2))) != cudaSuccess ||
        (e = cudaMemset(h->dCounter, 0, sizeof(unsigned) * ((size_t)maxBatch * nHeadKv + 2))) != cudaSuccess ||
        (e = cudaStreamCreateWithFlags(&h->stream, cudaStreamNonBlocking)) != cudaSuccess ||
        (e = cudaDeviceSynchronize()) != cudaSuccess)
        return cleanup(fail(TL_ERR_CUDA, "handle setup failed: %s", cudaGetErrorString(e)));
    *out = h;
    return TL_OK;
}

void tl_dist_finalize(tl_attn *h);

void tl_attn_destroy(tl_attn *h) {
    if (!h) return;
    DeviceGuard g(h->device);
    tl_dist_finalize(h);
    if (h->stream) cudaStreamSynchronize(h->stream);
    cudaFree(h->kv.k);
    cudaFree(h->kv.v);
    cudaFree(h->dPos);
    cudaFree(h->dErr);
    cudaFree(h->dCounter);
    cudaFree(h->dPartial);
    cudaFree(h->dIo);
    cudaFree(h->dQb);
    cudaFree(h->dGather);
    if (h->hPinned) cudaFreeHost(h->hPinned);
    for (int j = 0; j < 4; ++j) {
        if (h->evIn[j]) cudaEventDestroy(h->evIn[j]);
        if (h->evOut[j]) cudaEventDestroy(h->evOut[j]);
    }
    if (h->evDone) cudaEventDestroy(h->evDone);
    if (h->cpIn) cudaStreamDestroy(h->cpIn);
    if (h->cpOut) cudaStreamDestroy(h->cpOut);
    if (h->stream) cudaStreamDestroy(h->stream);
    delete h;
}

int tl_kv_get_len(const tl_attn *h, int slot, int *len) {
    if (!h || !len) return fail(TL_ERR_INVALID, "NULL argument");
    if (slot < 0 || slot >= h->maxBatch) return fail(TL_ERR_INVALID, "slot %d out of range", slot);
    *len = h->curLen[slot];
    return TL_OK;
}

int tl_kv_set_len(tl_attn *h, int slot, int len) {
    if (!h) return fail(TL_ERR_INVALID, "NULL handle");
    if (slot < 0 || slot >= h->maxBatch) return fail(TL_ERR_INVALID, "slot %d out of range", slot);
    if (len < 0 || len > h->maxLen) return fail(TL_ERR_RANGE, "length %d outside [0, %d]", len, h->maxLen);
    h->curLen[slot] = len;
    return TL_OK;
}

int tl_kv_reset(tl_attn *h) {
    if (!h) return fail(TL_ERR_INVALID, "NULL handle");
    DeviceGuard g(h->device);
    const size_t bytes = (size_t)h->nLayer * h->maxBatch * h->nHeadKv * (size_t)h->maxLen * h->headDim *
                         esize(h->kvDtype);
    TL_CUDA(cudaMemsetAsync(h->kv.k, 0, bytes, h->stream));
    TL_CUDA(cudaMemsetAsync(h->kv.v, 0, bytes, h->stream));
    TL_CUDA(cudaStreamSynchronize(h->stream));
    std::fill(h->curLen.begin(), h->curLen.end(), 0);
    return TL_OK;
}

int tl_kv_clone(tl_attn *dst, const tl_attn *src) {
    if (!dst || !src) return fail(TL_ERR_INVALID, "NULL handle");
    if (dst->nLayer != src->nLayer || dst->maxBatch != src->maxBatch || dst->nHeadKv != src->nHeadKv ||
        dst->maxLen != src->maxLen || dst->headDim != src->headDim || dst->kvDtype != src->kvDtype)
        return fail(TL_ERR_INVALID, "cloneCache: handles differ in shape");
    DeviceGuard g(dst->device);
    const size_t bytes = (size_t)src->nLayer * src->maxBatch * src->nHeadKv * (size_t)src->maxLen *
                         src->headDim * esize(src->kvDtype);
    if (dst->device == src->device) {
        TL_CUDA(cudaMemcpyAsync(dst->kv.k, src->kv.k, bytes, cudaMemcpyDeviceToDevice, dst->stream));
        TL_CUDA(cudaMemcpyAsync(dst->kv.v, src->kv.v, bytes, cudaMemcpyDeviceToDevice, dst->stream));
    } else {
        TL_CUDA(cudaMemcpyPeerAsync(dst->kv.k, dst->device, src->kv.k, src->device, bytes, dst->stream));
        TL_CUDA(cudaMemcpyPeerAsync(dst->kv.v, dst->device, src->kv.v, src->device, bytes, dst->stream));
    }
    TL_CUDA(cudaStreamSynchronize(dst->stream));
    dst->curLen = src->curLen;
    return TL_OK;
}

int tl_kv_read(tl_attn *h, int layer, int slot, float *k, float *v) {
    if (!h || !k || !v) return fail(TL_ERR_INVALID, "NULL argument");
    TL_TRY(check_layer_slot(h, layer, slot));
    DeviceGuard g(h->device);
    const int D = h->headDim, L = h->maxLen, H = h->nHeadKv;
    const size_t n = (size_t)H * L * D;
    const size_t es = esize(h->kvDtype);
    std::vector<uint8_t> kb(n * es), vb(n * es);
    const size_t off = (size_t)h->kv.row(layer, slot, 0, 0) * D * es;
    TL_CUDA(cudaMemcpyAsync(kb.data(), (const uint8_t *)h->kv.k + off, n * es, cudaMemcpyDeviceToHost, h->stream));
    TL_CUDA(cudaMemcpyAsync(vb.data(), (const uint8_t *)h->kv.v + off, n * es, cudaMemcpyDeviceToHost, h->stream));
    TL_CUDA(cudaStreamSynchronize(h->stream));
    auto get = [&](const std::vector<uint8_t> &buf, size_t i) -> float {
        if (es == 4) {
            float f;
            memcpy(&f, buf.data() + i * 4, 4);
            return f;
        }
        uint16_t b16;
        memcpy(&b16, buf.data() + i * 2, 2);
        uint32_t u = (uint32_t)b16 << 16;
        float f;
        memcpy(&f, &u, 4);
        return f;
    };
    // head-major [H][L][D] -> reference dim-major [H*D, L]
    for (int hh = 0; hh < H; ++hh)
        for (int p = 0; p < L; ++p)
            for (int d = 0; d < D; ++d) {
                const size_t src = ((size_t)hh * L + p) * D + d;
                const size_t dst = ((size_t)hh * D + d) * L + p;
                k[dst] = get(kb, src);
                v[dst] = get(vb, src);
            }
    return TL_OK;
}

// ---- host tier -------------------------------------------------------------------------------

int tl_rope_single_host(tl_attn *h, float *x, int nHead, int headDim, int ropeDim, float base,
                        int seqLen) {
    if (!h || !x) return fail(TL_ERR_INVALID, "NULL argument");
    if (nHead <= 0 || headDim <= 0 || (headDim & 1) || ropeDim < 0 || ropeDim > headDim ||
        ropeDim / 2 > kMaxRopePairs || seqLen < 0)
        return fail(TL_ERR_INVALID, "rope: bad shape");
    if (seqLen == 0) return TL_OK;
    DeviceGuard g(h->device);
    const size_t n = (size_t)nHead * headDim * seqLen;
    TL_TRY(ensure_io(h, n));
    TL_CUDA(cudaMemcpyAsync(h->dIo, x, n * 4, cudaMemcpyHostToDevice, h->stream));
    RopeAppendArgs a = rope_args(h);
    a.q = col_view(h->dIo, nHead, headDim, seqLen);
    a.nseq = 1;
    a.ntok = seqLen;
    a.nHead = nHead;
    a.nHeadKv = 1;
    a.headDim = headDim;
    a.pos0 = nullptr;
    a.pos0_scalar = 0;
    a.rope_q = true;
    TL_CUDA(launch_rope_append(a, make_rope_tab(ropeDim, base), h->stream));
    TL_CUDA(cudaMemcpyAsync(x, h->dIo, n * 4, cudaMemcpyDeviceToHost, h->stream));
    return finish(h, h->stream);
}

int tl_rope_at_pos_host(tl_attn *h, float *x, int nHead, int headDim, int ropeDim, float base,
                        int pos, int seqLen) {
    if (!h || !x) return fail(TL_ERR_INVALID, "NULL argument");
    if (nHead <= 0 || headDim <= 0 || (headDim & 1) || ropeDim < 0 || ropeDim > headDim ||
        ropeDim / 2 > kMaxRopePairs || seqLen <= 0)
        return fail(TL_ERR_INVALID, "rope: bad shape");
    DeviceGuard g(h->device);
    const size_t n = (size_t)nHead * headDim * seqLen;
    TL_TRY(ensure_io(h, n));
    TL_CUDA(cudaMemcpyAsync(h->dIo, x, n * 4, cudaMemcpyHostToDevice, h->stream));
    RopeAppendArgs a = rope_args(h);
    a.q = col_view(h->dIo, nHead, headDim, seqLen);
    a.q.st = 0;  // only column 0
    a.nseq = 1;
    a.ntok = 1;
    a.nHead = nHead;
    a.nHeadKv = 1;
    a.headDim = headDim;
    a.pos0 = nullptr;
    a.pos0_scalar = pos;
    a.rope_q = true;
    TL_CUDA(launch_rope_append(a, make_rope_tab(ropeDim, base), h->stream));
    TL_CUDA(cudaMemcpyAsync(x, h->dIo, n * 4, cudaMemcpyDeviceToHost, h->stream));
    return finish(h, h->stream);
}

int tl_kv_store_host(tl_attn *h, int layer, int slot, int startPos, const float *k,
                     const float *v, int cols) {
    if (!h || !k || !v) return fail(TL_ERR_INVALID, "NULL argument");
    TL_TRY(check_layer_slot(h, layer, slot));
    if (cols < 0 || startPos < 0) return fail(TL_ERR_INVALID, "storeKVRange: negative position or width");
    if ((long long)startPos + cols > h->maxLen)
        return fail(TL_ERR_RANGE, "storeKVRange: columns [%d, %d) exceed maxLen %d", startPos,
                    startPos + cols, h->maxLen);
    if (cols == 0) return TL_OK;
    DeviceGuard g(h->device);
    const int D = h->headDim, H = h->nHeadKv;
    const size_t n = (size_t)H * D * cols;
    TL_TRY(ensure_io(h, 2 * n));
    TL_CUDA(cudaMemcpyAsync(h->dIo, k, n * 4, cudaMemcpyHostToDevice, h->stream));
    TL_CUDA(cudaMemcpyAsync(h->dIo + n, v, n * 4, cudaMemcpyHostToDevice, h->stream));
    RopeAppendArgs a = rope_args(h);
    a.k = col_view(h->dIo, H, D, cols);
    a.v = col_view(h->dIo + n, H, D, cols);
    a.nseq = 1;
    a.ntok = cols;
    a.nHead = h->nHead;
    a.nHeadKv = H;
    a.headDim = D;
    a.pos0_scalar = startPos;
    a.store = true;
    a.layer = layer;
    a.slot0 = slot;
    TL_CUDA(launch_rope_append(a, make_rope_tab(h->ropeDim, h->ropeBase), h->stream));
    return finish(h, h->stream);
}

int tl_attention_full_host(tl_attn *h, const float *q, const float *k, const float *v,
                           int seqLen, int nHead, int nHeadKv, int headDim, float *ctx) {
    if (!h || !q || !k || !v || !ctx) return fail(TL_ERR_INVALID, "NULL argument");
    TL_TRY(check_shape(nHead, nHeadKv, headDim));
    if (seqLen < 0) return fail(TL_ERR_INVALID, "seqLen < 0");
    if (seqLen == 0) return TL_OK;
    DeviceGuard g(h->device);
    const size_t nq = (size_t)nHead * headDim * seqLen, nk = (size_t)nHeadKv * headDim * seqLen;
    TL_TRY(ensure_io(h, 2 * nq + 2 * nk));
    float *dq = h->dIo, *dk = dq + nq, *dv = dk + nk, *dc = dv + nk;
    TL_CUDA(cudaMemcpyAsync(dq, q, nq * 4, cudaMemcpyHostToDevice, h->stream));
    TL_CUDA(cudaMemcpyAsync(dk, k, nk * 4, cudaMemcpyHostToDevice, h->stream));
    TL_CUDA(cudaMemcpyAsync(dv, v, nk * 4, cudaMemcpyHostToDevice, h->stream));
    PrefillArgs a{};
    a.q = col_view(dq, nHead, headDim, seqLen);
    a.out = col_view(dc, nHead, headDim, seqLen);
    a.kf = col_view(dk, nHeadKv, headDim, seqLen);
    a.vf = col_view(dv, nHeadKv, headDim, seqLen);
    a.pos0 = nullptr;
    a.nseq = 1;
    a.ntok = seqLen;
    a.nHead = nHead;
    a.nHeadKv = nHeadKv;
    a.headDim = headDim;
    a.kv = h->kv;
    a.err = h->dErr;
    cudaError_t e = launch_prefill_f32(a, h->stream);
    if (e == cudaErrorNotSupported) return fail(TL_ERR_UNSUPPORTED, "attentionFull: shape not covered");
    TL_CUDA(e);
    TL_CUDA(cudaMemcpyAsync(ctx, dc, nq * 4, cudaMemcpyDeviceToHost, h->stream));
    return finish(h, h->stream);
}

int tl_attention_cached_host(tl_attn *h, int layer, int slot, const float *q, int curLen,
                             int nHead, int nHeadKv, int headDim, float *ctx) {
    if (!h || !q || !ctx) return fail(TL_ERR_INVALID, "NULL argument");
    TL_TRY(check_layer_slot(h, layer, slot));
    TL_TRY(check_handle_shape(h, nHead, nHeadKv, headDim));
    if (curLen < 1 || curLen > h->maxLen)
        return fail(TL_ERR_RANGE, "attentionCached: curLen %d outside [1, %d]", curLen, h->maxLen);
    DeviceGuard g(h->device);
    const size_t nq = (size_t)nHead * headDim;
    TL_TRY(ensure_io(h, 2 * nq));
    TL_CUDA(cudaMemcpyAsync(h->dIo, q, nq * 4, cudaMemcpyHostToDevice, h->stream));
    const int pos = curLen - 1;
    TL_CUDA(cudaMemcpyAsync(h->dPos, &pos, sizeof(int), cudaMemcpyHostToDevice, h->stream));
    TL_TRY(run_decode(h, layer, slot, 1, h->dPos, &pos, h->dIo, h->dIo + nq, h->stream, 0, nullptr));
    TL_CUDA(cudaMemcpyAsync(ctx, h->dIo + nq, nq * 4, cudaMemcpyDeviceToHost, h->stream));
    return finish(h, h->stream);
}

int tl_decode_layer_host(tl_attn *h, int layer, int slot, const float *q, const float *k,
                         const float *v, int pos, float *ctx) {
    if (!h || !q || !k || !v || !ctx) return fail(TL_ERR_INVALID, "NULL argument");
    TL_TRY(check_layer_slot(h, layer, slot));
    if (pos >= h->maxLen) return fail(TL_ERR_KV_FULL, "KV cache full");
    if (pos < 0) return fail(TL_ERR_INVALID, "negative position");
    return tl_decode_batch_host(h, layer, slot, 1, &pos, q, k, v, ctx);
}

int tl_decode_batch_host(tl_attn *h, int layer, int slot0, int nseq, const int *pos,
                         const float *q, const float *k, const float *v, float *out) {
    if (!h || !pos || !q || !k || !v || !out) return fail(TL_ERR_INVALID, "NULL argument");
    TL_TRY(check_layer_slot(h, layer, slot0, nseq));
    long long kv_rows = 0;
    for (int b = 0; b < nseq; ++b) {
        if (pos[b] >= h->maxLen) return fail(TL_ERR_KV_FULL, "KV cache full");
        if (pos[b] < 0) return fail(TL_ERR_INVALID, "negative position");
        kv_rows += pos[b] + 1;
    }
    DeviceGuard g(h->device);
    const int rc = decode_batch_host_impl(h, layer, slot0, nseq, pos, q, k, v, out, kv_rows);
    if (rc != TL_OK) {
        // what was queued may still read the caller's buffers: wait for it
        if (h->cpIn) cudaStreamSynchronize(h->cpIn);
        cudaStreamSynchronize(h->stream);
        if (h->cpOut) cudaStreamSynchronize(h->cpOut);
        return rc;
    }
    return finish(h, h->stream);
}

static int prefill_layer_host_impl(tl_attn *h, int layer, int slot, int startPos, const float *q,
                                   const float *k, const float *v, int seqLen, float *ctx) {
    if (!h || !q || !k || !v || !ctx) return fail(TL_ERR_INVALID, "NULL argument");
    TL_TRY(check_layer_slot(h, layer, slot));
    if (seqLen < 0) return fail(TL_ERR_INVALID, "seqLen < 0");
    if (startPos < 0) return fail(TL_ERR_INVALID, "negative start position");
    if ((long long)startPos + seqLen > h->maxLen)
        return fail(TL_ERR_RANGE, "prefill of positions [%d, %d) exceeds the KV cache (maxLen %d)", startPos,
                    startPos + seqLen, h->maxLen);
    if (seqLen == 0) return TL_OK;
    DeviceGuard g(h->device);
    const int D = h->headDim, Hq = h->nHead, Hk = h->nHeadKv;
    const size_t nq = (size_t)Hq * D * seqLen, nk = (size_t)Hk * D * seqLen;
    TL_TRY(ensure_io(h, 2 * nq + 2 * nk));
    float *dq = h->dIo, *dk = dq + nq, *dv = dk + nk, *dc = dv + nk;
    TL_CUDA(cudaMemcpyAsync(dq, q, nq * 4, cudaMemcpyHostToDevice, h->stream));
    TL_CUDA(cudaMemcpyAsync(dk, k, nk * 4, cudaMemcpyHostToDevice, h->stream));
    TL_CUDA(cudaMemcpyAsync(dv, v, nk * 4, cudaMemcpyHostToDevice, h->stream));
    const int *pos0_dev = nullptr;
    if (startPos > 0) {
        // the attention kernels take the start position from device memory
        TL_CUDA(cudaMemcpyAsync(h->dPos, &startPos, sizeof(int), cudaMemcpyHostToDevice, h->stream));
        pos0_dev = h->dPos;
    }
    const bool tc = tc_prefill_eligible(h);
    if (tc) TL_TRY(ensure_qb(h, nq * 2));
    RopeAppendArgs a = rope_args(h);
    a.q = col_view(dq, Hq, D, seqLen);
    a.k = col_view(dk, Hk, D, seqLen);
    a.v = col_view(dv, Hk, D, seqLen);
    a.nseq = 1;
    a.ntok = seqLen;
    a.nHead = Hq;
    a.nHeadKv = Hk;
    a.headDim = D;
    a.pos0_scalar = startPos;
    a.rope_q = a.rope_k = a.store = true;
    a.layer = layer;
    a.slot0 = slot;
    a.qb = tc ? h->dQb : nullptr;
    TL_CUDA(launch_rope_append(a, make_rope_tab(h->ropeDim, h->ropeBase), h->stream));
    TL_TRY(prefill_attention(h, layer, slot, 1, seqLen, col_view(dq, Hq, D, seqLen),
                             col_view(dc, Hq, D, seqLen), tc, false, h->stream, pos0_dev));
    TL_CUDA(cudaMemcpyAsync(ctx, dc, nq * 4, cudaMemcpyDeviceToHost, h->stream));
    return finish(h, h->stream);
}

int tl_prefill_layer_host(tl_attn *h, int layer, int slot, const float *q, const float *k,
                          const float *v, int seqLen, float *ctx) {
    return prefill_layer_host_impl(h, layer, slot, 0, q, k, v, seqLen, ctx);
}

int tl_prefill_layer_at_host(tl_attn *h, int layer, int slot, int startPos, const float *q, const float *k,
                             const float *v, int seqLen, float *ctx) {
    return prefill_layer_host_impl(h, layer, slot, startPos, q, k, v, seqLen, ctx);
}

// ---- device tier -------------------------------------------------------------------------------

int tl_decode_step(tl_attn *h, int layer, int slot0, int nseq, const int *pos_dev,
                   const int *pos_host, float *q, float *k, const float *v, float *out,
                   void *stream) {
    if (!h || !pos_dev || !q || !k || !v || !out) return fail(TL_ERR_INVALID, "NULL argument");
    TL_TRY(check_layer_slot(h, layer, slot0, nseq));
    if (pos_host)
        for (int b = 0; b < nseq; ++b)
            if (pos_host[b] >= h->maxLen) return fail(TL_ERR_KV_FULL, "KV cache full");
    DeviceGuard g(h->device);
    cudaStream_t s = pick(h, stream);
    const int D = h->headDim;
    RopeAppendArgs a = rope_args(h);
    a.q = tok_view(q, h->nHead, D, 1);
    a.k = tok_view(k, h->nHeadKv, D, 1);
    a.v = tok_view(const_cast<float *>(v), h->nHeadKv, D, 1);
    a.nseq = nseq;
    a.ntok = 1;
    a.nHead = h->nHead;
    a.nHeadKv = h->nHeadKv;
    a.headDim = D;
    a.pos0 = pos_dev;
    a.rope_q = a.rope_k = a.store = true;
    a.layer = layer;
    a.slot0 = slot0;
    return run_decode(h, layer, slot0, nseq, pos_dev, pos_host, q, out, s, 0, nullptr, nullptr, &a);
}

int tl_decode_attention(tl_attn *h, int layer, int slot0, int nseq, const int *pos_dev,
                        const int *pos_host, const float *q, float *out, void *stream) {
    if (!h || !pos_dev || !q || !out) return fail(TL_ERR_INVALID, "NULL argument");
    TL_TRY(check_layer_slot(h, layer, slot0, nseq));
    if (pos_host)
        for (int b = 0; b < nseq; ++b)
            if (pos_host[b] >= h->maxLen) return fail(TL_ERR_KV_FULL, "KV cache full");
    DeviceGuard g(h->device);
    return run_decode(h, layer, slot0, nseq, pos_dev, pos_host, q, out, pick(h, stream), 0, nullptr);
}

static int prefill_step_impl(tl_attn *h, int layer, int slot0, int nseq, int seqLen, float *q,
                             float *k, const float *v, float *out, void *stream, bool force_f32,
                             const int *pos0_dev = nullptr, const int *pos0_host = nullptr) {
    if (!h || !q || !k || !v || !out) return fail(TL_ERR_INVALID, "NULL argument");
    TL_TRY(check_layer_slot(h, layer, slot0, nseq));
    if (seqLen < 0) return fail(TL_ERR_INVALID, "seqLen < 0");
    if (seqLen > h->maxLen)
        return fail(TL_ERR_RANGE, "prefill of %d tokens exceeds the KV cache (maxLen %d)", seqLen, h->maxLen);
    if (pos0_host)
        for (int b = 0; b < nseq; ++b) {
            if (pos0_host[b] < 0) return fail(TL_ERR_INVALID, "negative start position");
            if ((long long)pos0_host[b] + seqLen > h->maxLen)
                return fail(TL_ERR_RANGE, "prefill of positions [%d, %d) exceeds the KV cache (maxLen %d)",
                            pos0_host[b], pos0_host[b] + seqLen, h->maxLen);
        }
    if (seqLen == 0) return TL_OK;
    DeviceGuard g(h->device);
    cudaStream_t s = pick(h, stream);
    const int D = h->headDim, Hq = h->nHead, Hk = h->nHeadKv;
    const bool tc = !force_f32 && tc_prefill_eligible(h);
    if (tc) TL_TRY(ensure_qb(h, (size_t)nseq * Hq * seqLen * D * 2));
    RopeAppendArgs a = rope_args(h);
    a.q = tok_view(q, Hq, D, seqLen);
    a.k = tok_view(k, Hk, D, seqLen);
    a.v = tok_view(const_cast<float *>(v), Hk, D, seqLen);
    a.nseq = nseq;
    a.ntok = seqLen;
    a.nHead = Hq;
    a.nHeadKv = Hk;
    a.headDim = D;
    a.pos0 = pos0_dev;
    a.pos0_scalar = 0;
    a.rope_q = a.rope_k = a.store = true;
    // the tensor-core path reads the bf16 copy of q and the cache, so the rotated fp32 q and k
    // need not be written back
    a.q_inplace = a.k_inplace = !tc;
    a.layer = layer;
    a.slot0 = slot0;
    a.qb = tc ? h->dQb : nullptr;
    TL_CUDA(launch_rope_append(a, make_rope_tab(h->ropeDim, h->ropeBase), s));
    return prefill_attention(h, layer, slot0, nseq, seqLen, tok_view(q, Hq, D, seqLen),
                             tok_view(out, Hq, D, seqLen), tc, force_f32, s, pos0_dev, !tc);
}

int tl_prefill_step_at(tl_attn *h, int layer, int slot0, int nseq, int seqLen, const int *pos0_dev,
                       const int *pos0_host, float *q, float *k, const float *v, float *out, void *stream) {
    if (!pos0_dev) return fail(TL_ERR_INVALID, "NULL argument");
    return prefill_step_impl(h, layer, slot0, nseq, seqLen, q, k, v, out, stream, false, pos0_dev, pos0_host);
}

int tl_prefill_step(tl_attn *h, int layer, int slot0, int nseq, int seqLen, float *q, float *k,
                    const float *v, float *out, void *stream) {
    return prefill_step_impl(h, layer, slot0, nseq, seqLen, q, k, v, out, stream, false);
}

int tl_prefill_step_f32(tl_attn *h, int layer, int slot0, int nseq, int seqLen, float *q,
                        float *k, const float *v, float *out, void *stream) {
    return prefill_step_impl(h, layer, slot0, nseq, seqLen, q, k, v, out, stream, true);
}

int tl_kv_store(tl_attn *h, int layer, int slot, int startPos, const float *k, const float *v,
                int cols, void *stream) {
    if (!h || !k || !v) return fail(TL_ERR_INVALID, "NULL argument");
    TL_TRY(check_layer_slot(h, layer, slot));
    if (cols < 0 || startPos < 0) return fail(TL_ERR_INVALID, "storeKVRange: negative position or width");
    if ((long long)startPos + cols > h->maxLen)
        return fail(TL_ERR_RANGE, "storeKVRange: columns [%d, %d) exceed maxLen %d", startPos,
                    startPos + cols, h->maxLen);
    if (cols == 0) return TL_OK;
    DeviceGuard g(h->device);
    RopeAppendArgs a = rope_args(h);
    a.k = tok_view(const_cast<float *>(k), h->nHeadKv, h->headDim, cols);
    a.v = tok_view(const_cast<float *>(v), h->nHeadKv, h->headDim, cols);
    a.nseq = 1;
    a.ntok = cols;
    a.nHead = h->nHead;
    a.nHeadKv = h->nHeadKv;
    a.headDim = h->headDim;
    a.pos0_scalar = startPos;
    a.store = true;
    a.layer = layer;
    a.slot0 = slot;
    TL_CUDA(launch_rope_append(a, make_rope_tab(h->ropeDim, h->ropeBase), pick(h, stream)));
    return TL_OK;
}

int tl_check_device(tl_attn *h, void *stream) {
    if (!h) return fail(TL_ERR_INVALID, "NULL handle");
    DeviceGuard g(h->device);
    return finish(h, pick(h, stream));
}

}  // extern "C"

// Used by dist.cu.
namespace tl {
int api_run_decode_lse(tl_attn *h, int layer, int slot0, int nseq, const int *pos_dev,
                       const int *pos_host, const float *q, float *lse_out, cudaStream_t s,
                       int pos_offset) {
    return run_decode(h, layer, slot0, nseq, pos_dev, pos_host, q, nullptr, s, pos_offset, lse_out);
}

int api_run_decode_peer(tl_attn *h, int layer, int slot0, int nseq, const int *pos_dev,
                        const int *pos_host, const float *q, float *out, cudaStream_t s, int pos_offset,
                        const DecodeArgs::Peer &px) {
    return run_decode(h, layer, slot0, nseq, pos_dev, pos_host, q, out, s, pos_offset, nullptr, &px);
}
int api_fail(int code, const char *msg) { return fail(code, "%s", msg); }
}  // namespace tl
