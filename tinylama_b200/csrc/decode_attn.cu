// decode_attn.cu -- split-KV ("flash-decoding") decode attention over the head-major cache.
//
// Replaces attentionCached (src/forward.nim:179-211): for every q-head h of a sequence,
//   s_j = q_h . k_{kvh,j} / sqrt(d),  p = softmax(s over j < curLen),  ctx_h = sum_j p_j v_{kvh,j}
// with kvh = h / (nHead / nHeadKv).  The reference reads the dim-major cache with stride
// maxLen and re-reads each kv-head once per q-head; here one CTA work unit (sequence, kv-head,
// chunk of positions) reads each K/V row from HBM once and serves all G = nHead/nHeadKv
// q-heads of the group.
//
// Structure (persistent kernel, grid = CTAs resident on the device):
//   * warp 4 (producer): streams contiguous K and V tiles of T positions (head-major layout
//     makes a tile one contiguous block) with cp.async.bulk into an NS-stage shared-memory
//     ring guarded by full/empty mbarriers.  No tensor map, no multicast.
//   * warps 0..3 (consumers): each owns PPW = T/4 positions of every tile, computes the G*PPW
//     dot products with lanes over head_dim, reduces them with a multi-value butterfly
//     (log2 shuffles per value), and keeps its own online-softmax state (m, l, o) in the
//     log2 domain.  At the end of a unit the four warp states are merged through shared
//     memory.
//   * a unit that covers a whole sequence writes ctx directly; otherwise it writes its
//     (o, m, l) partial to scratch and the last CTA to finish a (sequence, kv-head) merges
//     all chunks (threadfence + arrival counter; nobody waits on anybody).
#include <float.h>
#include <math.h>

#include <mutex>

#include "common.cuh"
#include "decode_common.cuh"
#include "internal.h"

namespace tl {
namespace {

constexpr float kLog2e = 1.4426950408889634f;


template <typename KV, int D, int G>
struct DecCfg {
    static constexpr int VPL = D / 32;          // head_dim values per lane
    static constexpr int T = 32;                // positions per tile
    static constexpr int NW = 4;                // consumer warps
    static constexpr int PPW = T / NW;          // positions per warp per tile
    static constexpr int NV = G * PPW;          // dot products per warp per tile
    static constexpr int THREADS = 32 * (NW + 1);
    static constexpr int TILE_BYTES = T * D * (int)sizeof(KV);
    static constexpr int STAGE_BYTES = 2 * TILE_BYTES;
    // bytes in flight per CTA: 96 KB for f32 KV (2 CTAs/SM), 48 KB for bf16 KV, whose GQA
    // consumers need more warps per SM to hide latency (3 CTAs/SM)
    static constexpr int NS_RAW = (sizeof(KV) == 2 ? 49152 : 98304) / STAGE_BYTES;
    static constexpr int NS = NS_RAW < 2 ? 2 : (NS_RAW > 8 ? 8 : NS_RAW);
    // shared memory carve-up (bytes, all 16-aligned)
    static constexpr int OFF_STAGES = 0;
    static constexpr int OFF_BARS = OFF_STAGES + NS * STAGE_BYTES;
    static constexpr int OFF_UQ = OFF_BARS + 2 * NS * 8 + 16;           // unit queue
    static constexpr int OFF_SC = OFF_UQ + kUnitQBytes;                 // [NW][NV] scores
    static constexpr int OFF_WM = OFF_SC + NW * NV * 4;                 // [NW][G] m
    static constexpr int OFF_WL = OFF_WM + NW * G * 4;                  // [NW][G] l
    static constexpr int OFF_WO = OFF_WL + NW * G * 4;                  // [NW][G][D] o
    static constexpr int OFF_CW = OFF_WO + NW * G * D * 4;              // [256][G] chunk weights
    static constexpr int OFF_PREFIX = OFF_CW + kMaxChunksPerSeq * G * 4;
    static size_t smem_bytes(int nseq) { return (size_t)OFF_PREFIX + 4 * (size_t)(nseq + 1) + 16; }
};

// Multi-value butterfly: N partial sums per lane -> after the call, lane holds the full
// (over 32 lanes) sum of R = max(1, N/32) of the N values in v[0..R).  The original index of
// v[r] is butterfly_index<N>(lane) + r.
template <int N>
__device__ __forceinline__ void butterfly(float (&v)[N], int lane) {
    int h = N / 2;
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) {
        if (h >= 1) {
            const bool upper = (lane & m) != 0;
#pragma unroll
            for (int i = 0; i < N / 2; ++i) {
                if (i < h) {
                    const float send = upper ? v[i] : v[i + h];
                    const float keep = upper ? v[i + h] : v[i];
                    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, m);
                }
            }
            h >>= 1;
        } else {
            v[0] += __shfl_xor_sync(0xffffffffu, v[0], m);
        }
    }
}
template <int N>
__device__ __forceinline__ int butterfly_index(int lane) {
    int idx = 0, h = N / 2;
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) {
        if (h >= 1) {
            if (lane & m) idx += h;
            h >>= 1;
        }
    }
    return idx;
}

template <typename KV, int D, int G>
__global__ void __launch_bounds__(DecCfg<KV, D, G>::THREADS)
decode_kernel(const DecodeArgs a) {
    using C = DecCfg<KV, D, G>;
    extern __shared__ __align__(1024) uint8_t smem[];
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + C::OFF_BARS);
    uint64_t *empty = full + C::NS;
    volatile int *abort_flag = reinterpret_cast<volatile int *>(empty + C::NS);
    int *is_last_flag = const_cast<int *>(reinterpret_cast<volatile int *>(abort_flag) + 1);
    int *max_nch = is_last_flag + 1;
    float *sc = reinterpret_cast<float *>(smem + C::OFF_SC);
    float *wm = reinterpret_cast<float *>(smem + C::OFF_WM);
    float *wl = reinterpret_cast<float *>(smem + C::OFF_WL);
    float *wo = reinterpret_cast<float *>(smem + C::OFF_WO);
    float *cw = reinterpret_cast<float *>(smem + C::OFF_CW);
    int *prefix = reinterpret_cast<int *>(smem + C::OFF_PREFIX);
    // lens are kept in the high part of the prefix region: prefix[nseq+1], lens after it
    int *lens = prefix + (a.nseq + 1);
    UnitQueue *uq = reinterpret_cast<UnitQueue *>(smem + C::OFF_UQ);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    unsigned *err = a.err;

    // ---- schedule: per-sequence chunk counts and their exclusive prefix (warp 0) ----------
    if (tid == 0) {
        for (int s = 0; s < C::NS; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], C::NW);
        }
        for (int s = 0; s < kUnitQ; ++s) {
            mbar_init(&uq->full[s], 1);
            mbar_init(&uq->empty[s], C::NW);
        }
        *abort_flag = 0;
        fence_mbar_init();
    }
    // launched behind the RoPE/append kernel: positions, q and the cache are read after it
    pdl_wait();
    if (warp == 0) build_schedule(a, prefix, lens, max_nch, lane, err);
    __syncthreads();
    const int total_units = prefix[a.nseq] * a.nHeadKv;
    // The host sizes the scratch and the chunk length; refuse (uniformly) if they do not fit.
    if (max_nch[0] > kMaxChunksPerSeq ||
        (max_nch[0] > 1 && decode_partial_floats_dev(total_units, G, D) > a.partial_cap)) {
        if (tid == 0) atomicOr(err, TL_DEVERR_BAD_ARG);
        return;
    }
    const float qscale = kLog2e / sqrtf((float)D);

    if (warp == C::NW) {
        // ================= producer ==================
        if (lane == 0) {
            const uint64_t pol = policy_evict_first();
            int stage = 0;
            uint32_t phase = 0;
            long issued = 0;
            bool ok = true;
            int qs = 0, u = 0;
            uint32_t qp = 0;
            bool first = true;
            while (ok) {
                if (!unitq_push(a, uq, prefix, total_units, qs, qp, u, first, err, abort_flag)) { ok = false; break; }
                if (u < 0) break;
                const Unit un = decode_unit(a, prefix, lens, u);
                const int64_t row0 = a.kv.row(a.layer, a.slot0 + un.b, un.g, 0);
                const KV *kb = reinterpret_cast<const KV *>(a.kv.k) + row0 * D;
                const KV *vb = reinterpret_cast<const KV *>(a.kv.v) + row0 * D;
                for (int p = un.p0; p < un.p1; p += C::T) {
                    const int np = min(C::T, un.p1 - p);
                    if (!mbar_wait(&empty[stage], phase ^ 1u, err, abort_flag)) { ok = false; break; }
                    const uint32_t bytes = (uint32_t)(np * D * sizeof(KV));
                    uint8_t *st = smem + C::OFF_STAGES + stage * C::STAGE_BYTES;
                    mbar_arrive_expect_tx(&full[stage], 2 * bytes);
                    bulk_g2s_evict_first(st, kb + (int64_t)p * D, bytes, &full[stage], pol);
                    bulk_g2s_evict_first(st + C::TILE_BYTES, vb + (int64_t)p * D, bytes, &full[stage], pol);
                    ++issued;
                    if (++stage == C::NS) { stage = 0; phase ^= 1u; }
                }
            }
            if (ok) unitq_finish(a);
            if (!ok) {
                // drain: wait (bounded) for the copies this thread issued into the ring
                const int outstanding = issued < (long)C::NS ? (int)issued : C::NS;
                int s = stage;
                uint32_t ph = phase;
                for (int i = 0; i < outstanding; ++i) {
                    if (--s < 0) { s = C::NS - 1; ph ^= 1u; }
                    mbar_wait(&full[s], ph, err, nullptr);
                }
            }
        }
        return;
    }

    // ================= consumers ==================
    int stage = 0;
    uint32_t phase = 0;
    int qs = 0;
    uint32_t qp = 0;
    while (true) {
        const int u = unitq_pop(uq, qs, qp, err, abort_flag, lane);
        if (u < 0) break;
        const Unit un = decode_unit(a, prefix, lens, u);
        // q for the G heads of this group, pre-scaled so that scores are in log2 units
        float qf[G][C::VPL];
        const float *qrow = a.q + ((int64_t)un.b * a.nHead + (int64_t)un.g * G) * D + lane * C::VPL;
#pragma unroll
        for (int h = 0; h < G; ++h) {
#pragma unroll
            for (int v = 0; v < C::VPL; ++v) qf[h][v] = qrow[(int64_t)h * D + v] * qscale;
        }
        float m[G], l[G], o[G][C::VPL];
#pragma unroll
        for (int h = 0; h < G; ++h) {
            m[h] = -INFINITY;
            l[h] = 0.f;
#pragma unroll
            for (int v = 0; v < C::VPL; ++v) o[h][v] = 0.f;
        }
        bool ok = true;
        for (int p = un.p0; p < un.p1; p += C::T) {
            const int np = min(C::T, un.p1 - p);
            // warp-uniform verdict, so that the warp's shuffles and barriers stay converged
            ok = __all_sync(0xffffffffu, mbar_wait(&full[stage], phase, err, abort_flag));
            if (!ok) break;
            const KV *ks = reinterpret_cast<const KV *>(smem + C::OFF_STAGES + stage * C::STAGE_BYTES);
            const KV *vs = reinterpret_cast<const KV *>(smem + C::OFF_STAGES + stage * C::STAGE_BYTES + C::TILE_BYTES);
            const int jb = warp * C::PPW;
            // dot products: part[h*PPW + jj]
            float part[C::NV];
#pragma unroll
            for (int jj = 0; jj < C::PPW; ++jj) {
                float kv[C::VPL];
                VecLoad<KV, C::VPL>::run(ks + (jb + jj) * D + lane * C::VPL, kv);
#pragma unroll
                for (int h = 0; h < G; ++h) {
                    float acc = 0.f;
#pragma unroll
                    for (int v = 0; v < C::VPL; ++v) acc = fmaf(qf[h][v], kv[v], acc);
                    part[h * C::PPW + jj] = acc;
                }
            }
            butterfly<C::NV>(part, lane);
            constexpr int R = C::NV >= 32 ? C::NV / 32 : 1;
            const int base = butterfly_index<C::NV>(lane);
            // owners publish their scores, masking positions past the end of the tile
            float own[R];
#pragma unroll
            for (int r = 0; r < R; ++r) {
                const int idx = base + r;
                own[r] = (jb + idx % C::PPW < np) ? part[r] : -INFINITY;
                sc[warp * C::NV + idx] = own[r];
            }
            __syncwarp();
            // per-head tile maximum (every lane reads the G*PPW scores)
            float mnew[G];
#pragma unroll
            for (int h = 0; h < G; ++h) {
                float tmax = -INFINITY;
#pragma unroll
                for (int jj = 0; jj < C::PPW; jj += 4) {
                    const float4 t4 = *reinterpret_cast<const float4 *>(&sc[warp * C::NV + h * C::PPW + jj]);
                    tmax = fmaxf(tmax, fmaxf(fmaxf(t4.x, t4.y), fmaxf(t4.z, t4.w)));
                }
                mnew[h] = fmaxf(m[h], tmax);
            }
            __syncwarp();
            // each lane exponentiates only the score(s) it owns
#pragma unroll
            for (int r = 0; r < R; ++r) {
                const int idx = base + r;
                const int hidx = idx / C::PPW;
                float mh = mnew[0];
#pragma unroll
                for (int h = 1; h < G; ++h)
                    if (hidx == h) mh = mnew[h];
                sc[warp * C::NV + idx] = (own[r] == -INFINITY) ? 0.f : exp2f(own[r] - mh);
            }
            __syncwarp();
            float pr[G][C::PPW];
#pragma unroll
            for (int h = 0; h < G; ++h) {
                float psum = 0.f;
#pragma unroll
                for (int jj = 0; jj < C::PPW; jj += 4) {
                    const float4 t4 = *reinterpret_cast<const float4 *>(&sc[warp * C::NV + h * C::PPW + jj]);
                    pr[h][jj] = t4.x; pr[h][jj + 1] = t4.y; pr[h][jj + 2] = t4.z; pr[h][jj + 3] = t4.w;
                    psum += (t4.x + t4.y) + (t4.z + t4.w);
                }
                if (mnew[h] != m[h]) {  // warp-uniform: rescale only when the maximum moved
                    const float alpha = safe_exp2_diff(m[h], mnew[h]);
                    l[h] *= alpha;
#pragma unroll
                    for (int v = 0; v < C::VPL; ++v) o[h][v] *= alpha;
                    m[h] = mnew[h];
                }
                l[h] += psum;
            }
#pragma unroll
            for (int jj = 0; jj < C::PPW; ++jj) {
                if (jb + jj < np) {
                    float vv[C::VPL];
                    VecLoad<KV, C::VPL>::run(vs + (jb + jj) * D + lane * C::VPL, vv);
#pragma unroll
                    for (int h = 0; h < G; ++h) {
#pragma unroll
                        for (int v = 0; v < C::VPL; ++v) o[h][v] = fmaf(pr[h][jj], vv[v], o[h][v]);
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[stage]);
            if (++stage == C::NS) { stage = 0; phase ^= 1u; }
        }
        // ---- merge the four warp states (reached even after an abort, so that every
        // consumer warp arrives at the same named barriers) ----
#pragma unroll
        for (int h = 0; h < G; ++h) {
            if (lane == 0) { wm[warp * G + h] = m[h]; wl[warp * G + h] = l[h]; }
#pragma unroll
            for (int v = 0; v < C::VPL; ++v) wo[(warp * G + h) * D + lane * C::VPL + v] = o[h][v];
        }
        unit_epilogue<G, D, C::NW>(a, un, u, prefix, wm, wl, wo, cw, is_last_flag, tid, warp, lane);
        // shared scratch is reused by the next unit; leave together if any warp aborted
        if (named_bar_or(1, C::NW * 32, (!ok) || (*abort_flag != 0))) break;
    }
    // split-KV across GPUs: this CTA's share of the cross-rank merges, after its own units
    if (a.px.nranks > 0 && *abort_flag == 0) peer_merge_pairs<G, D, C::NW>(a, tid);
}

// Merge G per-rank (o, m, l) partials into the final context.
__global__ void lse_merge_kernel(const float *__restrict__ parts, int nparts, int rows, int D,
                                 float *__restrict__ out) {
    const int row = blockIdx.x;
    if (row >= rows) return;
    const int64_t stride_rank = (int64_t)rows * (D + 2);
    float M = -INFINITY;
    for (int r = 0; r < nparts; ++r) M = fmaxf(M, parts[r * stride_rank + (int64_t)row * (D + 2) + D]);
    float L = 0.f;
    for (int r = 0; r < nparts; ++r) {
        const float *pp = parts + r * stride_rank + (int64_t)row * (D + 2);
        L = fmaf(pp[D + 1], safe_exp2_diff(pp[D], M), L);
    }
    for (int dd = threadIdx.x; dd < D; dd += blockDim.x) {
        float O = 0.f;
        for (int r = 0; r < nparts; ++r) {
            const float *pp = parts + r * stride_rank + (int64_t)row * (D + 2);
            O = fmaf(pp[dd], safe_exp2_diff(pp[D], M), O);
        }
        out[(int64_t)row * D + dd] = (L > 0.f) ? O / L : 0.f;
    }
}

template <typename KV, int D, int G>
size_t smem_t(int nseq) {
    return DecCfg<KV, D, G>::smem_bytes(nseq) + 4 * (size_t)nseq;
}

template <typename KV, int D, int G>
cudaError_t launch_t(const DecodeArgs &a, int num_ctas, cudaStream_t s) {
    using C = DecCfg<KV, D, G>;
    const size_t smem = smem_t<KV, D, G>(a.nseq);
    auto kern = decode_kernel<KV, D, G>;
    // set the shared-memory limit only when it grows, so that steady-state launches (and CUDA
    // graph capture of them) make no attribute calls
    static size_t smem_set[64] = {};  // per device: attributes are per context
    int dev = 0;
    cudaGetDevice(&dev);
    size_t &cur = smem_set[dev & 63];
    if (smem > cur) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        cur = smem;
    }
    return launch_pdl(kern, dim3(num_ctas), dim3(C::THREADS), smem, s, a);
}

template <typename KV, int D>
cudaError_t launch_g(const DecodeArgs &a, int num_ctas, cudaStream_t s) {
    switch (a.nHead / a.nHeadKv) {
        case 1: return launch_t<KV, D, 1>(a, num_ctas, s);
        case 2: return launch_t<KV, D, 2>(a, num_ctas, s);
        case 4: return launch_t<KV, D, 4>(a, num_ctas, s);
        case 8: return launch_t<KV, D, 8>(a, num_ctas, s);
        default: return cudaErrorNotSupported;
    }
}

template <typename KV, int D, int G>
int occ_t(int nseq) {
    using C = DecCfg<KV, D, G>;
    int n = 0;
    const size_t smem = smem_t<KV, D, G>(nseq);
    cudaFuncSetAttribute(decode_kernel<KV, D, G>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, decode_kernel<KV, D, G>, C::THREADS, smem) != cudaSuccess) n = 1;
    return n < 1 ? 1 : n;
}

}  // namespace

cudaError_t launch_decode(const DecodeArgs &a, int num_ctas, cudaStream_t s) {
    if (decode_mma_covers(a.headDim, a.nHead / a.nHeadKv, a.kv.dtype)) {
        // bf16 caches, and f32 caches with G >= 4: tensor-core kernel; the CUDA-core kernel
        // below is used only if its tensor maps cannot be built
        const cudaError_t e = launch_decode_mma(a, num_ctas, s);
        if (e != cudaErrorNotSupported) return e;
    }
    if (a.cluster > 0) return cudaErrorNotSupported;  // cluster mode exists only in the tensor-core kernel
    if (a.headDim == 64) {
        return a.kv.dtype == TL_KV_F32 ? launch_g<float, 64>(a, num_ctas, s)
                                       : launch_g<__nv_bfloat16, 64>(a, num_ctas, s);
    }
    if (a.headDim == 128) {
        return a.kv.dtype == TL_KV_F32 ? launch_g<float, 128>(a, num_ctas, s)
                                       : launch_g<__nv_bfloat16, 128>(a, num_ctas, s);
    }
    return cudaErrorNotSupported;
}

static int decode_ctas_per_sm_uncached(int headDim, int group, int dtype, int nseq);

// The CTAs of one launch must all be resident at once (the split-KV exchange waits on CTAs of
// the same launch), and the shared memory of a launch grows with nseq: the occupancy is taken
// at the launch's own size, rounded up to a power of two (at least 256 sequences).
int decode_ctas_per_sm(int headDim, int group, int dtype, int nseq) {
    int bucket = 256, lg = 0;
    while (bucket < nseq && lg < 15) { bucket <<= 1; ++lg; }
    if (bucket < nseq) bucket = nseq;
    static int cache[16][2][2][9][16];  // [device][headDim 64/128][dtype][group][size bucket]
    static std::mutex mu;
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 16 || group < 1 || group > 8 || bucket > (256 << 15))
        return decode_ctas_per_sm_uncached(headDim, group, dtype, bucket);
    std::lock_guard<std::mutex> lock(mu);
    int &slot = cache[dev][headDim == 128][dtype == TL_KV_BF16][group][lg];
    if (slot == 0) slot = decode_ctas_per_sm_uncached(headDim, group, dtype, bucket);
    return slot;
}

static int decode_ctas_per_sm_uncached(int headDim, int group, int dtype, int nseq) {
    if (decode_mma_covers(headDim, group, dtype)) return decode_mma_ctas_per_sm(headDim, group, dtype, nseq);
#define TL_OCC(KV, D)                                  \
    switch (group) {                                   \
        case 1: return occ_t<KV, D, 1>(nseq);          \
        case 2: return occ_t<KV, D, 2>(nseq);          \
        case 4: return occ_t<KV, D, 4>(nseq);          \
        case 8: return occ_t<KV, D, 8>(nseq);          \
        default: return 1;                             \
    }
    if (headDim == 64) {
        if (dtype == TL_KV_F32) { TL_OCC(float, 64) } else { TL_OCC(__nv_bfloat16, 64) }
    } else if (headDim == 128) {
        if (dtype == TL_KV_F32) { TL_OCC(float, 128) } else { TL_OCC(__nv_bfloat16, 128) }
    }
#undef TL_OCC
    return 1;
}

size_t decode_smem_bytes(int headDim, int group, int dtype, int nseq) {
    if (decode_mma_covers(headDim, group, dtype)) return decode_mma_smem_bytes(headDim, group, dtype, nseq);
#define TL_SMEM(KV, D)                                     \
    switch (group) {                                       \
        case 1: return smem_t<KV, D, 1>(nseq);             \
        case 2: return smem_t<KV, D, 2>(nseq);             \
        case 4: return smem_t<KV, D, 4>(nseq);             \
        case 8: return smem_t<KV, D, 8>(nseq);             \
        default: return 0;                                 \
    }
    if (headDim == 64) {
        if (dtype == TL_KV_F32) { TL_SMEM(float, 64) } else { TL_SMEM(__nv_bfloat16, 64) }
    } else if (headDim == 128) {
        if (dtype == TL_KV_F32) { TL_SMEM(float, 128) } else { TL_SMEM(__nv_bfloat16, 128) }
    }
#undef TL_SMEM
    return 0;
}

size_t decode_partial_floats(int total_units, int group, int headDim) {
    return (size_t)total_units * group * (headDim + 2);
}

cudaError_t launch_lse_merge(const float *parts, int nparts, int nseq, int nHead, int headDim,
                             float *out, cudaStream_t s) {
    const int rows = nseq * nHead;
    lse_merge_kernel<<<rows, headDim, 0, s>>>(parts, nparts, rows, headDim, out);
    return cudaGetLastError();
}

}  // namespace tl
