// decode_mma.cu -- split-KV decode attention for bf16 KV caches on the tensor cores.
//
// Same contract and schedule as the CUDA-core kernel in decode_attn.cu (attentionCached,
// src/forward.nim:179-211, batched), for caches stored in bf16.  With grouped-query attention
// the G q-heads of a kv-head share every K/V row, so per row the work is a tiny matrix product:
// S[G x T] = Q[G x d] K^T[d x T] and O[G x d] += P[G x T] V[T x d].  On the CUDA cores that costs
// ~G*d/16 FMAs plus cross-lane reductions per row; here it is a few warp-level
// mma.sync.m16n8k16 (bf16 in, fp32 accumulate) per 8 rows, with the G heads as the M rows of
// the fragment, so the kernel stays at the HBM roofline for any G <= 8.
//
//  * warp 4 (producer): 2-D TMA (tensor map over the whole cache, 64-column boxes with the
//    128-byte swizzle, no multicast) brings K and V tiles of T = 64 positions into an
//    NS-stage ring guarded by full/empty mbarriers.
//  * warps 0..3 (consumers): warp w owns positions 16w..16w+15 of every tile.
//      S = Q K^T: A = q with its bf16 hi part in fragment rows 0..7 and lo part in rows 8..15
//        (q keeps ~16 mantissa bits at the cost of one instruction), B = K fragments from
//        ldmatrix on the swizzled tile;
//      online softmax on the C fragment (row = head, reductions over the 4 lanes of a quad,
//        log2 domain, rescale only when the maximum grows past 2^8);
//      O += P V: the C fragment of S becomes the A fragment of P (hi rows 0..7, lo rows 8..15),
//        B = V fragments from ldmatrix.trans.
//  * end of unit: the warps' states go through shared memory to the shared merge
//    (decode_common.cuh).
//
// f32 caches with G >= 4 take the same path (on the CUDA cores such groups need ~G*2 flops per
// byte, more than the FP32 pipe delivers at HBM speed), on mma.sync.m16n8k8 with tf32 inputs.
// The f32 tiles arrive through TMA in 32-column boxes (128-byte swizzle); every q, K, V and P
// value is split in registers into a tf32 "big" part and the tf32 "small" remainder (x = big +
// small to 2^-22 relative).  q and p put big in fragment rows 0..7 and small in rows 8..15, and
// each product takes two MMAs (K big, K small; V big, V small), so all four cross terms are
// kept and the products are as accurate as fp32 ones.  A thread reads whole 16-byte chunks of
// the swizzled tile (conflict-free), which fixes the head_dim columns it serves: for S the k16
// block kt takes chunk 2*tq + (kt & 1) of box kt/2, for O the n8 tile nt holds column
// 32*(nt/4) + 4*n + (nt % 4).  q and the output use the same column order.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <math.h>

#include <mutex>

#include "common.cuh"
#include "decode_common.cuh"
#include "internal.h"

namespace tl {
namespace {

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescale = 8.0f;

template <typename KV, int D, int G>
struct MmaCfg {
    static constexpr bool F32 = sizeof(KV) == 4;
    static constexpr int T = 64;                     // positions per tile
    static constexpr int NW = 4;                     // consumer warps, 16 positions each
    static constexpr int THREADS = 32 * (NW + 1);
    static constexpr int BOX_COLS = 128 / (int)sizeof(KV);  // columns per 128-byte box row
    static constexpr int HALVES = D / BOX_COLS;      // boxes per row
    static constexpr int HALF_BYTES = T * 128;       // one box: 64 rows x 128 B
    static constexpr int TILE_BYTES = HALVES * HALF_BYTES;
    static constexpr int STAGE_BYTES = 2 * TILE_BYTES;
#ifndef TL_NS_BF16_64
#define TL_NS_BF16_64 3
#endif
#ifndef TL_MIN_BF16_64
#define TL_MIN_BF16_64 2
#endif
    static constexpr int NS = F32 ? 2 : (D == 128 ? 3 : TL_NS_BF16_64);
    static constexpr int MIN_CTAS = (F32 && D == 128) ? 1 : ((!F32 && D == 64) ? TL_MIN_BF16_64 : 2);  // register cap
    static constexpr int KT = D / 16;                // k16 steps over head_dim
    static constexpr int NT = D / 8;                 // n8 tiles over head_dim
    static constexpr int OFF_STAGES = 0;             // 1024-aligned (swizzle atoms)
    static constexpr int OFF_BARS = NS * STAGE_BYTES;
    static constexpr int OFF_UQ = OFF_BARS + 2 * NS * 8 + 16;  // unit queue
    static constexpr int OFF_WM = OFF_UQ + kUnitQBytes;
    static constexpr int OFF_WL = OFF_WM + NW * G * 4;
    static constexpr int OFF_WO = OFF_WL + NW * G * 4;
    static constexpr int OFF_CW = OFF_WO + NW * G * D * 4;
    static constexpr int OFF_CX = (OFF_CW + kMaxChunksPerSeq * G * 4 + 15) / 16 * 16;  // cluster mode:
    static constexpr int OFF_PREFIX = OFF_CX + 16 + G * (D + 2) * 4;  // o (16-B aligned), then (m, l) pairs
    static size_t smem_bytes(int nseq) { return 1024 + (size_t)OFF_PREFIX + 4 * (2 * (size_t)nseq + 1) + 16; }
};

__device__ __forceinline__ void tma_load_2d(void *smem_dst, const CUtensorMap *map, int x, int y, uint64_t *bar,
                                            uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(smem_dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

// D += A * B, m16n8k16, bf16 inputs, fp32 accumulators.  With G <= 8 heads, A rows 0..7 carry
// the bf16 "hi" part of q (or p) and rows 8..15 the "lo" remainder, so one instruction yields
// both products: d0,d1 = hi . B (row gid) and d2,d3 = lo . B (row gid+8), summed by the lane.
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t *>(&v);
}
// bf16 hi/lo split of a pair: x = hi + lo with |lo| <= 2^-9 |x|, both bf16
__device__ __forceinline__ void split2(float x0, float x1, uint32_t &hi, uint32_t &lo) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(x0, x1);
    hi = *reinterpret_cast<const uint32_t *>(&h);
    lo = pack2(x0 - __low2float(h), x1 - __high2float(h));
}

// D += A * B, m16n8k8, tf32 inputs, fp32 accumulators (f32 caches).  A rows 0..7 carry the
// tf32 "big" part of q (or p), rows 8..15 the "small" remainder.
__device__ __forceinline__ void mma1688(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                        uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// tf32 big/small split: x = big + small + e with |e| <= 2^-22 |x| (big, small: tf32 bit patterns)
__device__ __forceinline__ void split_tf32(float x, uint32_t &big, uint32_t &small) {
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(big) : "f"(x));
    const float r = x - __uint_as_float(big);
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(small) : "f"(r));
}

// address of 16-byte chunk `chunk` (0..7) of row `row` in a swizzled 64-column box
__device__ __forceinline__ uint32_t swz(uint32_t box, int row, int chunk) {
    return box + row * 128 + ((chunk ^ (row & 7)) << 4);
}

// ---- cluster mode: one cluster of CL CTAs per (sequence, kv-head), merged in shared memory ----
constexpr int kMaxCluster = 16;  // 8 is the portable size; 16 with the non-portable attribute
__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t cluster_size() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// address of the same shared-memory location in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t cluster_addr(const void *p, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
    return r;
}
// Distributed shared-memory loads of another CTA's (m, l) pair and four o values.  Volatile,
// so they stay after the cluster barrier, without a memory clobber, so that a thread's loads of
// all the ranks issue back to back and their latencies overlap.
__device__ __forceinline__ float2 ld_cluster_v2(uint32_t addr) {
    float2 v;
    asm volatile("ld.shared::cluster.v2.f32 {%0, %1}, [%2];" : "=f"(v.x), "=f"(v.y) : "r"(addr));
    return v;
}
__device__ __forceinline__ float4 ld_cluster_v4(uint32_t addr) {
    float4 v;
    asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "r"(addr));
    return v;
}
// The hardware cluster barrier, in its unaligned form (the producer warp's lanes reach it on
// different paths).  Every thread of every CTA of the cluster reaches each of the two barriers
// of the epilogue on every path, errors included, so neither can wait for a thread that has left.
__device__ __forceinline__ void cluster_barrier() {
    asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}

// The merged (O, M, L) of one head element: ctx = O / L, or (O, M, L) to the (o, lse) output,
// or to every rank's exchange buffer (split-KV across GPUs).
template <int D>
__device__ __forceinline__ void cluster_final(const DecodeArgs &a, int b, int head, int dd, float O, float M, float L) {
    if (a.px.nranks > 0) {
        peer_store_final<D>(a, b, head, dd, O, M, L);
    } else if (a.lse_out != nullptr) {
        float *dst = a.lse_out + ((int64_t)b * a.nHead + head) * (D + 2);
        dst[dd] = O;
        if (dd == 0) { dst[D] = M; dst[D + 1] = L; }
    } else {
        a.out[((int64_t)b * a.nHead + head) * D + dd] = (L > 0.f) ? O / L : 0.f;
    }
}

// Fused decode step: the cluster's G heads of q are rotated in place (the tl_decode_step
// contract), but only once every CTA of the cluster has read q.  Each CTA writes the groups of
// four q values it also merges (at most two per thread), from a copy loaded at the start.
template <int G, int D>
struct QStash {
    static constexpr int MAXG = (G * D / 4 + 127) / 128;  // groups per thread with one CTA
    float4 v[MAXG];
};
// first group and group count of this CTA's share: G*D/4 groups of four values split over CL
template <int G, int D>
__device__ __forceinline__ void cluster_share(uint32_t CL, uint32_t rank, int &j0, int &j1) {
    constexpr int E4 = G * D / 4;
    const int per = (E4 + (int)CL - 1) / (int)CL;
    j0 = min(E4, (int)rank * per);
    j1 = min(E4, j0 + per);
}
template <int G, int D, int NW>
__device__ __forceinline__ void q_stash_load(const DecodeArgs &a, const Unit &un, QStash<G, D> &qs, int tid) {
    int j0, j1;
    cluster_share<G, D>(cluster_size(), cluster_rank(), j0, j1);
#pragma unroll
    for (int k = 0; k < QStash<G, D>::MAXG; ++k) {
        const int j = j0 + tid + k * NW * 32;
        if (j < j1) {
            const int e = 4 * j, h = e / D, dd = e - h * D;
            qs.v[k] = *reinterpret_cast<const float4 *>(a.fz.q + ((int64_t)un.b * a.nHead + un.g * G + h) * D + dd);
        }
    }
}
template <int G, int D, int NW>
__device__ __forceinline__ void q_stash_write(const DecodeArgs &a, const Unit &un, const QStash<G, D> &qs,
                                              const float2 *cs, int tid) {
    int j0, j1;
    cluster_share<G, D>(cluster_size(), cluster_rank(), j0, j1);
#pragma unroll
    for (int k = 0; k < QStash<G, D>::MAXG; ++k) {
        const int j = j0 + tid + k * NW * 32;
        if (j < j1) {
            const int e = 4 * j, h = e / D, dd = e - h * D, i = dd >> 1;
            float4 x = qs.v[k];
            if (i < a.fz.tab.pairs) rope_rotate(x.x, x.y, cs[i].x, cs[i].y, x.x, x.y);
            if (i + 1 < a.fz.tab.pairs) rope_rotate(x.z, x.w, cs[i + 1].x, cs[i + 1].y, x.z, x.w);
            *reinterpret_cast<float4 *>(a.fz.q + ((int64_t)un.b * a.nHead + un.g * G + h) * D + dd) = x;
        }
    }
}

// End of the unit in cluster mode, run by the NW*32 consumer threads (the producer warp meets
// them at the two cluster barriers: producer_cluster_barriers).
//  1. The warps' (m, l, o) are merged into this CTA's own (cm, cl) pairs and co row.
//  2. Cluster barrier: every CTA's values are in its shared memory (and every CTA has read q).
//  3. CTA `rank` merges its 1/CL share of the G*D elements from all CTAs of the cluster through
//     distributed shared memory,
//       M = max_r m_r,  L = sum_r l_r 2^(m_r - M),  ctx = sum_r o_r 2^(m_r - M) / L,
//     with a thread's loads of every rank issued back to back, and writes that share of ctx (and
//     of the rotated q for a fused step).
//  4. Cluster barrier: no CTA leaves while another may still read its shared memory.
template <int G, int D, int NW>
__device__ __forceinline__ void cluster_epilogue(const DecodeArgs &a, const Unit &un, const float *wm, const float *wl,
                                                 const float *wo, float *cx, int tid, const QStash<G, D> &qst,
                                                 const float2 *fz_cs) {
    named_bar(1, NW * 32);
    float *co = cx;                                       // [G*D], 16-byte aligned
    float2 *cml = reinterpret_cast<float2 *>(cx + G * D);  // [G] (m, l)
    for (int e = tid; e < G * D; e += NW * 32) {
        const int h = e / D, dd = e - h * D;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < NW; ++w) M = fmaxf(M, wm[w * G + h]);
        float L = 0.f, O = 0.f;
#pragma unroll
        for (int w = 0; w < NW; ++w) {
            const float sw = safe_exp2_diff(wm[w * G + h], M);
            L = fmaf(wl[w * G + h], sw, L);
            O = fmaf(wo[(w * G + h) * D + dd], sw, O);
        }
        co[e] = O;
        if (dd == 0) cml[h] = make_float2(M, L);
    }
    const uint32_t CL = cluster_size(), rank = cluster_rank();
    named_bar(1, NW * 32);
    if (CL > 1) cluster_barrier();
    int j0, j1;
    cluster_share<G, D>(CL, rank, j0, j1);
    // With an exchange across GPUs each thread takes one (group, destination rank) pair, so
    // that the remote stores of a group go out from R threads at once rather than one after
    // the other from a single thread (the merge of the group is repeated by those threads).
    const int R = a.px.nranks > 0 ? a.px.nranks : 1;
    for (int q = tid; q < (j1 - j0) * R; q += NW * 32) {
        const int j = j0 + q / R, dest = q - (q / R) * R;
        const int e = 4 * j, h = e / D, dd = e - h * D;
        // the ranks in groups of 8 (registers), merged online: one group for clusters of up to 8
        constexpr int RG = 8;
        float M = -INFINITY, L = 0.f;
        float4 O = make_float4(0.f, 0.f, 0.f, 0.f);
        for (uint32_t r0 = 0; r0 < CL; r0 += RG) {
            float2 ml[RG];
            float4 o4[RG];
            if (CL == 1) {
                ml[0] = cml[h];
                o4[0] = *reinterpret_cast<const float4 *>(co + e);
            } else {
#pragma unroll
                for (uint32_t r = 0; r < (uint32_t)RG; ++r) {
                    if (r0 + r < CL) {
                        ml[r] = ld_cluster_v2(cluster_addr(&cml[h], r0 + r));
                        o4[r] = ld_cluster_v4(cluster_addr(co + e, r0 + r));
                    }
                }
            }
            float Mn = M;
#pragma unroll
            for (uint32_t r = 0; r < (uint32_t)RG; ++r)
                if (r0 + r < CL) Mn = fmaxf(Mn, ml[r].x);
            const float sc = safe_exp2_diff(M, Mn);
            L *= sc;
            O.x *= sc;
            O.y *= sc;
            O.z *= sc;
            O.w *= sc;
#pragma unroll
            for (uint32_t r = 0; r < (uint32_t)RG; ++r) {
                if (r0 + r < CL) {
                    const float w = safe_exp2_diff(ml[r].x, Mn);
                    L = fmaf(ml[r].y, w, L);
                    O.x = fmaf(o4[r].x, w, O.x);
                    O.y = fmaf(o4[r].y, w, O.y);
                    O.z = fmaf(o4[r].z, w, O.z);
                    O.w = fmaf(o4[r].w, w, O.w);
                }
            }
            M = Mn;
        }
        const int head = un.g * G + h;
        if (a.px.nranks > 0) {
            peer_store_group<D>(a, dest, un.b, head, dd, O, M, L);
        } else {
            cluster_final<D>(a, un.b, head, dd, O.x, M, L);
            cluster_final<D>(a, un.b, head, dd + 1, O.y, M, L);
            cluster_final<D>(a, un.b, head, dd + 2, O.z, M, L);
            cluster_final<D>(a, un.b, head, dd + 3, O.w, M, L);
        }
    }
    if (a.fz.k != nullptr) q_stash_write<G, D, NW>(a, un, qst, fz_cs, tid);
    if (CL > 1) cluster_barrier();
}
// the producer warp's part of the epilogue: the same two cluster barriers
__device__ __forceinline__ void producer_cluster_barriers() {
    if (cluster_size() > 1) {
        cluster_barrier();
        cluster_barrier();
    }
}

template <typename KV, int D, int G, bool CLU>
__global__ void __launch_bounds__(MmaCfg<KV, D, G>::THREADS, MmaCfg<KV, D, G>::MIN_CTAS)
decode_mma_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
                  const DecodeArgs a) {
    using C = MmaCfg<KV, D, G>;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    uint8_t *smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + C::OFF_BARS);
    uint64_t *empty = full + C::NS;
    volatile int *abort_flag = reinterpret_cast<volatile int *>(empty + C::NS);
    int *is_last_flag = const_cast<int *>(reinterpret_cast<volatile int *>(abort_flag) + 1);
    int *max_nch = is_last_flag + 1;
    float *wm = reinterpret_cast<float *>(smem + C::OFF_WM);
    float *wl = reinterpret_cast<float *>(smem + C::OFF_WL);
    float *wo = reinterpret_cast<float *>(smem + C::OFF_WO);
    float *cw = reinterpret_cast<float *>(smem + C::OFF_CW);
    int *prefix = reinterpret_cast<int *>(smem + C::OFF_PREFIX);
    int *lens = prefix + (a.nseq + 1);
    UnitQueue *uq = reinterpret_cast<UnitQueue *>(smem + C::OFF_UQ);
    float *cx = reinterpret_cast<float *>(smem + C::OFF_CX + 16);  // cluster mode: this CTA's (o, m, l)

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    unsigned *err = a.err;
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
    // cluster mode: every CTA's barriers exist before any CTA arrives on them
    if constexpr (CLU) cluster_sync_all();
    // a fused decode step: this thread's RoPE frequency (a table of the handle, written by no
    // kernel) is fetched before the wait
    static_assert(D / 2 <= C::NW * 32, "one RoPE pair per consumer thread");
    const bool fuse = CLU && a.fz.k != nullptr;
    float fz_theta = 0.f;
    if (fuse && tid < D / 2 && tid < a.fz.tab.pairs) fz_theta = a.fz.tab.theta[tid];
    // launched behind the RoPE/append kernel: positions, q and the cache are read after it
    pdl_wait();
    // a kernel launched behind this one with programmatic serialisation may start its own
    // independent prologue (it waits for this grid's completion before reading its output).
    // Not with a split-KV exchange: there the next call's clusters, placed while this grid's
    // merging CTAs still hold their slots, left a cluster without room until the first ones
    // ended (a second wave of ~20 us at 16384 positions per GPU); the next call then starts
    // when this grid ends.
    if (a.px.nranks == 0) pdl_launch_dependents();
    int total_units = 0;
    Unit cu{};
    // producer state (lane 0 of warp NW): ring stage and phase, copies issued
    int pstage = 0, pspec = 0;
    uint32_t pphase = 0;
    long pissued = 0;
    const uint64_t pol = policy_evict_first();
    // one K/V tile (positions p .. p+T of the rows from row0) into the next stage of the ring
    auto issue_tile = [&](int row0, int p) {
        uint8_t *st = smem + C::OFF_STAGES + pstage * C::STAGE_BYTES;
        mbar_arrive_expect_tx(&full[pstage], C::STAGE_BYTES);
#pragma unroll
        for (int hh = 0; hh < C::HALVES; ++hh) {
            tma_load_2d(st + hh * C::HALF_BYTES, &kmap, C::BOX_COLS * hh, row0 + p, &full[pstage], pol);
            tma_load_2d(st + C::TILE_BYTES + hh * C::HALF_BYTES, &vmap, C::BOX_COLS * hh, row0 + p, &full[pstage], pol);
        }
        ++pissued;
        if (++pstage == C::NS) { pstage = 0; pphase ^= 1u; }
    };
    const int gid = lane >> 2, tq = lane & 3;  // fragment row (head) and column pair
    const bool row_ok = gid < G;
    float4 qpre[C::KT];  // cluster mode: this lane's q values, loaded before the position is known
    if constexpr (!CLU) {
        if (warp == 0) build_schedule(a, prefix, lens, max_nch, lane, err);
        __syncthreads();
        total_units = prefix[a.nseq] * a.nHeadKv;
        if (max_nch[0] > kMaxChunksPerSeq ||
            (max_nch[0] > 1 && decode_partial_floats_dev(total_units, G, D) > a.partial_cap)) {
            if (tid == 0) atomicOr(err, TL_DEVERR_BAD_ARG);
            return;
        }
    } else {
        // this CTA's unit: chunk `rank` of (sequence, kv-head) `cluster index`
        __syncthreads();
        const int cl = (int)cluster_size(), rank = (int)cluster_rank();
        const int pair = (int)blockIdx.x / cl;
        cu.b = pair / a.nHeadKv;
        cu.g = pair - cu.b * a.nHeadKv;
        cu.c = rank;
        cu.nch = cl;
        // Before the position is read, the producer starts the chunk's first tiles (at most the
        // ring's depth, into stages that start free) and the consumers load their q values.  A
        // chunk that turns out shorter leaves tiles unconsumed; the producer still waits for them.
        if (warp == C::NW && lane == 0) {
            const int row0 = (int)a.kv.row(a.layer, a.slot0 + cu.b, cu.g, 0);
            for (; pspec < C::NS && pspec * C::T < a.chunk; ++pspec) issue_tile(row0, rank * a.chunk + pspec * C::T);
        }
        if (warp < C::NW) {
            const float *qrow = a.q + ((int64_t)cu.b * a.nHead + (int64_t)cu.g * G + (row_ok ? gid : 0)) * D;
#pragma unroll
            for (int kt = 0; kt < C::KT; ++kt) {
                qpre[kt] = make_float4(0.f, 0.f, 0.f, 0.f);
                if (row_ok) {
                    if constexpr (C::F32) {
                        qpre[kt] = *reinterpret_cast<const float4 *>(qrow + 32 * (kt >> 1) + 4 * (2 * tq + (kt & 1)));
                    } else {
                        const float2 lo = *reinterpret_cast<const float2 *>(qrow + 16 * kt + 2 * tq);
                        const float2 hi = *reinterpret_cast<const float2 *>(qrow + 16 * kt + 2 * tq + 8);
                        qpre[kt] = make_float4(lo.x, lo.y, hi.x, hi.y);
                    }
                }
            }
        }
        cu.n = local_len(a, cu.b, err);
        cu.p0 = min(rank * a.chunk, cu.n);
        cu.p1 = min(cu.p0 + a.chunk, cu.n);
        // the host sized the chunks from its copy of the positions: a longer sequence on the
        // device would leave positions past the cluster's last chunk unread
        if (tid == 0 && rank == cl - 1 && (long long)cu.n > (long long)cl * a.chunk) atomicOr(err, TL_DEVERR_BAD_ARG);
    }
    // a decode step fused into this launch (cluster mode): this CTA's share of q for the in-place
    // rotation at the end, then the cos/sin of this sequence's position, for the rotation of q
    // (every CTA) and of the new k (the CTA whose chunk holds it)
    __shared__ float2 fz_cs[64];
    QStash<G, D> qst;
    if (fuse && warp < C::NW) q_stash_load<G, D, C::NW>(a, cu, qst, tid);
    const int fz_pos = fuse ? a.pos[cu.b] : -1;
    if (fuse && warp < C::NW) {
        if (tid < D / 2) fz_cs[tid] = tid < a.fz.tab.pairs ? rope_cos_sin(fz_pos, fz_theta) : make_float2(1.f, 0.f);
        named_bar(1, C::NW * 32);
    }

    if (warp == C::NW) {
        // ================= producer =================
        if (lane == 0) {
            bool ok = true;
            // the copies of one unit's tiles into the ring, from its tile `skip` on
            auto issue_unit = [&](const Unit &un, int skip) {
                const int row0 = (int)a.kv.row(a.layer, a.slot0 + un.b, un.g, 0);
                for (int p = un.p0 + skip * C::T; p < un.p1; p += C::T) {
                    if (!mbar_wait(&empty[pstage], pphase ^ 1u, err, abort_flag)) { ok = false; break; }
                    issue_tile(row0, p);
                }
            };
            if constexpr (CLU) {
                issue_unit(cu, pspec);
            } else {
                int qs = 0, u = 0;
                uint32_t qp = 0;
                bool first = true;
                while (ok) {
                    if (!unitq_push(a, uq, prefix, total_units, qs, qp, u, first, err, abort_flag)) { ok = false; break; }
                    if (u < 0) break;
                    issue_unit(decode_unit(a, prefix, lens, u), 0);
                }
            }
            if (!CLU && ok) unitq_finish(a);
            // wait (bounded) for every copy issued into this CTA's shared memory
            const int outstanding = pissued < (long)C::NS ? (int)pissued : C::NS;
            int s = pstage;
            uint32_t ph = pphase;
            for (int i = 0; i < outstanding; ++i) {
                if (--s < 0) { s = C::NS - 1; ph ^= 1u; }
                mbar_wait(&full[s], ph, err, nullptr);
            }
        }
        if constexpr (CLU) producer_cluster_barriers();
        return;
    }

    // ================= consumers =================
    const float C2 = kLog2e / sqrtf((float)D);
    int stage = 0;
    uint32_t phase = 0;
    int qs = 0;
    uint32_t qp = 0;
    // one unit: q fragments, the tile loop, then this warp's (m, l, o) into wm/wl/wo
    auto consume_unit = [&](const Unit &un) -> bool {
        // q fragments (A rows = heads of this kv group; rows >= G are zero): bf16 hi + lo for
        // bf16 caches; tf32 big + small of the four columns of one chunk per k16 block for f32
        uint32_t qh[C::KT][C::F32 ? 4 : 2], ql[C::KT][C::F32 ? 4 : 2];
        {
            const float *qrow = a.q + ((int64_t)un.b * a.nHead + (int64_t)un.g * G + (row_ok ? gid : 0)) * D;
#pragma unroll
            for (int kt = 0; kt < C::KT; ++kt) {
                if constexpr (C::F32) {
                    float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
                    if constexpr (CLU) x = qpre[kt];
                    else if (row_ok) x = *reinterpret_cast<const float4 *>(qrow + 32 * (kt >> 1) + 4 * (2 * tq + (kt & 1)));
                    if (fuse) {  // columns c, c+1 and c+2, c+3: pairs c/2 and c/2 + 1
                        const int pr0 = 16 * (kt >> 1) + 2 * (2 * tq + (kt & 1));
                        if (pr0 < a.fz.tab.pairs) rope_rotate(x.x, x.y, fz_cs[pr0].x, fz_cs[pr0].y, x.x, x.y);
                        if (pr0 + 1 < a.fz.tab.pairs) rope_rotate(x.z, x.w, fz_cs[pr0 + 1].x, fz_cs[pr0 + 1].y, x.z, x.w);
                    }
                    split_tf32(x.x, qh[kt][0], ql[kt][0]);
                    split_tf32(x.y, qh[kt][1], ql[kt][1]);
                    split_tf32(x.z, qh[kt][2], ql[kt][2]);
                    split_tf32(x.w, qh[kt][3], ql[kt][3]);
                } else {
                    float x0 = 0.f, x1 = 0.f, x2 = 0.f, x3 = 0.f;
                    if constexpr (CLU) {
                        x0 = qpre[kt].x; x1 = qpre[kt].y; x2 = qpre[kt].z; x3 = qpre[kt].w;
                    } else if (row_ok) {
                        const float2 lo = *reinterpret_cast<const float2 *>(qrow + 16 * kt + 2 * tq);
                        const float2 hi = *reinterpret_cast<const float2 *>(qrow + 16 * kt + 2 * tq + 8);
                        x0 = lo.x; x1 = lo.y; x2 = hi.x; x3 = hi.y;
                    }
                    if (fuse) {  // columns 16kt + 2tq (+1) and 16kt + 8 + 2tq (+1)
                        const int pr0 = 8 * kt + tq, pr1 = 8 * kt + 4 + tq;
                        if (pr0 < a.fz.tab.pairs) rope_rotate(x0, x1, fz_cs[pr0].x, fz_cs[pr0].y, x0, x1);
                        if (pr1 < a.fz.tab.pairs) rope_rotate(x2, x3, fz_cs[pr1].x, fz_cs[pr1].y, x2, x3);
                    }
                    split2(x0, x1, qh[kt][0], ql[kt][0]);
                    split2(x2, x3, qh[kt][1], ql[kt][1]);
                }
            }
        }
        float m = -INFINITY, l = 0.f;
        float o[C::NT][4];
#pragma unroll
        for (int nt = 0; nt < C::NT; ++nt) o[nt][0] = o[nt][1] = o[nt][2] = o[nt][3] = 0.f;
        bool ok = true;
        for (int p = un.p0; p < un.p1; p += C::T) {
            ok = __all_sync(0xffffffffu, mbar_wait(&full[stage], phase, err, abort_flag));
            if (!ok) break;
            const uint32_t kbox = smem_u32(smem + C::OFF_STAGES + stage * C::STAGE_BYTES);
            const uint32_t vbox = kbox + C::TILE_BYTES;
            const int r0 = warp * 16;  // first tile row of this warp
            if (fuse) {
                // the new token's row: the tile was loaded before the step's k and v were in the
                // cache, so the warp that owns the row writes it -- rotated k, and v -- into the
                // tile, into the cache and (k) back into its input
                const int rr = fz_pos - p;
                if (rr >= r0 && rr < r0 + 16 && fz_pos < un.p1) {
                    for (int i = lane; i < D / 2; i += 32) {
                        const int64_t src = ((int64_t)un.b * a.nHeadKv + un.g) * D + 2 * i;
                        float k0 = a.fz.k[src], k1 = a.fz.k[src + 1];
                        if (i < a.fz.tab.pairs) {
                            rope_rotate(k0, k1, fz_cs[i].x, fz_cs[i].y, k0, k1);
                            a.fz.k[src] = k0;
                            a.fz.k[src + 1] = k1;
                        }
                        const float v0 = a.fz.v[src], v1 = a.fz.v[src + 1];
                        const int64_t dst = a.kv.row(a.layer, a.slot0 + un.b, un.g, fz_pos) * D + 2 * i;
                        const int col = (2 * i) % C::BOX_COLS;
                        const uint32_t off = (uint32_t)((2 * i) / C::BOX_COLS) * C::HALF_BYTES;
                        const uint32_t byte = (uint32_t)(col * (int)sizeof(KV)) & 15u;
                        const int chunk = col * (int)sizeof(KV) / 16;
                        uint8_t *ks = smem_raw + (swz(kbox + off, rr, chunk) - raw) + byte;
                        uint8_t *vs = smem_raw + (swz(vbox + off, rr, chunk) - raw) + byte;
                        if constexpr (C::F32) {
                            *reinterpret_cast<float2 *>(reinterpret_cast<float *>(a.kv.k) + dst) = make_float2(k0, k1);
                            *reinterpret_cast<float2 *>(reinterpret_cast<float *>(a.kv.v) + dst) = make_float2(v0, v1);
                            *reinterpret_cast<float2 *>(ks) = make_float2(k0, k1);
                            *reinterpret_cast<float2 *>(vs) = make_float2(v0, v1);
                        } else {
                            const __nv_bfloat162 kb = __floats2bfloat162_rn(k0, k1), vb = __floats2bfloat162_rn(v0, v1);
                            *reinterpret_cast<__nv_bfloat162 *>(reinterpret_cast<__nv_bfloat16 *>(a.kv.k) + dst) = kb;
                            *reinterpret_cast<__nv_bfloat162 *>(reinterpret_cast<__nv_bfloat16 *>(a.kv.v) + dst) = vb;
                            *reinterpret_cast<__nv_bfloat162 *>(ks) = kb;
                            *reinterpret_cast<__nv_bfloat162 *>(vs) = vb;
                        }
                    }
                    __syncwarp();
                }
            }
            // ---- S = Q K^T for 16 positions: two n8 tiles ----
            float s[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
            if constexpr (C::F32) {
                // B[k][n] = K[position r0 + 8*nt + gid][column]: one 16-byte read per (k16 block,
                // n8 tile) covers two k8 steps (k = tq, tq+4 <- columns d0, d0+1, then d0+2,
                // d0+3); K big and K small each take one MMA per step
#pragma unroll
                for (int kt = 0; kt < C::KT; ++kt) {
                    const uint32_t box = kbox + (kt >> 1) * C::HALF_BYTES;
                    const int chunk = 2 * tq + (kt & 1);
#pragma unroll
                    for (int nt = 0; nt < 2; ++nt) {
                        const float4 x = *reinterpret_cast<const float4 *>(
                            smem_raw + (swz(box, r0 + 8 * nt + gid, chunk) - raw));
                        uint32_t kb[4], ks[4];
                        split_tf32(x.x, kb[0], ks[0]);
                        split_tf32(x.y, kb[1], ks[1]);
                        split_tf32(x.z, kb[2], ks[2]);
                        split_tf32(x.w, kb[3], ks[3]);
                        mma1688(s[nt], qh[kt][0], ql[kt][0], qh[kt][1], ql[kt][1], kb[0], kb[1]);
                        mma1688(s[nt], qh[kt][0], ql[kt][0], qh[kt][1], ql[kt][1], ks[0], ks[1]);
                        mma1688(s[nt], qh[kt][2], ql[kt][2], qh[kt][3], ql[kt][3], kb[2], kb[3]);
                        mma1688(s[nt], qh[kt][2], ql[kt][2], qh[kt][3], ql[kt][3], ks[2], ks[3]);
                    }
                }
            } else {
                const int krow = r0 + ((lane >> 4) << 3) + (lane & 7);  // n tile = lane >> 4
                const int kc = (lane >> 3) & 1;                          // 8-dim half of the k16 step
#pragma unroll
                for (int kt = 0; kt < C::KT; ++kt) {
                    const int dim = 16 * kt + 8 * kc;
                    uint32_t b00, b01, b10, b11;
                    ldsm_x4(swz(kbox + (dim >> 6) * C::HALF_BYTES, krow, (dim & 63) >> 3), b00, b01, b10, b11);
                    mma16816(s[0], qh[kt][0], ql[kt][0], qh[kt][1], ql[kt][1], b00, b01);
                    mma16816(s[1], qh[kt][0], ql[kt][0], qh[kt][1], ql[kt][1], b10, b11);
                }
            }
            // ---- online softmax on row gid (positions 2tq, 2tq+1 of each n8 tile) ----
            const int pbase = p + r0 + 2 * tq;
            // score = hi row + lo row of the fragment
            float v[4] = {(s[0][0] + s[0][2]) * C2, (s[0][1] + s[0][3]) * C2, (s[1][0] + s[1][2]) * C2,
                          (s[1][1] + s[1][3]) * C2};
            const int pos[4] = {pbase, pbase + 1, pbase + 8, pbase + 9};
#pragma unroll
            for (int i = 0; i < 4; ++i)
                if (pos[i] >= un.p1) v[i] = -INFINITY;
            float mx = fmaxf(fmaxf(v[0], v[1]), fmaxf(v[2], v[3]));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
            if (mx > m + kRescale || (m == -INFINITY && mx != -INFINITY)) {
                // quad-uniform: the four lanes of a row share mx and m
                const float alpha = (m == -INFINITY) ? 0.f : exp2f(m - mx);
                m = mx;
                l *= alpha;
#pragma unroll
                for (int nt = 0; nt < C::NT; ++nt) {
                    o[nt][0] *= alpha;
                    o[nt][1] *= alpha;
                    o[nt][2] *= alpha;
                    o[nt][3] *= alpha;
                }
            }
            float pr[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) pr[i] = (v[i] == -INFINITY) ? 0.f : exp2f(v[i] - m);
            float ps = (pr[0] + pr[1]) + (pr[2] + pr[3]);
            ps += __shfl_xor_sync(0xffffffffu, ps, 1);
            ps += __shfl_xor_sync(0xffffffffu, ps, 2);
            l += ps;
            // ---- O += P V: P as the A fragment (k = the 16 positions), hi + lo ----
            if constexpr (C::F32) {
                // tf32 k8 steps over positions: step 0 maps k = tq, tq+4 to this thread's
                // positions 2tq, 2tq+1 of n8 tile 0 of S, step 1 to 8+2tq, 9+2tq (so P stays
                // where S left it).  B[k][n] = V[that position][column of n8 tile nt, n = gid]: a
                // 16-byte read of chunk gid of box j at one position gives n = gid of tiles
                // 4j .. 4j+3.  V big and V small each take one MMA per step.
                uint32_t pb[4], ps[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) split_tf32(pr[i], pb[i], ps[i]);
#pragma unroll
                for (int j = 0; j < C::HALVES; ++j) {
                    const uint32_t box = vbox + j * C::HALF_BYTES;
                    const float4 x0 = *reinterpret_cast<const float4 *>(smem_raw + (swz(box, r0 + 2 * tq, gid) - raw));
                    const float4 x1 = *reinterpret_cast<const float4 *>(smem_raw + (swz(box, r0 + 2 * tq + 1, gid) - raw));
                    const float4 x8 = *reinterpret_cast<const float4 *>(smem_raw + (swz(box, r0 + 2 * tq + 8, gid) - raw));
                    const float4 x9 = *reinterpret_cast<const float4 *>(smem_raw + (swz(box, r0 + 2 * tq + 9, gid) - raw));
                    const float a0[4] = {x0.x, x0.y, x0.z, x0.w}, a1[4] = {x1.x, x1.y, x1.z, x1.w};
                    const float a8[4] = {x8.x, x8.y, x8.z, x8.w}, a9[4] = {x9.x, x9.y, x9.z, x9.w};
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        uint32_t v0b, v0s, v1b, v1s, v8b, v8s, v9b, v9s;
                        split_tf32(a0[u], v0b, v0s);
                        split_tf32(a1[u], v1b, v1s);
                        split_tf32(a8[u], v8b, v8s);
                        split_tf32(a9[u], v9b, v9s);
                        mma1688(o[4 * j + u], pb[0], ps[0], pb[1], ps[1], v0b, v1b);
                        mma1688(o[4 * j + u], pb[0], ps[0], pb[1], ps[1], v0s, v1s);
                        mma1688(o[4 * j + u], pb[2], ps[2], pb[3], ps[3], v8b, v9b);
                        mma1688(o[4 * j + u], pb[2], ps[2], pb[3], ps[3], v8s, v9s);
                    }
                }
            } else {
                uint32_t ph0, pl0, ph1, pl1;
                split2(pr[0], pr[1], ph0, pl0);  // row gid, k = 2tq, 2tq+1
                split2(pr[2], pr[3], ph1, pl1);  // row gid, k = 2tq+8, 2tq+9
                const int vrow = r0 + (((lane >> 3) & 1) << 3) + (lane & 7);
                const int vc = lane >> 4;  // which n8 tile of the pair
#pragma unroll
                for (int dp = 0; dp < C::NT / 2; ++dp) {
                    const int dim = 16 * dp + 8 * vc;
                    uint32_t b00, b01, b10, b11;
                    ldsm_x4_t(swz(vbox + (dim >> 6) * C::HALF_BYTES, vrow, (dim & 63) >> 3), b00, b01, b10, b11);
                    mma16816(o[2 * dp], ph0, pl0, ph1, pl1, b00, b01);
                    mma16816(o[2 * dp + 1], ph0, pl0, ph1, pl1, b10, b11);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[stage]);
            if (++stage == C::NS) { stage = 0; phase ^= 1u; }
        }
        // ---- hand this warp's state to the merge (rows gid < G) ----
        if (row_ok) {
            if (tq == 0) {
                wm[warp * G + gid] = m;
                wl[warp * G + gid] = l;
            }
#pragma unroll
            for (int nt = 0; nt < C::NT; ++nt) {
                float *row = wo + (warp * G + gid) * D;
                if constexpr (C::F32) {
                    const int c = 32 * (nt >> 2) + (nt & 3);  // column of n = 2tq is c + 8tq
                    row[c + 8 * tq] = o[nt][0] + o[nt][2];       // hi rows + lo rows
                    row[c + 8 * tq + 4] = o[nt][1] + o[nt][3];
                } else {
                    row[8 * nt + 2 * tq] = o[nt][0] + o[nt][2];  // hi rows + lo rows
                    row[8 * nt + 2 * tq + 1] = o[nt][1] + o[nt][3];
                }
            }
        }
        return ok;
    };
    if constexpr (CLU) {
        consume_unit(cu);
        cluster_epilogue<G, D, C::NW>(a, cu, wm, wl, wo, cx, tid, qst, fz_cs);
        // split-KV across GPUs: this CTA's share of the cross-rank merge (every cluster is
        // resident: the host checks)
        if (a.px.nranks > 0 && *abort_flag == 0) peer_merge_pairs<G, D, C::NW>(a, tid);
    } else {
        while (true) {
            const int u = unitq_pop(uq, qs, qp, err, abort_flag, lane);
            if (u < 0) break;
            const Unit un = decode_unit(a, prefix, lens, u);
            const bool ok = consume_unit(un);
            unit_epilogue<G, D, C::NW>(a, un, u, prefix, wm, wl, wo, cw, is_last_flag, tid, warp, lane);
            if (named_bar_or(1, C::NW * 32, (!ok) || (*abort_flag != 0))) break;
        }
        // split-KV across GPUs: this CTA's share of the cross-rank merges, after its own units
        if (a.px.nranks > 0 && *abort_flag == 0) peer_merge_pairs<G, D, C::NW>(a, tid);
    }
}

PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

// 2-D map over a whole cache: rows = layer*slot*kvHead*pos, D columns; box = 128 bytes of
// columns (64 bf16 or 32 f32) x 64 rows.
bool make_cache_map(CUtensorMap *m, const void *ptr, uint64_t rows, int D, bool f32) {
    auto enc = get_encode();
    if (!enc) return false;
    const int es = f32 ? 4 : 2;
    cuuint64_t dims[2] = {(cuuint64_t)D, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)D * es};
    cuuint32_t box[2] = {(cuuint32_t)(128 / es), 64};
    cuuint32_t estr[2] = {1, 1};
    return enc(m, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
               const_cast<void *>(ptr), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <typename KV, int D, int G>
cudaError_t launch_t(const DecodeArgs &a, int num_ctas, cudaStream_t s) {
    using C = MmaCfg<KV, D, G>;
    const uint64_t rows = (uint64_t)a.kv.nLayer * a.kv.maxBatch * a.kv.nHeadKv * a.kv.maxLen;
    if (rows + C::T > (uint64_t)INT32_MAX) return cudaErrorNotSupported;
    CUtensorMap km, vm;
    if (!make_cache_map(&km, a.kv.k, rows, D, C::F32) || !make_cache_map(&vm, a.kv.v, rows, D, C::F32))
        return cudaErrorNotSupported;
    const size_t smem = C::smem_bytes(a.nseq);
    int dev = 0;
    cudaGetDevice(&dev);
    // only when it grows (per device and kernel): steady-state launches make no attribute calls
    auto ensure_smem = [&](auto kern, size_t *set) -> cudaError_t {
        size_t &cur = set[dev & 63];
        if (smem > cur) {
            cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            if (e != cudaSuccess) return e;
            cur = smem;
        }
        return cudaSuccess;
    };
    if (a.cluster > 0) {
        if (a.cluster > kMaxCluster || num_ctas % a.cluster != 0) return cudaErrorInvalidValue;
        static size_t smem_set_clu[64] = {};
        auto kern = decode_mma_kernel<KV, D, G, true>;
        cudaError_t e = ensure_smem(kern, smem_set_clu);
        if (e != cudaSuccess) return e;
        if (a.cluster > 8) {
            e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
            if (e != cudaSuccess) return e;
        }
        return launch_pdl_cluster(kern, dim3(num_ctas), dim3(C::THREADS), smem, a.cluster, s, km, vm, a);
    }
    static size_t smem_set[64] = {};
    auto kern = decode_mma_kernel<KV, D, G, false>;
    cudaError_t e = ensure_smem(kern, smem_set);
    if (e != cudaSuccess) return e;
    return launch_pdl(kern, dim3(num_ctas), dim3(C::THREADS), smem, s, km, vm, a);
}

template <typename KV, int D, int G>
int occ_t(int nseq) {
    using C = MmaCfg<KV, D, G>;
    int n = 0;
    const size_t smem = C::smem_bytes(nseq);
    auto kern = decode_mma_kernel<KV, D, G, false>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, C::THREADS, smem) != cudaSuccess)
        n = 1;
    return n < 1 ? 1 : n;
}

}  // namespace

bool decode_mma_covers(int headDim, int group, int dtype) {
    if (headDim != 64 && headDim != 128) return false;
    if (dtype == TL_KV_BF16) return group == 1 || group == 2 || group == 4 || group == 8;
    // f32: the CUDA-core kernel stays at the HBM roofline up to G = 2
    return dtype == TL_KV_F32 && (group == 4 || group == 8);
}

cudaError_t launch_decode_mma(const DecodeArgs &a, int num_ctas, cudaStream_t s) {
    const int G = a.nHead / a.nHeadKv;
    if (!decode_mma_covers(a.headDim, G, a.kv.dtype)) return cudaErrorNotSupported;
#define TL_MMA_CASE(DD)                                                     \
    switch (G) {                                                            \
        case 1: return launch_t<__nv_bfloat16, DD, 1>(a, num_ctas, s);      \
        case 2: return launch_t<__nv_bfloat16, DD, 2>(a, num_ctas, s);      \
        case 4: return launch_t<__nv_bfloat16, DD, 4>(a, num_ctas, s);      \
        case 8: return launch_t<__nv_bfloat16, DD, 8>(a, num_ctas, s);      \
        default: return cudaErrorNotSupported;                              \
    }
#define TL_MMA_CASE_F32(DD)                                                 \
    switch (G) {                                                            \
        case 4: return launch_t<float, DD, 4>(a, num_ctas, s);              \
        case 8: return launch_t<float, DD, 8>(a, num_ctas, s);              \
        default: return cudaErrorNotSupported;                              \
    }
    if (a.kv.dtype == TL_KV_F32) {
        if (a.headDim == 64) { TL_MMA_CASE_F32(64) }
        if (a.headDim == 128) { TL_MMA_CASE_F32(128) }
    } else {
        if (a.headDim == 64) { TL_MMA_CASE(64) }
        if (a.headDim == 128) { TL_MMA_CASE(128) }
    }
#undef TL_MMA_CASE
#undef TL_MMA_CASE_F32
    return cudaErrorNotSupported;
}

namespace {
template <typename KV, int D, int G>
int cluster_capacity_t(int cluster) {
    using C = MmaCfg<KV, D, G>;
    const size_t smem = C::smem_bytes(512);  // at least what a cluster-mode launch uses (nseq <= 512)
    auto kern = decode_mma_kernel<KV, D, G, true>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) return 0;
    if (cluster > 8 && cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(cluster);
    cfg.blockDim = dim3(C::THREADS);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)cluster;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return n;
}
}  // namespace

int decode_mma_cluster_capacity(int headDim, int group, int dtype, int cluster) {
    if (!decode_mma_covers(headDim, group, dtype) || cluster < 1 || cluster > kMaxCluster) return 0;
    // cached per (device, dtype, head_dim, group, cluster size)
    static int cache[16][2][2][4][kMaxCluster + 1];
    static std::mutex mu;
    int dev = 0;
    cudaGetDevice(&dev);
    const int gi = group == 1 ? 0 : group == 2 ? 1 : group == 4 ? 2 : 3;
    const int di = dtype == TL_KV_F32 ? 0 : 1, hi = headDim == 64 ? 0 : 1;
    if (dev < 0 || dev >= 16) return 0;
    std::lock_guard<std::mutex> lock(mu);
    int &c = cache[dev][di][hi][gi][cluster];
    if (c > 0) return c;
    int n = 0;
#define TL_CAP(KV, DD)                                               \
    switch (group) {                                                 \
        case 1: n = cluster_capacity_t<KV, DD, 1>(cluster); break;   \
        case 2: n = cluster_capacity_t<KV, DD, 2>(cluster); break;   \
        case 4: n = cluster_capacity_t<KV, DD, 4>(cluster); break;   \
        case 8: n = cluster_capacity_t<KV, DD, 8>(cluster); break;   \
    }
    if (dtype == TL_KV_F32) {
        if (headDim == 64) n = group == 8 ? cluster_capacity_t<float, 64, 8>(cluster) : cluster_capacity_t<float, 64, 4>(cluster);
        else n = group == 8 ? cluster_capacity_t<float, 128, 8>(cluster) : cluster_capacity_t<float, 128, 4>(cluster);
    } else if (headDim == 64) {
        TL_CAP(__nv_bfloat16, 64)
    } else {
        TL_CAP(__nv_bfloat16, 128)
    }
#undef TL_CAP
    c = n;
    return n;
}

int decode_mma_ctas_per_sm(int headDim, int group, int dtype, int nseq) {
#define TL_MMA_OCC(KV, DD)                             \
    switch (group) {                                   \
        case 1: return occ_t<KV, DD, 1>(nseq);         \
        case 2: return occ_t<KV, DD, 2>(nseq);         \
        case 4: return occ_t<KV, DD, 4>(nseq);         \
        case 8: return occ_t<KV, DD, 8>(nseq);         \
        default: return 1;                             \
    }
    if (dtype == TL_KV_F32) {
        if (headDim == 64) return group == 8 ? occ_t<float, 64, 8>(nseq) : occ_t<float, 64, 4>(nseq);
        if (headDim == 128) return group == 8 ? occ_t<float, 128, 8>(nseq) : occ_t<float, 128, 4>(nseq);
    } else {
        if (headDim == 64) { TL_MMA_OCC(__nv_bfloat16, 64) }
        if (headDim == 128) { TL_MMA_OCC(__nv_bfloat16, 128) }
    }
#undef TL_MMA_OCC
    return 1;
}

size_t decode_mma_smem_bytes(int headDim, int group, int dtype, int nseq) {
#define TL_MMA_SMEM(KV, DD)                                              \
    switch (group) {                                                     \
        case 1: return MmaCfg<KV, DD, 1>::smem_bytes(nseq);              \
        case 2: return MmaCfg<KV, DD, 2>::smem_bytes(nseq);              \
        case 4: return MmaCfg<KV, DD, 4>::smem_bytes(nseq);              \
        case 8: return MmaCfg<KV, DD, 8>::smem_bytes(nseq);              \
        default: return 0;                                               \
    }
    if (dtype == TL_KV_F32) {
        if (headDim == 64) { TL_MMA_SMEM(float, 64) }
        if (headDim == 128) { TL_MMA_SMEM(float, 128) }
    } else {
        if (headDim == 64) { TL_MMA_SMEM(__nv_bfloat16, 64) }
        if (headDim == 128) { TL_MMA_SMEM(__nv_bfloat16, 128) }
    }
#undef TL_MMA_SMEM
    return 0;
}

}  // namespace tl
