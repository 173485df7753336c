// prefill_tc.cu -- causal GQA prefill attention on the 5th-generation tensor cores (sm_100a).
//
// Replaces the context part of attentionFull (src/forward.nim:141-176) on the bf16 KV path:
// for q-head h and query i, s_j = q_i . k_j / sqrt(d) for j <= i, softmax, ctx_i = sum p_j v_j.
// Inputs are bf16 (Q staged by the RoPE kernel, K/V from the cache the same launch sequence
// appended to), products accumulate in fp32 in tensor memory, softmax runs in fp32.
//
// One CTA owns 256 query rows (two tiles of 128) of one (sequence, q-head).  A TMA warp brings
// Q once and K/V tiles of 128 positions (2-D tensor maps, 128-byte swizzle, no multicast) into a
// three-deep ring; a single MMA thread issues S_q = Q_q K^T (4 x tcgen05.mma kind::f16, M=128,
// N=128, K=16, A and B K-major from shared memory) and O_q += P_q V (8 MMAs, A = P from TMEM,
// B = V MN-major from shared memory); two softmax groups of 128 threads (thread = query row =
// TMEM lane) load S, mask causally, keep the online max/sum in fp32 (log2 domain), write P as
// packed bf16 into TMEM and rescale O in TMEM only when a row's maximum grows past 2^8.  S and
// P have separate TMEM columns, so S_q(j+1) runs on the tensor core while the softmax of
// S_q(j) is still in flight, and the two query tiles alternate.  KV tiles past the diagonal are
// skipped.  Every mbarrier wait is bounded (common.cuh); TMEM is released on every exit path
// after the MMA thread has seen its own last commit.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <math.h>

#include <mutex>

#include "common.cuh"
#include "internal.h"

namespace tl {
namespace {

constexpr int BM = 128;             // query rows per CTA
constexpr int BN = 128;             // keys per KV tile
constexpr int HD = 64;              // head_dim covered by this kernel
constexpr int TILE_BYTES = BM * HD * 2;  // 16 KB, one 128 x 64 bf16 tile
constexpr float kLog2e = 1.4426950408889634f;

// ---- PTX wrappers ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_load_2d(void *smem_dst, const CUtensorMap *map, int x, int y,
                                            uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
            "r"(smem_u32(smem_dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void tmem_alloc(uint32_t *smem_slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_slot)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
// D[tmem] (+)= A[smem desc] * B[smem desc]
__device__ __forceinline__ void mma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem desc]
__device__ __forceinline__ void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

#define TL_LD32(taddr, r)                                                                          \
    asm volatile(                                                                                  \
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14," \
        "%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"               \
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),      \
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),  \
          "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),            \
          "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),            \
          "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])             \
        : "r"(taddr))

#define TL_ST32(taddr, r)                                                                          \
    asm volatile(                                                                                  \
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"  \
        "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr), \
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),    \
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),           \
        "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),         \
        "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),         \
        "r"(r[29]), "r"(r[30]), "r"(r[31])                                                          \
        : "memory")

#define TL_LD16(taddr, r)                                                                          \
    asm volatile(                                                                                  \
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14," \
        "%15}, [%16];"                                                                             \
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),      \
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),  \
          "=r"(r[14]), "=r"(r[15])                                                                 \
        : "r"(taddr))

#define TL_ST16(taddr, r)                                                                          \
    asm volatile(                                                                                  \
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"  \
        "%14,%15,%16};" ::"r"(taddr),                                                              \
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),    \
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),           \
        "r"(r[15])                                                                                  \
        : "memory")

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor, 128-byte swizzle, 8-row groups 1024 bytes apart.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr, uint32_t lbo_bytes) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)(1024u >> 4) << 32;  // stride byte offset
    d |= (uint64_t)1 << 46;             // descriptor version (sm_100)
    d |= (uint64_t)2 << 61;             // SWIZZLE_128B
    return d;
}

// Instruction descriptor, kind::f16: bf16 x bf16 -> f32, M = 128.
__host__ __device__ constexpr uint32_t idesc_bf16(int N, bool b_mn_major) {
    return (1u << 4)                      // D format f32
           | (1u << 7)                    // A bf16
           | (1u << 10)                   // B bf16
           | ((b_mn_major ? 1u : 0u) << 16)
           | ((uint32_t)(N >> 3) << 17)
           | ((uint32_t)(BM >> 4) << 24);
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t *>(&v);
}

struct TcParams {
    HeadView out;
    int nseq, ntok, nHead, nHeadKv;
    int64_t kv_row_layer;  // cache row of (layer, slot0, kvh=0, pos=0)
    int kv_rows_per_slot;  // nHeadKv * maxLen
    int maxLen;
    unsigned *err;
};

constexpr int NS_KV = 3;                       // K/V ring depth (32 KB per stage)
constexpr int THREADS = 384;                   // 3 warpgroups: control, softmax tile 0, softmax tile 1
constexpr int TMEM_ALL = 512;
// TMEM columns: S0 | S1 | P0 | P1 | O0 | O1
__host__ __device__ constexpr int col_s(int q) { return q * 128; }
__host__ __device__ constexpr int col_p(int q) { return 256 + q * 64; }
__host__ __device__ constexpr int col_o(int q) { return 384 + q * 64; }
constexpr float kRescaleThreshold = 8.0f;      // log2 units: O is rescaled only past 2^8

// Each scheduler partition runs one control warp and two softmax warps (warp w sits on
// partition w % 4).  Registers move from the control warpgroup (104 per thread) to the softmax
// groups (200): 104 + 2*200 = 504 = 3*168, the allotment of three warps launched at 168.
__device__ __forceinline__ void setmaxnreg_dec() { asm volatile("setmaxnreg.dec.sync.aligned.u32 104;"); }
__device__ __forceinline__ void setmaxnreg_inc() { asm volatile("setmaxnreg.inc.sync.aligned.u32 200;"); }

__device__ __forceinline__ float max3f(float a, float b, float c) {
    float r;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
    return r;
}

// packed fp32 pair arithmetic (one instruction for two lanes of work)
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
    unsigned long long d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;"
        : "=l"(d)
        : "l"(*reinterpret_cast<unsigned long long *>(&a)), "l"(*reinterpret_cast<unsigned long long *>(&b)),
          "l"(*reinterpret_cast<unsigned long long *>(&c)));
    return *reinterpret_cast<float2 *>(&d);
}
__device__ __forceinline__ float2 fadd2(float2 a, float2 b) {
    unsigned long long d;
    asm("add.f32x2 %0, %1, %2;"
        : "=l"(d)
        : "l"(*reinterpret_cast<unsigned long long *>(&a)), "l"(*reinterpret_cast<unsigned long long *>(&b)));
    return *reinterpret_cast<float2 *>(&d);
}

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}


struct Bars {
    uint64_t q_full, kv_full[NS_KV], kv_empty[NS_KV], s_full[2], s_free[2], p_ready[2], o_bar[2],
        o_done[2], mma_final;
    uint32_t tmem_base;
    int abort;
};

// Causal prefill, one CTA = 256 query rows (two 128-row tiles) of one (sequence, q-head).
//   warpgroup 0: warp 0 lane 0 = TMA producer; warp 1 = TMEM owner, its lane 0 the MMA issuer
//   warpgroups 1 / 2: softmax of query tile 0 / 1, thread = row = TMEM lane (warp w reaches
//   TMEM lanes 32*(w%4)..)
// Per KV tile j and query tile q the MMA issuer runs S_q(j+1) = Q_q K_{j+1}^T as soon as the
// softmax group has pulled S_q(j) into registers (s_free), and O_q += P_q(j) V_j once P_q(j) is
// in TMEM (p_ready), so the tensor core works on one tile while the other group's softmax runs.
// A group overwrites P_q and rescales O_q only after PV_q(j-1) has completed (o_bar).
__global__ void __launch_bounds__(THREADS, 1)
prefill_tc_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap,
                  const __grid_constant__ CUtensorMap vmap, const TcParams p) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    uint8_t *base = smem_raw + (((raw + 1023u) & ~1023u) - raw);
    uint8_t *sQ[2] = {base, base + TILE_BYTES};
    uint8_t *sK = base + 2 * TILE_BYTES;                  // [NS_KV] tiles
    uint8_t *sV = base + (2 + NS_KV) * TILE_BYTES;        // [NS_KV] tiles
    Bars *bars = reinterpret_cast<Bars *>(base + (2 + 2 * NS_KV) * TILE_BYTES);
    volatile int *abort_flag = &bars->abort;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int npairs = (p.ntok + 2 * BM - 1) / (2 * BM);
    const int pair = npairs - 1 - (int)blockIdx.x;  // heavy (late) tiles first
    const int h = blockIdx.y, b = blockIdx.z;
    const int g = h / (p.nHead / p.nHeadKv);
    const int q0 = pair * 2 * BM;
    int nt[2];
#pragma unroll
    for (int q = 0; q < 2; ++q) {
        const int start = q0 + q * BM;
        nt[q] = start < p.ntok ? (min(start + BM, p.ntok) + BN - 1) / BN : 0;
    }
    const int nkv = max(nt[0], nt[1]);

    if (tid == 0) {
        mbar_init(&bars->q_full, 1);
        for (int i = 0; i < NS_KV; ++i) {
            mbar_init(&bars->kv_full[i], 1);
            mbar_init(&bars->kv_empty[i], 1);
        }
        for (int q = 0; q < 2; ++q) {
            mbar_init(&bars->s_full[q], 1);
            mbar_init(&bars->s_free[q], BM);
            mbar_init(&bars->p_ready[q], BM);
            mbar_init(&bars->o_bar[q], 1);
            mbar_init(&bars->o_done[q], 1);
        }
        mbar_init(&bars->mma_final, 1);
        bars->abort = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(&bars->tmem_base, TMEM_ALL);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = bars->tmem_base;
    const int qrow = (int)(((int64_t)b * p.nHead + h) * p.ntok + q0);
    const int kvrow0 = (int)(p.kv_row_layer + (int64_t)b * p.kv_rows_per_slot + (int64_t)g * p.maxLen);

    if (warp < 4) {
        setmaxnreg_dec();
        if (warp == 0 && lane == 0) {
            // ---------------- TMA producer ----------------
            mbar_arrive_expect_tx(&bars->q_full, (nt[1] > 0 ? 2 : 1) * TILE_BYTES);
            tma_load_2d(sQ[0], &qmap, 0, qrow, &bars->q_full);
            if (nt[1] > 0) tma_load_2d(sQ[1], &qmap, 0, qrow + BM, &bars->q_full);
            int issued = 0;
            bool ok = true;
            for (int j = 0; j < nkv && ok; ++j) {
                const int st = j % NS_KV;
                if (!mbar_wait(&bars->kv_empty[st], ((j / NS_KV) & 1) ^ 1, p.err, abort_flag)) { ok = false; break; }
                mbar_arrive_expect_tx(&bars->kv_full[st], 2 * TILE_BYTES);
                tma_load_2d(sK + st * TILE_BYTES, &kmap, 0, kvrow0 + j * BN, &bars->kv_full[st]);
                tma_load_2d(sV + st * TILE_BYTES, &vmap, 0, kvrow0 + j * BN, &bars->kv_full[st]);
                ++issued;
            }
            // wait (bounded) until every copy issued into this CTA's shared memory has landed
            mbar_wait(&bars->q_full, 0, nullptr, nullptr);
            for (int j = max(0, issued - NS_KV); j < issued; ++j)
                mbar_wait(&bars->kv_full[j % NS_KV], (j / NS_KV) & 1, nullptr, nullptr);
        } else if (warp == 1 && lane == 0) {
            // ---------------- MMA issuer ----------------
            const uint32_t idesc_s = idesc_bf16(BN, false);
            const uint32_t idesc_o = idesc_bf16(HD, true);
            bool ok = mbar_wait(&bars->q_full, 0, p.err, abort_flag) &&
                      mbar_wait(&bars->kv_full[0], 0, p.err, abort_flag);
            auto issue_s = [&](int q, int j) {
                const uint32_t qa = smem_u32(sQ[q]), ka = smem_u32(sK + (j % NS_KV) * TILE_BYTES);
#pragma unroll
                for (int kk = 0; kk < HD / 16; ++kk)
                    mma_ss(tmem + col_s(q), sw128_desc(qa + kk * 32, 16), sw128_desc(ka + kk * 32, 16), idesc_s,
                           kk > 0 ? 1u : 0u);
                tc_commit(&bars->s_full[q]);
            };
            if (ok) {
                tc_fence_after();
                for (int q = 0; q < 2; ++q)
                    if (nt[q] > 0) issue_s(q, 0);
            }
            for (int j = 0; j < nkv && ok; ++j) {
                for (int q = 0; q < 2 && ok; ++q) {
                    if (j >= nt[q]) continue;
                    if (j + 1 < nt[q]) {
                        ok = mbar_wait(&bars->s_free[q], j & 1, p.err, abort_flag) &&
                             mbar_wait(&bars->kv_full[(j + 1) % NS_KV], ((j + 1) / NS_KV) & 1, p.err, abort_flag);
                        if (!ok) break;
                        tc_fence_after();
                        issue_s(q, j + 1);
                    }
                    if (!mbar_wait(&bars->p_ready[q], j & 1, p.err, abort_flag)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t va = smem_u32(sV + (j % NS_KV) * TILE_BYTES);
#pragma unroll
                    for (int kk = 0; kk < BN / 16; ++kk)
                        mma_ts(tmem + col_o(q), tmem + col_p(q) + kk * 8, sw128_desc(va + kk * 2048, TILE_BYTES),
                               idesc_o, (j > 0 || kk > 0) ? 1u : 0u);
                    tc_commit(&bars->o_bar[q]);
                    if (j == nt[q] - 1) tc_commit(&bars->o_done[q]);
                }
                if (ok) tc_commit(&bars->kv_empty[j % NS_KV]);
            }
            // every MMA this thread issued has completed before TMEM can be released
            tc_commit(&bars->mma_final);
            mbar_wait(&bars->mma_final, 0, p.err, nullptr);
        }
    } else {
        setmaxnreg_inc();
        // ---------------- softmax of query tile q ----------------
        const int q = (warp - 4) >> 2;
        const int r = (warp & 3) * 32 + lane;
        const int row = q0 + q * BM + r;
        const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
        const float C = kLog2e / 8.0f;  // log2(e) / sqrt(64)
        float m_run = -INFINITY, l = 0.f;
        bool ok = true;
        for (int j = 0; j < nt[q] && ok; ++j) {
            // warp-uniform verdict: the TMEM loads below are warp-collective
            ok = __all_sync(0xffffffffu, mbar_wait(&bars->s_full[q], j & 1, p.err, abort_flag));
            if (!ok) break;
            tc_fence_after();
            // S in two halves: the second half's TMEM load overlaps the first half's maximum
            uint32_t sr[BN];
            const int k0 = j * BN;
            const bool diag = (j == nt[q] - 1);  // diagonal / ragged tile: causal and length mask
            float mq[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                if (half == 0) {
#pragma unroll
                    for (int c = 0; c < 2; ++c) {
                        uint32_t *rr = sr + 32 * c;
                        TL_LD32(tmem + lane_base + col_s(q) + 32 * c, rr);
                    }
                    tmem_wait_ld();
#pragma unroll
                    for (int c = 2; c < 4; ++c) {
                        uint32_t *rr = sr + 32 * c;
                        TL_LD32(tmem + lane_base + col_s(q) + 32 * c, rr);
                    }
                } else {
                    tmem_wait_ld();
                    tc_fence_before();
                    mbar_arrive(&bars->s_free[q]);  // S_q(j) is in registers: the next S may overwrite it
                }
                const int c0 = half * (BN / 2);
                if (diag) {
#pragma unroll
                    for (int c = c0; c < c0 + BN / 2; ++c)
                        if (k0 + c > row || k0 + c >= p.ntok) sr[c] = __float_as_uint(-INFINITY);
                }
                // row maximum: four independent chains of three-input max
#pragma unroll
                for (int c = c0; c < c0 + BN / 2; c += 8) {
#pragma unroll
                    for (int u = 0; u < 4; ++u)
                        mq[u] = max3f(mq[u], __uint_as_float(sr[c + 2 * u]), __uint_as_float(sr[c + 2 * u + 1]));
                }
            }
            const float mx = max3f(mq[0], mq[1], fmaxf(mq[2], mq[3]));
            const float ms = mx * C;
            const bool grow = ms > m_run + kRescaleThreshold || m_run == -INFINITY;
            float alpha = 1.f;
            if (grow) {
                alpha = (m_run == -INFINITY) ? 0.f : ex2(m_run - ms);
                m_run = ms;
                l *= alpha;
            }
            if (j > 0) {
                // PV_q(j-1) must be complete before P_q is overwritten (and before O_q is rescaled)
                ok = __all_sync(0xffffffffu, mbar_wait(&bars->o_bar[q], (j - 1) & 1, p.err, abort_flag));
                if (!ok) break;
                tc_fence_after();
            }
            if (__any_sync(0xffffffffu, grow && j > 0)) {
                // O_q holds the sum through tile j-1: rescale it in TMEM
#pragma unroll
                for (int c = 0; c < HD / 16; ++c) {  // 16 columns at a time: S stays in registers
                    uint32_t orr[16];
                    TL_LD16(tmem + lane_base + col_o(q) + 16 * c, orr);
                    tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < 16; ++i) orr[i] = __float_as_uint(__uint_as_float(orr[i]) * alpha);
                    TL_ST16(tmem + lane_base + col_o(q) + 16 * c, orr);
                }
            }
            // p = 2^(s*C - m): the argument in packed pairs, the sum in four packed accumulators
            const float2 c2 = make_float2(C, C), n2 = make_float2(-m_run, -m_run);
            float2 acc[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                             make_float2(0.f, 0.f)};
            uint32_t pk[BN / 2];
#pragma unroll
            for (int c = 0; c < BN; c += 2) {
                const float2 x = ffma2(make_float2(__uint_as_float(sr[c]), __uint_as_float(sr[c + 1])), c2, n2);
                const float2 pp = make_float2(ex2(x.x), ex2(x.y));
                acc[(c >> 1) & 3] = fadd2(acc[(c >> 1) & 3], pp);
                pk[c / 2] = pack_bf16(pp.x, pp.y);
            }
            const float2 a01 = fadd2(acc[0], acc[1]), a23 = fadd2(acc[2], acc[3]);
            const float2 a = fadd2(a01, a23);
            l += a.x + a.y;
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                uint32_t *rr = pk + 32 * c;
                TL_ST32(tmem + lane_base + col_p(q) + 32 * c, rr);
            }
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(&bars->p_ready[q]);
        }
        if (ok && nt[q] > 0) ok = __all_sync(0xffffffffu, mbar_wait(&bars->o_done[q], 0, p.err, abort_flag));
        if (ok && nt[q] > 0) {
            tc_fence_after();
            uint32_t orr[HD];
#pragma unroll
            for (int c = 0; c < HD / 32; ++c) {
                uint32_t *rr = orr + 32 * c;
                TL_LD32(tmem + lane_base + col_o(q) + 32 * c, rr);
            }
            tmem_wait_ld();
            if (row < p.ntok) {
                const float inv = l > 0.f ? 1.f / l : 0.f;
                float *dst = p.out.ptr;
#pragma unroll
                for (int i = 0; i < HD; i += 4) {
                    const int64_t o = p.out.at(b, row, h, i);
                    if (p.out.sd == 1 && (o & 3) == 0) {
                        *reinterpret_cast<float4 *>(dst + o) =
                            make_float4(__uint_as_float(orr[i]) * inv, __uint_as_float(orr[i + 1]) * inv,
                                        __uint_as_float(orr[i + 2]) * inv, __uint_as_float(orr[i + 3]) * inv);
                    } else {
#pragma unroll
                        for (int u = 0; u < 4; ++u) dst[p.out.at(b, row, h, i + u)] = __uint_as_float(orr[i + u]) * inv;
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, TMEM_ALL);
    }
}

// ---- host side ------------------------------------------------------------------------------
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

bool make_map(CUtensorMap *m, const void *ptr, uint64_t rows) {
    auto enc = get_encode();
    if (!enc) return false;
    cuuint64_t dims[2] = {(cuuint64_t)HD, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)HD * 2};
    cuuint32_t box[2] = {(cuuint32_t)HD, (cuuint32_t)BM};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(ptr), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

}  // namespace

cudaError_t launch_prefill_tc(const PrefillArgs &a, cudaStream_t s) {
    static_assert(BM == BN, "one tensor map box serves Q, K and V tiles");
    if (a.headDim != HD || a.kv.dtype != TL_KV_BF16 || a.qb == nullptr || a.pos0 != nullptr ||
        a.kf.ptr != nullptr)
        return cudaErrorNotSupported;
    const int64_t q_rows = (int64_t)a.nseq * a.nHead * a.ntok;
    const int64_t kv_rows = (int64_t)a.kv.nLayer * a.kv.maxBatch * a.kv.nHeadKv * a.kv.maxLen;
    if (q_rows + 2 * BM > INT32_MAX || kv_rows + BN > INT32_MAX) return cudaErrorNotSupported;
    CUtensorMap qm, km, vm;
    if (!make_map(&qm, a.qb, (uint64_t)q_rows) || !make_map(&km, a.kv.k, (uint64_t)kv_rows) ||
        !make_map(&vm, a.kv.v, (uint64_t)kv_rows))
        return cudaErrorNotSupported;
    TcParams p;
    p.out = a.out;
    p.nseq = a.nseq;
    p.ntok = a.ntok;
    p.nHead = a.nHead;
    p.nHeadKv = a.nHeadKv;
    p.kv_row_layer = a.kv.row(a.layer, a.slot0, 0, 0);
    p.kv_rows_per_slot = a.kv.nHeadKv * a.kv.maxLen;
    p.maxLen = a.kv.maxLen;
    p.err = a.err;
    const int smem = (2 + 2 * NS_KV) * TILE_BYTES + (int)sizeof(Bars) + 1024;
    cudaError_t e = cudaFuncSetAttribute(prefill_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    dim3 grid((a.ntok + 2 * BM - 1) / (2 * BM), a.nHead, a.nseq);
    prefill_tc_kernel<<<grid, THREADS, smem, s>>>(qm, km, vm, p);
    return cudaGetLastError();
}

}  // namespace tl
