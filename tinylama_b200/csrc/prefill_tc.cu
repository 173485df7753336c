// prefill_tc.cu -- causal GQA prefill attention on the 5th-generation tensor cores (sm_100a).
//
// Replaces the context part of attentionFull (src/forward.nim:141-176) on the bf16 KV path:
// for q-head h and query i, s_j = q_i . k_j / sqrt(d) for j <= i, softmax, ctx_i = sum p_j v_j.
// Inputs are bf16 (Q staged by the RoPE kernel, K/V from the cache the same launch sequence
// appended to), products accumulate in fp32 in tensor memory, softmax runs in fp32.
//
// One CTA owns 128 query rows of one (sequence, q-head); warp w owns TMEM lanes 32w..32w+31,
// i.e. query rows 32w..32w+31 (thread = row).  Per KV tile of 128 positions:
//   1. TMA (tensor maps, 128-byte swizzle, no multicast) has brought Q once and K_j/V_j into a
//      two-deep ring; thread 0 issues S = Q K_j^T as 4 tcgen05.mma (M=128, N=128, K=16 each,
//      A and B K-major from shared memory) into TMEM columns [0,128) and commits to an mbarrier.
//   2. Every thread loads its row of S (tcgen05.ld), applies the causal mask, updates the
//      running max / sum (online softmax, log2 domain) and writes P = 2^(s - m) as packed bf16
//      into TMEM columns [192,256).
//   3. Thread 0 issues O_j = P V_j as 8 tcgen05.mma with A = P from TMEM and B = V_j from shared
//      memory (MN-major: V rows are positions, head_dim contiguous) into TMEM columns
//      [128,192); threads fold O_j into their register accumulator with the rescale factor.
// KV tiles past the diagonal are skipped.  Every mbarrier wait is bounded (common.cuh); TMEM is
// released on every exit path.
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
constexpr int TMEM_COLS = 256;
constexpr int COL_S = 0, COL_O = 128, COL_P = 192;
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
    int64_t q_row0;      // staging row of (b=0, h=0, t=0)
    int64_t kv_row_layer;  // cache row of (layer, slot0, kvh=0, pos=0)
    int kv_rows_per_slot;  // nHeadKv * maxLen
    int maxLen;
    unsigned *err;
};

__global__ void __launch_bounds__(128, 1)
prefill_tc_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap,
                  const __grid_constant__ CUtensorMap vmap, const TcParams p) {
    extern __shared__ uint8_t smem_raw[];
    // 1024-aligned carve-up: Q | K0 | K1 | V0 | V1 | barriers
    const uint32_t raw = smem_u32(smem_raw);
    uint8_t *base = smem_raw + (((raw + 1023u) & ~1023u) - raw);
    uint8_t *sQ = base;
    uint8_t *sK[2] = {base + TILE_BYTES, base + 2 * TILE_BYTES};
    uint8_t *sV[2] = {base + 3 * TILE_BYTES, base + 4 * TILE_BYTES};
    uint64_t *bar = reinterpret_cast<uint64_t *>(base + 5 * TILE_BYTES);
    uint64_t *bar_q = bar, *bar_kv = bar + 1 /*[2]*/, *bar_mma = bar + 3;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bar + 4);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(bar + 5);

    const int tid = threadIdx.x, warp = tid >> 5;
    const int ntiles_q = (p.ntok + BM - 1) / BM;
    const int qt = ntiles_q - 1 - (int)blockIdx.x;  // heavy (late) tiles first
    const int h = blockIdx.y, b = blockIdx.z;
    const int G = p.nHead / p.nHeadKv;
    const int g = h / G;
    const int q0 = qt * BM;
    const int row = q0 + tid;  // this thread's query position
    const int nkv = min((q0 + BM + BN - 1) / BN, (p.ntok + BN - 1) / BN);

    if (tid == 0) {
        mbar_init(bar_q, 1);
        mbar_init(&bar_kv[0], 1);
        mbar_init(&bar_kv[1], 1);
        mbar_init(bar_mma, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 0) {
        tmem_alloc(tmem_slot, TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    const int qrow = (int)(p.q_row0 + ((int64_t)b * p.nHead + h) * p.ntok + q0);
    const int kvrow0 = (int)(p.kv_row_layer + (int64_t)b * p.kv_rows_per_slot + (int64_t)g * p.maxLen);
    if (tid == 0) {
        mbar_arrive_expect_tx(bar_q, TILE_BYTES);
        tma_load_2d(sQ, &qmap, 0, qrow, bar_q);
        mbar_arrive_expect_tx(&bar_kv[0], 2 * TILE_BYTES);
        tma_load_2d(sK[0], &kmap, 0, kvrow0, &bar_kv[0]);
        tma_load_2d(sV[0], &vmap, 0, kvrow0, &bar_kv[0]);
    }

    const float scale = kLog2e / 8.0f;  // log2(e) / sqrt(64)
    float m = -INFINITY, l = 0.f;
    float o[HD];
#pragma unroll
    for (int i = 0; i < HD; ++i) o[i] = 0.f;
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
    const uint32_t idesc_s = idesc_bf16(BN, false);
    const uint32_t idesc_o = idesc_bf16(HD, true);
    uint32_t mma_phase = 0;
    bool ok = mbar_wait(bar_q, 0, p.err, abort_flag);

    for (int j = 0; j < nkv && ok; ++j) {
        const int buf = j & 1;
        if (!mbar_wait(&bar_kv[buf], (j >> 1) & 1, p.err, abort_flag)) { ok = false; break; }
        if (tid == 0) {
            // prefetch the next KV tile into the other buffer (its previous MMAs are complete:
            // every iteration waits for its own MMAs before the next begins)
            if (j + 1 < nkv) {
                const int nb = buf ^ 1;
                mbar_arrive_expect_tx(&bar_kv[nb], 2 * TILE_BYTES);
                tma_load_2d(sK[nb], &kmap, 0, kvrow0 + (j + 1) * BN, &bar_kv[nb]);
                tma_load_2d(sV[nb], &vmap, 0, kvrow0 + (j + 1) * BN, &bar_kv[nb]);
            }
            tc_fence_after();
            const uint32_t qa = smem_u32(sQ), ka = smem_u32(sK[buf]);
#pragma unroll
            for (int kk = 0; kk < HD / 16; ++kk)
                mma_ss(tmem + COL_S, sw128_desc(qa + kk * 32, 16), sw128_desc(ka + kk * 32, 16), idesc_s,
                       kk > 0 ? 1u : 0u);
            tc_commit(bar_mma);
        }
        if (!mbar_wait(bar_mma, mma_phase, p.err, abort_flag)) { ok = false; break; }
        mma_phase ^= 1u;
        tc_fence_after();

        // ---- softmax on this thread's row ----
        uint32_t sr[BN];
#pragma unroll
        for (int c = 0; c < BN / 32; ++c) {
            uint32_t *r = sr + 32 * c;
            TL_LD32(tmem + lane_base + COL_S + 32 * c, r);
        }
        tmem_wait_ld();
        const int k0 = j * BN;
        const bool diag = (k0 + BN - 1 > row) || (k0 + BN > p.ntok);
        float mt = -INFINITY;
#pragma unroll
        for (int c = 0; c < BN; ++c) {
            float s = __uint_as_float(sr[c]) * scale;
            if (diag && (k0 + c > row || k0 + c >= p.ntok)) s = -INFINITY;
            sr[c] = __float_as_uint(s);
            mt = fmaxf(mt, s);
        }
        const float mnew = fmaxf(m, mt);
        const float alpha = (m == -INFINITY) ? 0.f : exp2f(m - mnew);
        float ps = 0.f;
        uint32_t pk[BN / 2];
#pragma unroll
        for (int c = 0; c < BN; c += 2) {
            const float s0 = __uint_as_float(sr[c]), s1 = __uint_as_float(sr[c + 1]);
            const float p0 = (s0 == -INFINITY) ? 0.f : exp2f(s0 - mnew);
            const float p1 = (s1 == -INFINITY) ? 0.f : exp2f(s1 - mnew);
            ps += p0 + p1;
            pk[c / 2] = pack_bf16(p0, p1);
        }
        l = l * alpha + ps;
        m = mnew;
#pragma unroll
        for (int c = 0; c < 2; ++c) {
            uint32_t *r = pk + 32 * c;
            TL_ST32(tmem + lane_base + COL_P + 32 * c, r);
        }
        tmem_wait_st();
        tc_fence_before();
        __syncthreads();
        if (tid == 0) {
            tc_fence_after();
            const uint32_t va = smem_u32(sV[buf]);
#pragma unroll
            for (int kk = 0; kk < BN / 16; ++kk)
                mma_ts(tmem + COL_O, tmem + COL_P + kk * 8, sw128_desc(va + kk * 2048, TILE_BYTES), idesc_o,
                       kk > 0 ? 1u : 0u);
            tc_commit(bar_mma);
        }
        if (!mbar_wait(bar_mma, mma_phase, p.err, abort_flag)) { ok = false; break; }
        mma_phase ^= 1u;
        tc_fence_after();
        uint32_t orr[HD];
#pragma unroll
        for (int c = 0; c < HD / 32; ++c) {
            uint32_t *r = orr + 32 * c;
            TL_LD32(tmem + lane_base + COL_O + 32 * c, r);
        }
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < HD; ++i) o[i] = fmaf(o[i], alpha, __uint_as_float(orr[i]));
        tc_fence_before();
        __syncthreads();  // all rows done with S/P/O before the next tile's MMAs overwrite them
    }

    if (ok && row < p.ntok) {
        const float inv = l > 0.f ? 1.f / l : 0.f;
        float *dst = p.out.ptr;
#pragma unroll
        for (int i = 0; i < HD; ++i) dst[p.out.at(b, row, h, i)] = o[i] * inv;
    }
    // drain outstanding TMA into this CTA's shared memory before it is released
    if (tid == 0 && !ok) {
        mbar_wait(&bar_kv[0], 0, nullptr, nullptr);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, TMEM_COLS);
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
    if (q_rows + BM > INT32_MAX || kv_rows + BN > INT32_MAX) return cudaErrorNotSupported;
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
    p.q_row0 = 0;
    p.kv_row_layer = a.kv.row(a.layer, a.slot0, 0, 0);
    p.kv_rows_per_slot = a.kv.nHeadKv * a.kv.maxLen;
    p.maxLen = a.kv.maxLen;
    p.err = a.err;
    const int smem = 5 * TILE_BYTES + 128 + 1024;
    cudaError_t e = cudaFuncSetAttribute(prefill_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    dim3 grid((a.ntok + BM - 1) / BM, a.nHead, a.nseq);
    prefill_tc_kernel<<<grid, 128, smem, s>>>(qm, km, vm, p);
    return cudaGetLastError();
}

}  // namespace tl
