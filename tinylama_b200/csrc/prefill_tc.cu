// prefill_tc.cu -- causal GQA prefill attention on the 5th-generation tensor cores (sm_100a).
//
// Replaces the context part of attentionFull (src/forward.nim:141-176) on the bf16 KV path:
// for q-head h and query i, s_j = q_i . k_j / sqrt(d) for j <= i, softmax, ctx_i = sum p_j v_j.
// A prefill may also continue a cached prefix (the prompt of a later turn, which the reference
// feeds token by token through forwardDecode, src/tinylama.nim:70-73): query i of a sequence
// whose chunk starts at position pos0 attends cache positions j <= pos0 + i.
// Inputs are bf16 (Q staged by the RoPE kernel, K/V from the cache the same launch sequence
// appended to), products accumulate in fp32 in tensor memory, softmax runs in fp32.
//
// Persistent: one CTA per SM walks work tiles of NQ x 128 query rows (NQ = 2) of one (sequence,
// q-head), heaviest first, keeping its TMEM and pipelines across tiles.  A TMA warp brings each
// tile's Q into one of two buffers and K/V tiles of BN = 128 positions (2-D tensor maps, 128-byte
// swizzle, no multicast) into a three-deep ring that runs on across tiles.  tcgen05.mma issue is
// spread over three warps of the control warpgroup, each a converged warp with one elected lane
// issuing: one issues S_q = Q_q K^T (4 x kind::f16, M=128, N=128, K=16, A and B K-major from
// shared memory), two issue O_q += P_q V (A = P from TMEM, B = V MN-major from shared memory).
// Issuing an MMA occupies the issuing warp's scheduler partition, and spreading it keeps the four
// softmax warps of a group in step.  NQ softmax warpgroups (thread = query row = TMEM lane) load
// S, mask causally, keep the online max/sum in fp32 (log2 domain), write P as packed bf16 into
// TMEM and rescale O in TMEM only when a row's maximum grows past 2^8.  One pair in four of the
// exponentials runs as a polynomial on the FMA pipe, the rest on MUFU.  S and P have separate
// TMEM columns, so S_q(j+1) runs on the tensor core while the softmax of S_q(j) is still in
// flight.  KV tiles past the diagonal are skipped.  Every mbarrier wait is bounded (common.cuh);
// TMEM is released on every exit path after all issued MMAs have completed.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <math.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "internal.h"

namespace tl {
namespace {

constexpr int BM = 128;             // query rows per CTA
constexpr int HD = 64;              // head_dim covered by this kernel
constexpr int TILE_BYTES = BM * HD * 2;  // 16 KB, one 128 x 64 bf16 tile
constexpr float kLog2e = 1.4426950408889634f;

// ---- PTX wrappers ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_load_2d(void *smem_dst, const CUtensorMap *map, int x, int y,
                                            uint64_t *bar, uint32_t issue) {
    asm volatile(
        "{\n\t.reg .pred e;\n\t"
        "setp.ne.b32 e, %5, 0;\n\t"
        "@e cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];\n\t}" ::
            "r"(smem_u32(smem_dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar)), "r"(issue)
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
// One lane of a converged warp is elected to issue; the rest of the warp runs the same code with
// the instruction predicated off.  Keeping the issuing warp converged lets the compiler hold the
// descriptors in uniform registers instead of moving them lane by lane around every issue.
__device__ __forceinline__ uint32_t elect_one() {
    uint32_t e;
    asm volatile(
        "{\n\t.reg .pred e;\n\t"
        "elect.sync _|e, 0xffffffff;\n\t"
        "selp.u32 %0, 1, 0, e;\n\t}"
        : "=r"(e));
    return e;
}
__device__ __forceinline__ void tc_commit(uint64_t *bar, uint32_t issue) {
    asm volatile(
        "{\n\t.reg .pred e;\n\t"
        "setp.ne.b32 e, %1, 0;\n\t"
        "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(smem_u32(bar)),
        "r"(issue)
        : "memory");
}
// S = Q K^T for one 128 x BN tile, K = 64 as four K=16 MMAs in one block: the predicates are set
// once and the descriptors step by 32 bytes (the K=16 slice of a 128-byte swizzled row), so the
// issuing warp spends a few instructions per MMA.
__device__ __forceinline__ void mma_s_k64(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                          uint32_t issue) {
    asm volatile(
        "{\n\t.reg .pred e, t, f;\n\t.reg .b64 a1, a2, a3, b1, b2, b3;\n\t"
        "setp.ne.b32 e, %4, 0;\n\t"
        "setp.eq.b32 t, %4, %4;\n\t"
        "setp.ne.b32 f, %4, %4;\n\t"
        "add.s64 a1, %1, 2;\n\tadd.s64 a2, %1, 4;\n\tadd.s64 a3, %1, 6;\n\t"
        "add.s64 b1, %2, 2;\n\tadd.s64 b2, %2, 4;\n\tadd.s64 b3, %2, 6;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, f;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], a1, b1, %3, t;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], a2, b2, %3, t;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], a3, b3, %3, t;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(issue)
        : "memory");
}
// O += P V over 64 keys: four K=16 MMAs, A = P from TMEM (8 columns of packed bf16 per step), B = V
// MN-major from shared memory (16 rows of 128 bytes = 2048 bytes per step).
__device__ __forceinline__ void mma_pv_k64(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate, uint32_t issue) {
    asm volatile(
        "{\n\t.reg .pred e, t, p;\n\t.reg .b32 a1, a2, a3;\n\t.reg .b64 b1, b2, b3;\n\t"
        "setp.ne.b32 e, %5, 0;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "setp.eq.b32 t, %5, %5;\n\t"
        "add.u32 a1, %1, 8;\n\tadd.u32 a2, %1, 16;\n\tadd.u32 a3, %1, 24;\n\t"
        "add.s64 b1, %2, 128;\n\tadd.s64 b2, %2, 256;\n\tadd.s64 b3, %2, 384;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [a1], b1, %3, t;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [a2], b2, %3, t;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [a3], b3, %3, t;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(issue)
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
    const int *pos0;       // device [nseq]: token t of sequence b sits at position pos0[b] + t, or
                           // nullptr (all zero).  Its keys are cache positions [0, pos0[b] + t].
    int nseq, ntok, nHead, nHeadKv;
    int64_t kv_row_layer;  // cache row of (layer, slot0, kvh=0, pos=0)
    int kv_rows_per_slot;  // nHeadKv * maxLen
    int maxLen;
    unsigned *err;
};

// Kernel shape: NQ query tiles of 128 rows per CTA and KV tiles of BN positions.  One control
// warpgroup (TMA warp, MMA warp) and NQ softmax warpgroups; each scheduler partition holds one
// control warp and NQ softmax warps, and more softmax warps per partition hide more latency.
// TMEM per query tile: S (BN columns) + P (BN/2, packed bf16) + O (64).
template <int NQ, int BN_>
struct TcShape {
    static constexpr int THREADS = 128 * (NQ + 1);
    static constexpr int KV_TILE = BN_ * HD * 2;                      // bytes of one K or V tile
    static constexpr int NS = (96 * 1024) / (2 * KV_TILE);            // K/V ring depth: 96 KB
    static constexpr int REG_LAUNCH = (65536 / THREADS) / 8 * 8;       // 168 for 384 threads
    static constexpr int REG_CTRL = 104;
    static constexpr int REG_SOFT = 200;
    static_assert(REG_CTRL + NQ * REG_SOFT <= (NQ + 1) * REG_LAUNCH, "register split exceeds the launch allotment");
    static constexpr int COL_P0 = NQ * BN_;
    static constexpr int COL_O0 = COL_P0 + NQ * BN_ / 2;
    static_assert(COL_O0 + NQ * 64 <= 512, "TMEM columns");
    __host__ __device__ static constexpr int col_s(int q) { return q * BN_; }
    __host__ __device__ static constexpr int col_p(int q) { return COL_P0 + q * (BN_ / 2); }
    __host__ __device__ static constexpr int col_o(int q) { return COL_O0 + q * 64; }
    static constexpr int SMEM = 2 * NQ * TILE_BYTES + NS * 2 * KV_TILE;  // two Q buffers + K/V ring (+ barriers)
};

constexpr int TMEM_ALL = 512;
// Output staging: each softmax warp writes 16 of its rows (64 floats, padded to 68) to shared
// memory and stores them back as whole 256-byte rows, 2 rows per instruction; a thread storing
// its own row would touch 32 rows (lines) per instruction.
constexpr int kStgRow = HD + 4;
constexpr int kStgFloats = 16 * kStgRow;  // per softmax warp
constexpr int kIssuers = 3;  // warps that issue tcgen05.mma: one for S, two for P V
constexpr float kRescaleThreshold = 8.0f;  // log2 units: O is rescaled only past 2^8

template <int N>
__device__ __forceinline__ void setmaxnreg_dec() { asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N)); }
template <int N>
__device__ __forceinline__ void setmaxnreg_inc() { asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N)); }

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

// 2^x for a pair on the FMA pipe, to take part of the exponentials off the MUFU unit (whose
// throughput, 16 per SM per clock, bounds this kernel).  Range reduction by the round-to-nearest
// magic constant 1.5 * 2^23: t = x + M keeps n = round(x) in its low mantissa bits, f = x - n lies
// in [-0.5, 0.5], 2^f comes from a degree-3 polynomial fitted for minimax relative error on that
// interval (7.5e-5 relative, below the bf16 rounding of P), and 2^n is added to the exponent
// field.  x is clamped to -125 so that the exponent never underflows (2^-125 stands in for 0).
__device__ __forceinline__ float2 fsub2(float2 a, float2 b) {
    unsigned long long d;
    asm("sub.rn.f32x2 %0, %1, %2;"
        : "=l"(d)
        : "l"(*reinterpret_cast<unsigned long long *>(&a)), "l"(*reinterpret_cast<unsigned long long *>(&b)));
    return *reinterpret_cast<float2 *>(&d);
}
__device__ __forceinline__ float2 fadd2_rn(float2 a, float2 b) {
    unsigned long long d;
    asm("add.rn.f32x2 %0, %1, %2;"
        : "=l"(d)
        : "l"(*reinterpret_cast<unsigned long long *>(&a)), "l"(*reinterpret_cast<unsigned long long *>(&b)));
    return *reinterpret_cast<float2 *>(&d);
}
__device__ __forceinline__ float2 exp2_poly2(float2 x) {
    constexpr float kM = 12582912.0f;  // 1.5 * 2^23
    x.x = fmaxf(x.x, -125.f);
    x.y = fmaxf(x.y, -125.f);
    const float2 t = fadd2_rn(x, make_float2(kM, kM));
    const float2 f = fsub2(x, fsub2(t, make_float2(kM, kM)));
    float2 p = ffma2(make_float2(0.05517132207751274f, 0.05517132207751274f), f,
                     make_float2(0.24261054396629333f, 0.24261054396629333f));
    p = ffma2(p, f, make_float2(0.6932609677314758f, 0.6932609677314758f));
    p = ffma2(p, f, make_float2(0.9999281167984009f, 0.9999281167984009f));
    return make_float2(__uint_as_float(__float_as_uint(p.x) + (__float_as_uint(t.x) << 23)),
                       __uint_as_float(__float_as_uint(p.y) + (__float_as_uint(t.y) << 23)));
}

#ifndef TL_POLY_MOD
#define TL_POLY_MOD 4
#endif
// every TL_POLY_MOD-th pair of a row's exponentials runs on the FMA pipe (0: none)
constexpr int kPolyMod = TL_POLY_MOD;

template <int NQ, int NS>
struct Bars {
    uint64_t q_full[2], q_empty[2], kv_full[NS], kv_empty[NS], s_full[NQ], s_free[NQ], p_ready[NQ], o_bar[NQ],
        o_done[NQ], o_free[NQ], mma_final;
    uint32_t tmem_base;
    int abort;
};

// One work tile: NQ*128 query rows of one (sequence, q-head).  Tiles are numbered heaviest first
// (the last query rows of a sequence attend to the most keys); CTA i takes tiles i, i + gridDim,
// ... so every CTA gets a similar mix.  off = the position of the sequence's first query (a
// prefill that continues a cached prefix); query row r attends keys [0, off + r].
template <int NQ, int BN_>
struct TileInfo {
    int b, h, g, q0, off, nkv, nq_live, qrow, kvrow0;
    int nt[NQ];
    __device__ __forceinline__ TileInfo(const TcParams &p, int t) {
        const int ngroups = (p.ntok + NQ * BM - 1) / (NQ * BM);
        const int per = p.nHead * p.nseq;
        const int rank = t / per, rem = t - rank * per;
        h = rem / p.nseq;
        b = rem - h * p.nseq;
        g = h / (p.nHead / p.nHeadKv);
        q0 = (ngroups - 1 - rank) * NQ * BM;
        // the host checks 0 <= pos0 and pos0 + ntok <= maxLen; the clamp keeps every K/V tile
        // inside this (sequence, kv-head)'s rows whatever the device array holds
        off = p.pos0 ? min(max(p.pos0[b], 0), p.maxLen - p.ntok) : 0;
        nkv = 0;
        nq_live = 0;
#pragma unroll
        for (int q = 0; q < NQ; ++q) {
            const int start = q0 + q * BM;
            nt[q] = start < p.ntok ? (off + min(start + BM, p.ntok) + BN_ - 1) / BN_ : 0;
            nkv = max(nkv, nt[q]);
            nq_live += nt[q] > 0;
        }
        qrow = (int)(((int64_t)b * p.nHead + h) * p.ntok + q0);
        kvrow0 = (int)(p.kv_row_layer + (int64_t)b * p.kv_rows_per_slot + (int64_t)g * p.maxLen);
    }
};

// Causal prefill, persistent: one CTA per SM walks work tiles (NQ*128 query rows of one
// (sequence, q-head)) and keeps its TMEM, barriers and pipelines across them.
//   warp 0: TMA (elected lane) -- Q of each tile into one of two Q buffers, K/V tiles into a ring
//     that runs on across tiles, so the next tile's Q and first K/V arrive while this one ends;
//   warp 1: TMEM owner and S issuer; warps 2, 3: P V issuers (query tile 0, 1);
//   warpgroup 1+q: softmax of query tile q, thread = row = TMEM lane (warp w reaches TMEM lanes
//     32*(w%4)..).
// Per KV tile j and query tile q the S issuer runs S_q(j+1) = Q_q K_{j+1}^T as soon as group q
// has pulled S_q(j) into registers (s_free), and O_q += P_q(j) V_j once P_q(j) is in TMEM
// (p_ready), so the tensor core works on one tile while the softmax runs.  A group overwrites
// P_q and rescales O_q only after PV_q(j-1) has completed (o_bar); a tile's first P V (which
// overwrites O_q) waits until the group has read out the previous tile's O_q (o_free).  Every
// barrier phase comes from per-role running counts, not from the tile-local index.
template <int NQ, int BN_>
__global__ void __launch_bounds__(TcShape<NQ, BN_>::THREADS, 1)
prefill_tc_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap,
                  const __grid_constant__ CUtensorMap vmap, const TcParams p) {
    static_assert(NQ == 2, "one P V issuer warp per query tile: warps 2 and 3");
    using S_ = TcShape<NQ, BN_>;
    using T_ = TileInfo<NQ, BN_>;
    constexpr int BNK = BN_;
    constexpr int NS = S_::NS;
    using B_ = Bars<NQ, NS>;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    uint8_t *base = smem_raw + (((raw + 1023u) & ~1023u) - raw);
    uint8_t *sQ = base;                                  // [2 buffers][NQ] 16 KB tiles
    uint8_t *sK = base + 2 * NQ * TILE_BYTES;            // [NS] tiles
    uint8_t *sV = sK + NS * S_::KV_TILE;                 // [NS] tiles
    B_ *bars = reinterpret_cast<B_ *>(sV + NS * S_::KV_TILE);
    float *stage = reinterpret_cast<float *>(reinterpret_cast<uint8_t *>(bars) + (sizeof(B_) + 15) / 16 * 16);
    volatile int *abort_flag = &bars->abort;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int ngroups = (p.ntok + NQ * BM - 1) / (NQ * BM);
    const int ntiles = ngroups * p.nHead * p.nseq;

    if (tid == 0) {
        for (int i = 0; i < 2; ++i) {
            mbar_init(&bars->q_full[i], 1);
            mbar_init(&bars->q_empty[i], 1);
        }
        for (int i = 0; i < NS; ++i) {
            mbar_init(&bars->kv_full[i], 1);
            mbar_init(&bars->kv_empty[i], kIssuers);
        }
        for (int q = 0; q < NQ; ++q) {
            mbar_init(&bars->s_full[q], 1);
            mbar_init(&bars->s_free[q], BM);
            mbar_init(&bars->p_ready[q], BM);
            mbar_init(&bars->o_bar[q], 1);
            mbar_init(&bars->o_done[q], 1);
            mbar_init(&bars->o_free[q], BM);
        }
        mbar_init(&bars->mma_final, kIssuers);
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

    if (warp < 4) {
        setmaxnreg_dec<S_::REG_CTRL>();
        // bounded wait by the whole warp with a warp-uniform verdict
        auto wait_all = [&](uint64_t *bar, uint32_t parity, unsigned *err, volatile int *ab) {
            return __all_sync(0xffffffffu, mbar_wait(bar, parity, err, ab));
        };
        if (warp == 0) {
            // ---------------- TMA producer (one elected lane issues) ----------------
            const uint32_t leader = elect_one();
            int it = 0, kvit = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x, ++it) {
                const T_ ti(p, t);
                const int qb = it & 1;
                // Q buffer qb is free once the S MMAs of tile it-2 have completed
                if (!wait_all(&bars->q_empty[qb], ((it >> 1) & 1) ^ 1, p.err, abort_flag)) { ok = false; break; }
                if (leader) mbar_arrive_expect_tx(&bars->q_full[qb], ti.nq_live * TILE_BYTES);
                __syncwarp();
#pragma unroll
                for (int q = 0; q < NQ; ++q)
                    if (ti.nt[q] > 0)
                        tma_load_2d(sQ + (qb * NQ + q) * TILE_BYTES, &qmap, 0, ti.qrow + q * BM, &bars->q_full[qb], leader);
                for (int j = 0; j < ti.nkv; ++j, ++kvit) {
                    const int st = kvit % NS;
                    if (!wait_all(&bars->kv_empty[st], ((kvit / NS) & 1) ^ 1, p.err, abort_flag)) { ok = false; break; }
                    if (leader) mbar_arrive_expect_tx(&bars->kv_full[st], 2 * S_::KV_TILE);
                    __syncwarp();
                    tma_load_2d(sK + st * S_::KV_TILE, &kmap, 0, ti.kvrow0 + j * BNK, &bars->kv_full[st], leader);
                    tma_load_2d(sV + st * S_::KV_TILE, &vmap, 0, ti.kvrow0 + j * BNK, &bars->kv_full[st], leader);
                }
                if (!ok) { ++it; break; }
            }
            // wait (bounded) until every copy issued into this CTA's shared memory has landed
            for (int i = max(0, it - 2); i < it; ++i) wait_all(&bars->q_full[i & 1], (i >> 1) & 1, nullptr, nullptr);
            for (int j = max(0, kvit - NS); j < kvit; ++j)
                wait_all(&bars->kv_full[j % NS], (j / NS) & 1, nullptr, nullptr);
        } else if (warp == 1) {
            // ---------------- S issuer: S_q(j) = Q_q K_j^T ----------------
            // Issuing a tcgen05.mma holds the issuing warp's scheduler for a while, so the MMAs
            // are spread over three warps (three scheduler partitions): this one issues every S,
            // warps 2 and 3 issue O += P V.
            const uint32_t leader = elect_one();
            const uint32_t idesc_s = idesc_bf16(BNK, false);
            int it = 0, kvit = 0;
            int ns[NQ] = {};
            bool ok = true;
            for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x, ++it) {
                const T_ ti(p, t);
                const int qb = it & 1;
                ok = wait_all(&bars->q_full[qb], (it >> 1) & 1, p.err, abort_flag);
                for (int j = 0; j < ti.nkv && ok; ++j, ++kvit) {
                    const int st = kvit % NS;
                    ok = wait_all(&bars->kv_full[st], (kvit / NS) & 1, p.err, abort_flag);
                    if (!ok) break;
                    const uint32_t ka = smem_u32(sK + st * S_::KV_TILE);
#pragma unroll
                    for (int q = 0; q < NQ; ++q) {
                        if (!ok || j >= ti.nt[q]) continue;
                        // the previous S_q must be in the softmax group's registers before it is overwritten
                        if (ns[q] > 0) ok = wait_all(&bars->s_free[q], (ns[q] - 1) & 1, p.err, abort_flag);
                        if (!ok) continue;
                        tc_fence_after();
                        mma_s_k64(tmem + S_::col_s(q), sw128_desc(smem_u32(sQ + (qb * NQ + q) * TILE_BYTES), 16),
                                  sw128_desc(ka, 16), idesc_s, leader);
                        tc_commit(&bars->s_full[q], leader);
                        ++ns[q];
                    }
                    tc_commit(&bars->kv_empty[st], leader);  // K_j is free once these S MMAs complete
                }
                if (ok) tc_commit(&bars->q_empty[qb], leader);  // Q buffer free once this tile's S complete
            }
            // every MMA of the CTA has completed before TMEM can be released
            tc_commit(&bars->mma_final, leader);
            wait_all(&bars->mma_final, 0, p.err, nullptr);
        } else {
            // ---------------- P V issuer for query tile q = warp - 2 ----------------
            const int q = warp - 2;
            const uint32_t leader = elect_one();
            const uint32_t idesc_o = idesc_bf16(HD, true);
            int kvit = 0, npv = 0, nto = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
                const T_ ti(p, t);
                const int ntq = q == 0 ? ti.nt[0] : ti.nt[1];
                for (int j = 0; j < ti.nkv && ok; ++j, ++kvit) {
                    // tile kvit's phase of kv_full has completed, so this warp's kv_empty arrival
                    // belongs to it even when it issues nothing for it
                    const int st = kvit % NS;
                    ok = wait_all(&bars->kv_full[st], (kvit / NS) & 1, p.err, abort_flag);
                    if (!ok) break;
                    if (j < ntq) {
                        // the tile's first P V overwrites O_q: the group has read the previous tile's out
                        if (j == 0 && nto > 0) ok = wait_all(&bars->o_free[q], (nto - 1) & 1, p.err, abort_flag);
                        if (ok) ok = wait_all(&bars->p_ready[q], npv & 1, p.err, abort_flag);
                        if (!ok) break;
                        tc_fence_after();
                        const uint32_t va = smem_u32(sV + st * S_::KV_TILE);
#pragma unroll
                        for (int kb = 0; kb < BNK / 64; ++kb)
                            mma_pv_k64(tmem + S_::col_o(q), tmem + S_::col_p(q) + kb * 32,
                                       sw128_desc(va + kb * 4 * 2048, S_::KV_TILE), idesc_o,
                                       (j > 0 || kb > 0) ? 1u : 0u, leader);
                        tc_commit(&bars->o_bar[q], leader);
                        if (j == ntq - 1) tc_commit(&bars->o_done[q], leader);
                        ++npv;
                    }
                    tc_commit(&bars->kv_empty[st], leader);  // V_j is free once these P V MMAs complete
                }
                if (ntq > 0) ++nto;
            }
            tc_commit(&bars->mma_final, leader);
        }
    } else {
        setmaxnreg_inc<S_::REG_SOFT>();
        // ---------------- softmax of query tile q ----------------
        const int q = (warp - 4) >> 2;
        const int r = (warp & 3) * 32 + lane;
        const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
        const float C = kLog2e / 8.0f;  // log2(e) / sqrt(64)
        int ns = 0, npv = 0, nto = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
            const T_ ti(p, t);
            const int ntq = q == 0 ? ti.nt[0] : ti.nt[1];
            if (ntq == 0) continue;
            const int row_first = ti.q0 + q * BM;
            const int row = row_first + r;
            const int kpos_first = ti.off + row_first, kpos = ti.off + row;  // last key of a row
            float m_run = -INFINITY, l = 0.f;
            for (int j = 0; j < ntq && ok; ++j) {
                // warp-uniform verdict: the TMEM loads below are warp-collective
                ok = __all_sync(0xffffffffu, mbar_wait(&bars->s_full[q], ns & 1, p.err, abort_flag));
                if (!ok) break;
                ++ns;
                tc_fence_after();
                uint32_t sr[BNK];
#pragma unroll
                for (int c = 0; c < BNK / 32; ++c) {
                    uint32_t *rr = sr + 32 * c;
                    TL_LD32(tmem + lane_base + S_::col_s(q) + 32 * c, rr);
                }
                tmem_wait_ld();
                tc_fence_before();
                mbar_arrive(&bars->s_free[q]);  // S_q(j) is in registers: the next S may overwrite it
                const int k0 = j * BNK;
                const int kend = ti.off + p.ntok;
                if (k0 + BNK - 1 > kpos_first || k0 + BNK > kend) {  // tile crosses the diagonal or the end
#pragma unroll
                    for (int c = 0; c < BNK; ++c)
                        if (k0 + c > kpos || k0 + c >= kend) sr[c] = __float_as_uint(-INFINITY);
                }
                // row maximum: four independent chains of three-input max
                float mq[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
                for (int c = 0; c < BNK; c += 8) {
#pragma unroll
                    for (int u = 0; u < 4; ++u)
                        mq[u] = max3f(mq[u], __uint_as_float(sr[c + 2 * u]), __uint_as_float(sr[c + 2 * u + 1]));
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
                    // PV_q(j-1) must be complete before P_q is overwritten (and before O_q is
                    // rescaled); at j == 0 the previous tile's last P V has completed (o_done)
                    ok = __all_sync(0xffffffffu, mbar_wait(&bars->o_bar[q], (npv - 1) & 1, p.err, abort_flag));
                    if (!ok) break;
                    tc_fence_after();
                }
                if (__any_sync(0xffffffffu, grow && j > 0)) {
                    // O_q holds the sum through tile j-1: rescale it in TMEM, 16 columns at a time
#pragma unroll
                    for (int c = 0; c < HD / 16; ++c) {
                        uint32_t orr[16];
                        TL_LD16(tmem + lane_base + S_::col_o(q) + 16 * c, orr);
                        tmem_wait_ld();
#pragma unroll
                        for (int i = 0; i < 16; ++i) orr[i] = __float_as_uint(__uint_as_float(orr[i]) * alpha);
                        TL_ST16(tmem + lane_base + S_::col_o(q) + 16 * c, orr);
                    }
                }
                // p = 2^(s*C - m): the argument in packed pairs, the sum in four packed accumulators
                const float2 c2 = make_float2(C, C), n2 = make_float2(-m_run, -m_run);
                float2 acc[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                                 make_float2(0.f, 0.f)};
                uint32_t pk[BNK / 2];
#pragma unroll
                for (int c = 0; c < BNK; c += 2) {
                    const float2 x = ffma2(make_float2(__uint_as_float(sr[c]), __uint_as_float(sr[c + 1])), c2, n2);
                    const float2 pp = (kPolyMod > 0 && (c >> 1) % (kPolyMod > 0 ? kPolyMod : 1) == (kPolyMod > 0 ? kPolyMod : 1) - 1)
                                          ? exp2_poly2(x)
                                          : make_float2(ex2(x.x), ex2(x.y));
                    acc[(c >> 1) & 3] = fadd2(acc[(c >> 1) & 3], pp);
                    pk[c / 2] = pack_bf16(pp.x, pp.y);
                }
                const float2 a01 = fadd2(acc[0], acc[1]), a23 = fadd2(acc[2], acc[3]);
                const float2 a = fadd2(a01, a23);
                l += a.x + a.y;
#pragma unroll
                for (int c = 0; c < BNK / 64; ++c) {
                    uint32_t *rr = pk + 32 * c;
                    TL_ST32(tmem + lane_base + S_::col_p(q) + 32 * c, rr);
                }
                tmem_wait_st();
                tc_fence_before();
                mbar_arrive(&bars->p_ready[q]);
                ++npv;
            }
            if (!ok) break;
            // epilogue: O_q out of TMEM (then it may be overwritten by the next tile), normalise, store
            ok = __all_sync(0xffffffffu, mbar_wait(&bars->o_done[q], nto & 1, p.err, abort_flag));
            if (!ok) break;
            ++nto;
            tc_fence_after();
            uint32_t orr[HD];
#pragma unroll
            for (int c = 0; c < HD / 32; ++c) {
                uint32_t *rr = orr + 32 * c;
                TL_LD32(tmem + lane_base + S_::col_o(q) + 32 * c, rr);
            }
            tmem_wait_ld();
            tc_fence_before();
            mbar_arrive(&bars->o_free[q]);
            const float inv = l > 0.f ? 1.f / l : 0.f;
            float *dst = p.out.ptr;
            const int wrow0 = row_first + (warp & 3) * 32;  // this warp's first row
            const int64_t o0 = p.out.at(ti.b, wrow0, ti.h, 0), rs = p.out.st;
            const bool staged = p.out.sd == 1 && (o0 & 3) == 0 && (rs & 3) == 0 &&
                                (reinterpret_cast<uintptr_t>(dst) & 15) == 0;
            if (staged) {
                float *stg = stage + (warp - 4) * kStgFloats;
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    if ((lane >> 4) == half) {
                        float *srow = stg + (lane & 15) * kStgRow;
#pragma unroll
                        for (int i = 0; i < HD; i += 4)
                            *reinterpret_cast<float4 *>(srow + i) =
                                make_float4(__uint_as_float(orr[i]) * inv, __uint_as_float(orr[i + 1]) * inv,
                                            __uint_as_float(orr[i + 2]) * inv, __uint_as_float(orr[i + 3]) * inv);
                    }
                    __syncwarp();
#pragma unroll
                    for (int k = 0; k < 8; ++k) {
                        const int idx = k * 32 + lane, rr = idx >> 4, c4 = idx & 15;
                        if (wrow0 + half * 16 + rr < p.ntok)
                            *reinterpret_cast<float4 *>(dst + o0 + (int64_t)(half * 16 + rr) * rs + 4 * c4) =
                                *reinterpret_cast<const float4 *>(stg + rr * kStgRow + 4 * c4);
                    }
                    __syncwarp();
                }
            } else if (row < p.ntok) {
#pragma unroll
                for (int i = 0; i < HD; i += 4) {
                    const int64_t o = p.out.at(ti.b, row, ti.h, i);
                    if (p.out.sd == 1 && (o & 3) == 0) {
                        *reinterpret_cast<float4 *>(dst + o) =
                            make_float4(__uint_as_float(orr[i]) * inv, __uint_as_float(orr[i + 1]) * inv,
                                        __uint_as_float(orr[i + 2]) * inv, __uint_as_float(orr[i + 3]) * inv);
                    } else {
#pragma unroll
                        for (int u = 0; u < 4; ++u)
                            dst[p.out.at(ti.b, row, ti.h, i + u)] = __uint_as_float(orr[i + u]) * inv;
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

bool make_map(CUtensorMap *m, const void *ptr, uint64_t rows, int box_rows) {
    auto enc = get_encode();
    if (!enc) return false;
    cuuint64_t dims[2] = {(cuuint64_t)HD, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)HD * 2};
    cuuint32_t box[2] = {(cuuint32_t)HD, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(ptr), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

template <int NQ, int BN_>
cudaError_t launch_shape(const PrefillArgs &a, cudaStream_t s) {
    using S_ = TcShape<NQ, BN_>;
    const int64_t q_rows = (int64_t)a.nseq * a.nHead * a.ntok;
    const int64_t kv_rows = (int64_t)a.kv.nLayer * a.kv.maxBatch * a.kv.nHeadKv * a.kv.maxLen;
    if (q_rows + NQ * BM > INT32_MAX || kv_rows + BN_ > INT32_MAX) return cudaErrorNotSupported;
    CUtensorMap qm, km, vm;
    if (!make_map(&qm, a.qb, (uint64_t)q_rows, BM) || !make_map(&km, a.kv.k, (uint64_t)kv_rows, BN_) ||
        !make_map(&vm, a.kv.v, (uint64_t)kv_rows, BN_))
        return cudaErrorNotSupported;
    TcParams p;
    p.out = a.out;
    p.pos0 = a.pos0;
    p.nseq = a.nseq;
    p.ntok = a.ntok;
    p.nHead = a.nHead;
    p.nHeadKv = a.nHeadKv;
    p.kv_row_layer = a.kv.row(a.layer, a.slot0, 0, 0);
    p.kv_rows_per_slot = a.kv.nHeadKv * a.kv.maxLen;
    p.maxLen = a.kv.maxLen;
    p.err = a.err;
    const int smem = S_::SMEM + (int)sizeof(Bars<NQ, S_::NS>) + 16 + NQ * 4 * kStgFloats * (int)sizeof(float) + 1024;
    auto kern = prefill_tc_kernel<NQ, BN_>;
    static int smem_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (smem_set[dev & 63] < smem) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        smem_set[dev & 63] = smem;
    }
    // persistent: one CTA per SM (TMEM and shared memory allow one), at most one per tile
    static int sms[64] = {};
    if (sms[dev & 63] == 0) {
        int n = 0;
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        sms[dev & 63] = n > 0 ? n : 1;
    }
    const long long ntiles = (long long)((a.ntok + NQ * BM - 1) / (NQ * BM)) * a.nHead * a.nseq;
    if (ntiles > INT32_MAX) return cudaErrorNotSupported;
    const int grid = (int)std::min<long long>(ntiles, sms[dev & 63]);
    kern<<<grid, S_::THREADS, smem, s>>>(qm, km, vm, p);
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_prefill_tc(const PrefillArgs &a, cudaStream_t s) {
    if (a.headDim != HD || a.kv.dtype != TL_KV_BF16 || a.qb == nullptr || a.kf.ptr != nullptr ||
        a.ntok > a.kv.maxLen)
        return cudaErrorNotSupported;
    return launch_shape<2, 128>(a, s);
}

}  // namespace tl
