// model_gpu.cu -- the llama forward pass of tinylama on one B200 (tl_model.h).
//
// The reference computes every step of a token on the CPU in float32 (src/forward.nim:243-329)
// from weights dequantised at load time.  Here the weights stay in HBM as the GGUF stores them
// (Q2_K: 84 bytes per 256 weights, src/quant.nim:49-87; or float32) and are dequantised inside
// the matrix-vector kernel, whose cost is the weight bytes it streams.
//
// Kernels of one token (S tokens for the prefill):
//   embed_kernel       embeddingLookup (src/forward.nim:15-38): the token's row, dequantised if
//                      Q2_K; the token id comes from device memory.
//   gemv_kernel        linearGGMLCol (src/forward.nim:40-83), y[s][o] = sum_k W[o][k] x[s][k],
//                      with what is around it folded in: the rmsnormCols of its input
//                      (src/tensor.nim:97-113) in the prologue, and in the epilogue the
//                      residual add (x = add(x, ...)), or silu(gate) * up of ffn
//                      (src/forward.nim:213-217) when it computes the gate and up rows together.
//                      q, k and v are one launch (three matrices, one input).
//   argmax_kernel      argmaxLast (src/infer_core.nim:6-32) and the top-2 gap; it writes the
//                      next token and position for the following decode step.
// Attention between them is the path of tl_attn.h: tl_decode_step (RoPE, append, split-KV decode)
// and tl_prefill_step, on an f32 cache like the reference's.
//
// Q2_K in the matrix-vector kernel.  Weight w of a 256-weight block is
//   d * (sc & 15) * q - dmin * (sc >> 4),
// q two bits of byte 32n + 16h + l (n = w / 128, h = w / 16 % 2, l = w % 16) at bit 2*it
// (it = w / 32 % 4), sc byte 8n + 2it + h of the 16 scales.  A lane takes one (block, n, h):
// 16 bytes of q, i.e. four 16-weight sub-blocks (it = 0..3) that each share one (d*sc, dmin*sc).
// Per sub-block it forms
//   F = sum_l (1 + q_l / 4) x_l      (the float 1 + q/4 is the bit pattern 0x3F800000 | q << 21)
// and adds  d*sc * 4 * (F - X) - dmin*sc * X,  X = sum_l x_l of the sub-block, which the block
// computes once for all rows in its prologue.  For one token (the decode step) the bit
// patterns of four weights come from one word of bytes 0x80 | q << 5 by one byte permutation
// each, two weights share a packed multiply-add (fma.rn.f32x2), and the two rows of a gate/up
// or RoPE pair share their loads of x: about two and a half instructions per weight against
// 2.6 bits of HBM traffic; the several-token prefill path keeps a shift and a logic op per
// weight and one multiply-add per weight and token.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdio.h>

#include <algorithm>
#include <map>
#include <string>
#include <vector>

#include "../../include/tl_model.h"
#include "common.cuh"
#include "internal.h"

namespace tl {
int api_fail(int code, const char *msg);
}  // namespace tl

using namespace tl;

namespace {

constexpr int QK = 256;          // weights per Q2_K block
constexpr int Q2K_BYTES = 84;    // 16 scales, 64 bytes of 2-bit q, d, dmin (f16)
constexpr int kThreads = 256;    // gemv block: 8 warps, a warp per output row
constexpr int kMaxS = 4;         // tokens per gemv launch
constexpr unsigned kErrToken = 8u;  // a token id outside [0, nVocab)

struct GTensor {
    int type = -1;
    int64_t ne0 = 0, ne1 = 0;
    void *dev = nullptr;
};

struct GMat {
    int type;        // TL_GGML_F32 or TL_GGML_Q2_K
    int rows;
    const void *w;   // rows x in
    float *y;        // [S][rows]
};

enum GemvMode { kPlain = 0, kResidual = 1, kSwiGLU = 2 };

struct GemvArgs {
    GMat m[3];
    int nmat;
    int in;             // input length (multiple of 256 for Q2_K)
    const float *x;     // [S][in]
    int S;
    const float *norm;  // rmsnorm weight [in] applied to x first, or nullptr
    float eps;
    int mode;
};

// x in shared memory, four floats of padding after every 128: the lanes of a warp read float4s
// 16 floats apart within a 256-float stride, which would otherwise meet in the same banks.
__device__ __forceinline__ int xpad(int i) { return i + ((i >> 7) << 2); }
__host__ __device__ constexpr int xpad_len(int in) { return in + ((in >> 7) << 2) + 4; }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// f16 bits to float: exact (src/quant.nim:28-47 builds the same value)
__device__ __forceinline__ float h2f(uint32_t bits) { return __half2float(__ushort_as_half((unsigned short)bits)); }

// One (block, n, h) quarter of a Q2_K block: its 16 bytes of q, the 8 scale bytes of half n
// (sa, sb) and (d, dmin) as f16 bits.
struct Q2Part {
    uint32_t q[4], sa, sb, dd;
};

__device__ __forceinline__ void q2_load(Q2Part &p, const uint8_t *B, int n, int h) {
    const uint32_t *q32 = reinterpret_cast<const uint32_t *>(B + 16 + 32 * n + 16 * h);
    p.q[0] = __ldg(q32);
    p.q[1] = __ldg(q32 + 1);
    p.q[2] = __ldg(q32 + 2);
    p.q[3] = __ldg(q32 + 3);
    const uint32_t *s32 = reinterpret_cast<const uint32_t *>(B + 8 * n);
    p.sa = __ldg(s32);
    p.sb = __ldg(s32 + 1);
    p.dd = __ldg(reinterpret_cast<const uint32_t *>(B + 80));
}

// The quarter against NS inputs.  xs = padded x of token 0 (the others follow at stride
// xstride), xsum = sub-block sums, base = first weight index of the block.
template <int NS>
__device__ __forceinline__ void q2_compute(const Q2Part &p, int n, int h, const float *xs, int xstride,
                                           const float *xsum, int sstride, int base, int S, float *acc) {
    const float d = h2f(p.dd & 0xFFFFu), dmin = h2f(p.dd >> 16);
#pragma unroll
    for (int it = 0; it < 4; ++it) {
        // scale byte 8n + 2it + h: byte 2it + h of (sa, sb)
        const uint32_t word = it < 2 ? p.sa : p.sb;
        const uint32_t sc = (word >> (8 * (2 * (it & 1) + h))) & 0xFFu;
        const float dl = __fmul_rn(d, (float)(sc & 15u)), ml = __fmul_rn(dmin, (float)(sc >> 4));
        const int w0 = base + 128 * n + 32 * it + 16 * h;  // first weight of the sub-block
        float F[NS];
#pragma unroll
        for (int s = 0; s < NS; ++s) F[s] = 0.f;
#pragma unroll
        for (int c = 0; c < 4; ++c) {  // weights 4c .. 4c+3: bytes of q[c]
            float f[4];
#pragma unroll
            for (int b = 0; b < 4; ++b) {
                const int sh = 8 * b + 2 * it;  // bit of q in q[c]
                const uint32_t bits = sh <= 21 ? (p.q[c] << (21 - sh)) : (p.q[c] >> (sh - 21));
                f[b] = __uint_as_float((bits & 0x00600000u) | 0x3F800000u);  // 1 + q/4
            }
#pragma unroll
            for (int s = 0; s < NS; ++s) {
                if (s < S) {
                    const float4 xv = *reinterpret_cast<const float4 *>(xs + s * xstride + xpad(w0 + 4 * c));
                    F[s] = fmaf(f[0], xv.x, F[s]);
                    F[s] = fmaf(f[1], xv.y, F[s]);
                    F[s] = fmaf(f[2], xv.z, F[s]);
                    F[s] = fmaf(f[3], xv.w, F[s]);
                }
            }
        }
#pragma unroll
        for (int s = 0; s < NS; ++s) {
            if (s < S) {
                const float X = xsum[s * sstride + (w0 >> 4)];
                acc[s] = fmaf(dl, 4.f * (F[s] - X), fmaf(-ml, X, acc[s]));
            }
        }
    }
}

// One token (the decode step): the same sums with two weights per packed multiply-add
// (fma.rn.f32x2: even and odd weights in two partial sums, added at the end of the sub-block),
// and the float 1 + q/4 of each weight made by one byte permutation from a word that holds four
// weights' bytes 0x80 | q << 5 (a shift and two logic ops per four weights).
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
    unsigned long long d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;"
        : "=l"(d)
        : "l"(*reinterpret_cast<unsigned long long *>(&a)), "l"(*reinterpret_cast<unsigned long long *>(&b)),
          "l"(*reinterpret_cast<unsigned long long *>(&c)));
    return *reinterpret_cast<float2 *>(&d);
}
__device__ __forceinline__ void q2_compute1(const Q2Part &p, int n, int h, const float *xs, const float *xsum,
                                            int base, float &acc) {
    const float d = h2f(p.dd & 0xFFFFu), dmin = h2f(p.dd >> 16);
    // the four scale bytes of this quarter (byte 2it + h of sa, sb), low and high nibbles apart;
    // a nibble v becomes the float v as the bits 0x4B000000 | v minus 2^23 (exact)
    const uint32_t S4 = __byte_perm(p.sa, p.sb, h ? 0x7531u : 0x6420u);
    const uint32_t SL = S4 & 0x0F0F0F0Fu, SH = (S4 >> 4) & 0x0F0F0F0Fu;
#pragma unroll
    for (int it = 0; it < 4; ++it) {
        const uint32_t sel = 0x5440u | (uint32_t)it;  // bytes (nibble it, 0, 0, 0x4B)
        const float scl = __uint_as_float(__byte_perm(SL, 0x4B00u, sel)) - 8388608.f;
        const float sch = __uint_as_float(__byte_perm(SH, 0x4B00u, sel)) - 8388608.f;
        const float dl = __fmul_rn(d, scl), ml = __fmul_rn(dmin, sch);
        const int w0 = base + 128 * n + 32 * it + 16 * h;  // first weight of the sub-block
        float2 F = make_float2(0.f, 0.f);
#pragma unroll
        for (int c = 0; c < 4; ++c) {  // weights 4c .. 4c+3: bytes of q[c]
            const uint32_t T = (((p.q[c] >> (2 * it)) & 0x03030303u) << 5) | 0x80808080u;
            const float4 xv = *reinterpret_cast<const float4 *>(xs + xpad(w0 + 4 * c));
            // bytes (0, 0, 0x80 | q << 5, 0x3F): the float 1 + q/4
            const float f0 = __uint_as_float(__byte_perm(T, 0x3F00u, 0x5044u));
            const float f1 = __uint_as_float(__byte_perm(T, 0x3F00u, 0x5144u));
            const float f2 = __uint_as_float(__byte_perm(T, 0x3F00u, 0x5244u));
            const float f3 = __uint_as_float(__byte_perm(T, 0x3F00u, 0x5344u));
            F = ffma2(make_float2(f0, f1), make_float2(xv.x, xv.y), F);
            F = ffma2(make_float2(f2, f3), make_float2(xv.z, xv.w), F);
        }
        const float X = xsum[w0 >> 4];
        acc = fmaf(dl, 4.f * ((F.x + F.y) - X), fmaf(-ml, X, acc));
    }
}

// Two rows' quarters at the same place of x (gate and up, or the two rows of a RoPE pair):
// the sums of q2_compute1, with each float4 of x and each sub-block sum loaded once for both.
__device__ __forceinline__ void q2_compute1x2(const Q2Part &pa, const Q2Part &pb, int n, int h, const float *xs,
                                              const float *xsum, int base, float &acca, float &accb) {
    const float da = h2f(pa.dd & 0xFFFFu), dmina = h2f(pa.dd >> 16);
    const float db = h2f(pb.dd & 0xFFFFu), dminb = h2f(pb.dd >> 16);
    const uint32_t Sa = __byte_perm(pa.sa, pa.sb, h ? 0x7531u : 0x6420u);
    const uint32_t Sb = __byte_perm(pb.sa, pb.sb, h ? 0x7531u : 0x6420u);
    const uint32_t SLa = Sa & 0x0F0F0F0Fu, SHa = (Sa >> 4) & 0x0F0F0F0Fu;
    const uint32_t SLb = Sb & 0x0F0F0F0Fu, SHb = (Sb >> 4) & 0x0F0F0F0Fu;
#pragma unroll
    for (int it = 0; it < 4; ++it) {
        const uint32_t sel = 0x5440u | (uint32_t)it;
        const float dla = __fmul_rn(da, __uint_as_float(__byte_perm(SLa, 0x4B00u, sel)) - 8388608.f);
        const float mla = __fmul_rn(dmina, __uint_as_float(__byte_perm(SHa, 0x4B00u, sel)) - 8388608.f);
        const float dlb = __fmul_rn(db, __uint_as_float(__byte_perm(SLb, 0x4B00u, sel)) - 8388608.f);
        const float mlb = __fmul_rn(dminb, __uint_as_float(__byte_perm(SHb, 0x4B00u, sel)) - 8388608.f);
        const int w0 = base + 128 * n + 32 * it + 16 * h;
        float2 Fa = make_float2(0.f, 0.f), Fb = make_float2(0.f, 0.f);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const float4 xv = *reinterpret_cast<const float4 *>(xs + xpad(w0 + 4 * c));
            const float2 x01 = make_float2(xv.x, xv.y), x23 = make_float2(xv.z, xv.w);
            const uint32_t Ta = (((pa.q[c] >> (2 * it)) & 0x03030303u) << 5) | 0x80808080u;
            const uint32_t Tb = (((pb.q[c] >> (2 * it)) & 0x03030303u) << 5) | 0x80808080u;
            Fa = ffma2(make_float2(__uint_as_float(__byte_perm(Ta, 0x3F00u, 0x5044u)),
                                   __uint_as_float(__byte_perm(Ta, 0x3F00u, 0x5144u))), x01, Fa);
            Fa = ffma2(make_float2(__uint_as_float(__byte_perm(Ta, 0x3F00u, 0x5244u)),
                                   __uint_as_float(__byte_perm(Ta, 0x3F00u, 0x5344u))), x23, Fa);
            Fb = ffma2(make_float2(__uint_as_float(__byte_perm(Tb, 0x3F00u, 0x5044u)),
                                   __uint_as_float(__byte_perm(Tb, 0x3F00u, 0x5144u))), x01, Fb);
            Fb = ffma2(make_float2(__uint_as_float(__byte_perm(Tb, 0x3F00u, 0x5244u)),
                                   __uint_as_float(__byte_perm(Tb, 0x3F00u, 0x5344u))), x23, Fb);
        }
        const float X = xsum[w0 >> 4];
        acca = fmaf(dla, 4.f * ((Fa.x + Fa.y) - X), fmaf(-mla, X, acca));
        accb = fmaf(dlb, 4.f * ((Fb.x + Fb.y) - X), fmaf(-mlb, X, accb));
    }
}

template <int NS>
__device__ __forceinline__ void row_dot(const GMat &M, int row, int in, const float *xs, int xstride,
                                        const float *xsum, int sstride, int S, int lane, float *acc) {
#pragma unroll
    for (int s = 0; s < NS; ++s) acc[s] = 0.f;
    if (M.type == TL_GGML_Q2_K) {
        const int nb = in / QK;
        const uint8_t *R = static_cast<const uint8_t *>(M.w) + (size_t)row * nb * Q2K_BYTES;
        for (int t = lane; t < nb * 4; t += 32) {
            const int blk = t >> 2, n = (t >> 1) & 1, h = t & 1;
            Q2Part part;
            q2_load(part, R + (size_t)blk * Q2K_BYTES, n, h);
            q2_compute<NS>(part, n, h, xs, xstride, xsum, sstride, blk * QK, S, acc);
        }
    } else {
        const float *R = static_cast<const float *>(M.w) + (size_t)row * in;
        for (int i = lane * 4; i < in; i += 128) {
            const float4 wv = __ldg(reinterpret_cast<const float4 *>(R + i));
#pragma unroll
            for (int s = 0; s < NS; ++s) {
                if (s < S) {
                    const float4 xv = *reinterpret_cast<const float4 *>(xs + s * xstride + xpad(i));
                    acc[s] = fmaf(wv.x, xv.x, fmaf(wv.y, xv.y, fmaf(wv.z, xv.z, fmaf(wv.w, xv.w, acc[s]))));
                }
            }
        }
    }
#pragma unroll
    for (int s = 0; s < NS; ++s) acc[s] = warp_sum(acc[s]);
}

// The block's copy of x in shared memory: normalised (rmsnormCols) when a.norm is set, and the
// sums of its 16-element sub-blocks.  Each thread loads its share of a token's x (and of the
// norm weights) as float4s in one batch, so the row costs one round trip to L2, not one per
// element.  The norm's sum of squares takes one barrier per token (red holds every token's
// warp partials, each thread adds the 8 of its token); a sub-block's sum is formed in
// registers by the four lanes that hold its float4s.  V4 float4s per thread: inputs up to
// V4 * 1024 wide.  red: kMaxS * 8 floats.  Ends with a barrier.
constexpr int kMaxIn = 8192;
constexpr int kV4 = kMaxIn / 4 / kThreads;  // float4s per thread at the widest input

template <int V4>
__device__ __forceinline__ void stage_x(const GemvArgs &a, float *xs, float *xsum, float *red) {
    const int xstride = xpad_len(a.in), sstride = a.in / 16;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int n4 = a.in / 4;
    for (int s = 0; s < a.S; ++s) {
        const float4 *xr = reinterpret_cast<const float4 *>(a.x + (size_t)s * a.in);
        const float4 *wr = reinterpret_cast<const float4 *>(a.norm);
        float4 v[V4], w[V4];
#pragma unroll
        for (int k = 0; k < V4; ++k) {
            const int i4 = tid + k * kThreads;
            if (i4 < n4) {
                v[k] = xr[i4];
                if (a.norm) w[k] = __ldg(wr + i4);
            }
        }
        float inv = 1.f;
        if (a.norm) {
            // rmsnormCols: inv = 1 / sqrt(sum x^2 / dim + eps); out = x * inv * w
            float ss = 0.f;
#pragma unroll
            for (int k = 0; k < V4; ++k) {
                if (tid + k * kThreads < n4) {
                    ss = fmaf(v[k].x, v[k].x, ss);
                    ss = fmaf(v[k].y, v[k].y, ss);
                    ss = fmaf(v[k].z, v[k].z, ss);
                    ss = fmaf(v[k].w, v[k].w, ss);
                }
            }
            ss = warp_sum(ss);
            if (lane == 0) red[s * (kThreads / 32) + warp] = ss;
            __syncthreads();
            float t = 0.f;
#pragma unroll
            for (int i = 0; i < kThreads / 32; ++i) t += red[s * (kThreads / 32) + i];
            inv = 1.f / sqrtf(t / (float)a.in + a.eps);
        }
#pragma unroll
        for (int k = 0; k < V4; ++k) {
            const int i4 = tid + k * kThreads;
            float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
            if (i4 < n4) {
                o = v[k];
                if (a.norm) {
                    o.x = __fmul_rn(__fmul_rn(o.x, inv), w[k].x);
                    o.y = __fmul_rn(__fmul_rn(o.y, inv), w[k].y);
                    o.z = __fmul_rn(__fmul_rn(o.z, inv), w[k].z);
                    o.w = __fmul_rn(__fmul_rn(o.w, inv), w[k].w);
                }
                *reinterpret_cast<float4 *>(xs + s * xstride + xpad(4 * i4)) = o;
            }
            // the sub-block of float4s 4j .. 4j+3 sits in four consecutive lanes
            float t = (o.x + o.y) + (o.z + o.w);
            t += __shfl_xor_sync(0xffffffffu, t, 1);
            t += __shfl_xor_sync(0xffffffffu, t, 2);
            if ((lane & 3) == 0 && (i4 >> 2) < sstride) xsum[s * sstride + (i4 >> 2)] = t;
        }
    }
    __syncthreads();
}

template <int NS>
__global__ void __launch_bounds__(kThreads) gemv_kernel(const GemvArgs a) {
    extern __shared__ float sm[];
    const int xstride = xpad_len(a.in), sstride = a.in / 16;
    float *xs = sm;                     // [NS][xstride]
    float *xsum = sm + NS * xstride;    // [NS][in/16]
    __shared__ float red[kMaxS * (kThreads / 32)];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    stage_x<kV4>(a, xs, xsum, red);
    // ---- rows: a warp per row task ----
    const int rows0 = a.m[0].rows;
    const int tasks = a.mode == kSwiGLU ? rows0 : rows0 + (a.nmat > 1 ? a.m[1].rows : 0) + (a.nmat > 2 ? a.m[2].rows : 0);
    const int gw = blockIdx.x * (kThreads / 32) + warp, nw = gridDim.x * (kThreads / 32);
    for (int task = gw; task < tasks; task += nw) {
        // the matrix of this row, chosen without indexing the parameter array (which would copy
        // it to local memory)
        int row = task;
        GMat M = a.m[0];
        if (a.mode != kSwiGLU && a.nmat > 1 && row >= a.m[0].rows) {
            row -= a.m[0].rows;
            M = a.m[1];
            if (a.nmat > 2 && row >= a.m[1].rows) {
                row -= a.m[1].rows;
                M = a.m[2];
            }
        }
        float acc[NS];
        row_dot<NS>(M, row, a.in, xs, xstride, xsum, sstride, a.S, lane, acc);
        if (a.mode == kSwiGLU) {
            float up[NS];
            row_dot<NS>(a.m[1], row, a.in, xs, xstride, xsum, sstride, a.S, lane, up);
            if (lane == 0) {
#pragma unroll
                for (int s = 0; s < NS; ++s) {
                    if (s < a.S) {
                        // silu(g) = g / (1 + exp(-g)) (src/tensor.nim:52-56), times up
                        const float g = acc[s];
                        const float sl = __fdiv_rn(g, __fadd_rn(1.f, expf(-g)));
                        M.y[(size_t)s * rows0 + row] = __fmul_rn(sl, up[s]);
                    }
                }
            }
        } else if (lane == 0) {
#pragma unroll
            for (int s = 0; s < NS; ++s) {
                if (s < a.S) {
                    float *dst = M.y + (size_t)s * M.rows + row;
                    *dst = a.mode == kResidual ? __fadd_rn(*dst, acc[s]) : acc[s];
                }
            }
        }
    }
}

// RoPE and the cache append folded into the q/k/v product of a decode step (S = 1): a warp
// computes rows 2i and 2i+1 of a head together, rotates q and k at the token's position like
// applyRopeAtPos (src/forward.nim:125-139), writes q for the attention and k, v straight into
// the f32 cache (storeKVRange, :232-241).
struct RopeFuse {
    const float *theta;  // [pairs] per-pair frequencies
    int pairs, hd, layer;
    const int *pos;      // device: the token's position
    float *kc, *vc;      // the cache
    KvLayout kv;
    unsigned *err;
};

// Q2_K matrices only, launched with programmatic dependent launch.  Before the kernel waits for
// the one before it, each warp loads the quantised data of its first PRE row tasks into
// registers -- the weights depend on nothing, so their fetch overlaps the tail of the previous
// kernel; later tasks are loaded PRE ahead of their use.  A task is RP consecutive rows (2 for
// the RoPE pairs).  SWI: gate and up rows together, silu(gate) * up out.
template <int NS, int TPL, bool SWI, int RP>
struct Q2Cfg {
    static constexpr int PER = RP * TPL * (SWI ? 2 : 1);  // Q2Part per task and lane
    static constexpr int PRE = PER * 7 * 3 <= 48 ? 3 : (PER * 7 * 2 <= 48 ? 2 : 1);
};

template <int NS, int TPL, bool SWI, int RP>
__global__ void __launch_bounds__(kThreads, 2) gemv_q2k_kernel(const GemvArgs a, const RopeFuse rf) {
    using Cf = Q2Cfg<NS, TPL, SWI, RP>;
    constexpr int PRE = Cf::PRE;
    extern __shared__ float sm[];
    const int xstride = xpad_len(a.in), sstride = a.in / 16;
    float *xs = sm;
    float *xsum = sm + NS * xstride;
    __shared__ float red[kMaxS * (kThreads / 32)];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int nb = a.in / QK, ntask = nb * 4;
    const size_t rowBytes = (size_t)nb * Q2K_BYTES;
    const int rows0 = a.m[0].rows;
    const int rowsAll = SWI ? rows0 : rows0 + (a.nmat > 1 ? a.m[1].rows : 0) + (a.nmat > 2 ? a.m[2].rows : 0);
    const int tasks = rowsAll / RP;
    const int gw = blockIdx.x * (kThreads / 32) + warp, nw = gridDim.x * (kThreads / 32);
    const int count = gw < tasks ? (tasks - gw + nw - 1) / nw : 0;  // tasks of this warp
    // task -> (matrix, first row), without indexing the parameter array
    auto locate = [&](int task, GMat &M, int &row, int &mi) {
        row = task * RP;
        M = a.m[0];
        mi = 0;
        if (!SWI && a.nmat > 1 && row >= a.m[0].rows) {
            row -= a.m[0].rows;
            M = a.m[1];
            mi = 1;
            if (a.nmat > 2 && row >= a.m[1].rows) {
                row -= a.m[1].rows;
                M = a.m[2];
                mi = 2;
            }
        }
    };
    auto load_task = [&](Q2Part (&P)[Cf::PER], int task) {
        GMat M;
        int row, mi;
        locate(task, M, row, mi);
#pragma unroll
        for (int r = 0; r < RP; ++r) {
#pragma unroll
            for (int k = 0; k < TPL; ++k) {
                const int t = lane + 32 * k;
                if (t < ntask) {
                    const size_t off = (size_t)(row + r) * rowBytes + (size_t)(t >> 2) * Q2K_BYTES;
                    q2_load(P[r * TPL + k], static_cast<const uint8_t *>(M.w) + off, (t >> 1) & 1, t & 1);
                    if (SWI) q2_load(P[RP * TPL + r * TPL + k], static_cast<const uint8_t *>(a.m[1].w) + off, (t >> 1) & 1, t & 1);
                }
            }
        }
    };
    Q2Part buf[PRE][Cf::PER];
#pragma unroll
    for (int j = 0; j < PRE; ++j)
        if (j < count) load_task(buf[j], gw + j * nw);
    pdl_launch_dependents();  // the next kernel may start fetching its own weights
    pdl_wait();               // x comes from the kernel before
    stage_x<2 * TPL>(a, xs, xsum, red);
    int pos = 0;
    if (RP == 2 && rf.pos) pos = *rf.pos;
    for (int j0 = 0; j0 < count; j0 += PRE) {
#pragma unroll
        for (int jj = 0; jj < PRE; ++jj) {
            const int j = j0 + jj;
            if (j >= count) break;
            const int task = gw + j * nw;
            float acc[RP][NS], up[RP][NS];
#pragma unroll
            for (int r = 0; r < RP; ++r)
#pragma unroll
                for (int s = 0; s < NS; ++s) acc[r][s] = up[r][s] = 0.f;
#pragma unroll
            for (int r = 0; r < RP; ++r) {
#pragma unroll
                for (int k = 0; k < TPL; ++k) {
                    const int t = lane + 32 * k;
                    if (t < ntask) {
                        const int n = (t >> 1) & 1, h = t & 1, base = (t >> 2) * QK;
                        if constexpr (NS == 1 && SWI) {
                            q2_compute1x2(buf[jj][r * TPL + k], buf[jj][RP * TPL + r * TPL + k], n, h, xs, xsum, base,
                                          acc[r][0], up[r][0]);
                        } else if constexpr (NS == 1 && RP == 2) {
                            if (r == 0)  // both rows of the pair at once
                                q2_compute1x2(buf[jj][k], buf[jj][TPL + k], n, h, xs, xsum, base, acc[0][0], acc[RP - 1][0]);
                        } else if constexpr (NS == 1) {
                            q2_compute1(buf[jj][r * TPL + k], n, h, xs, xsum, base, acc[r][0]);
                        } else {
                            q2_compute<NS>(buf[jj][r * TPL + k], n, h, xs, xstride, xsum, sstride, base, a.S, acc[r]);
                            if (SWI) q2_compute<NS>(buf[jj][RP * TPL + r * TPL + k], n, h, xs, xstride, xsum, sstride, base, a.S, up[r]);
                        }
                    }
                }
            }
            // this slot is free: fetch the task PRE ahead into it
            if (j + PRE < count) load_task(buf[jj], task + PRE * nw);
#pragma unroll
            for (int r = 0; r < RP; ++r)
#pragma unroll
                for (int s = 0; s < NS; ++s) {
                    acc[r][s] = warp_sum(acc[r][s]);
                    if (SWI) up[r][s] = warp_sum(up[r][s]);
                }
            if (lane != 0) continue;
            GMat M;
            int row, mi;
            locate(task, M, row, mi);
            if (RP == 2 && rf.pos) {
                // decode step: rows (row, row+1) are a RoPE pair of head row / hd
                float y0 = acc[0][0], y1 = acc[RP - 1][0];
                const int head = row / rf.hd, d = row - head * rf.hd;
                if (mi < 2 && (d >> 1) < rf.pairs) {
                    const float angle = __fmul_rn((float)pos, rf.theta[d >> 1]);
                    double sd, cd;
                    sincos((double)angle, &sd, &cd);
                    const float c = (float)cd, sn = (float)sd;
                    const float r0 = __fsub_rn(__fmul_rn(y0, c), __fmul_rn(y1, sn));
                    const float r1 = __fadd_rn(__fmul_rn(y0, sn), __fmul_rn(y1, c));
                    y0 = r0;
                    y1 = r1;
                }
                if (mi == 0) {
                    M.y[row] = y0;
                    M.y[row + 1] = y1;
                } else if (pos >= 0 && pos < rf.kv.maxLen) {
                    float *dst = (mi == 1 ? rf.kc : rf.vc) + rf.kv.row(rf.layer, 0, head, pos) * rf.hd + d;
                    dst[0] = y0;
                    dst[1] = y1;
                } else if (rf.err) {
                    atomicOr(rf.err, TL_DEVERR_POS_RANGE);
                }
                continue;
            }
#pragma unroll
            for (int r = 0; r < RP; ++r) {
#pragma unroll
                for (int s = 0; s < NS; ++s) {
                    if (s < a.S) {
                        if (SWI) {
                            // silu(g) = g / (1 + exp(-g)) (src/tensor.nim:52-56), times up
                            const float g = acc[r][s];
                            const float sl = __fdiv_rn(g, __fadd_rn(1.f, expf(-g)));
                            M.y[(size_t)s * rows0 + row + r] = __fmul_rn(sl, up[r][s]);
                        } else {
                            float *dst = M.y + (size_t)s * M.rows + row + r;
                            *dst = a.mode == kResidual ? __fadd_rn(*dst, acc[r][s]) : acc[r][s];
                        }
                    }
                }
            }
        }
    }
}

// embeddingLookup: the row of each token (nEmb contiguous values in both layouts the reference
// accepts), dequantised if Q2_K.  tokens == nullptr: the token is state[0].
__global__ void embed_kernel(int type, const void *emb, int nVocab, int nEmb, const int32_t *tokens, const int *state,
                             float *x, unsigned *err) {
    const int s = blockIdx.x;
    int tok = tokens ? tokens[s] : state[0];
    if (tok < 0 || tok >= nVocab) {
        if (threadIdx.x == 0) atomicOr(err, kErrToken);
        tok = 0;
    }
    float *dst = x + (size_t)s * nEmb;
    if (type == TL_GGML_F32) {
        const float *row = static_cast<const float *>(emb) + (size_t)tok * nEmb;
        for (int e = threadIdx.x; e < nEmb; e += blockDim.x) dst[e] = row[e];
        return;
    }
    const uint8_t *row = static_cast<const uint8_t *>(emb) + (size_t)tok * (nEmb / QK) * Q2K_BYTES;
    for (int e = threadIdx.x; e < nEmb; e += blockDim.x) {
        const uint8_t *B = row + (size_t)(e / QK) * Q2K_BYTES;
        const int w = e % QK, n = w >> 7, it = (w >> 5) & 3, h = (w >> 4) & 1, l = w & 15;
        const uint32_t dd = *reinterpret_cast<const uint32_t *>(B + 80);
        const uint32_t sc = B[8 * n + 2 * it + h];
        const uint32_t q = (B[16 + 32 * n + 16 * h + l] >> (2 * it)) & 3u;
        const float dl = __fmul_rn(h2f(dd & 0xFFFFu), (float)(sc & 15u));
        const float ml = __fmul_rn(h2f(dd >> 16), (float)(sc >> 4));
        dst[e] = __fsub_rn(__fmul_rn(dl, (float)q), ml);  // dl * q - ml (src/quant.nim:75)
    }
}

// argmaxLast over one logits column with the top-2 gap.  The first index of the maximum wins,
// as in the reference's strict comparison.  Writes ids[step], gaps[step], the next token, and
// advances the position when `advance`.
__global__ void __launch_bounds__(1024) argmax_kernel(const float *logits, int n, int *state, int32_t *ids,
                                                      float *gaps, int advance) {
    __shared__ float sv[32], sv2[32];
    __shared__ int si[32];
    float best = -INFINITY, second = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float v = logits[i];
        if (v > best || (v == best && i < bi)) {
            second = fmaxf(second, best);
            best = v;
            bi = i;
        } else {
            second = fmaxf(second, v);
        }
    }
    // merge (best, index, second) across the block
    auto merge = [](float &b, int &i, float &s2, float ob, int oi, float os2) {
        if (ob > b || (ob == b && oi < i)) {
            s2 = fmaxf(fmaxf(s2, b), os2);
            b = ob;
            i = oi;
        } else {
            s2 = fmaxf(s2, fmaxf(ob, os2));
        }
    };
    for (int o = 16; o >= 1; o >>= 1) {
        const float ob = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        const float os = __shfl_xor_sync(0xffffffffu, second, o);
        merge(best, bi, second, ob, oi, os);
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) { sv[warp] = best; si[warp] = bi; sv2[warp] = second; }
    __syncthreads();
    if (warp == 0) {
        const int nw = blockDim.x >> 5;
        best = lane < nw ? sv[lane] : -INFINITY;
        bi = lane < nw ? si[lane] : 0x7fffffff;
        second = lane < nw ? sv2[lane] : -INFINITY;
        for (int o = 16; o >= 1; o >>= 1) {
            const float ob = __shfl_xor_sync(0xffffffffu, best, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            const float os = __shfl_xor_sync(0xffffffffu, second, o);
            merge(best, bi, second, ob, oi, os);
        }
        if (lane == 0) {
            const int step = state[2];
            ids[step] = bi;
            if (gaps) gaps[step] = best - second;
            state[0] = bi;
            state[2] = step + 1;
            if (advance) state[1] += 1;
        }
    }
}

}  // namespace

struct tl_model {
    tl_model_config c{};
    int device = 0, numSms = 0, headDim = 0;
    std::map<std::string, GTensor> w;
    tl_attn *attn = nullptr;
    cudaStream_t stream = nullptr;
    int capTok = 0;
    float *x = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *ctx = nullptr, *hb = nullptr, *logits = nullptr;
    int *state = nullptr;       // [0] token of the next step, [1] its position, [2] step index
    unsigned *err = nullptr;
    int32_t *tokens = nullptr;
    int capPrompt = 0;
    int32_t *ids = nullptr;
    float *gaps = nullptr;
    int capIds = 0;
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t graphExec = nullptr;
    cudaEvent_t ev[3] = {};
    float prefillMs = 0.f, decodeMs = 0.f;
    float *ropeTheta = nullptr;  // per-pair RoPE frequencies (device), for the fused decode q/k/v
    int ropePairs = 0;
};

namespace {

int cuda_fail(cudaError_t e, const char *what) {
    char m[256];
    snprintf(m, sizeof m, "%s failed: %s", what, cudaGetErrorString(e));
    return api_fail(e == cudaErrorMemoryAllocation ? TL_ERR_NOMEM : TL_ERR_CUDA, m);
}
#define TLM_CUDA(call)                                   \
    do {                                                 \
        cudaError_t e_ = (call);                         \
        if (e_ != cudaSuccess) return cuda_fail(e_, #call); \
    } while (0)
#define TLM_TRY(expr)               \
    do {                            \
        int r_ = (expr);            \
        if (r_ != TL_OK) return r_; \
    } while (0)

struct DevGuard {
    int prev = -1;
    explicit DevGuard(int dev) {
        cudaGetDevice(&prev);
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DevGuard() {
        int cur = -1;
        cudaGetDevice(&cur);
        if (prev >= 0 && cur != prev) cudaSetDevice(prev);
    }
};

const GTensor *find(const tl_model *m, const std::string &a, const std::string &b = "") {
    auto it = m->w.find(a);
    if (it != m->w.end()) return &it->second;
    if (!b.empty()) {
        it = m->w.find(b);
        if (it != m->w.end()) return &it->second;
    }
    return nullptr;
}

int need(const tl_model *m, const GTensor **out, const std::string &name, int64_t ne0, int64_t ne1,
         const std::string &alt = "") {
    const GTensor *t = find(m, name, alt);
    if (!t) return api_fail(TL_ERR_INVALID, ("missing tensor: " + name).c_str());
    if (t->ne0 != ne0 || t->ne1 != ne1) {
        char msg[256];
        snprintf(msg, sizeof msg, "tensor %s has shape [%lld, %lld], expected [%lld, %lld]", name.c_str(),
                 (long long)t->ne0, (long long)t->ne1, (long long)ne0, (long long)ne1);
        return api_fail(TL_ERR_INVALID, msg);
    }
    *out = t;
    return TL_OK;
}

int launch_gemv(tl_model *m, int mode, const GTensor *const *W, int nmat, float *const *y, const float *x, int S,
                const float *norm, const RopeFuse *rope = nullptr) {
    const int in = (int)W[0]->ne0;
    if (in > kMaxIn || in % 4 != 0) return api_fail(TL_ERR_UNSUPPORTED, "tl_model: matrix inputs wider than 8192");
    for (int s0 = 0; s0 < S; s0 += kMaxS) {
        GemvArgs a{};
        a.nmat = nmat;
        a.in = in;
        a.S = std::min(kMaxS, S - s0);
        a.x = x + (size_t)s0 * in;
        a.norm = norm;
        a.eps = m->c.rmsEps;
        a.mode = mode;
        int tasks = 0;
        for (int i = 0; i < nmat; ++i) {
            a.m[i].type = W[i]->type;
            a.m[i].rows = (int)W[i]->ne1;
            a.m[i].w = W[i]->dev;
            a.m[i].y = y[i] + (size_t)s0 * W[i]->ne1;
            if (mode != kSwiGLU || i == 0) tasks += a.m[i].rows;
        }
        if (rope) tasks /= 2;  // a warp takes a RoPE pair of rows
        const int blocks = std::max(1, std::min((tasks + 7) / 8, 2 * m->numSms));
        bool q2 = in % QK == 0 && in <= 4 * 2048;
        for (int i = 0; i < nmat; ++i) q2 = q2 && W[i]->type == TL_GGML_Q2_K;
        const int tpl = (in + 2047) / 2048;
        const bool swi = mode == kSwiGLU;
        const size_t smem = (size_t)(a.S == 1 ? 1 : kMaxS) * (xpad_len(in) + in / 16) * sizeof(float);
        if (rope && !(q2 && S == 1)) return api_fail(TL_ERR_UNSUPPORTED, "fused RoPE needs Q2_K q/k/v and one token");
        if (q2) {
            cudaError_t e = cudaErrorInvalidValue;
            const RopeFuse rf = rope ? *rope : RopeFuse{};
#define TLM_Q2(NS_, T_)                                                                                         \
    e = swi ? launch_pdl(gemv_q2k_kernel<NS_, T_, true, 1>, dim3(blocks), dim3(kThreads), smem, m->stream, a, rf) \
            : launch_pdl(gemv_q2k_kernel<NS_, T_, false, 1>, dim3(blocks), dim3(kThreads), smem, m->stream, a, rf)
#define TLM_Q2R(T_) e = launch_pdl(gemv_q2k_kernel<1, T_, false, 2>, dim3(blocks), dim3(kThreads), smem, m->stream, a, rf)
            if (rope) {
                switch (tpl) {
                    case 1: TLM_Q2R(1); break;
                    case 2: TLM_Q2R(2); break;
                    case 3: TLM_Q2R(3); break;
                    default: TLM_Q2R(4); break;
                }
            } else if (a.S == 1) {
                switch (tpl) {
                    case 1: TLM_Q2(1, 1); break;
                    case 2: TLM_Q2(1, 2); break;
                    case 3: TLM_Q2(1, 3); break;
                    default: TLM_Q2(1, 4); break;
                }
            } else {
                switch (tpl) {
                    case 1: TLM_Q2(kMaxS, 1); break;
                    case 2: TLM_Q2(kMaxS, 2); break;
                    case 3: TLM_Q2(kMaxS, 3); break;
                    default: TLM_Q2(kMaxS, 4); break;
                }
            }
#undef TLM_Q2
#undef TLM_Q2R
            TLM_CUDA(e);
        } else if (a.S == 1) {
            gemv_kernel<1><<<blocks, kThreads, smem, m->stream>>>(a);
        } else {
            gemv_kernel<kMaxS><<<blocks, kThreads, smem, m->stream>>>(a);
        }
        TLM_CUDA(cudaGetLastError());
    }
    return TL_OK;
}

struct LayerW {
    const GTensor *an, *fn, *wq, *wk, *wv, *wo, *wg, *wu, *wd;
};

int resolve(tl_model *m, std::vector<LayerW> &L, const GTensor **emb, const GTensor **onorm, const GTensor **out) {
    const tl_model_config &c = m->c;
    const int hd = m->headDim, kv = c.nHeadKv * hd;
    L.resize(c.nLayer);
    for (int l = 0; l < c.nLayer; ++l) {
        const std::string p = "blk." + std::to_string(l) + ".";
        LayerW &w = L[l];
        TLM_TRY(need(m, &w.an, p + "attn_norm.weight", c.nEmb, 1));
        TLM_TRY(need(m, &w.fn, p + "ffn_norm.weight", c.nEmb, 1));
        TLM_TRY(need(m, &w.wq, p + "attn_q.weight", c.nEmb, c.nHead * hd));
        TLM_TRY(need(m, &w.wk, p + "attn_k.weight", c.nEmb, kv));
        TLM_TRY(need(m, &w.wv, p + "attn_v.weight", c.nEmb, kv));
        TLM_TRY(need(m, &w.wo, p + "attn_output.weight", c.nHead * hd, c.nEmb));
        TLM_TRY(need(m, &w.wg, p + "ffn_gate.weight", c.nEmb, c.nFfn));
        TLM_TRY(need(m, &w.wu, p + "ffn_up.weight", c.nEmb, c.nFfn));
        TLM_TRY(need(m, &w.wd, p + "ffn_down.weight", c.nFfn, c.nEmb));
        if (w.wg->type != w.wu->type) return api_fail(TL_ERR_UNSUPPORTED, "ffn_gate and ffn_up of different types");
    }
    // embeddingLookup and linearOut accept both orientations; the data is nVocab rows of nEmb
    const GTensor *e = find(m, "token_embd.weight", "tok_embeddings.weight");
    if (!e || e->ne0 * e->ne1 != (int64_t)c.nEmb * c.nVocab || !(e->ne0 == c.nEmb || e->ne0 == c.nVocab))
        return api_fail(TL_ERR_INVALID, "embedding shape mismatch");
    if (e->type == TL_GGML_Q2_K && e->ne0 != c.nEmb)
        return api_fail(TL_ERR_UNSUPPORTED, "Q2_K embedding stored vocab-innermost");
    *emb = e;
    TLM_TRY(need(m, onorm, "output_norm.weight", c.nEmb, 1, "norm.weight"));
    const GTensor *o = find(m, "output.weight");
    if (!o || o->ne0 * o->ne1 != (int64_t)c.nEmb * c.nVocab) return api_fail(TL_ERR_INVALID, "output weight shape mismatch");
    if (o->type == TL_GGML_Q2_K && o->ne0 != c.nEmb)
        return api_fail(TL_ERR_UNSUPPORTED, "Q2_K output weight stored vocab-innermost");
    *out = o;
    return TL_OK;
}

// One forward pass over S tokens at positions pos0.. (S == 1 with tokens == nullptr: the decode
// step, token and position from m->state).  Ends with the logits of the last token and its argmax.
int forward(tl_model *m, const std::vector<LayerW> &L, const GTensor *emb, const GTensor *onorm, const GTensor *out,
            int S, const int32_t *tokens, bool decode) {
    const tl_model_config &c = m->c;
    const int hd = m->headDim;
    embed_kernel<<<S, 256, 0, m->stream>>>(emb->type, emb->dev, c.nVocab, c.nEmb, tokens, m->state, m->x, m->err);
    TLM_CUDA(cudaGetLastError());
    for (int l = 0; l < c.nLayer; ++l) {
        const LayerW &w = L[l];
        const GTensor *qkv[3] = {w.wq, w.wk, w.wv};
        float *qkvy[3] = {m->q, m->k, m->v};
        const bool fuse = decode && w.wq->type == TL_GGML_Q2_K && w.wk->type == TL_GGML_Q2_K &&
                          w.wv->type == TL_GGML_Q2_K && m->ropeTheta != nullptr;
        if (fuse) {
            // q/k/v with RoPE at the step's position and k, v written into the cache; then the
            // attention alone (src/forward.nim:314-317)
            RopeFuse rf{};
            rf.theta = m->ropeTheta;
            rf.pairs = m->ropePairs;
            rf.hd = hd;
            rf.layer = l;
            rf.pos = m->state + 1;
            rf.kv = m->attn->kv;
            rf.kc = static_cast<float *>(m->attn->kv.k);
            rf.vc = static_cast<float *>(m->attn->kv.v);
            rf.err = m->err;
            TLM_TRY(launch_gemv(m, kPlain, qkv, 3, qkvy, m->x, 1, static_cast<const float *>(w.an->dev), &rf));
            TLM_TRY(tl_decode_attention(m->attn, l, 0, 1, m->state + 1, nullptr, m->q, m->ctx, m->stream));
        } else if (decode) {
            TLM_TRY(launch_gemv(m, kPlain, qkv, 3, qkvy, m->x, S, static_cast<const float *>(w.an->dev)));
            TLM_TRY(tl_decode_step(m->attn, l, 0, 1, m->state + 1, nullptr, m->q, m->k, m->v, m->ctx, m->stream));
        } else {
            TLM_TRY(launch_gemv(m, kPlain, qkv, 3, qkvy, m->x, S, static_cast<const float *>(w.an->dev)));
            TLM_TRY(tl_prefill_step(m->attn, l, 0, 1, S, m->q, m->k, m->v, m->ctx, m->stream));
        }
        const GTensor *wo[1] = {w.wo};
        float *xo[1] = {m->x};
        TLM_TRY(launch_gemv(m, kResidual, wo, 1, xo, m->ctx, S, nullptr));
        const GTensor *gu[2] = {w.wg, w.wu};
        float *hy[2] = {m->hb, m->hb};
        TLM_TRY(launch_gemv(m, kSwiGLU, gu, 2, hy, m->x, S, static_cast<const float *>(w.fn->dev)));
        const GTensor *wd[1] = {w.wd};
        TLM_TRY(launch_gemv(m, kResidual, wd, 1, xo, m->hb, S, nullptr));
    }
    // linearOut of the last token only: argmaxLast reads the last column
    GTensor ow = *out;
    ow.ne0 = c.nEmb;
    ow.ne1 = c.nVocab;
    const GTensor *ows[1] = {&ow};
    float *ly[1] = {m->logits};
    TLM_TRY(launch_gemv(m, kPlain, ows, 1, ly, m->x + (size_t)(S - 1) * c.nEmb, 1,
                        static_cast<const float *>(onorm->dev)));
    argmax_kernel<<<1, 1024, 0, m->stream>>>(m->logits, c.nVocab, m->state, m->ids, m->gaps, decode ? 1 : 0);
    TLM_CUDA(cudaGetLastError());
    return TL_OK;
}

int ensure_buffers(tl_model *m, int nPrompt, int nNew) {
    const tl_model_config &c = m->c;
    const int hd = m->headDim;
    if (nPrompt > m->capTok) {
        const int cap = std::max(nPrompt, 16);
        cudaFree(m->x); cudaFree(m->q); cudaFree(m->k); cudaFree(m->v); cudaFree(m->ctx); cudaFree(m->hb);
        m->x = m->q = m->k = m->v = m->ctx = m->hb = nullptr;
        m->capTok = 0;
        TLM_CUDA(cudaMalloc(&m->x, sizeof(float) * cap * c.nEmb));
        TLM_CUDA(cudaMalloc(&m->q, sizeof(float) * cap * c.nHead * hd));
        TLM_CUDA(cudaMalloc(&m->k, sizeof(float) * cap * c.nHeadKv * hd));
        TLM_CUDA(cudaMalloc(&m->v, sizeof(float) * cap * c.nHeadKv * hd));
        TLM_CUDA(cudaMalloc(&m->ctx, sizeof(float) * cap * c.nHead * hd));
        TLM_CUDA(cudaMalloc(&m->hb, sizeof(float) * cap * c.nFfn));
        m->capTok = cap;
        // the decode graph captured the old addresses
        if (m->graphExec) { cudaGraphExecDestroy(m->graphExec); m->graphExec = nullptr; }
        if (m->graph) { cudaGraphDestroy(m->graph); m->graph = nullptr; }
    }
    if (nPrompt > m->capPrompt) {
        cudaFree(m->tokens);
        m->tokens = nullptr;
        m->capPrompt = 0;
        TLM_CUDA(cudaMalloc(&m->tokens, sizeof(int32_t) * nPrompt));
        m->capPrompt = nPrompt;
    }
    if (nNew > m->capIds) {
        cudaFree(m->ids);
        cudaFree(m->gaps);
        m->ids = nullptr;
        m->gaps = nullptr;
        m->capIds = 0;
        TLM_CUDA(cudaMalloc(&m->ids, sizeof(int32_t) * nNew));
        TLM_CUDA(cudaMalloc(&m->gaps, sizeof(float) * nNew));
        m->capIds = nNew;
        if (m->graphExec) { cudaGraphExecDestroy(m->graphExec); m->graphExec = nullptr; }
        if (m->graph) { cudaGraphDestroy(m->graph); m->graph = nullptr; }
    }
    return TL_OK;
}

}  // namespace

extern "C" {

int tl_model_create(tl_model **out, const tl_model_config *cfg, int device) {
    if (!out || !cfg) return api_fail(TL_ERR_INVALID, "NULL argument");
    *out = nullptr;
    const tl_model_config &c = *cfg;
    if (c.nLayer < 1 || c.nEmb < 1 || c.nHead < 1 || c.nHeadKv < 1 || c.nFfn < 1 || c.nVocab < 1 || c.maxLen < 1)
        return api_fail(TL_ERR_INVALID, "tl_model_create: sizes must be positive");
    if (c.nHead % c.nHeadKv != 0) return api_fail(TL_ERR_INVALID, "GQA requires head_count divisible by head_count_kv");
    if (c.nEmb % c.nHead != 0) return api_fail(TL_ERR_INVALID, "nEmb must be a multiple of nHead");
    if (c.nEmb > kMaxIn || c.nFfn > kMaxIn)
        return api_fail(TL_ERR_UNSUPPORTED, "tl_model: nEmb and nFfn up to 8192");
    if (c.nEmb % QK != 0 || c.nFfn % QK != 0)
        return api_fail(TL_ERR_UNSUPPORTED, "tl_model: nEmb and nFfn must be multiples of 256");
    tl_model *m = new tl_model();
    m->c = c;
    m->device = device;
    m->headDim = c.nEmb / c.nHead;
    const int ropeDim = c.ropeDim > 0 ? c.ropeDim : m->headDim;
    int rc = tl_attn_create(&m->attn, c.nLayer, c.nHead, c.nHeadKv, m->headDim, ropeDim, c.ropeFreqBase, c.maxLen, 1,
                            TL_KV_F32, device);
    if (rc != TL_OK) {
        delete m;
        return rc;
    }
    DevGuard g(device);
    cudaDeviceGetAttribute(&m->numSms, cudaDevAttrMultiProcessorCount, device);
    if (m->numSms < 1) m->numSms = 1;
    cudaError_t e = cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaMalloc(&m->state, sizeof(int) * 4);
    if (e == cudaSuccess) e = cudaMalloc(&m->err, sizeof(unsigned));
    if (e == cudaSuccess) e = cudaMemset(m->err, 0, sizeof(unsigned));
    for (int i = 0; i < 3 && e == cudaSuccess; ++i) e = cudaEventCreate(&m->ev[i]);
    if (e == cudaSuccess && ropeDim <= m->headDim && ropeDim % 2 == 0 && ropeDim / 2 <= kMaxRopePairs) {
        const RopeTab tab = make_rope_tab(ropeDim, c.ropeFreqBase);  // the frequencies of the RoPE kernels
        e = cudaMalloc(&m->ropeTheta, sizeof(float) * (tab.pairs > 0 ? tab.pairs : 1));
        if (e == cudaSuccess && tab.pairs > 0)
            e = cudaMemcpy(m->ropeTheta, tab.theta, sizeof(float) * tab.pairs, cudaMemcpyHostToDevice);
        m->ropePairs = tab.pairs;
    }
    // the largest gemv (kMaxS tokens of the ffn input) needs more than the default 48 KB
    const int big = std::max(c.nEmb, c.nFfn);
    const int smem = kMaxS * (xpad_len(big) + big / 16) * (int)sizeof(float);
    if (e == cudaSuccess) e = cudaFuncSetAttribute(gemv_kernel<kMaxS>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(gemv_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (xpad_len(big) + big / 16) * (int)sizeof(float));
    // the pipelined Q2_K kernels take inputs up to 8192 wide
    const int smem1 = (xpad_len(8192) + 8192 / 16) * (int)sizeof(float), smem4 = kMaxS * smem1;
#define TLM_ATTR(NS_, T_, SW_)                                                                             \
    if (e == cudaSuccess)                                                                                 \
        e = cudaFuncSetAttribute(gemv_q2k_kernel<NS_, T_, SW_, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                                 NS_ == 1 ? smem1 : smem4);                                              \
    if (e == cudaSuccess && NS_ == 1 && !SW_)                                                            \
        e = cudaFuncSetAttribute(gemv_q2k_kernel<1, T_, false, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem1);
    TLM_ATTR(1, 1, false) TLM_ATTR(1, 2, false) TLM_ATTR(1, 3, false) TLM_ATTR(1, 4, false)
    TLM_ATTR(1, 1, true) TLM_ATTR(1, 2, true) TLM_ATTR(1, 3, true) TLM_ATTR(1, 4, true)
    TLM_ATTR(kMaxS, 1, false) TLM_ATTR(kMaxS, 2, false) TLM_ATTR(kMaxS, 3, false) TLM_ATTR(kMaxS, 4, false)
    TLM_ATTR(kMaxS, 1, true) TLM_ATTR(kMaxS, 2, true) TLM_ATTR(kMaxS, 3, true) TLM_ATTR(kMaxS, 4, true)
#undef TLM_ATTR
    if (e != cudaSuccess) {
        tl_model_destroy(m);
        return cuda_fail(e, "tl_model_create");
    }
    *out = m;
    return TL_OK;
}

void tl_model_destroy(tl_model *m) {
    if (!m) return;
    DevGuard g(m->device);
    if (m->stream) cudaStreamSynchronize(m->stream);
    if (m->graphExec) cudaGraphExecDestroy(m->graphExec);
    if (m->graph) cudaGraphDestroy(m->graph);
    for (auto &kv : m->w) cudaFree(kv.second.dev);
    cudaFree(m->x); cudaFree(m->q); cudaFree(m->k); cudaFree(m->v); cudaFree(m->ctx); cudaFree(m->hb);
    cudaFree(m->logits); cudaFree(m->state); cudaFree(m->err); cudaFree(m->tokens); cudaFree(m->ids);
    cudaFree(m->gaps);
    cudaFree(m->ropeTheta);
    for (auto &ev : m->ev)
        if (ev) cudaEventDestroy(ev);
    if (m->stream) cudaStreamDestroy(m->stream);
    if (m->attn) tl_attn_destroy(m->attn);
    delete m;
}

int tl_model_set_tensor(tl_model *m, const char *name, int ggmlType, const void *data, long long ne0, long long ne1) {
    if (!m || !name || !data) return api_fail(TL_ERR_INVALID, "NULL argument");
    if (ne0 < 1 || ne1 < 1) return api_fail(TL_ERR_INVALID, "tensor dimensions must be positive");
    size_t bytes = 0;
    if (ggmlType == TL_GGML_F32) {
        bytes = (size_t)ne0 * ne1 * sizeof(float);
    } else if (ggmlType == TL_GGML_Q2_K) {
        if (ne0 % QK != 0) return api_fail(TL_ERR_INVALID, "q2_K row size must be multiple of 256");
        bytes = (size_t)(ne0 / QK) * Q2K_BYTES * ne1;
    } else {
        return api_fail(TL_ERR_UNSUPPORTED, "tl_model_set_tensor: type must be F32 or Q2_K");
    }
    DevGuard g(m->device);
    // the captured decode step holds the old tensors' addresses
    if (m->graphExec) { cudaGraphExecDestroy(m->graphExec); m->graphExec = nullptr; }
    if (m->graph) { cudaGraphDestroy(m->graph); m->graph = nullptr; }
    GTensor &t = m->w[name];
    if (t.dev) {
        cudaStreamSynchronize(m->stream);  // no queued work may still read it
        cudaFree(t.dev);
    }
    t = GTensor{};
    void *p = nullptr;
    TLM_CUDA(cudaMalloc(&p, bytes));
    cudaError_t e = cudaMemcpy(p, data, bytes, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        cudaFree(p);
        m->w.erase(name);
        return cuda_fail(e, "cudaMemcpy(tensor)");
    }
    t.type = ggmlType;
    t.ne0 = ne0;
    t.ne1 = ne1;
    t.dev = p;
    return TL_OK;
}

int tl_model_generate(tl_model *m, const int32_t *prompt, int nPrompt, int nNew, int32_t *outIds, float *gaps) {
    if (!m || !prompt || !outIds) return api_fail(TL_ERR_INVALID, "NULL argument");
    if (nPrompt < 1 || nNew < 1) return api_fail(TL_ERR_INVALID, "nPrompt and nNew must be positive");
    if ((long long)nPrompt + nNew - 1 > m->c.maxLen) return api_fail(TL_ERR_KV_FULL, "KV cache full");
    for (int i = 0; i < nPrompt; ++i)
        if (prompt[i] < 0 || prompt[i] >= m->c.nVocab) return api_fail(TL_ERR_INVALID, "token id out of range");
    DevGuard g(m->device);
    std::vector<LayerW> L;
    const GTensor *emb = nullptr, *onorm = nullptr, *out = nullptr;
    TLM_TRY(resolve(m, L, &emb, &onorm, &out));
    TLM_TRY(ensure_buffers(m, nPrompt, nNew));
    if (!m->logits) TLM_CUDA(cudaMalloc(&m->logits, sizeof(float) * m->c.nVocab));
    const int st[4] = {0, nPrompt, 0, 0};  // after the prefill: the first generated token sits at nPrompt
    TLM_CUDA(cudaMemcpyAsync(m->tokens, prompt, sizeof(int32_t) * nPrompt, cudaMemcpyHostToDevice, m->stream));
    TLM_CUDA(cudaMemcpyAsync(m->state, st, sizeof st, cudaMemcpyHostToDevice, m->stream));
    TLM_CUDA(cudaEventRecord(m->ev[0], m->stream));
    TLM_TRY(forward(m, L, emb, onorm, out, nPrompt, m->tokens, false));
    TLM_CUDA(cudaEventRecord(m->ev[1], m->stream));
    int done = 1;
    if (nNew > 1 && !m->graphExec) {
        // one step eagerly (it sizes the attention scratch), then capture a step
        TLM_TRY(forward(m, L, emb, onorm, out, 1, nullptr, true));
        ++done;
        if (done < nNew) {
            TLM_CUDA(cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal));
            const int rc = forward(m, L, emb, onorm, out, 1, nullptr, true);
            cudaGraph_t graph = nullptr;
            const cudaError_t ec = cudaStreamEndCapture(m->stream, &graph);
            if (rc != TL_OK) {
                if (graph) cudaGraphDestroy(graph);
                return rc;
            }
            TLM_CUDA(ec);
            m->graph = graph;
            TLM_CUDA(cudaGraphInstantiate(&m->graphExec, graph, 0));
        }
    }
    for (; done < nNew; ++done) TLM_CUDA(cudaGraphLaunch(m->graphExec, m->stream));
    TLM_CUDA(cudaEventRecord(m->ev[2], m->stream));
    TLM_CUDA(cudaMemcpyAsync(outIds, m->ids, sizeof(int32_t) * nNew, cudaMemcpyDeviceToHost, m->stream));
    if (gaps) TLM_CUDA(cudaMemcpyAsync(gaps, m->gaps, sizeof(float) * nNew, cudaMemcpyDeviceToHost, m->stream));
    unsigned word = 0;
    TLM_CUDA(cudaMemcpyAsync(&word, m->err, sizeof word, cudaMemcpyDeviceToHost, m->stream));
    TLM_CUDA(cudaStreamSynchronize(m->stream));
    cudaEventElapsedTime(&m->prefillMs, m->ev[0], m->ev[1]);
    cudaEventElapsedTime(&m->decodeMs, m->ev[1], m->ev[2]);
    if (word) {
        cudaMemsetAsync(m->err, 0, sizeof(unsigned), m->stream);
        cudaStreamSynchronize(m->stream);
        return api_fail(TL_ERR_DEVICE, (word & kErrToken) ? "tl_model: a token id outside the vocabulary reached the device"
                                                          : "tl_model: a position outside the KV cache reached the device");
    }
    return tl_check_device(m->attn, m->stream);
}

int tl_model_last_logits(tl_model *m, float *logits) {
    if (!m || !logits) return api_fail(TL_ERR_INVALID, "NULL argument");
    if (!m->logits) return api_fail(TL_ERR_INVALID, "no forward pass has run");
    DevGuard g(m->device);
    TLM_CUDA(cudaMemcpyAsync(logits, m->logits, sizeof(float) * m->c.nVocab, cudaMemcpyDeviceToHost, m->stream));
    TLM_CUDA(cudaStreamSynchronize(m->stream));
    return TL_OK;
}

int tl_model_last_timing(tl_model *m, float *prefill_ms, float *decode_ms) {
    if (!m) return api_fail(TL_ERR_INVALID, "NULL argument");
    if (prefill_ms) *prefill_ms = m->prefillMs;
    if (decode_ms) *decode_ms = m->decodeMs;
    return TL_OK;
}

}  // extern "C"
