// rope_append.cu -- RoPE on q/k and append of (k, v) into the head-major KV cache.
//
// Replaces applyRopeSingle (src/forward.nim:108-123), applyRopeAtPos (:125-139) and
// storeKVRange (:232-241).  Three kernels share one per-element arithmetic:
//   * rope_append_pos_kernel: token-major rows with positions pos0 + t shared by all sequences
//     (prefill, storeKVRange): a block takes one position for up to 8 sequences;
//   * rope_append_tok_kernel: token-major rows with a position per sequence (decode);
//   * rope_append_kernel: any strides: a thread rotates pair (2i, 2i+1) of up to 8 heads of one
//     token with one cos/sin evaluation and appends the rotated k pairs; v pairs are appended by
//     a second set of threads.  The rotation reproduces the reference's float32 arithmetic operation by
// operation: theta_i comes from the host (glibc powf, see make_rope_tab), the angle is the
// float32 product float32(pos) * theta_i, cos/sin are evaluated in double and rounded to
// float32 (the correctly rounded value glibc's cosf/sinf return), and
//   x0' = x0*c - x1*s,  x1' = x0*s + x1*c
// is evaluated with explicit round-to-nearest multiplies and adds, so no multiply-add is
// contracted.  Rotated values therefore match the reference bit for bit whenever the two
// libm results agree.
#include <math.h>

#include "common.cuh"
#include "internal.h"

namespace tl {

RopeTab make_rope_tab(int ropeDim, float base) {
    RopeTab t{};
    t.pairs = ropeDim / 2;
    if (t.pairs > kMaxRopePairs) t.pairs = kMaxRopePairs;
    for (int i = 0; i < t.pairs; ++i) {
        // src/forward.nim:116: pow(1.0'f32 / base, float32(2*i) / float32(ropeDim))
        volatile float inv = 1.0f / base;
        volatile float ex = (float)(2 * i) / (float)ropeDim;
        t.theta[i] = powf(inv, ex);
    }
    return t;
}

namespace {

__device__ __forceinline__ void rotate_cs(float x0, float x1, float c, float s, float &y0,
                                          float &y1) {
    rope_rotate(x0, x1, c, s, y0, y1);
}

template <typename KV>
__device__ __forceinline__ void store_pair(void *base, int64_t idx, float a, float b) {
    if constexpr (sizeof(KV) == 4) {
        *reinterpret_cast<float2 *>(reinterpret_cast<float *>(base) + idx) = make_float2(a, b);
    } else {
        *reinterpret_cast<__nv_bfloat162 *>(reinterpret_cast<__nv_bfloat16 *>(base) + idx) =
            __floats2bfloat162_rn(a, b);
    }
}

constexpr int kHeadsPerThread = 8;

// Thread layout: segment A has one thread per (sequence, token, head group of 8, pair i),
// with i fastest so that a warp touches consecutive pairs of one head; the thread computes
// cos/sin of (pos, i) once and applies them to the q heads and then the k heads of its group
// (the angle depends only on the position and the pair).  Segment B appends v.
template <typename KV>
__global__ void rope_append_kernel(const RopeAppendArgs a, const RopeTab tab) {
    pdl_launch_dependents();  // a decode kernel launched behind this one may be scheduled
    const int half = a.headDim / 2;
    const int hq = a.rope_q ? a.nHead : 0;
    const int hk = (a.rope_k || a.store) ? a.nHeadKv : 0;
    const int ngroups = (hq + hk + kHeadsPerThread - 1) / kHeadsPerThread;
    const int64_t na = (int64_t)a.nseq * a.ntok * ngroups * half;
    const int64_t nv = a.store ? (int64_t)a.nseq * a.ntok * a.nHeadKv * half : 0;
    const int64_t total = na + nv;
    for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
         idx += (int64_t)gridDim.x * blockDim.x) {
        if (idx < na) {
            const int i = (int)(idx % half);
            int64_t rest = idx / half;
            const int hg = (int)(rest % ngroups);
            rest /= ngroups;
            const int t = (int)(rest % a.ntok);
            const int b = (int)(rest / a.ntok);
            const int pos = (a.pos0 ? a.pos0[b] : a.pos0_scalar) + t;
            const bool rot = i < tab.pairs;
            float c = 1.f, sn = 0.f;
            if (rot) {
                const float2 cs = rope_cos_sin(pos, tab.theta[i]);
                c = cs.x;
                sn = cs.y;
            }
            const bool in_range = pos >= 0 && pos < a.kv.maxLen;
            const int h_end = min(hq + hk, (hg + 1) * kHeadsPerThread);
            for (int hh = hg * kHeadsPerThread; hh < h_end; ++hh) {
                if (hh < hq) {
                    const HeadView &v = a.q;
                    const int64_t i0 = v.at(b, t, hh, 2 * i), i1 = v.at(b, t, hh, 2 * i + 1);
                    float y0 = v.ptr[i0], y1 = v.ptr[i1];
                    if (rot) rotate_cs(y0, y1, c, sn, y0, y1);
                    if (a.q_inplace) {
                        v.ptr[i0] = y0;
                        v.ptr[i1] = y1;
                    }
                    if (a.qb) {
                        __nv_bfloat16 *qb = reinterpret_cast<__nv_bfloat16 *>(a.qb);
                        const int64_t o = (((int64_t)b * a.nHead + hh) * a.ntok + t) * a.headDim + 2 * i;
                        *reinterpret_cast<__nv_bfloat162 *>(qb + o) = __floats2bfloat162_rn(y0, y1);
                    }
                } else {
                    const int h = hh - hq;
                    const HeadView &v = a.k;
                    const int64_t i0 = v.at(b, t, h, 2 * i), i1 = v.at(b, t, h, 2 * i + 1);
                    float y0 = v.ptr[i0], y1 = v.ptr[i1];
                    if (a.rope_k && rot) {
                        rotate_cs(y0, y1, c, sn, y0, y1);
                        if (a.k_inplace) {
                            v.ptr[i0] = y0;
                            v.ptr[i1] = y1;
                        }
                    }
                    if (a.store) {
                        if (!in_range) {
                            atomicOr(a.err, TL_DEVERR_POS_RANGE);
                            continue;
                        }
                        const int64_t dst = a.kv.row(a.layer, a.slot0 + b, h, pos) * a.headDim + 2 * i;
                        store_pair<KV>(a.kv.k, dst, y0, y1);
                    }
                }
            }
        } else {
            const int64_t r = idx - na;
            const int i = (int)(r % half);
            int64_t rest = r / half;
            const int h = (int)(rest % a.nHeadKv);
            rest /= a.nHeadKv;
            const int t = (int)(rest % a.ntok);
            const int b = (int)(rest / a.ntok);
            const int pos = (a.pos0 ? a.pos0[b] : a.pos0_scalar) + t;
            if (pos < 0 || pos >= a.kv.maxLen) {
                atomicOr(a.err, TL_DEVERR_POS_RANGE);
                continue;
            }
            const HeadView &v = a.v;
            const float y0 = v.ptr[v.at(b, t, h, 2 * i)], y1 = v.ptr[v.at(b, t, h, 2 * i + 1)];
            const int64_t dst = a.kv.row(a.layer, a.slot0 + b, h, pos) * a.headDim + 2 * i;
            store_pair<KV>(a.kv.v, dst, y0, y1);
        }
    }
}

// Token-major fast path: q, k and v are [nseq][ntok][heads*headDim] rows (the layout of a
// prefill's projections), so one block walks tokens and a thread moves four consecutive floats
// (two pairs) of one head with a 16-byte load.  The cos/sin pairs of a token are evaluated once,
// by the first half-headDim threads, into shared memory: for 32 q and 8 kv heads that is 40x
// fewer double-precision sincos than one per (head group, pair), and no 64-bit index division
// is left in the inner loop.  The arithmetic per element is the one above, so the results are
// bit-identical to the generic kernel.
template <typename KV, int D4T>
__global__ void __launch_bounds__(256) rope_append_tok_kernel(const RopeAppendArgs a, const RopeTab tab) {
    pdl_launch_dependents();  // a decode kernel launched behind this one may be scheduled
    __shared__ float2 cs[kMaxRopePairs];
    const int D = a.headDim;
    const int D4 = D4T > 0 ? D4T : D / 4;
    const int half = D / 2;
    const int hq = a.rope_q ? a.nHead : 0;
    const int hk = (a.rope_k || a.store) ? a.nHeadKv : 0;
    const int hv = a.store ? a.nHeadKv : 0;
    const int nq4 = hq * D4, nk4 = hk * D4;
    const int per_tok = nq4 + nk4 + hv * D4;
    const int64_t ntokens = (int64_t)a.nseq * a.ntok;
    for (int64_t tok = blockIdx.x; tok < ntokens; tok += gridDim.x) {
        const int b = (int)(tok / a.ntok);
        const int t = (int)(tok - (int64_t)b * a.ntok);
        const int pos = (a.pos0 ? a.pos0[b] : a.pos0_scalar) + t;
        __syncthreads();  // the previous token's cos/sin are no longer read
        for (int i = threadIdx.x; i < half; i += blockDim.x) {
            cs[i] = i < tab.pairs ? rope_cos_sin(pos, tab.theta[i]) : make_float2(1.f, 0.f);
        }
        __syncthreads();
        const bool in_range = pos >= 0 && pos < a.kv.maxLen;
        if (a.store && !in_range && threadIdx.x == 0) atomicOr(a.err, TL_DEVERR_POS_RANGE);
        for (int e = threadIdx.x; e < per_tok; e += blockDim.x) {
            int seg = e < nq4 ? 0 : (e < nq4 + nk4 ? 1 : 2);
            const int r = e - (seg == 0 ? 0 : (seg == 1 ? nq4 : nq4 + nk4));
            const int hh = r / D4;
            const int d = (r - hh * D4) * 4;
            const int p0 = d >> 1;
            if (seg == 0) {
                float *src = a.q.ptr + tok * ((int64_t)a.nHead * D) + hh * D + d;
                float4 x = *reinterpret_cast<const float4 *>(src);
                if (p0 < tab.pairs) rotate_cs(x.x, x.y, cs[p0].x, cs[p0].y, x.x, x.y);
                if (p0 + 1 < tab.pairs) rotate_cs(x.z, x.w, cs[p0 + 1].x, cs[p0 + 1].y, x.z, x.w);
                if (a.q_inplace) *reinterpret_cast<float4 *>(src) = x;
                if (a.qb) {
                    __nv_bfloat16 *qb = reinterpret_cast<__nv_bfloat16 *>(a.qb) +
                                        (((int64_t)b * a.nHead + hh) * a.ntok + t) * D + d;
                    __nv_bfloat162 lo = __floats2bfloat162_rn(x.x, x.y), hi = __floats2bfloat162_rn(x.z, x.w);
                    uint2 w;
                    w.x = *reinterpret_cast<uint32_t *>(&lo);
                    w.y = *reinterpret_cast<uint32_t *>(&hi);
                    *reinterpret_cast<uint2 *>(qb) = w;
                }
            } else {
                const bool is_k = seg == 1;
                float *src = (is_k ? a.k.ptr : a.v.ptr) + tok * ((int64_t)a.nHeadKv * D) + hh * D + d;
                float4 x = *reinterpret_cast<const float4 *>(src);
                if (is_k && a.rope_k) {
                    if (p0 < tab.pairs) rotate_cs(x.x, x.y, cs[p0].x, cs[p0].y, x.x, x.y);
                    if (p0 + 1 < tab.pairs) rotate_cs(x.z, x.w, cs[p0 + 1].x, cs[p0 + 1].y, x.z, x.w);
                    if (a.k_inplace) *reinterpret_cast<float4 *>(src) = x;
                }
                if (a.store && in_range) {
                    const int64_t dst = a.kv.row(a.layer, a.slot0 + b, hh, pos) * D + d;
                    void *base = is_k ? a.kv.k : a.kv.v;
                    store_pair<KV>(base, dst, x.x, x.y);
                    store_pair<KV>(base, dst + 2, x.z, x.w);
                }
            }
        }
    }
}

// Same rows, positions shared by all sequences (pos = pos0_scalar + t, the prefill case): a
// block takes one position t for up to 8 sequences, so the cos/sin of t are evaluated once for
// all of them, and a thread keeps the loads of four sequences in flight before it rotates and
// stores.
template <typename KV, int D4T>
__global__ void __launch_bounds__(256) rope_append_pos_kernel(const RopeAppendArgs a, const RopeTab tab) {
    pdl_launch_dependents();  // a decode kernel launched behind this one may be scheduled
    __shared__ float2 cs[kMaxRopePairs];
    const int D = a.headDim;
    const int D4 = D4T > 0 ? D4T : D / 4;
    const int half = D / 2;
    const int hq = a.rope_q ? a.nHead : 0;
    const int hk = (a.rope_k || a.store) ? a.nHeadKv : 0;
    const int hv = a.store ? a.nHeadKv : 0;
    const int nq4 = hq * D4, nk4 = hk * D4;
    const int per_tok = nq4 + nk4 + hv * D4;
    const int b0 = blockIdx.y * 8;
    const int nb = min(8, a.nseq - b0);
    for (int t = blockIdx.x; t < a.ntok; t += gridDim.x) {
        const int pos = a.pos0_scalar + t;
        __syncthreads();  // the previous position's cos/sin are no longer read
        for (int i = threadIdx.x; i < half; i += blockDim.x) {
            cs[i] = i < tab.pairs ? rope_cos_sin(pos, tab.theta[i]) : make_float2(1.f, 0.f);
        }
        __syncthreads();
        const bool in_range = pos >= 0 && pos < a.kv.maxLen;
        if (a.store && !in_range && threadIdx.x == 0) atomicOr(a.err, TL_DEVERR_POS_RANGE);
        for (int e = threadIdx.x; e < per_tok; e += blockDim.x) {
            const int seg = e < nq4 ? 0 : (e < nq4 + nk4 ? 1 : 2);
            const int r = e - (seg == 0 ? 0 : (seg == 1 ? nq4 : nq4 + nk4));
            const int hh = r / D4;
            const int d = (r - hh * D4) * 4;
            const int p0 = d >> 1;
            const bool rot0 = p0 < tab.pairs, rot1 = p0 + 1 < tab.pairs;
            const float2 cs0 = cs[p0], cs1 = cs[p0 + 1 < half ? p0 + 1 : p0];
            const int64_t row = (int64_t)(seg == 0 ? a.nHead : a.nHeadKv) * D;
            float *base = (seg == 0 ? a.q.ptr : (seg == 1 ? a.k.ptr : a.v.ptr)) + hh * D + d;
            for (int bb0 = 0; bb0 < nb; bb0 += 4) {
                float4 x[4];
#pragma unroll
                for (int u = 0; u < 4; ++u)
                    if (bb0 + u < nb)
                        x[u] = *reinterpret_cast<const float4 *>(base + ((int64_t)(b0 + bb0 + u) * a.ntok + t) * row);
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    if (bb0 + u >= nb) continue;
                    const int b = b0 + bb0 + u;
                    float *src = base + ((int64_t)b * a.ntok + t) * row;
                    if (seg == 0) {
                        if (rot0) rotate_cs(x[u].x, x[u].y, cs0.x, cs0.y, x[u].x, x[u].y);
                        if (rot1) rotate_cs(x[u].z, x[u].w, cs1.x, cs1.y, x[u].z, x[u].w);
                        if (a.q_inplace) *reinterpret_cast<float4 *>(src) = x[u];
                        if (a.qb) {
                            __nv_bfloat16 *qb = reinterpret_cast<__nv_bfloat16 *>(a.qb) +
                                                (((int64_t)b * a.nHead + hh) * a.ntok + t) * D + d;
                            __nv_bfloat162 lo = __floats2bfloat162_rn(x[u].x, x[u].y);
                            __nv_bfloat162 hi = __floats2bfloat162_rn(x[u].z, x[u].w);
                            uint2 w;
                            w.x = *reinterpret_cast<uint32_t *>(&lo);
                            w.y = *reinterpret_cast<uint32_t *>(&hi);
                            *reinterpret_cast<uint2 *>(qb) = w;
                        }
                    } else {
                        if (seg == 1 && a.rope_k) {
                            if (rot0) rotate_cs(x[u].x, x[u].y, cs0.x, cs0.y, x[u].x, x[u].y);
                            if (rot1) rotate_cs(x[u].z, x[u].w, cs1.x, cs1.y, x[u].z, x[u].w);
                            if (a.k_inplace) *reinterpret_cast<float4 *>(src) = x[u];
                        }
                        if (a.store && in_range) {
                            const int64_t dst = a.kv.row(a.layer, a.slot0 + b, hh, pos) * D + d;
                            void *cbase = seg == 1 ? a.kv.k : a.kv.v;
                            store_pair<KV>(cbase, dst, x[u].x, x[u].y);
                            store_pair<KV>(cbase, dst + 2, x[u].z, x[u].w);
                        }
                    }
                }
            }
        }
    }
}

bool token_major(const HeadView &v, int heads, int D, int ntok) {
    if (!v.ptr) return false;
    return v.sd == 1 && v.sh == D && v.st == (int64_t)heads * D && v.sb == (int64_t)ntok * heads * D &&
           (reinterpret_cast<uintptr_t>(v.ptr) & 15) == 0;
}

}  // namespace

cudaError_t launch_rope_append(const RopeAppendArgs &a, const RopeTab &tab, cudaStream_t s) {
    const int half = a.headDim / 2;
    const int hq = a.rope_q ? a.nHead : 0;
    const int hk = (a.rope_k || a.store) ? a.nHeadKv : 0;
    const int ngroups = (hq + hk + kHeadsPerThread - 1) / kHeadsPerThread;
    const int64_t total = (int64_t)a.nseq * a.ntok * half *
                          (ngroups + (a.store ? a.nHeadKv : 0));
    if (total == 0) return cudaSuccess;
    const bool fast = a.headDim % 4 == 0 && a.headDim / 2 <= kMaxRopePairs &&
                      (!a.rope_q || token_major(a.q, a.nHead, a.headDim, a.ntok)) &&
                      (!(a.rope_k || a.store) || token_major(a.k, a.nHeadKv, a.headDim, a.ntok)) &&
                      (!a.store || token_major(a.v, a.nHeadKv, a.headDim, a.ntok)) &&
                      (reinterpret_cast<uintptr_t>(a.kv.k) & 15) == 0 && (reinterpret_cast<uintptr_t>(a.kv.v) & 15) == 0 &&
                      (reinterpret_cast<uintptr_t>(a.qb) & 7) == 0;
    if (fast && a.pos0 == nullptr) {
        const int bx = a.ntok < 148 * 8 ? a.ntok : 148 * 8;
        const dim3 grid(bx, (a.nseq + 7) / 8);
        const bool bf = a.kv.dtype == TL_KV_BF16;
        if (a.headDim == 64)
            bf ? rope_append_pos_kernel<__nv_bfloat16, 16><<<grid, 256, 0, s>>>(a, tab)
               : rope_append_pos_kernel<float, 16><<<grid, 256, 0, s>>>(a, tab);
        else if (a.headDim == 128)
            bf ? rope_append_pos_kernel<__nv_bfloat16, 32><<<grid, 256, 0, s>>>(a, tab)
               : rope_append_pos_kernel<float, 32><<<grid, 256, 0, s>>>(a, tab);
        else
            bf ? rope_append_pos_kernel<__nv_bfloat16, 0><<<grid, 256, 0, s>>>(a, tab)
               : rope_append_pos_kernel<float, 0><<<grid, 256, 0, s>>>(a, tab);
        return cudaGetLastError();
    }
    if (fast) {
        const int64_t ntokens = (int64_t)a.nseq * a.ntok;
        const int blocks = (int)(ntokens < 148 * 8 ? ntokens : 148 * 8);
        const bool bf = a.kv.dtype == TL_KV_BF16;
        if (a.headDim == 64)
            bf ? rope_append_tok_kernel<__nv_bfloat16, 16><<<blocks, 256, 0, s>>>(a, tab)
               : rope_append_tok_kernel<float, 16><<<blocks, 256, 0, s>>>(a, tab);
        else if (a.headDim == 128)
            bf ? rope_append_tok_kernel<__nv_bfloat16, 32><<<blocks, 256, 0, s>>>(a, tab)
               : rope_append_tok_kernel<float, 32><<<blocks, 256, 0, s>>>(a, tab);
        else
            bf ? rope_append_tok_kernel<__nv_bfloat16, 0><<<blocks, 256, 0, s>>>(a, tab)
               : rope_append_tok_kernel<float, 0><<<blocks, 256, 0, s>>>(a, tab);
        return cudaGetLastError();
    }
    const int threads = 256;
    int64_t blocks = (total + threads - 1) / threads;
    if (blocks > 148 * 32) blocks = 148 * 32;
    if (a.kv.dtype == TL_KV_BF16)
        rope_append_kernel<__nv_bfloat16><<<(int)blocks, threads, 0, s>>>(a, tab);
    else
        rope_append_kernel<float><<<(int)blocks, threads, 0, s>>>(a, tab);
    return cudaGetLastError();
}

}  // namespace tl
