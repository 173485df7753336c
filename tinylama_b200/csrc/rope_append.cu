// rope_append.cu -- RoPE on q/k and append of (k, v) into the head-major KV cache.
//
// Replaces applyRopeSingle (src/forward.nim:108-123), applyRopeAtPos (:125-139) and
// storeKVRange (:232-241).  A thread rotates pair (2i, 2i+1) of up to 8 heads of one token
// with one cos/sin evaluation, and appends the rotated k pairs; v pairs are appended by a
// second set of threads.  The rotation reproduces the reference's float32 arithmetic operation by
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
    y0 = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
    y1 = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
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
                const float angle = __fmul_rn((float)pos, tab.theta[i]);
                double sd, cd;
                sincos((double)angle, &sd, &cd);
                c = (float)cd;
                sn = (float)sd;
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

}  // namespace

cudaError_t launch_rope_append(const RopeAppendArgs &a, const RopeTab &tab, cudaStream_t s) {
    const int half = a.headDim / 2;
    const int hq = a.rope_q ? a.nHead : 0;
    const int hk = (a.rope_k || a.store) ? a.nHeadKv : 0;
    const int ngroups = (hq + hk + kHeadsPerThread - 1) / kHeadsPerThread;
    const int64_t total = (int64_t)a.nseq * a.ntok * half *
                          (ngroups + (a.store ? a.nHeadKv : 0));
    if (total == 0) return cudaSuccess;
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
