// rope_append.cu -- RoPE on q/k and append of (k, v) into the head-major KV cache.
//
// Replaces applyRopeSingle (src/forward.nim:108-123), applyRopeAtPos (:125-139) and
// storeKVRange (:232-241).  One thread per rotation pair (2i, 2i+1) of q and k and per pair
// of v elements.  The rotation reproduces the reference's float32 arithmetic operation by
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

__device__ __forceinline__ void rotate(float x0, float x1, float theta, int pos, float &y0,
                                       float &y1) {
    const float angle = __fmul_rn((float)pos, theta);
    double sd, cd;
    sincos((double)angle, &sd, &cd);
    const float c = (float)cd, s = (float)sd;
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

template <typename KV>
__global__ void rope_append_kernel(const RopeAppendArgs a, const RopeTab tab) {
    const int half = a.headDim / 2;
    const int64_t nq = a.rope_q ? (int64_t)a.nseq * a.ntok * a.nHead * half : 0;
    const int64_t nk = (a.rope_k || a.store) ? (int64_t)a.nseq * a.ntok * a.nHeadKv * half : 0;
    const int64_t nv = a.store ? nk : 0;
    const int64_t total = nq + nk + nv;
    for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
         idx += (int64_t)gridDim.x * blockDim.x) {
        int64_t r = idx;
        int which;  // 0 q, 1 k, 2 v
        if (r < nq) which = 0;
        else if ((r -= nq) < nk) which = 1;
        else { r -= nk; which = 2; }
        const int nh = which == 0 ? a.nHead : a.nHeadKv;
        const int i = (int)(r % half);
        int64_t rest = r / half;
        const int h = (int)(rest % nh);
        rest /= nh;
        const int t = (int)(rest % a.ntok);
        const int b = (int)(rest / a.ntok);
        const int pos = (a.pos0 ? a.pos0[b] : a.pos0_scalar) + t;
        if (which == 0) {
            const HeadView &v = a.q;
            const int64_t i0 = v.at(b, t, h, 2 * i), i1 = v.at(b, t, h, 2 * i + 1);
            float y0 = v.ptr[i0], y1 = v.ptr[i1];
            if (i < tab.pairs) rotate(y0, y1, tab.theta[i], pos, y0, y1);
            v.ptr[i0] = y0;
            v.ptr[i1] = y1;
            if (a.qb) {
                __nv_bfloat16 *qb = reinterpret_cast<__nv_bfloat16 *>(a.qb);
                const int64_t o = (((int64_t)b * a.nHead + h) * a.ntok + t) * a.headDim + 2 * i;
                *reinterpret_cast<__nv_bfloat162 *>(qb + o) = __floats2bfloat162_rn(y0, y1);
            }
        } else {
            const HeadView &v = which == 1 ? a.k : a.v;
            const int64_t i0 = v.at(b, t, h, 2 * i), i1 = v.at(b, t, h, 2 * i + 1);
            float y0 = v.ptr[i0], y1 = v.ptr[i1];
            if (which == 1 && a.rope_k && i < tab.pairs) {
                rotate(y0, y1, tab.theta[i], pos, y0, y1);
                v.ptr[i0] = y0;
                v.ptr[i1] = y1;
            }
            if (a.store) {
                if (pos < 0 || pos >= a.kv.maxLen) {
                    atomicOr(a.err, TL_DEVERR_POS_RANGE);
                    continue;
                }
                const int64_t dst = a.kv.row(a.layer, a.slot0 + b, h, pos) * a.headDim + 2 * i;
                store_pair<KV>(which == 1 ? a.kv.k : a.kv.v, dst, y0, y1);
            }
        }
    }
}

}  // namespace

cudaError_t launch_rope_append(const RopeAppendArgs &a, const RopeTab &tab, cudaStream_t s) {
    const int half = a.headDim / 2;
    const int64_t total = (a.rope_q ? (int64_t)a.nseq * a.ntok * a.nHead * half : 0) +
                          ((a.rope_k || a.store) ? (int64_t)a.nseq * a.ntok * a.nHeadKv * half : 0) *
                              (a.store ? 2 : 1);
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
