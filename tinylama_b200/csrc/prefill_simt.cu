// prefill_simt.cu -- causal GQA prefill attention in fp32 on the CUDA cores.
//
// Replaces the context part of attentionFull (src/forward.nim:141-176): for q-head h and
// query i, s_j = q_{h,i} . k_{kvh,j} / sqrt(d) for j <= i, softmax, ctx = sum_j p_j v_{kvh,j}.
// This is the fp32 path (fp32 cache, or the reference's fresh fp32 projections) used where the
// 1e-3 bound applies; the bf16 tensor-core path lives in prefill_tc.cu.
//
// One CTA (4 warps) owns one (sequence, kv-head, tile of QT query tokens) and all G q-heads of
// the group: R = G*QT = 32 query rows, 8 per warp, so each K/V tile staged in shared memory is
// reused by 32 rows.  Lane j scores key j of the 32-key tile; the online softmax runs per row
// with warp reductions; lanes then own head_dim columns of the output.
#include <math.h>

#include "common.cuh"
#include "internal.h"

namespace tl {
namespace {

constexpr float kLog2e = 1.4426950408889634f;
constexpr int kRows = 32, kRpw = 8, kKeys = 32;

template <typename KV, int D, int G>
__global__ void __launch_bounds__(128) prefill_f32_kernel(const PrefillArgs a) {
    constexpr int QT = kRows / G;
    constexpr int DPL = D / 32;
    extern __shared__ float psm[];
    float(*Qs)[D] = reinterpret_cast<float(*)[D]>(psm);
    float(*Ks)[D + 1] = reinterpret_cast<float(*)[D + 1]>(psm + kRows * D);
    float(*Vs)[D + 1] = reinterpret_cast<float(*)[D + 1]>(psm + kRows * D + kKeys * (D + 1));

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int t0 = blockIdx.x * QT;
    const int g = blockIdx.y;
    const int b = blockIdx.z;
    const int pos0 = a.pos0 ? a.pos0[b] : 0;
    const int ntile = min(QT, a.ntok - t0);
    if (ntile <= 0) return;
    const float qscale = kLog2e / sqrtf((float)D);

    for (int e = tid; e < kRows * D; e += 128) {
        const int r = e / D, d = e - r * D;
        const int hh = r / QT, tt = r - hh * QT;
        float x = 0.f;
        if (tt < ntile) x = a.q.ptr[a.q.at(b, t0 + tt, g * G + hh, d)] * qscale;
        Qs[r][d] = x;
    }
    int qpos[kRpw];
    bool rvalid[kRpw];
#pragma unroll
    for (int rr = 0; rr < kRpw; ++rr) {
        const int r = warp * kRpw + rr;
        const int tt = r % QT;
        rvalid[rr] = tt < ntile;
        qpos[rr] = pos0 + t0 + tt;
    }
    float m[kRpw], l[kRpw], o[kRpw][DPL];
#pragma unroll
    for (int rr = 0; rr < kRpw; ++rr) {
        m[rr] = -INFINITY;
        l[rr] = 0.f;
#pragma unroll
        for (int k = 0; k < DPL; ++k) o[rr][k] = 0.f;
    }
    const int kmax = pos0 + t0 + ntile;  // keys [0, kmax)
    const bool fresh = a.kf.ptr != nullptr;
    const KV *kc = reinterpret_cast<const KV *>(a.kv.k);
    const KV *vc = reinterpret_cast<const KV *>(a.kv.v);
    for (int k0 = 0; k0 < kmax; k0 += kKeys) {
        __syncthreads();
        for (int e = tid; e < kKeys * D; e += 128) {
            const int j = e / D, d = e - j * D;
            const int kp = k0 + j;
            float kx = 0.f, vx = 0.f;
            if (kp < kmax) {
                if (fresh) {
                    kx = a.kf.ptr[a.kf.at(b, kp, g, d)];
                    vx = a.vf.ptr[a.vf.at(b, kp, g, d)];
                } else {
                    const int64_t o2 = a.kv.row(a.layer, a.slot0 + b, g, kp) * D + d;
                    kx = KvT<KV>::to_f(kc[o2]);
                    vx = KvT<KV>::to_f(vc[o2]);
                }
            }
            Ks[j][d] = kx;
            Vs[j][d] = vx;
        }
        __syncthreads();
        float acc[kRpw];
#pragma unroll
        for (int rr = 0; rr < kRpw; ++rr) acc[rr] = 0.f;
#pragma unroll 8
        for (int d = 0; d < D; ++d) {
            const float kd = Ks[lane][d];
#pragma unroll
            for (int rr = 0; rr < kRpw; ++rr) acc[rr] = fmaf(Qs[warp * kRpw + rr][d], kd, acc[rr]);
        }
        const int kp = k0 + lane;
#pragma unroll
        for (int rr = 0; rr < kRpw; ++rr) {
            const float s = (rvalid[rr] && kp <= qpos[rr]) ? acc[rr] : -INFINITY;
            float tmax = s;
#pragma unroll
            for (int off = 16; off >= 1; off >>= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, off));
            const float mnew = fmaxf(m[rr], tmax);
            const float alpha = (m[rr] == -INFINITY) ? 0.f : exp2f(m[rr] - mnew);
            const float p = (s == -INFINITY) ? 0.f : exp2f(s - mnew);
            float psum = p;
#pragma unroll
            for (int off = 16; off >= 1; off >>= 1) psum += __shfl_xor_sync(0xffffffffu, psum, off);
            l[rr] = l[rr] * alpha + psum;
            m[rr] = mnew;
#pragma unroll
            for (int k = 0; k < DPL; ++k) o[rr][k] *= alpha;
            acc[rr] = p;
        }
#pragma unroll 4
        for (int j = 0; j < kKeys; ++j) {
            float vv[DPL];
#pragma unroll
            for (int k = 0; k < DPL; ++k) vv[k] = Vs[j][lane + 32 * k];
#pragma unroll
            for (int rr = 0; rr < kRpw; ++rr) {
                const float p = __shfl_sync(0xffffffffu, acc[rr], j);
#pragma unroll
                for (int k = 0; k < DPL; ++k) o[rr][k] = fmaf(p, vv[k], o[rr][k]);
            }
        }
    }
#pragma unroll
    for (int rr = 0; rr < kRpw; ++rr) {
        if (!rvalid[rr]) continue;
        const int r = warp * kRpw + rr;
        const int hh = r / QT, tt = r % QT;
        const float inv = l[rr] > 0.f ? 1.f / l[rr] : 0.f;
#pragma unroll
        for (int k = 0; k < DPL; ++k)
            a.out.ptr[a.out.at(b, t0 + tt, g * G + hh, lane + 32 * k)] = o[rr][k] * inv;
    }
}

template <typename KV, int D, int G>
cudaError_t launch_t(const PrefillArgs &a, cudaStream_t s) {
    constexpr int QT = kRows / G;
    dim3 grid((a.ntok + QT - 1) / QT, a.nHeadKv, a.nseq);
    const int smem = (kRows * D + 2 * kKeys * (D + 1)) * (int)sizeof(float);
    cudaError_t e = cudaFuncSetAttribute(prefill_f32_kernel<KV, D, G>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    prefill_f32_kernel<KV, D, G><<<grid, 128, smem, s>>>(a);
    return cudaGetLastError();
}

template <typename KV, int D>
cudaError_t launch_g(const PrefillArgs &a, cudaStream_t s) {
    switch (a.nHead / a.nHeadKv) {
        case 1: return launch_t<KV, D, 1>(a, s);
        case 2: return launch_t<KV, D, 2>(a, s);
        case 4: return launch_t<KV, D, 4>(a, s);
        case 8: return launch_t<KV, D, 8>(a, s);
        default: return cudaErrorNotSupported;
    }
}

}  // namespace

cudaError_t launch_prefill_f32(const PrefillArgs &a, cudaStream_t s) {
    if (a.ntok <= 0 || a.nseq <= 0) return cudaSuccess;
    const bool bf = (a.kf.ptr == nullptr) && a.kv.dtype == TL_KV_BF16;
    if (a.headDim == 64) return bf ? launch_g<__nv_bfloat16, 64>(a, s) : launch_g<float, 64>(a, s);
    if (a.headDim == 128) return bf ? launch_g<__nv_bfloat16, 128>(a, s) : launch_g<float, 128>(a, s);
    return cudaErrorNotSupported;
}

}  // namespace tl
