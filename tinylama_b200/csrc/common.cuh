// common.cuh -- shared device helpers for the tinylama B200 attention library (sm_100a).
//
// Every spin-wait in this library is bounded: it gives up after TL_WAIT_NS nanoseconds of
// %globaltimer, records TL_DEVERR_TIMEOUT in the handle's device error word and lets the
// kernel return.  No kernel here traps.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#define TL_DEVERR_POS_RANGE 1u    // a position/length was outside [0, maxLen)
#define TL_DEVERR_TIMEOUT 2u      // an mbarrier wait ran out of time
#define TL_DEVERR_BAD_ARG 4u      // a kernel saw an argument the host should have rejected

#ifndef TL_WAIT_NS
#define TL_WAIT_NS 2000000000ull  // 2 s per wait
#endif

namespace tl {

// Programmatic dependent launch.  A kernel launched with programmatic stream serialisation may
// start while the previous kernel on its stream still runs; it must wait here before it reads
// anything that kernel writes.  A kernel that others depend on signals early that they may be
// scheduled.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- mbarrier ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
                 : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile(
        "{\n\t.reg .b64 st;\n\t"
        "mbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile(
        "{\n\t.reg .b64 st;\n\t"
        "mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(smem_u32(bar)),
        "r"(bytes)
        : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Non-blocking probe: has the phase with the given parity completed?
__device__ __forceinline__ bool mbar_test(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait for the phase with the given parity to complete.  Returns false (and sets
// TL_DEVERR_TIMEOUT in *err) if it did not complete within TL_WAIT_NS, or if *abort_flag
// (shared) becomes non-zero while waiting.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, unsigned *err,
                                          volatile int *abort_flag) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
        if (abort_flag && *abort_flag) return false;
        if (globaltimer_ns() - t0 > TL_WAIT_NS) {
            if (err) atomicOr(err, TL_DEVERR_TIMEOUT);
            if (abort_flag) *abort_flag = 1;
            return false;
        }
    }
}

// ---- bulk (non-tensor) async copy global -> shared, completion on an mbarrier ------------
// Both addresses must be 16-byte aligned and bytes a multiple of 16.  No multicast.
__device__ __forceinline__ void bulk_g2s(void *smem_dst, const void *gmem_src, uint32_t bytes,
                                         uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
            "r"(smem_u32(smem_dst)),
        "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// Same, with an L2 eviction hint: KV streamed once per step should not evict other data.
__device__ __forceinline__ void bulk_g2s_evict_first(void *smem_dst, const void *gmem_src,
                                                     uint32_t bytes, uint64_t *bar,
                                                     uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], "
        "[%1], %2, [%3], %4;" ::"r"(smem_u32(smem_dst)),
        "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// Named barrier over `count` threads (a multiple of 32), id 1..15.
__device__ __forceinline__ void named_bar(int id, int count) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// Named barrier that also ORs a predicate over the participating threads.
__device__ __forceinline__ bool named_bar_or(int id, int count, bool pred) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 q, %1, 0;\n\t"
        "bar.red.or.pred p, %2, %3, q;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)pred), "r"(id), "r"(count)
        : "memory");
    return r != 0;
}

// ---- RoPE --------------------------------------------------------------------------------
// Pair rotation (x0, x1) -> (x0*c - x1*s, x0*s + x1*c) with explicit round-to-nearest
// multiplies and adds (no contraction into multiply-adds), as the reference evaluates it in
// float32 (src/forward.nim:119-123).
__device__ __forceinline__ void rope_rotate(float x0, float x1, float c, float s, float &y0, float &y1) {
    y0 = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
    y1 = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
}

// cos/sin of the float32 angle float32(pos) * theta: evaluated in double and rounded to float32
// (the correctly rounded values a libm's cosf/sinf return).
__device__ __forceinline__ float2 rope_cos_sin(int pos, float theta) {
    const float angle = __fmul_rn((float)pos, theta);
    double sd, cd;
    sincos((double)angle, &sd, &cd);
    return make_float2((float)cd, (float)sd);
}

// ---- element conversion ------------------------------------------------------------------
template <typename T> struct KvT;
template <> struct KvT<float> {
    static constexpr int kBytes = 4;
    __device__ __forceinline__ static float to_f(float x) { return x; }
    __device__ __forceinline__ static float from_f(float x) { return x; }
};
template <> struct KvT<__nv_bfloat16> {
    static constexpr int kBytes = 2;
    __device__ __forceinline__ static float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
    __device__ __forceinline__ static __nv_bfloat16 from_f(float x) { return __float2bfloat16_rn(x); }
};

// Load VPL consecutive KV elements from shared memory as floats.
template <typename T, int VPL> struct VecLoad;
template <> struct VecLoad<float, 4> {
    __device__ __forceinline__ static void run(const float *p, float *o) {
        const float4 v = *reinterpret_cast<const float4 *>(p);
        o[0] = v.x; o[1] = v.y; o[2] = v.z; o[3] = v.w;
    }
};
template <> struct VecLoad<float, 2> {
    __device__ __forceinline__ static void run(const float *p, float *o) {
        const float2 v = *reinterpret_cast<const float2 *>(p);
        o[0] = v.x; o[1] = v.y;
    }
};
template <> struct VecLoad<__nv_bfloat16, 4> {
    __device__ __forceinline__ static void run(const __nv_bfloat16 *p, float *o) {
        const uint2 v = *reinterpret_cast<const uint2 *>(p);
        o[0] = __uint_as_float(v.x << 16); o[1] = __uint_as_float(v.x & 0xffff0000u);
        o[2] = __uint_as_float(v.y << 16); o[3] = __uint_as_float(v.y & 0xffff0000u);
    }
};
template <> struct VecLoad<__nv_bfloat16, 2> {
    __device__ __forceinline__ static void run(const __nv_bfloat16 *p, float *o) {
        const uint32_t v = *reinterpret_cast<const uint32_t *>(p);
        o[0] = __uint_as_float(v << 16); o[1] = __uint_as_float(v & 0xffff0000u);
    }
};

}  // namespace tl
