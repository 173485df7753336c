// decode_noalloc.cu -- decode attention that allocates nothing.
//
// Some callers cannot call cudaMalloc: a host whose allocator owns all device memory (a
// serving engine that carves one pre-reserved pool and forbids other allocations), or a
// real-time loop in which an allocation's latency and possible implicit synchronisation are
// not allowed.  For them
// tl_decode_attention_noalloc runs the same split-KV decode kernel as tl_decode_attention,
// but without a tl_attn handle: the caller passes q, the K/V cache and the output, and the
// kernel's scratch -- chunk partials, arrival counters and the device error word -- lives in
// the file-scope array below, which the CUDA module reserves on every GPU that loads this
// library, for the life of the process.
//
// Limits: the array holds kNoAllocBytes = 16 MiB.  At most kNoAllocCounters = 65536
// (sequence, kv-head) pairs per call; the chunk length is raised until the partials fit in
// what remains, and a call that cannot fit is refused with TL_ERR_INVALID.  The decode kernel
// keeps two ints per sequence in shared memory, so the number of sequences is also bounded by
// the device's shared memory per block (checked before the launch, TL_ERR_INVALID).
//
// With no handle there is no tl_check_device: when the kernel refuses a call on the device
// (positions on the device that disagree with pos_host, a position past maxLen, a timed-out
// wait), a second small kernel fills `out` with NaN, so that the caller can see it.
//
// The first call on a device looks the array's device address up with cudaGetSymbolAddress
// (with that device current); make that first call before any stream capture.  Every call
// shares the one array and clears the part it needs at its start (cudaMemsetAsync on the
// caller's stream): calls that may overlap on the GPU -- on different streams without
// ordering between them -- race on it and must not be issued.
#include <cuda_runtime.h>
#include <stdio.h>

#include <algorithm>
#include <mutex>
#include <string>

#include "common.cuh"
#include "internal.h"

namespace tl {
int api_fail(int code, const char *msg);
}  // namespace tl

using namespace tl;

namespace {

constexpr size_t kNoAllocBytes = 16u << 20;
constexpr int kNoAllocCounters = 1 << 16;
constexpr size_t kCounterBytes = sizeof(unsigned) * kNoAllocCounters;  // 256 KiB
constexpr size_t kErrBytes = 256;
constexpr size_t kPartialOffset = kCounterBytes + kErrBytes;
constexpr size_t kPartialFloats = (kNoAllocBytes - kPartialOffset) / sizeof(float);
constexpr int kMaxChunksPerSeq = 64;  // the decode kernels' limit (decode_common.cuh)
constexpr int kMaxDevices = 64;

// The scratch.  Host code must not take this name's address: on the host it is only a
// stand-in symbol, not device memory.  The device address comes from cudaGetSymbolAddress.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocBytes];

std::mutex g_mu;
void *g_scratch_dev[kMaxDevices] = {};

// After the decode kernel: if it recorded an error, every output element becomes NaN.
__global__ void poison_on_error_kernel(const unsigned *err, float *out, size_t n) {
    if (*reinterpret_cast<const volatile unsigned *>(err) == 0u) return;
    const float nan = __int_as_float(0x7fc00000);
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        out[i] = nan;
}

int scratch_for_current_device(void **out) {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
        return api_fail(TL_ERR_CUDA, "no current CUDA device");
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_scratch_dev[dev]) {
        void *p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || p == nullptr) {
            std::string m = std::string("cudaGetSymbolAddress(scratch) failed: ") + cudaGetErrorString(e);
            return api_fail(TL_ERR_CUDA, m.c_str());
        }
        g_scratch_dev[dev] = p;
    }
    *out = g_scratch_dev[dev];
    return TL_OK;
}

}  // namespace

extern "C" int tl_decode_attention_noalloc(const float *q, const void *k_cache, const void *v_cache,
                                           int kvDtype, int nHead, int nHeadKv, int headDim, int maxLen,
                                           int nseq, const int *pos_dev, const int *pos_host, float *out,
                                           void *stream) {
    if (!q || !k_cache || !v_cache || !pos_dev || !pos_host || !out)
        return api_fail(TL_ERR_INVALID, "NULL argument (pos_host is required by the no-alloc entry point)");
    if ((reinterpret_cast<uintptr_t>(q) & 15u) != 0) return api_fail(TL_ERR_INVALID, "q must be 16-byte aligned");
    if (kvDtype != TL_KV_F32 && kvDtype != TL_KV_BF16) return api_fail(TL_ERR_INVALID, "bad kvDtype");
    if (nHead <= 0 || nHeadKv <= 0 || nHead % nHeadKv != 0)
        return api_fail(TL_ERR_INVALID, "GQA requires head_count divisible by head_count_kv");
    const int G = nHead / nHeadKv;
    if ((headDim != 64 && headDim != 128) || !(G == 1 || G == 2 || G == 4 || G == 8))
        return api_fail(TL_ERR_UNSUPPORTED, "decode: shape not covered (headDim 64/128, group 1/2/4/8)");
    if (nseq < 1 || maxLen < 1) return api_fail(TL_ERR_INVALID, "nseq and maxLen must be positive");
    if ((long long)nseq * nHeadKv > kNoAllocCounters) {
        char m[160];
        snprintf(m, sizeof m, "nseq*nHeadKv = %lld exceeds the no-alloc scratch limit of %d",
                 (long long)nseq * nHeadKv, kNoAllocCounters);
        return api_fail(TL_ERR_INVALID, m);
    }
    long long tot = 0;
    int nmax = 0;
    for (int b = 0; b < nseq; ++b) {
        if (pos_host[b] >= maxLen) return api_fail(TL_ERR_KV_FULL, "KV cache full");
        if (pos_host[b] < 0) return api_fail(TL_ERR_INVALID, "negative position");
        tot += pos_host[b] + 1;
        nmax = std::max(nmax, pos_host[b] + 1);
    }
    void *scratch = nullptr;
    int rc = scratch_for_current_device(&scratch);
    if (rc != TL_OK) return rc;
    int dev = 0, sms = 0, smem_max = 0;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0 ||
        cudaDeviceGetAttribute(&smem_max, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess)
        return api_fail(TL_ERR_CUDA, "cudaDeviceGetAttribute failed");
    const size_t smem = decode_smem_bytes(headDim, G, kvDtype, nseq);
    if (smem > (size_t)smem_max) {
        char m[200];
        snprintf(m, sizeof m,
                 "nseq %d needs %zu bytes of shared memory in the decode kernel, more than the %d per block "
                 "of this device: split the batch",
                 nseq, smem, smem_max);
        return api_fail(TL_ERR_INVALID, m);
    }
    const int ctas = sms * decode_ctas_per_sm(headDim, G, kvDtype, nseq);

    // chunk length: the usual balance target, raised until the partials fit the scratch
    long long want = (tot * nHeadKv + (long long)ctas * 4 - 1) / ((long long)ctas * 4);
    int chunk = (int)std::min<long long>(1024, std::max<long long>(32, want));
    chunk = (chunk + 31) / 32 * 32;
    chunk = std::max(chunk, ((nmax + kMaxChunksPerSeq - 1) / kMaxChunksPerSeq + 31) / 32 * 32);
    long long units = 0;
    size_t need = 0;
    for (;;) {
        units = 0;
        bool multi = false;
        for (int b = 0; b < nseq; ++b) {
            const int n = pos_host[b] + 1;
            const int nch = (n + chunk - 1) / chunk;
            multi |= nch > 1;
            units += (long long)nch * nHeadKv;
        }
        need = multi ? decode_partial_floats((int)units, G, headDim) : 0;
        if (need <= kPartialFloats) break;
        if (chunk >= nmax) break;  // one chunk per sequence needs no partials: cannot happen
        chunk = std::min(((chunk * 2) + 31) / 32 * 32, ((nmax + 31) / 32) * 32);
    }
    if (need > kPartialFloats) return api_fail(TL_ERR_INVALID, "decode partials exceed the no-alloc scratch");

    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    unsigned char *base = static_cast<unsigned char *>(scratch);
    // counters of this call's (sequence, kv-head) pairs and the error word start at zero
    cudaError_t e = cudaMemsetAsync(base, 0, sizeof(unsigned) * (size_t)nseq * nHeadKv, s);
    if (e == cudaSuccess) e = cudaMemsetAsync(base + kCounterBytes, 0, kErrBytes, s);
    if (e != cudaSuccess) return api_fail(TL_ERR_CUDA, cudaGetErrorString(e));

    DecodeArgs a{};
    a.q = q;
    a.out = out;
    a.pos = pos_dev;
    a.nseq = nseq;
    a.nHead = nHead;
    a.nHeadKv = nHeadKv;
    a.headDim = headDim;
    a.layer = 0;
    a.slot0 = 0;
    a.pos_offset = 0;
    a.chunk = chunk;
    a.kv.k = const_cast<void *>(k_cache);
    a.kv.v = const_cast<void *>(v_cache);
    a.kv.nLayer = 1;
    a.kv.maxBatch = nseq;
    a.kv.nHeadKv = nHeadKv;
    a.kv.maxLen = maxLen;
    a.kv.headDim = headDim;
    a.kv.dtype = kvDtype;
    a.partial = reinterpret_cast<float *>(base + kPartialOffset);
    a.partial_cap = kPartialFloats;
    a.counter = reinterpret_cast<unsigned *>(base);
    a.err = reinterpret_cast<unsigned *>(base + kCounterBytes);
    a.work = reinterpret_cast<unsigned *>(base + kCounterBytes + 16);  // inside the cleared error block
    a.lse_out = nullptr;
    e = launch_decode(a, (int)std::max<long long>(1, std::min<long long>(units, ctas)), s);
    if (e == cudaErrorNotSupported) return api_fail(TL_ERR_UNSUPPORTED, "decode: shape not covered");
    if (e != cudaSuccess) return api_fail(TL_ERR_CUDA, cudaGetErrorString(e));
    const size_t n_out = (size_t)nseq * nHead * headDim;
    const int blocks = (int)std::min<size_t>((n_out + 1023) / 1024, (size_t)sms * 4);
    poison_on_error_kernel<<<blocks, 256, 0, s>>>(a.err, out, n_out);
    e = cudaGetLastError();
    if (e != cudaSuccess) return api_fail(TL_ERR_CUDA, cudaGetErrorString(e));
    return TL_OK;
}
