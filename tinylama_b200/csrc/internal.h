// internal.h -- the handle behind tl_attn* and the kernel launchers shared between the .cu
// files of libtlattn.so.  Nothing here is part of the C ABI (include/tl_attn.h is).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <string>
#include <utility>
#include <vector>

#include "../../include/tl_attn.h"

namespace tl {

constexpr int kMaxRopePairs = 128;  // headDim <= 256
constexpr int kMaxPeers = 8;        // GPUs in a split-KV group (one NVSwitch domain of an HGX node)

// RoPE frequencies, computed on the host with the same float32 powf as src/forward.nim:116
// (theta_i = powf(1/base, 2i/ropeDim)) and passed by value to the kernels, so device and
// reference angles are the same float32 product float32(pos) * theta_i.
struct RopeTab {
    float theta[kMaxRopePairs];
    int pairs;  // ropeDim / 2
};

RopeTab make_rope_tab(int ropeDim, float base);

// Strided view of a float tensor of per-head vectors: element (sequence b, token t, head h,
// dim d) is at ptr[b*sb + t*st + h*sh + d*sd].  The reference's column layout [H*D, S] is
// (sb=0, st=1, sh=D*S, sd=S); a token-major [B][S][H*D] buffer is (S*H*D, H*D, D, 1).
struct HeadView {
    float *ptr;
    int64_t sb, st, sh, sd;
    __host__ __device__ int64_t at(int b, int t, int h, int d) const {
        return b * sb + t * st + h * sh + d * sd;
    }
};

struct KvLayout {
    // Head-major cache: element (layer, slot, kvHead, pos, dim) of K (and of V) is at
    // (((layer*maxBatch + slot)*nHeadKv + kvHead)*maxLen + pos)*headDim + dim.
    void *k;
    void *v;
    int nLayer, maxBatch, nHeadKv, maxLen, headDim;
    int dtype;  // TL_KV_F32 / TL_KV_BF16
    __host__ __device__ int64_t row(int layer, int slot, int kvh, int pos) const {
        return (((int64_t)layer * maxBatch + slot) * nHeadKv + kvh) * (int64_t)maxLen + pos;
    }
};

}  // namespace tl

struct tl_attn {
    int device = 0;
    int nLayer = 0, nHead = 0, nHeadKv = 0, headDim = 0, ropeDim = 0;
    float ropeBase = 10000.f;
    int maxLen = 0, maxBatch = 0, kvDtype = TL_KV_F32;
    int numSms = 0;
    tl::KvLayout kv{};
    std::vector<int> curLen;        // host copy of each slot's length (KvCache.curLen)
    int *dPos = nullptr;            // device positions scratch [maxBatch]
    unsigned *dErr = nullptr;       // device error word
    // split-KV scratch: partial (m, l) pairs and partial outputs, and per-(slot,kvHead)
    // arrival counters used by the last CTA of a sequence to merge its chunks.
    float *dPartial = nullptr;
    size_t partialCap = 0;          // floats
    unsigned *dCounter = nullptr;   // [maxBatch * nHeadKv] + 2 work counters, zero between launches
    // host-tier staging (device side) for q/k/v/ctx copies
    float *dIo = nullptr;
    size_t ioCap = 0;               // floats
    float *hPinned = nullptr;       // pinned host staging
    size_t pinnedCap = 0;
    // bf16 Q staging for the tensor-core prefill [maxBatch][nHead][S][headDim]
    void *dQb = nullptr;
    size_t qbCap = 0;               // bytes
    cudaStream_t stream = nullptr;  // the handle's own stream (host tier)
    // host-tier batched decode: copy streams (in, out) and per-part events, so that the copies
    // of one part of the batch overlap the attention of another
    cudaStream_t cpIn = nullptr, cpOut = nullptr;
    cudaEvent_t evIn[4] = {}, evOut[4] = {}, evDone = nullptr;
    // multi-GPU split-KV
    void *comm = nullptr;           // ncclComm_t (used to exchange the IPC handles)
    bool commNonblocking = false;   // set up non-blocking (TL_DIST_INIT_TIMEOUT_MS)
    int nranks = 1, rank = 0;
    float *dGather = nullptr;
    size_t gatherCap = 0;
    // peer-memory exchange: this rank's exported buffer ([2 halves][nranks][maxBatch*nHead]
    // [headDim+2] 8-byte words) and every rank's mapping of it
    void *dPeerBuf = nullptr;
    void *peerBase[tl::kMaxPeers] = {};
    size_t peerHalfWords = 0;
    unsigned epoch = 0;
    unsigned long long peerWaitNs = 2000000000ull;  // TL_DIST_WAIT_MS at tl_dist_init
    // host-side fault injection (TL_DIST_FAULT_SILENT_PEER=1 at tl_dist_init, one rank only):
    // the exchange runs as rank 0 of two, and rank 1 is a local buffer that nothing writes
    void *dSilentPeer = nullptr;
};

namespace tl {

// Launch a kernel with programmatic stream serialisation: its CTAs may be scheduled while the
// previous kernel on the stream still runs, and it waits (pdl_wait) before reading that
// kernel's output.  Used for the decode kernels, which follow the RoPE/append launch in a
// decode step.  (The persistent prefill kernel is launched normally: its CTAs, resident early,
// would take the SMs' shared memory from the RoPE kernel still running.)
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                       Args &&...args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// The same, with thread-block clusters of `cluster` CTAs along x.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl_cluster(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, int cluster,
                               cudaStream_t s, Args &&...args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = (unsigned)cluster;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// ---- launchers (return cudaError_t of the launch) -----------------------------------------
// RoPE on q and/or k plus optional append of (rotated k, v) into the cache.
//   positions: token t of sequence b sits at position pos0[b] + t (pos0 on the device, or
//   the scalar pos0_scalar when pos0 == nullptr).
struct RopeAppendArgs {
    HeadView q;      // nullable ptr: no q rotation
    HeadView k;      // nullable ptr
    HeadView v;      // nullable ptr: no append
    int nseq, ntok, nHead, nHeadKv, headDim;
    const int *pos0;
    int pos0_scalar;
    bool rope_q, rope_k, store;
    bool q_inplace = true, k_inplace = true;  // write rotated q / k back into their views
    int layer, slot0;  // cache layer and first slot (sequence b -> slot slot0 + b)
    KvLayout kv;
    void *qb;          // nullable: bf16 copy of rotated q, [nseq][nHead][ntok][headDim]
    unsigned *err;
};
cudaError_t launch_rope_append(const RopeAppendArgs &a, const RopeTab &tab, cudaStream_t s);

// Split-KV decode attention over the cache for nseq sequences (slots slot0..), one query
// token each at position pos[b]; attends over [0, pos[b]] (the token is already appended).
//   q: [nseq][nHead][headDim] f32 (already rotated), out: [nseq][nHead][headDim] f32.
struct DecodeArgs {
    const float *q;
    float *out;
    const int *pos;        // device [nseq]
    int nseq, nHead, nHeadKv, headDim;
    int layer, slot0;
    int pos_offset;        // cache position of index 0 of this shard (split-KV across GPUs)
    int chunk;             // positions per work unit (multiple of 32)
    int cluster;           // > 0: one thread-block cluster of this many CTAs per (sequence,
                           // kv-head), one chunk each, merged through distributed shared memory
    KvLayout kv;
    float *partial;        // scratch
    size_t partial_cap;    // floats
    unsigned *counter;     // [nseq * nHeadKv] zeroed
    unsigned *work;        // [2] zeroed: next unit to claim, producers done (reset by the last)
    unsigned *err;
    // When non-null the kernel writes un-normalised (m, l, o) per (seq, head) here instead
    // of the final output: [nseq][nHead][headDim + 2] = (o[0..d), m, l).
    float *lse_out;
    // Split-KV across GPUs over peer memory (dist.cu); inactive when nranks == 0.  The CTA that
    // finishes a (sequence, kv-head) pair stores its heads' (o, m, l) into slot `rank` of every
    // rank's gather buffer as 8-byte words (float bits, epoch): a word is single-copy atomic,
    // so a reader that sees the current epoch in a word also sees its value, and no fence or
    // flag is needed.  After its own units, CTA i merges the pairs p = i, i + gridDim, ...,
    // waiting (bounded) on each word it reads.
    struct Peer {
        unsigned long long *gather[kMaxPeers];  // rank r's half for this call: [nranks][nseq*nHead][D+2]
        unsigned epoch;
        int nranks, rank;
        unsigned long long wait_ns;             // limit of each wait for a peer's words
    } px;
    // A decode step fused into the attention launch (cluster mode only; inactive when k is
    // null): q [nseq][nHead*D] (a.q points to it) and k [nseq][nHeadKv*D] are rotated at
    // position pos[b] in place, and the rotated k and v are written into the cache at that
    // position, in the same kernel -- what launch_rope_append followed by the decode does, with
    // the same arithmetic.
    struct Fuse {
        float *q, *k;
        const float *v;
        RopeTab tab;
    } fz;
};
cudaError_t launch_decode(const DecodeArgs &a, int num_ctas, cudaStream_t s);
// Resident CTAs per SM of the decode kernel a launch for nseq sequences uses.
int decode_ctas_per_sm(int headDim, int group, int dtype, int nseq);
// Dynamic shared memory of that launch (bytes).
size_t decode_smem_bytes(int headDim, int group, int dtype, int nseq);
// tensor-core decode for bf16 caches (decode_mma.cu)
bool decode_mma_covers(int headDim, int group, int dtype);
cudaError_t launch_decode_mma(const DecodeArgs &a, int num_ctas, cudaStream_t s);
int decode_mma_ctas_per_sm(int headDim, int group, int dtype, int nseq);
size_t decode_mma_smem_bytes(int headDim, int group, int dtype, int nseq);
// Clusters of `cluster` CTAs of the tensor-core decode kernel that can be resident at once
// (cudaOccupancyMaxActiveClusters; 0 if the query fails).
int decode_mma_cluster_capacity(int headDim, int group, int dtype, int cluster);
size_t decode_partial_floats(int total_units, int group, int headDim);

// Merge G per-rank (o, m, l) partials [G][nseq][nHead][d+2] into out [nseq][nHead][d].
cudaError_t launch_lse_merge(const float *parts, int nparts, int nseq, int nHead, int headDim,
                             float *out, cudaStream_t s);

// Causal prefill attention, f32 SIMT: queries of sequence b at positions pos0[b]+t,
// t < ntok, attend over cache positions [0, pos0[b]+t].
struct PrefillArgs {
    HeadView q;       // rotated q
    HeadView out;
    HeadView kf, vf;  // when kf.ptr != nullptr: f32 K/V views (attentionFull's fresh
                      // projections, token t at position t) instead of the cache
    const int *pos0; // device [nseq] or nullptr (all zero)
    int nseq, ntok, nHead, nHeadKv, headDim;
    int layer, slot0;
    KvLayout kv;
    const void *qb;  // bf16 q staging (tensor-core path)
    unsigned *err;
};
cudaError_t launch_prefill_f32(const PrefillArgs &a, cudaStream_t s);
// tcgen05 / TMEM bf16 path (bf16 cache, headDim 64; pos0 as above).  Returns
// cudaErrorNotSupported when the shape is not covered.
cudaError_t launch_prefill_tc(const PrefillArgs &a, cudaStream_t s);

}  // namespace tl
