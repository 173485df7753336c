// dist.cu -- split-KV decode across GPUs: one process per GPU, NCCL over NVLink/NVSwitch.
//
// The reference has no parallelism on this path (attentionCached, src/forward.nim:179-211,
// is one CPU loop).  Long contexts are split along the sequence axis: rank r's cache holds
// global positions [r*maxLen, (r+1)*maxLen) of every sequence.  Each rank runs the split-KV
// decode kernel over its slice and writes per-(sequence, q-head) partials (o, m, l) -- m and l
// in the log2 domain -- into its own slot of a gather buffer; one in-place ncclAllGather
// exchanges the slots (B*nHead*(headDim+2) floats per rank) and a merge kernel combines them:
//   M = max_r m_r,  L = sum_r l_r 2^(m_r - M),  ctx = sum_r o_r 2^(m_r - M) / L.
#include <dlfcn.h>
#include <nccl.h>
#include <string.h>

#include <algorithm>
#include <mutex>

#include "internal.h"

namespace tl {
int api_run_decode_lse(tl_attn *h, int layer, int slot0, int nseq, const int *pos_dev,
                       const int *pos_host, const float *q, float *lse_out, cudaStream_t s,
                       int pos_offset);
int api_fail(int code, const char *msg);
}  // namespace tl

using namespace tl;

namespace {

// NCCL is resolved at first use with dlopen, not linked: the library then loads in processes
// that never use the multi-GPU calls, and a host that has already loaded an NCCL (PyTorch
// does) keeps using that one instead of a second copy with the same soname.
struct Nccl {
    ncclResult_t (*GetUniqueId)(ncclUniqueId *);
    ncclResult_t (*CommInitRank)(ncclComm_t *, int, ncclUniqueId, int);
    ncclResult_t (*AllGather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t);
    ncclResult_t (*CommDestroy)(ncclComm_t);
    const char *(*GetErrorString)(ncclResult_t);
    bool ok;
};

const Nccl &nccl() {
    static Nccl n{};
    static std::once_flag once;
    std::call_once(once, [] {
        void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (!h) return;
        n.GetUniqueId = reinterpret_cast<decltype(n.GetUniqueId)>(dlsym(h, "ncclGetUniqueId"));
        n.CommInitRank = reinterpret_cast<decltype(n.CommInitRank)>(dlsym(h, "ncclCommInitRank"));
        n.AllGather = reinterpret_cast<decltype(n.AllGather)>(dlsym(h, "ncclAllGather"));
        n.CommDestroy = reinterpret_cast<decltype(n.CommDestroy)>(dlsym(h, "ncclCommDestroy"));
        n.GetErrorString = reinterpret_cast<decltype(n.GetErrorString)>(dlsym(h, "ncclGetErrorString"));
        n.ok = n.GetUniqueId && n.CommInitRank && n.AllGather && n.CommDestroy && n.GetErrorString;
    });
    return n;
}

int nccl_fail(ncclResult_t r, const char *what) {
    char buf[256];
    snprintf(buf, sizeof buf, "%s: %s", what, nccl().ok ? nccl().GetErrorString(r) : "NCCL unavailable");
    return api_fail(TL_ERR_NCCL, buf);
}

#define TL_NEED_NCCL()                                                                   \
    do {                                                                                 \
        if (!nccl().ok) return api_fail(TL_ERR_NCCL, "libnccl.so.2 could not be loaded"); \
    } while (0)

}  // namespace

extern "C" {

int tl_dist_unique_id(char *id128) {
    if (!id128) return api_fail(TL_ERR_INVALID, "NULL id buffer");
    static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId is 128 bytes");
    TL_NEED_NCCL();
    ncclUniqueId id;
    ncclResult_t r = nccl().GetUniqueId(&id);
    if (r != ncclSuccess) return nccl_fail(r, "ncclGetUniqueId");
    memcpy(id128, &id, sizeof id);
    return TL_OK;
}

int tl_dist_init(tl_attn *h, const char *id128, int nranks, int rank) {
    if (!h || !id128) return api_fail(TL_ERR_INVALID, "NULL argument");
    if (nranks < 1 || rank < 0 || rank >= nranks) return api_fail(TL_ERR_INVALID, "bad rank/nranks");
    if (h->comm) return api_fail(TL_ERR_INVALID, "handle already joined a communicator");
    TL_NEED_NCCL();
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(h->device);
    ncclUniqueId id;
    memcpy(&id, id128, sizeof id);
    ncclComm_t comm;
    ncclResult_t r = nccl().CommInitRank(&comm, nranks, id, rank);
    cudaSetDevice(prev);
    if (r != ncclSuccess) return nccl_fail(r, "ncclCommInitRank");
    h->comm = comm;
    h->nranks = nranks;
    h->rank = rank;
    return TL_OK;
}

void tl_dist_finalize(tl_attn *h) {
    if (!h || !h->comm) return;
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(h->device);
    if (h->stream) cudaStreamSynchronize(h->stream);
    nccl().CommDestroy(reinterpret_cast<ncclComm_t>(h->comm));
    cudaSetDevice(prev);
    h->comm = nullptr;
    h->nranks = 1;
    h->rank = 0;
}

int tl_decode_attention_dist(tl_attn *h, int layer, int slot0, int nseq, const int *pos_dev,
                             const int *pos_host, const float *q, float *out, void *stream) {
    if (!h || !pos_dev || !q || !out) return api_fail(TL_ERR_INVALID, "NULL argument");
    if (!h->comm) return api_fail(TL_ERR_INVALID, "tl_dist_init has not been called");
    if (layer < 0 || layer >= h->nLayer || nseq < 1 || slot0 < 0 || slot0 + nseq > h->maxBatch)
        return api_fail(TL_ERR_INVALID, "layer or slots out of range");
    if (pos_host)
        for (int b = 0; b < nseq; ++b)
            if ((long long)pos_host[b] >= (long long)h->maxLen * h->nranks)
                return api_fail(TL_ERR_KV_FULL, "KV cache full");
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(h->device);
    cudaStream_t s = stream ? reinterpret_cast<cudaStream_t>(stream) : h->stream;
    const size_t rows = (size_t)nseq * h->nHead;
    const size_t per_rank = rows * (h->headDim + 2);
    const size_t need = per_rank * h->nranks;
    int rc = TL_OK;
    if (need > h->gatherCap) {
        cudaDeviceSynchronize();
        cudaFree(h->dGather);
        h->dGather = nullptr;
        h->gatherCap = 0;
        if (cudaMalloc(&h->dGather, need * sizeof(float)) != cudaSuccess) {
            cudaSetDevice(prev);
            return api_fail(TL_ERR_NOMEM, "gather buffer allocation failed");
        }
        h->gatherCap = need;
    }
    float *mine = h->dGather + per_rank * h->rank;
    rc = api_run_decode_lse(h, layer, slot0, nseq, pos_dev, pos_host, q, mine, s,
                            h->rank * h->maxLen);
    if (rc == TL_OK) {
        ncclResult_t r = nccl().AllGather(mine, h->dGather, per_rank, ncclFloat,
                                       reinterpret_cast<ncclComm_t>(h->comm), s);
        if (r != ncclSuccess) rc = nccl_fail(r, "ncclAllGather");
    }
    if (rc == TL_OK) {
        cudaError_t e = launch_lse_merge(h->dGather, h->nranks, nseq, h->nHead, h->headDim, out, s);
        if (e != cudaSuccess) rc = api_fail(TL_ERR_CUDA, cudaGetErrorString(e));
    }
    cudaSetDevice(prev);
    return rc;
}

}  // extern "C"
