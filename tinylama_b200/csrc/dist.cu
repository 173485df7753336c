// dist.cu -- split-KV decode across GPUs: one process per GPU on one NVSwitch domain.
//
// The reference has no parallelism on this path (attentionCached, src/forward.nim:179-211,
// is one CPU loop).  Long contexts are split along the sequence axis: rank r's cache holds
// global positions [r*maxLen, (r+1)*maxLen) of every sequence.  Each rank runs the split-KV
// decode kernel over its slice; the per-(sequence, q-head) results (o, m, l) -- m and l in the
// log2 domain -- are combined as
//   M = max_r m_r,  L = sum_r l_r 2^(m_r - M),  ctx = sum_r o_r 2^(m_r - M) / L.
//
// The exchange is fused into the decode kernel over peer memory.  At tl_dist_init every rank
// exports one buffer with CUDA IPC (two halves of [nranks][maxBatch*nHead][headDim+2] 8-byte
// words), the handles are all-gathered once over NCCL, and every rank maps every peer's
// buffer.  In a call, the CTA that finishes a (sequence, kv-head) stores its heads' (o, m, l)
// straight into slot `rank` of every rank's buffer (NVLink stores) as words that carry the
// value and the call's epoch; after its own units each CTA merges a share of the pairs, reading
// each word once it shows the current epoch (a bounded wait).  An aligned 8-byte store is
// single-copy atomic, so the epoch in a word vouches for its value: no fences, no flags, one
// launch per call and no collective.  Calls alternate between the two halves by epoch parity,
// so a rank that runs ahead into the next call never overwrites words a slower rank has not
// read yet.
//
// If the peers cannot be mapped (ranks in one process, or TL_DIST_NCCL=1 in the environment at
// tl_dist_init), the exchange falls back to writing the local slot, one in-place
// ncclAllGather and a merge launch.
#include <dlfcn.h>
#include <nccl.h>
#include <string.h>

#include <stdlib.h>

#include <sched.h>

#include <algorithm>
#include <chrono>
#include <mutex>
#include <thread>
#include <vector>

#include "internal.h"

namespace tl {
int api_run_decode_lse(tl_attn *h, int layer, int slot0, int nseq, const int *pos_dev,
                       const int *pos_host, const float *q, float *lse_out, cudaStream_t s,
                       int pos_offset);
int api_run_decode_peer(tl_attn *h, int layer, int slot0, int nseq, const int *pos_dev,
                        const int *pos_host, const float *q, float *out, cudaStream_t s, int pos_offset,
                        const DecodeArgs::Peer &px);
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
    // non-blocking set-up (NCCL >= 2.14): an init that a rank never joins can be given up
    ncclResult_t (*CommInitRankConfig)(ncclComm_t *, int, ncclUniqueId, int, ncclConfig_t *);
    ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t *);
    ncclResult_t (*CommAbort)(ncclComm_t);
    ncclResult_t (*CommFinalize)(ncclComm_t);
    bool ok, nonblocking;
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
        n.CommInitRankConfig = reinterpret_cast<decltype(n.CommInitRankConfig)>(dlsym(h, "ncclCommInitRankConfig"));
        n.CommGetAsyncError = reinterpret_cast<decltype(n.CommGetAsyncError)>(dlsym(h, "ncclCommGetAsyncError"));
        n.CommAbort = reinterpret_cast<decltype(n.CommAbort)>(dlsym(h, "ncclCommAbort"));
        n.CommFinalize = reinterpret_cast<decltype(n.CommFinalize)>(dlsym(h, "ncclCommFinalize"));
        n.ok = n.GetUniqueId && n.CommInitRank && n.AllGather && n.CommDestroy && n.GetErrorString;
        n.nonblocking = n.CommInitRankConfig && n.CommGetAsyncError && n.CommAbort && n.CommFinalize;
    });
    return n;
}

int nccl_fail(ncclResult_t r, const char *what) {
    char buf[256];
    snprintf(buf, sizeof buf, "%s: %s", what, nccl().ok ? nccl().GetErrorString(r) : "NCCL unavailable");
    return api_fail(TL_ERR_NCCL, buf);
}

long long env_ms(const char *name, long long dflt) {
    const char *e = getenv(name);
    if (!e || !*e) return dflt;
    const long long v = atoll(e);
    return v > 0 ? v : dflt;
}

// On a non-blocking communicator an NCCL call may return before its work is enqueued: poll
// until it is, or until the operation fails.  A blocking communicator returns at once.
ncclResult_t nccl_settle(const tl_attn *h, ncclResult_t r) {
    if (!h->commNonblocking || (r != ncclSuccess && r != ncclInProgress)) return r;
    const auto comm = reinterpret_cast<ncclComm_t>(h->comm);
    ncclResult_t st = ncclInProgress;
    while (true) {
        if (nccl().CommGetAsyncError(comm, &st) != ncclSuccess) return ncclInternalError;
        if (st != ncclInProgress) return st;
        sched_yield();
    }
}

#define TL_NEED_NCCL()                                                                   \
    do {                                                                                 \
        if (!nccl().ok) return api_fail(TL_ERR_NCCL, "libnccl.so.2 could not be loaded"); \
    } while (0)

// All ranks reach this point: an all-gather of one float per rank on the handle's stream.
int dist_barrier(tl_attn *h) {
    float *d = nullptr;
    if (cudaMalloc(&d, sizeof(float) * h->nranks) != cudaSuccess) return api_fail(TL_ERR_NOMEM, "barrier buffer");
    ncclResult_t r = nccl_settle(
        h, nccl().AllGather(d + h->rank, d, 1, ncclFloat, reinterpret_cast<ncclComm_t>(h->comm), h->stream));
    cudaStreamSynchronize(h->stream);
    cudaFree(d);
    return r == ncclSuccess ? TL_OK : nccl_fail(r, "ncclAllGather (barrier)");
}

void unmap_peers(tl_attn *h) {
    for (int r = 0; r < h->nranks && r < kMaxPeers; ++r) {
        if (r != h->rank && h->peerBase[r]) cudaIpcCloseMemHandle(h->peerBase[r]);
        h->peerBase[r] = nullptr;
    }
}

// Collective: export this rank's exchange buffer, all-gather the IPC handles, map the peers'.
// Returns TL_OK with peerBase[rank] == nullptr when the peers cannot be mapped (the NCCL
// exchange is used then).
int map_peers(tl_attn *h, bool silent_peer) {
    const char *env = getenv("TL_DIST_NCCL");
    const bool want = h->nranks <= kMaxPeers && !(env && env[0] == '1');
    const int slots = h->nranks + (silent_peer ? 1 : 0);
    const size_t half = (size_t)slots * h->maxBatch * h->nHead * (h->headDim + 2);
    const size_t bytes = 2 * half * sizeof(unsigned long long);
    if (want) {
        if (cudaMalloc(&h->dPeerBuf, bytes) != cudaSuccess)
            return api_fail(TL_ERR_NOMEM, "split-KV exchange buffer allocation failed");
        cudaMemset(h->dPeerBuf, 0, bytes);  // every word starts at epoch 0
        h->peerHalfWords = half;
        if (silent_peer) {
            // the injected rank's buffer: this rank stores into it, nothing ever writes ours
            if (cudaMalloc(&h->dSilentPeer, bytes) != cudaSuccess)
                return api_fail(TL_ERR_NOMEM, "split-KV exchange buffer allocation failed");
            cudaMemset(h->dSilentPeer, 0, bytes);
        }
    }
    // every rank takes part in the handle exchange, also one that does not map (all-or-nothing)
    cudaIpcMemHandle_t mine{};
    int ok = want && (h->nranks == 1 || cudaIpcGetMemHandle(&mine, h->dPeerBuf) == cudaSuccess);
    const size_t rec = sizeof(cudaIpcMemHandle_t) + 8;
    std::vector<char> host(rec * h->nranks);
    char *dev = nullptr;
    if (cudaMalloc(&dev, rec * h->nranks) != cudaSuccess) return api_fail(TL_ERR_NOMEM, "handle exchange buffer");
    std::vector<char> me(rec, 0);
    memcpy(me.data(), &mine, sizeof mine);
    memcpy(me.data() + sizeof mine, &ok, sizeof ok);
    cudaMemcpy(dev + rec * h->rank, me.data(), rec, cudaMemcpyHostToDevice);
    cudaDeviceSynchronize();  // the zeroed words are in place before any peer can map them
    ncclResult_t r = nccl_settle(h, nccl().AllGather(dev + rec * h->rank, dev, rec, ncclChar,
                                                     reinterpret_cast<ncclComm_t>(h->comm), h->stream));
    cudaStreamSynchronize(h->stream);
    cudaMemcpy(host.data(), dev, rec * h->nranks, cudaMemcpyDeviceToHost);
    cudaFree(dev);
    if (r != ncclSuccess) return nccl_fail(r, "ncclAllGather (IPC handles)");
    int all_ok = 1;
    for (int q = 0; q < h->nranks; ++q) {
        int o = 0;
        memcpy(&o, host.data() + rec * q + sizeof(cudaIpcMemHandle_t), sizeof o);
        all_ok &= o;
    }
    if (all_ok) {
        for (int q = 0; q < h->nranks; ++q) {
            if (q == h->rank) { h->peerBase[q] = h->dPeerBuf; continue; }
            cudaIpcMemHandle_t hq;
            memcpy(&hq, host.data() + rec * q, sizeof hq);
            if (cudaIpcOpenMemHandle(&h->peerBase[q], hq, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
                cudaGetLastError();
                h->peerBase[q] = nullptr;
                all_ok = 0;
            }
        }
    }
    // agree on the outcome: the fused exchange runs only if every rank mapped every peer
    int agreed = all_ok;
    {
        std::vector<char> again(rec, 0);
        memcpy(again.data() + sizeof(cudaIpcMemHandle_t), &all_ok, sizeof all_ok);
        char *d2 = nullptr;
        if (cudaMalloc(&d2, rec * h->nranks) != cudaSuccess) return api_fail(TL_ERR_NOMEM, "handle exchange buffer");
        cudaMemcpy(d2 + rec * h->rank, again.data(), rec, cudaMemcpyHostToDevice);
        r = nccl_settle(h, nccl().AllGather(d2 + rec * h->rank, d2, rec, ncclChar,
                                            reinterpret_cast<ncclComm_t>(h->comm), h->stream));
        cudaStreamSynchronize(h->stream);
        cudaMemcpy(host.data(), d2, rec * h->nranks, cudaMemcpyDeviceToHost);
        cudaFree(d2);
        if (r != ncclSuccess) return nccl_fail(r, "ncclAllGather (IPC outcome)");
        for (int q = 0; q < h->nranks; ++q) {
            int o = 0;
            memcpy(&o, host.data() + rec * q + sizeof(cudaIpcMemHandle_t), sizeof o);
            agreed &= o;
        }
    }
    if (!agreed) unmap_peers(h);
    return TL_OK;
}

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
    if (nranks > kMaxPeers) return api_fail(TL_ERR_INVALID, "at most 8 ranks (one NVSwitch domain)");
    if (h->comm) return api_fail(TL_ERR_INVALID, "handle already joined a communicator");
    TL_NEED_NCCL();
    const char *fault = getenv("TL_DIST_FAULT_SILENT_PEER");
    const bool silent = fault && fault[0] == '1';
    if (silent && nranks != 1)
        return api_fail(TL_ERR_INVALID, "TL_DIST_FAULT_SILENT_PEER injects a peer into a one-rank group only");
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(h->device);
    ncclUniqueId id;
    memcpy(&id, id128, sizeof id);
    ncclComm_t comm = nullptr;
    ncclResult_t r;
    const bool nonblocking = nccl().nonblocking && env_ms("TL_DIST_INIT_TIMEOUT_MS", 0) > 0;
    if (nonblocking) {
        // with TL_DIST_INIT_TIMEOUT_MS set: a non-blocking set-up, given up after that many
        // milliseconds if some rank never joins, so that the call fails instead of waiting for
        // ever (without it, NCCL's own blocking set-up)
        ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
        cfg.blocking = 0;
        const long long limit_ms = env_ms("TL_DIST_INIT_TIMEOUT_MS", 120000);
        r = nccl().CommInitRankConfig(&comm, nranks, id, rank, &cfg);
        if (r == ncclSuccess || r == ncclInProgress) {
            const auto t0 = std::chrono::steady_clock::now();
            ncclResult_t st = ncclInProgress;
            while (true) {
                if (nccl().CommGetAsyncError(comm, &st) != ncclSuccess) st = ncclInternalError;
                if (st != ncclInProgress) break;
                const auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(
                                    std::chrono::steady_clock::now() - t0).count();
                if (ms > limit_ms) break;
                std::this_thread::sleep_for(std::chrono::milliseconds(1));
            }
            if (st == ncclInProgress) {
                nccl().CommAbort(comm);
                cudaSetDevice(prev);
                char m[192];
                snprintf(m, sizeof m, "tl_dist_init: the group of %d ranks did not form within %lld ms (a rank "
                         "never joined); the communicator was aborted", nranks, limit_ms);
                return api_fail(TL_ERR_NCCL, m);
            }
            r = st;
            if (r != ncclSuccess) nccl().CommAbort(comm);
        }
    } else {
        r = nccl().CommInitRank(&comm, nranks, id, rank);
    }
    cudaSetDevice(prev);
    if (r != ncclSuccess) return nccl_fail(r, "ncclCommInitRank");
    h->comm = comm;
    h->commNonblocking = nonblocking;
    h->nranks = nranks;
    h->rank = rank;
    h->epoch = 0;
    h->peerWaitNs = (unsigned long long)env_ms("TL_DIST_WAIT_MS", 2000) * 1000000ull;
    cudaSetDevice(h->device);
    const int rc = map_peers(h, silent);
    cudaSetDevice(prev);
    return rc;
}

int tl_dist_resync(tl_attn *h) {
    if (!h) return api_fail(TL_ERR_INVALID, "NULL handle");
    if (!h->comm) return api_fail(TL_ERR_INVALID, "tl_dist_init has not been called");
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(h->device);
    // this rank's calls have ended (completed or given up): no kernel of it still writes words
    cudaError_t e = cudaDeviceSynchronize();
    int rc = TL_OK;
    unsigned *d = nullptr;
    if (e != cudaSuccess) {
        rc = api_fail(TL_ERR_CUDA, cudaGetErrorString(e));
    } else if (cudaMalloc(&d, sizeof(unsigned) * h->nranks) != cudaSuccess) {
        rc = api_fail(TL_ERR_NOMEM, "resync buffer");
    } else {
        std::vector<unsigned> all(h->nranks);
        cudaMemcpy(d + h->rank, &h->epoch, sizeof(unsigned), cudaMemcpyHostToDevice);
        ncclResult_t r = nccl_settle(h, nccl().AllGather(d + h->rank, d, 1, ncclUint32,
                                                         reinterpret_cast<ncclComm_t>(h->comm), h->stream));
        cudaStreamSynchronize(h->stream);
        if (r != ncclSuccess) {
            rc = nccl_fail(r, "ncclAllGather (resync)");
        } else {
            cudaMemcpy(all.data(), d, sizeof(unsigned) * h->nranks, cudaMemcpyDeviceToHost);
            // every word any rank has stored carries an epoch <= the largest one used so far:
            // the next call, at a larger epoch, reads none of them
            unsigned mx = 0;
            for (unsigned x : all) mx = std::max(mx, x);
            h->epoch = mx;
        }
        cudaFree(d);
    }
    cudaSetDevice(prev);
    return rc;
}

void tl_dist_finalize(tl_attn *h) {
    if (!h || !h->comm) return;
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(h->device);
    cudaDeviceSynchronize();
    if (h->dPeerBuf) {
        // every rank's kernels are done before any mapping goes, and every mapping is gone
        // before any exporter frees its buffer
        dist_barrier(h);
        unmap_peers(h);
        dist_barrier(h);
        cudaFree(h->dPeerBuf);
        h->dPeerBuf = nullptr;
        h->peerHalfWords = 0;
        h->epoch = 0;
    }
    if (h->dSilentPeer) {
        cudaFree(h->dSilentPeer);
        h->dSilentPeer = nullptr;
    }
    if (h->commNonblocking) nccl_settle(h, nccl().CommFinalize(reinterpret_cast<ncclComm_t>(h->comm)));
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
    // refused before the call takes an epoch, so that every rank refuses the same call alike
    if ((reinterpret_cast<uintptr_t>(q) & 15u) != 0) return api_fail(TL_ERR_INVALID, "q must be 16-byte aligned");
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
    if (h->peerBase[h->rank]) {
        DecodeArgs::Peer px{};
        px.epoch = ++h->epoch;
        const size_t half = (px.epoch & 1u) ? h->peerHalfWords : 0;
        for (int r = 0; r < h->nranks; ++r) px.gather[r] = reinterpret_cast<unsigned long long *>(h->peerBase[r]) + half;
        px.nranks = h->nranks;
        px.rank = h->rank;
        px.wait_ns = h->peerWaitNs;
        if (h->dSilentPeer) {
            // injected fault: a second rank whose words never arrive
            px.gather[1] = reinterpret_cast<unsigned long long *>(h->dSilentPeer) + half;
            px.nranks = 2;
        }
        const int rc = api_run_decode_peer(h, layer, slot0, nseq, pos_dev, pos_host, q, out, s,
                                           h->rank * h->maxLen, px);
        cudaSetDevice(prev);
        return rc;
    }
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
        ncclResult_t r = nccl_settle(h, nccl().AllGather(mine, h->dGather, per_rank, ncclFloat,
                                                         reinterpret_cast<ncclComm_t>(h->comm), s));
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
