/*
 * tl_attn.h -- C ABI of libtlattn.so, the B200 (sm_100a) attention path for tinylama.
 *
 * Plain C: opaque handle, plain pointers and sizes, int status codes.  No C++ or framework
 * types cross this boundary, so Nim (importc/dynlib), ctypes or any C caller can bind it.
 *
 * Reference interface replaced (paths inside the tinylama project):
 *   KvCache / initKvCache        src/forward.nim:85-106
 *   applyRopeSingle              src/forward.nim:108-123
 *   applyRopeAtPos               src/forward.nim:125-139
 *   attentionFull (ctx part)     src/forward.nim:141-176  (wo, :177, stays with the caller)
 *   attentionCached              src/forward.nim:179-211
 *   storeKVRange                 src/forward.nim:232-241
 *   call sites                   src/forward.nim:267-275 (prefill), :310-319,325 (decode)
 *   cloneCache                   bench/bench_tinylama.nim:18-32
 *
 * Layouts.
 *   Host tier (suffix _host): tensors are the reference's "ggml column layout" Tensor data,
 *   [rows, cols] with element (r, c) at r*cols + c (src/tensor.nim:11-26), i.e. q is
 *   [nHead*headDim, seqLen].  Calls are synchronous: they copy in, run on the handle's stream,
 *   copy out and return.
 *   Device tier: device pointers, token-major (sequence b, token t, head h, dim d at
 *   ((b*seqLen + t)*H + h)*headDim + d), asynchronous on the caller's cudaStream_t (passed as
 *   void*; NULL = the handle's own stream).  The decode calls read q in 16-byte vectors and
 *   refuse a q that is not 16-byte aligned (TL_ERR_INVALID).
 *   KV cache (owned by the handle, on the device): head-major, K and V each
 *   [nLayer][maxBatch][nHeadKv][maxLen][headDim] of f32 or bf16; one cache slot per
 *   sequence.  The reference's cache is the single-slot, dim-major special case.
 *
 * Errors.  Every call returns TL_OK (0) or a negative TL_ERR_*; tl_last_error() gives the
 * message of the calling thread's last failure.  Messages follow the reference where it has
 * one ("KV cache full", src/forward.nim:291; "GQA requires head_count divisible by
 * head_count_kv", :248).  Device kernels never trap: a kernel that sees a bad position or a
 * timed-out wait sets the handle's device error word, which the host tier checks after every
 * call and the device tier reports through tl_check_device().
 *
 * Threading.  A handle is bound to one device and is not thread-safe; use one handle per
 * host thread (the reference is single-threaded).  The library never retains host pointers.
 */
#ifndef TL_ATTN_H
#define TL_ATTN_H

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define TL_API __attribute__((visibility("default")))
#else
#define TL_API
#endif

#define TL_ATTN_VERSION 1

#define TL_KV_F32 0
#define TL_KV_BF16 1

#define TL_OK 0
#define TL_ERR_INVALID (-1)     /* bad argument (shape, NULL pointer, layer/slot range) */
#define TL_ERR_CUDA (-2)        /* a CUDA runtime call failed */
#define TL_ERR_KV_FULL (-3)     /* decode with curLen >= maxLen (src/forward.nim:290-291) */
#define TL_ERR_RANGE (-4)       /* write past maxLen (reference: IndexDefect in storeKVRange) */
#define TL_ERR_DEVICE (-5)      /* a kernel reported an error through the device error word */
#define TL_ERR_NCCL (-6)        /* an NCCL call failed or timed out */
#define TL_ERR_NOMEM (-7)       /* device or pinned allocation failed */
#define TL_ERR_UNSUPPORTED (-8) /* shape not covered by a kernel (headDim not 64/128, ...) */

typedef struct tl_attn tl_attn;

/* Message of the calling thread's last failed call ("" if none). */
TL_API const char *tl_last_error(void);
TL_API int tl_version(void);

/* ---- handle / KV cache ------------------------------------------------------------------- */

/* initKvCache (src/forward.nim:94-106) plus the hyper-parameters the attention procs take.
 * Allocates the zeroed device cache for nLayer layers and maxBatch sequences of maxLen
 * positions.  ropeDim 0 means headDim (src/forward.nim:250).  Fails with TL_ERR_INVALID if
 * nHead % nHeadKv != 0, as forwardPrefill does (src/forward.nim:247-248). */
TL_API int tl_attn_create(tl_attn **out, int nLayer, int nHead, int nHeadKv, int headDim, int ropeDim,
                   float ropeBase, int maxLen, int maxBatch, int kvDtype, int device);
TL_API void tl_attn_destroy(tl_attn *h);

/* KvCache.curLen of one slot (src/forward.nim:89): read and assign, as forwardPrefill
 * (:254) and forwardDecode (:325) do. */
TL_API int tl_kv_get_len(const tl_attn *h, int slot, int *len);
TL_API int tl_kv_set_len(tl_attn *h, int slot, int len);
/* Zero the cache and all lengths. */
TL_API int tl_kv_reset(tl_attn *h);
/* cloneCache (bench/bench_tinylama.nim:18-32): deep copy of cache contents and lengths into
 * a handle created with the same shape. */
TL_API int tl_kv_clone(tl_attn *dst, const tl_attn *src);
/* Copy one slot of one layer back to the host in the reference layout
 * KvCache.k[layer] = [nHeadKv*headDim, maxLen] f32 (bf16 caches are widened). */
TL_API int tl_kv_read(tl_attn *h, int layer, int slot, float *k, float *v);

/* ---- host tier: the reference procs, same arguments, ggml column layout -------------------- */

/* applyRopeSingle (src/forward.nim:108-123): rotates x = [nHead*headDim, seqLen] in place,
 * position of column p = p. */
TL_API int tl_rope_single_host(tl_attn *h, float *x, int nHead, int headDim, int ropeDim, float base,
                        int seqLen);
/* applyRopeAtPos (src/forward.nim:125-139): rotates column 0 of x = [nHead*headDim, seqLen]
 * at position pos. */
TL_API int tl_rope_at_pos_host(tl_attn *h, float *x, int nHead, int headDim, int ropeDim, float base,
                        int pos, int seqLen);
/* storeKVRange (src/forward.nim:232-241): k, v = [nHeadKv*headDim, cols] into columns
 * startPos.. of layer `layer`, slot `slot`.  Unlike the reference (IndexDefect) a write past
 * maxLen is refused with TL_ERR_RANGE before anything is written. */
TL_API int tl_kv_store_host(tl_attn *h, int layer, int slot, int startPos, const float *k,
                     const float *v, int cols);
/* attentionFull without its trailing wo projection (src/forward.nim:141-176): causal GQA over
 * the fresh projections q = [nHead*headDim, seqLen], k, v = [nHeadKv*headDim, seqLen];
 * ctx = [nHead*headDim, seqLen].  The caller applies wo (linearGGMLCol, :177). */
TL_API int tl_attention_full_host(tl_attn *h, const float *q, const float *k, const float *v,
                           int seqLen, int nHead, int nHeadKv, int headDim, float *ctx);
/* attentionCached (src/forward.nim:179-211) over cache.k[layer], cache.v[layer] of slot
 * `slot`: q = [nHead*headDim, 1], attends columns 0..curLen-1, ctx = [nHead*headDim, 1]. */
TL_API int tl_attention_cached_host(tl_attn *h, int layer, int slot, const float *q, int curLen,
                             int nHead, int nHeadKv, int headDim, float *ctx);

/* Fused per-layer calls: one host<->device round trip for the whole attention block.  The
 * inputs are the un-rotated projections; they are not modified (forwardDecode and
 * forwardPrefill do not read q or k after attention).
 * Decode (src/forward.nim:314-317): RoPE q and k at pos, store k, v at pos, attend over
 * pos+1 columns.  Fails with TL_ERR_KV_FULL when pos >= maxLen (:290-291).  Lengths are not
 * advanced (the caller sets curLen = pos+1 after the last layer, :325). */
TL_API int tl_decode_layer_host(tl_attn *h, int layer, int slot, const float *q, const float *k,
                         const float *v, int pos, float *ctx);
/* Prefill (src/forward.nim:271-274): RoPE q, k over positions 0..seqLen-1, store k, v at
 * column 0, causal attention -> ctx = [nHead*headDim, seqLen].  With a bf16 cache and
 * headDim 64 the attention runs on the tcgen05 tensor-core kernel. */
TL_API int tl_prefill_layer_host(tl_attn *h, int layer, int slot, const float *q, const float *k,
                          const float *v, int seqLen, float *ctx);
/* Prefill that continues a cached prefix: the tokens sit at positions startPos..startPos+seqLen-1
 * and token t attends cache positions 0..startPos+t.  It gives what the reference computes when
 * it feeds a later prompt token by token through forwardDecode (src/tinylama.nim:70-73, each
 * step src/forward.nim:314-317 with pos = curLen), in one call.  startPos = 0 is
 * tl_prefill_layer_host.  TL_ERR_RANGE when startPos + seqLen > maxLen. */
TL_API int tl_prefill_layer_at_host(tl_attn *h, int layer, int slot, int startPos, const float *q,
                             const float *k, const float *v, int seqLen, float *ctx);
/* Batched decode step with host buffers (the host-tier form of tl_decode_step): q
 * [nseq][nHead*headDim], k, v [nseq][nHeadKv*headDim], pos [nseq], out like q, all host
 * memory (pinned memory makes the copies asynchronous).  Synchronous.  A large batch (>= 0.3
 * GB of K/V) is cut into 2-4 parts of consecutive sequences: the copies of one part overlap
 * the attention of another (environment TL_HOST_PARTS=1..4 sets the number of parts). */
TL_API int tl_decode_batch_host(tl_attn *h, int layer, int slot0, int nseq, const int *pos,
                         const float *q, const float *k, const float *v, float *out);

/* ---- device tier: batched, token-major, asynchronous --------------------------------------- */

/* One decode step for nseq sequences in slots slot0..slot0+nseq-1 (src/forward.nim:314-317,
 * batched): q [nseq][nHead*headDim], k, v [nseq][nHeadKv*headDim], out
 * [nseq][nHead*headDim].  Sequence b's token sits at position pos_dev[b]; q and k are rotated
 * in place, k and v appended at that position, and attention runs over positions
 * 0..pos_dev[b].  pos_host (optional, same values on the host) lets the library size the
 * split-KV schedule exactly; without it the schedule assumes maxLen. */
TL_API int tl_decode_step(tl_attn *h, int layer, int slot0, int nseq, const int *pos_dev,
                   const int *pos_host, float *q, float *k, const float *v, float *out,
                   void *stream);
/* Attention only (no RoPE, no append): q already rotated, cache already holds positions
 * 0..pos_dev[b]. */
TL_API int tl_decode_attention(tl_attn *h, int layer, int slot0, int nseq, const int *pos_dev,
                        const int *pos_host, const float *q, float *out, void *stream);
/* Batched prefill from position 0 (src/forward.nim:271-274 per sequence): q
 * [nseq][seqLen][nHead*headDim], k, v [nseq][seqLen][nHeadKv*headDim], out like q.
 * bf16 cache + headDim 64: tcgen05 tensor-core attention, q and k are left unmodified;
 * otherwise fp32 CUDA cores, q and k are rotated in place. */
TL_API int tl_prefill_step(tl_attn *h, int layer, int slot0, int nseq, int seqLen, float *q, float *k,
                    const float *v, float *out, void *stream);
/* tl_prefill_step continuing cached prefixes: token t of sequence b sits at position
 * pos0_dev[b] + t and attends cache positions 0..pos0_dev[b]+t (the batched form of
 * tl_prefill_layer_at_host).  pos0_host (optional, the same values on the host) is checked
 * against maxLen before anything is launched. */
TL_API int tl_prefill_step_at(tl_attn *h, int layer, int slot0, int nseq, int seqLen, const int *pos0_dev,
                       const int *pos0_host, float *q, float *k, const float *v, float *out,
                       void *stream);
/* Same as tl_prefill_step but forces the fp32 CUDA-core attention kernel. */
TL_API int tl_prefill_step_f32(tl_attn *h, int layer, int slot0, int nseq, int seqLen, float *q,
                        float *k, const float *v, float *out, void *stream);
/* storeKVRange on device buffers (src/forward.nim:232-241, device tier): k, v token-major
 * [cols][nHeadKv*headDim] written to positions startPos.. of (layer, slot), no RoPE. */
TL_API int tl_kv_store(tl_attn *h, int layer, int slot, int startPos, const float *k, const float *v,
                int cols, void *stream);
/* Read and clear the device error word after synchronising the stream.  TL_OK or
 * TL_ERR_DEVICE (message names the bits). */
TL_API int tl_check_device(tl_attn *h, void *stream);

/* ---- allocation-free decode ------------------------------------------------------------- */

/* No counterpart in the reference.  For callers that cannot allocate device memory (a host
 * whose allocator has reserved all of it up front, or a loop that must not take an
 * allocation's latency and implicit synchronisation): the same split-KV decode attention as
 * tl_decode_attention, without a handle and without any allocation.  The caller passes q [nseq][nHead*headDim],
 * the cache K and V, each head-major [nseq][nHeadKv][maxLen][headDim] of f32 or bf16 with
 * RoPE already applied, positions pos_dev / pos_host (both required and equal: sequence b
 * attends positions 0..pos[b]; the schedule is sized from pos_host) and out
 * [nseq][nHead*headDim], all on the current device; the call is asynchronous on `stream`.
 * The kernel's scratch is a fixed 16 MiB array inside the library, held by every GPU that
 * loads it until exit: at most 65536 (sequence, kv-head) pairs per call, and at most as many
 * sequences as the decode kernel's shared memory holds (8 bytes per sequence beside a fixed
 * part, checked against the device's per-block limit: some 15000 to 22000 sequences,
 * depending on the shape); larger calls are refused with TL_ERR_INVALID.  There is no
 * handle, so a device-side refusal (pos_dev disagreeing with pos_host, a position past maxLen)
 * cannot be reported through tl_check_device: instead every element of `out` is set to NaN.
 * The first call on a device looks the array up (cudaGetSymbolAddress) and should come before
 * any stream capture.  All calls share the array and clear what they use at their start, so
 * calls that can overlap on the GPU race and must not be issued. */
TL_API int tl_decode_attention_noalloc(const float *q, const void *k_cache, const void *v_cache,
                                       int kvDtype, int nHead, int nHeadKv, int headDim, int maxLen,
                                       int nseq, const int *pos_dev, const int *pos_host, float *out,
                                       void *stream);

/* ---- multi-GPU split-KV (one process per GPU, peer memory over NVLink) --------------------- */

/* NCCL unique id (128 bytes) created on one rank and shared with the others by the caller. */
TL_API int tl_dist_unique_id(char *id128);
/* Collective.  Join the group as rank `rank` of `nranks` (at most 8, one process per GPU on
 * one NVSwitch domain), on this handle's device.  The handle's cache then holds positions
 * [rank*maxLen, (rank+1)*maxLen) of every sequence (its slice).  Every rank exports an exchange
 * buffer with CUDA IPC and maps every peer's; NCCL is used here only to pass the IPC handles.
 * If the peers cannot be mapped (or TL_DIST_NCCL=1 is set), the calls below exchange through
 * an NCCL all-gather instead.  With TL_DIST_INIT_TIMEOUT_MS set (environment, milliseconds)
 * the set-up is non-blocking: if some rank never joins, the call fails with TL_ERR_NCCL after
 * that time instead of waiting for ever (without it, NCCL's blocking set-up waits for all).  TL_DIST_WAIT_MS (default 2000) bounds each wait of a split-KV call for a peer's
 * values.  TL_DIST_FAULT_SILENT_PEER=1 (test only, one-rank groups) injects a second rank
 * whose values never arrive, so that every call runs into that bound. */
TL_API int tl_dist_init(tl_attn *h, const char *id128, int nranks, int rank);
/* Collective, after a split-KV call failed on some rank (a peer's values did not arrive in
 * time, reported by tl_check_device as a wait-timeout, or a rank skipped a call): waits for this
 * rank's queued work and agrees on a fresh epoch with every rank, so that the next call reads
 * none of the values left over from the failed one.  Every rank calls it, the same number of
 * times; afterwards the calls give correct results again. */
TL_API int tl_dist_resync(tl_attn *h);
/* Collective: every rank makes the same sequence of calls.  Split-KV decode across the ranks:
 * every rank passes the same q [nseq][nHead*headDim] (already rotated) and global positions
 * pos_dev/pos_host (the query attends global positions 0..pos[b]); each rank attends its
 * slice, the kernel stores each (sequence, head)'s (o, m, l) into every rank's buffer over
 * NVLink and merges them, and every rank receives the full out [nseq][nHead*headDim].  One
 * kernel launch per call on `stream`; its waits for the peers are bounded (2 s), after which
 * the device error word reports a timeout (tl_check_device). */
TL_API int tl_decode_attention_dist(tl_attn *h, int layer, int slot0, int nseq, const int *pos_dev,
                             const int *pos_host, const float *q, float *out, void *stream);
/* Collective: synchronises the device, waits for every rank, unmaps the peers' buffers and
 * leaves the group (tl_attn_destroy does this too). */
TL_API void tl_dist_finalize(tl_attn *h);

#ifdef __cplusplus
}
#endif
#endif /* TL_ATTN_H */
