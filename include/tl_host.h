/*
 * tl_host.h -- C ABI of libtlhost.so: tinylama's forward pass on the host with its attention
 * block behind a table of the reference's attention procs.
 *
 * This is the C++ counterpart of the Nim host a tinylama user keeps: GGUF loading and
 * dequantisation (src/gguf_loader.nim, src/quant.nim, src/model.nim), the CPU linear layers,
 * RMSNorm and FFN (src/forward.nim, src/tensor.nim), greedy decoding (src/infer_core.nim,
 * src/tinylama.nim).  Its attention procs -- initKvCache, applyRopeSingle, applyRopeAtPos,
 * storeKVRange, attentionFull (ctx part), attentionCached (src/forward.nim:94-241) -- are
 * called through tlh_attn_ops; tlh_gpu_attn_ops_create fills the table with libtlattn.so
 * (the B200 path).  Everything but attention stays on the CPU, as in the reference.
 */
#ifndef TL_HOST_H
#define TL_HOST_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define TLH_API __attribute__((visibility("default")))
#else
#define TLH_API
#endif

/* The reference's attention procs.  Tensors are float32 in the ggml column layout
 * [rows, cols] (src/tensor.nim:11-26).  Each returns 0 or a negative status. */
typedef struct tlh_attn_ops {
    void *ctx;
    /* initKvCache (src/forward.nim:94-106): a fresh cache of maxLen positions per layer */
    int (*init_cache)(void *ctx, int maxLen);
    /* applyRopeSingle (:108-123) / applyRopeAtPos (:125-139), in place */
    int (*rope_single)(void *ctx, float *x, int nHead, int headDim, int ropeDim, float base,
                       int seqLen);
    int (*rope_at_pos)(void *ctx, float *x, int nHead, int headDim, int ropeDim, float base,
                       int pos, int seqLen);
    /* storeKVRange (:232-241): k, v = [rows = nHeadKv*headDim, cols] at column startPos */
    int (*store_kv)(void *ctx, int layer, int startPos, const float *k, const float *v, int rows,
                    int cols);
    /* attentionFull without wo (:141-176) */
    int (*attention_full)(void *ctx, const float *q, const float *k, const float *v, int seqLen,
                          int nHead, int nHeadKv, int headDim, float *out);
    /* attentionCached (:179-211) over the cache of `layer` */
    int (*attention_cached)(void *ctx, int layer, const float *q, int curLen, int nHead,
                            int nHeadKv, int headDim, float *out);
    /* KvCache.curLen / maxLen */
    int curLen, maxLen;
    /* Optional (NULL when the table does not provide it).  The attention blocks of seqLen
     * successive forwardDecode steps from pos = startPos (src/forward.nim:314-317), in one
     * call: RoPE q, k at startPos + t, storeKVRange at startPos, token t attending positions
     * 0..startPos+t; out = [nHead*headDim, seqLen]. */
    int (*prefill_at)(void *ctx, int layer, int startPos, const float *q, const float *k, const float *v,
                      int seqLen, float *out);
} tlh_attn_ops;

typedef struct tlh_model tlh_model;

/* HParams (src/model.nim:18-29) */
typedef struct tlh_hparams {
    int nVocab, nCtx, nEmb, nLayer, nFfn, nHead, nHeadKv, ropeDim;
    float ropeFreqBase, rmsEps;
} tlh_hparams;

/* loadModel + getTensor for every tensor (src/model.nim:105-123): parse the GGUF file and
 * dequantise F32/F16/Q2_K/Q3_K/Q6_K tensors to float32.  nthreads > 1 parallelises
 * dequantisation and the linear layers the way the reference's Malebolgia build does
 * (32-row chunks, src/forward.nim:51-74); 1 is the default build.  NULL on failure, with a
 * message in err. */
TLH_API tlh_model *tlh_model_load(const char *path, int nthreads, char *err, int errlen);
/* The same file mapped read-only (mmap), with no float32 copy of the weights: for
 * tlh_model_to_gpu, which uploads Q2_K and float32 tensors straight from the mapping (the
 * gguf_loader.nim:327-331 view of the data, without model.nim:116-123's dequantised cache).
 * tlh_model_tensor dequantises on demand; the CPU forward pass refuses such a model. */
TLH_API tlh_model *tlh_model_open(const char *path, char *err, int errlen);
TLH_API void tlh_model_free(tlh_model *m);
TLH_API int tlh_model_hparams(const tlh_model *m, tlh_hparams *out);
/* Copy the dequantised float32 data of tensor `name` (getTensor, src/model.nim:116-123) into
 * out (cap floats); *n receives its element count.  0, or -1 if the tensor does not exist. */
TLH_API int tlh_model_tensor(const tlh_model *m, const char *name, float *out, long cap, long *n);

/* runPrompt of src/tinylama.nim:49-69 for one prompt: initKvCache(max(32, nNew + 32)),
 * forwardPrefill (src/forward.nim:243-284), argmaxLast (src/infer_core.nim:6-32), then
 * nNew - 1 forwardDecode steps (:286-329).  outIds[nNew] receives the greedy ids; gaps[nNew]
 * (optional) the difference between the best and second-best logit of each step; attnOut
 * (optional, attnCap floats) every attention output (ctx before wo) in call order: the prefill
 * [nLayer][nHead*headDim*nPrompt] then each decode step [nLayer][nHead*headDim].  Returns the
 * number of attention floats written, or a negative status. */
TLH_API long tlh_generate(tlh_model *m, tlh_attn_ops *ops, const int32_t *prompt, int nPrompt,
                          int nNew, int32_t *outIds, float *gaps, float *attnOut, long attnCap);

/* The REPL of src/tinylama.nim:45-100, one line at a time.  tlh_session_init is the
 * initKvCache(max(32, nNew + 32)) of :47 (the cache then lives across turns).  tlh_run_prompt
 * is runPrompt (:49-86) for one line's tokens: the first turn (curLen = 0) runs forwardPrefill;
 * a later turn feeds its tokens through forwardDecode one at a time (:70-73) -- or, with
 * chunked != 0 and a table that has prefill_at, through one forward pass over all of them at
 * positions curLen.. (the same attention, fewer passes over the weights) -- and both then
 * decode nNew - 1 greedy tokens.  Outputs as tlh_generate; the attention outputs of a chunked
 * later turn are [nLayer][nHead*headDim*nPrompt].  Returns the number of attention floats. */
TLH_API int tlh_session_init(tlh_attn_ops *ops, int nNew);
TLH_API long tlh_run_prompt(tlh_model *m, tlh_attn_ops *ops, const int32_t *prompt, int nPrompt, int nNew,
                            int chunked, int32_t *outIds, float *gaps, float *attnOut, long attnCap);

/* Upload every tensor of a loaded model to a GPU model (tl_model.h): Q2_K tensors as stored in
 * the file, the others as the float32 the loader produced.  0 or a negative status. */
struct tl_model;
TLH_API int tlh_model_to_gpu(const tlh_model *m, struct tl_model *g);

/* The attention procs on the B200 (libtlattn.so, one cache slot, f32 cache); the table has
 * prefill_at (tl_prefill_layer_at_host). */
TLH_API tlh_attn_ops *tlh_gpu_attn_ops_create(int nLayer, int nHead, int nHeadKv, int headDim,
                                              int ropeDim, float ropeBase, int device);
TLH_API void tlh_gpu_attn_ops_destroy(tlh_attn_ops *ops);
TLH_API const char *tlh_last_error(void);

#ifdef __cplusplus
}
#endif
#endif /* TL_HOST_H */
