/*
 * tl_model.h -- the llama forward pass of tinylama on one B200, weights resident in HBM.
 *
 * The reference runs the whole model on the CPU in float32 (src/forward.nim:243-329) with
 * weights dequantised at load time (src/model.nim:116-123).  Here the weights stay in HBM as
 * they are stored in the GGUF file -- Q2_K blocks of 84 bytes per 256 weights
 * (src/quant.nim:49-87), or float32 -- and every step of a token runs on the device:
 *   embeddingLookup (src/forward.nim:15-38), rmsnormCols (src/tensor.nim:97-113),
 *   linearGGMLCol (src/forward.nim:40-83, Q2_K dequantised inside the matrix-vector kernel),
 *   RoPE + storeKVRange + attention (the attention path of tl_attn.h), add, ffn with silu
 *   (src/forward.nim:213-217, src/tensor.nim:40-56), linearOut (src/forward.nim:219-230) and
 *   argmaxLast (src/infer_core.nim:6-32).
 * A decode step is one CUDA graph replay: its token and position come from device memory, and
 * the argmax of one step feeds the next, so a greedy generation makes no host round trip per
 * token.  The KV cache is float32, like the reference's.
 *
 * Errors: TL_* codes of tl_attn.h, message from tl_last_error().  A model is bound to its
 * device and stream and is not thread-safe; calls are synchronous.
 */
#ifndef TL_MODEL_H
#define TL_MODEL_H

#include <stdint.h>

#include "tl_attn.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct tl_model tl_model;

/* HParams (src/model.nim:18-29) and the cache length (initKvCache maxLen). */
typedef struct tl_model_config {
    int nVocab, nEmb, nLayer, nFfn, nHead, nHeadKv, ropeDim;
    float ropeFreqBase, rmsEps;
    int maxLen;
} tl_model_config;

/* ggml tensor types accepted by tl_model_set_tensor; other k-quants are uploaded as float32
 * after dequantisation on the host. */
#define TL_GGML_F32 0
#define TL_GGML_Q2_K 10

TL_API int tl_model_create(tl_model **out, const tl_model_config *cfg, int device);
TL_API void tl_model_destroy(tl_model *m);

/* Upload one tensor under its GGUF name ("token_embd.weight", "blk.3.attn_q.weight",
 * "output_norm.weight", ...).  ne0 = the innermost (input) dimension, ne1 = rows (1 for a
 * vector).  data: ne1 rows of ne0 float32 (TL_GGML_F32), or of ne0/256 Q2_K blocks
 * (TL_GGML_Q2_K).  Copied; the caller keeps its buffer.  Replacing a tensor drops the captured
 * decode step (the next tl_model_generate captures it again). */
TL_API int tl_model_set_tensor(tl_model *m, const char *name, int ggmlType, const void *data, long long ne0,
                               long long ne1);

/* runPrompt (src/tinylama.nim:49-69): reset the cache, forwardPrefill over the prompt,
 * argmaxLast, then nNew - 1 forwardDecode steps, each fed the previous greedy id.  outIds[nNew]
 * receives the ids; gaps[nNew] (optional) the best minus the second-best logit of each step.
 * TL_ERR_KV_FULL when nPrompt + nNew - 1 > maxLen (src/forward.nim:290-291). */
TL_API int tl_model_generate(tl_model *m, const int32_t *prompt, int nPrompt, int nNew, int32_t *outIds,
                             float *gaps);

/* The logits of the last forward pass (nVocab floats, the last token's column), for checks. */
TL_API int tl_model_last_logits(tl_model *m, float *logits);

/* Device time of the last tl_model_generate call, split into the prefill (through its argmax)
 * and the nNew - 1 decode steps, in milliseconds (CUDA events on the model's stream). */
TL_API int tl_model_last_timing(tl_model *m, float *prefill_ms, float *decode_ms);

#ifdef __cplusplus
}
#endif

#endif /* TL_MODEL_H */
