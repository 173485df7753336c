/* attn_oracle.h -- CPU restatement of tinylama's attention path (test infrastructure only).
 * See attn_oracle.c for what each function restates and why parity is unpinned. */
#ifndef TL_ATTN_ORACLE_H
#define TL_ATTN_ORACLE_H
#ifdef __cplusplus
extern "C" {
#endif

void ora_rope_single(float *x, int nHead, int headDim, int ropeDim, float base, int seqLen);
void ora_rope_at_pos(float *x, int nHead, int headDim, int ropeDim, float base, int pos,
                     int seqLen);
void ora_store_kv_range(float *kCache, float *vCache, int cacheCols, int startPos,
                        const float *k, const float *v, int rows, int cols);
void ora_attention_full_ctx(const float *q, const float *k, const float *v, int seqLen,
                            int nHead, int nHeadKv, int headDim, float *ctx);
void ora_linear_ggml_col(const float *x, const float *w, int inDim, int outDim, int seqLen,
                         float *out);
void ora_attention_full(const float *q, const float *k, const float *v, const float *wo,
                        int nEmb, int seqLen, int nHead, int nHeadKv, int headDim,
                        float *out);
void ora_attention_cached(const float *q, const float *kCache, const float *vCache,
                          int cacheCols, int curLen, int nHead, int nHeadKv, int headDim,
                          float *ctx);
void ora_decode_step(float *q, float *k, const float *v, float *kCache, float *vCache,
                     int cacheCols, int pos, int nHead, int nHeadKv, int headDim, int ropeDim,
                     float base, float *ctx);
void ora_prefill_step(float *q, float *k, const float *v, float *kCache, float *vCache,
                      int cacheCols, int seqLen, int nHead, int nHeadKv, int headDim,
                      int ropeDim, float base, float *ctx);
float ora_rope_theta(int i, int ropeDim, float base);

#ifdef __cplusplus
}
#endif
#endif
