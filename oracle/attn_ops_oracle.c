/*
 * attn_ops_oracle.c -- the reference's attention procs as a tlh_attn_ops table, computed by the
 * oracle (TEST INFRASTRUCTURE ONLY: the end-to-end tests run the host forward pass once with
 * this table and once with the B200 table, and compare).  The cache is the reference's:
 * per layer, K and V are [nHeadKv*headDim, maxLen] float32 (src/forward.nim:85-106).
 */
#include <stdlib.h>
#include <string.h>

#include "../include/tl_host.h"
#include "attn_oracle.h"

typedef struct {
    tlh_attn_ops ops;
    int nLayer, kvDim;
    float *k, *v; /* [nLayer][kvDim][maxLen] */
} OraOps;

static int o_init(void *c, int maxLen) {
    OraOps *o = (OraOps *)c;
    free(o->k);
    free(o->v);
    const size_t n = (size_t)o->nLayer * o->kvDim * maxLen;
    o->k = (float *)calloc(n, sizeof(float));
    o->v = (float *)calloc(n, sizeof(float));
    if (!o->k || !o->v) return -7;
    o->ops.curLen = 0;
    o->ops.maxLen = maxLen;
    return 0;
}
static int o_rope_single(void *c, float *x, int nH, int d, int rd, float base, int S) {
    (void)c;
    ora_rope_single(x, nH, d, rd, base, S);
    return 0;
}
static int o_rope_at_pos(void *c, float *x, int nH, int d, int rd, float base, int pos, int S) {
    (void)c;
    ora_rope_at_pos(x, nH, d, rd, base, pos, S);
    return 0;
}
static int o_store(void *c, int layer, int start, const float *k, const float *v, int rows, int cols) {
    OraOps *o = (OraOps *)c;
    const int maxLen = o->ops.maxLen;
    if (start + cols > maxLen) return -4; /* the reference would raise IndexDefect */
    const size_t off = (size_t)layer * o->kvDim * maxLen;
    ora_store_kv_range(o->k + off, o->v + off, maxLen, start, k, v, rows, cols);
    return 0;
}
static int o_full(void *c, const float *q, const float *k, const float *v, int S, int nH, int nKv, int d,
                  float *out) {
    (void)c;
    ora_attention_full_ctx(q, k, v, S, nH, nKv, d, out);
    return 0;
}
static int o_cached(void *c, int layer, const float *q, int curLen, int nH, int nKv, int d, float *out) {
    OraOps *o = (OraOps *)c;
    const int maxLen = o->ops.maxLen;
    const size_t off = (size_t)layer * o->kvDim * maxLen;
    ora_attention_cached(q, o->k + off, o->v + off, maxLen, curLen, nH, nKv, d, out);
    return 0;
}

tlh_attn_ops *ora_attn_ops_create(int nLayer, int nHeadKv, int headDim) {
    OraOps *o = (OraOps *)calloc(1, sizeof(OraOps));
    o->nLayer = nLayer;
    o->kvDim = nHeadKv * headDim;
    o->ops.ctx = o;
    o->ops.init_cache = o_init;
    o->ops.rope_single = o_rope_single;
    o->ops.rope_at_pos = o_rope_at_pos;
    o->ops.store_kv = o_store;
    o->ops.attention_full = o_full;
    o->ops.attention_cached = o_cached;
    return &o->ops;
}

void ora_attn_ops_destroy(tlh_attn_ops *ops) {
    if (!ops) return;
    OraOps *o = (OraOps *)ops->ctx;
    free(o->k);
    free(o->v);
    free(o);
}
