/* nc_oracle.h -- CPU restatement of nanocompile's Qwen2 decode step (TEST INFRASTRUCTURE).
 *
 * This library is the checker, never the product: only tests/, the smoke check and
 * bench.py's cpu_baseline leg load it.  It restates, in plain C compiled with
 * -ffp-contract=off, the arithmetic of the C that nanocompile generates for
 * fuse(optimize(quantize(build_qwen2(...)))) -- same operations, same order, same
 * fmaf where the reference has an Fma node and nowhere else -- so its outputs are
 * bit-identical to the reference's CBackend.  It is pinned against golden vectors
 * produced by the reference itself (tests/golden/make_golden.py).
 */
#ifndef NC_ORACLE_H
#define NC_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    int64_t vocab, hidden, inter, layers, heads, kv_heads, head_dim;
    float eps;          /* float32(rms_norm_eps) */
    float attn_scale;   /* float32(head_dim ** -0.5) */
    int32_t quant;      /* 0 = float32 projections, 1 = int8-vnni (block 32), 2 = int8 weights, float32 activations */
    int32_t threads;    /* worker threads for row-parallel loops; <= 0 keeps the last setting */
} orc_config;

/* One decoder layer's parameters (host arrays, row-major [out, in]). */
typedef struct {
    const float *in_norm, *post_norm;                 /* [H] */
    const float *bq, *bk, *bv;                        /* [heads*d], [kv*d], [kv*d] */
    const float *wq, *wk, *wv, *wo, *wg, *wu, *wd;    /* float32 weights (quant == 0) */
    const int8_t *qq, *qk, *qv, *qo, *qg, *qu, *qd;   /* int8 weights (quant == 1, 2) */
    const float *sq, *sk, *sv, *so, *sg, *su, *sd;    /* per-row scales (quant == 1, 2) */
} orc_layer;

/* One step of the model: the reference graph `build_qwen2(config, last_only)`
 * evaluated on `seq` new tokens after `past` cached ones.
 *   past_keys/values: [layers, kv_heads, past_cap, head_dim]; positions 0..past-1 are read.
 *   logits: [last_only ? 1 : seq, vocab];  keys/values out: [layers, kv_heads, seq, head_dim].
 * Returns 0, or 1 when a token id is outside 0..vocab-1 (*bad_index gets the first one). */
int32_t orc_qwen2_step(const orc_config *c, const float *embed, const float *final_norm,
                       const orc_layer *layers, const float *inv_freq,
                       const int64_t *ids, int64_t seq,
                       const float *past_keys, const float *past_values, int64_t past, int64_t past_cap,
                       int32_t last_only, float *logits, float *keys, float *values,
                       int64_t *bad_index);

/* Block-32 activation quantization of `rows` rows of width k (quantize.py:102-124).
 * block_sums may be NULL. */
void orc_quantize_blocks(const float *x, int64_t rows, int64_t k, int8_t *xq, float *xs,
                         float *offset, int32_t *block_sums);

/* matmul_i8: out[m, n] = int8_dots(q[n], x[m]) * scales[n], float32 activations
 * (lower.py:320-356, lower.py:398-412). */
void orc_matmul_i8(const float *x, const int8_t *q, const float *scales, int64_t rows, int64_t n, int64_t k,
                   float *out);

/* matmul_i8_vnni: out[m, n] for m < rows (lower.py:363-397 + fusion.py:677-711).
 * lanes (nullable): the int32 Dp4 value of every (row m, output n, 4-byte lane),
 * [rows, n, k/4]. */
void orc_matmul_i8_vnni(const int8_t *xq, const float *xs, const float *offset,
                        const int8_t *q, const float *scales, int64_t rows, int64_t n, int64_t k,
                        float *out, int32_t *lanes);

/* The SwiGLU epilogue (nn.py:41-55): out = silu(g) * u with glibc's expf. */
void orc_swiglu(const float *g, const float *u, int64_t n, float *out);

/* In-order float32 rms_norm row kernel (fusion.py:631-650); residual may be NULL. */
void orc_rms_norm(const float *x, const float *residual, const float *w, int64_t rows, int64_t n,
                  float eps, float *out);

/* The tied fp32 LM head (one row) and greedy argmax, first maximum wins. */
void orc_lm_head(const float *x, const float *embed, int64_t vocab, int64_t hidden, float *logits);
int64_t orc_argmax(const float *v, int64_t n);

/* glibc's expf, and the table-driven restatement of its published method that the
 * device implements (exact on every float; tests compare the two). */
float orc_expf_libm(float x);
float orc_expf_restated(float x);
float orc_cosf_libm(float x);
float orc_sinf_libm(float x);
/* Element-wise over arrays: which = 0 glibc expf, 1 the restatement, 2 cosf, 3 sinf. */
void orc_map(int32_t which, const float *x, int64_t n, float *out);

/* Per-head decode attention over a cache, in the reference's order (calls 14-17 of a
 * fused block): q [heads, d]; keys/values [kv, len, d] (len = past + 1, the last
 * position being the new token); out [heads, d]; probs (nullable) [heads, len]. */
void orc_attention_decode(const float *q, const float *keys, const float *values, int64_t heads,
                          int64_t kv_heads, int64_t len, int64_t d, int64_t cap, float scale,
                          float *out, float *probs);

#ifdef __cplusplus
}
#endif
#endif
