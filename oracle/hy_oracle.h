/* hy_oracle.h — CPU restatement of the hymt2 decode/prefill hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This is the checker the CUDA backend is compared
 * against; it is never linked into, loaded by, or called from the product
 * library.  Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline
 * leg may use it.
 *
 * Parity is pinned: tests/test_oracle_pin.py compares every function here with
 * the reference's own implementation compiled from its sources (oracle/_ref)
 * and with the committed golden fixtures in tests/golden/.
 */
#ifndef HY_ORACLE_H
#define HY_ORACLE_H

#include "../include/hy_device_abi.h"

#ifdef __cplusplus
extern "C" {
#endif

float orc_f16_to_f32(uint16_t h);
uint16_t orc_f32_to_bf16(float f);
float orc_bf16_to_f32(uint16_t h);

void orc_quantize_q8k(const float *x, int k, q8k_block *y);
void orc_quantize_rows(const float *x, int nt, int k, q8k_block *y);

size_t orc_row_size(int type, int k);
void orc_panel_repack(int type, const uint8_t *data, size_t row_bytes, int n, int k, uint8_t *pk, float *ps);

/* Exact per-block integer accumulators.  `out` is [nt][n][nblk] int32 where
 * nblk = k/256 (panel, Q6_K, Q2_0C halves) or 2*k/256 for Q4_K (sumi, summ
 * pairs).  Returns the number of int32 per (t, r). */
int orc_block_ints(const weight_t *w, const q8k_block *xq, int nt, int32_t *out);

void orc_matmul(const weight_t *w, const float *xf, const q8k_block *xq, int nt, float *out);
void orc_dequant_row(const weight_t *w, int row, float *dst);

/* ---- model-level forward (reference src/model.c:719-958, CPU path) ---- */
typedef struct orc_model orc_model;
typedef struct {
    int n_layer, hidden, ffn, heads, kv_heads, hdim, ctx, rope_half;
    float eps, rope_base;            /* effective base (alpha already folded in) */
    weight_t embd, outw;             /* outw may alias embd */
    const float *out_norm;
    const float **attn_norm, **ffn_norm, **q_norm, **k_norm; /* [n_layer] */
    weight_t *wq, *wk, *wv, *wo, *wg, *wu, *wd;              /* [n_layer] (panels built) */
} orc_model_desc;

orc_model *orc_model_create(const orc_model_desc *d);
void orc_model_free(orc_model *m);
void orc_model_reset(orc_model *m);
/* Tokens at positions pos0..pos0+nt-1; writes logits of the last one when
 * logits != NULL.  h_out (optional) receives the final residual [nt*hidden]. */
void orc_forward(orc_model *m, const int *toks, int nt, int pos0, float *logits, float *h_out);
/* Greedy decode from token ids: prefill ids[0..n) in chunks of `chunk`, then
 * `ngen` greedy tokens (no stop check).  Optional step_logits [ngen][vocab]. */
int orc_greedy(orc_model *m, const int *ids, int n, int ngen, int chunk, int *out, float *step_logits);
int orc_vocab_out(const orc_model *m);
/* Read back the bf16 KV cache of one layer: [ctx * kvdim] each. */
const uint16_t *orc_kcache(const orc_model *m, int layer);
const uint16_t *orc_vcache(const orc_model *m, int layer);

void orc_attention(int heads, int kv_heads, int hd, int rope_half, float *q, float *k, const float *v, int nt,
                   int pos0, uint16_t *kc, uint16_t *vc, const float *q_norm, const float *k_norm,
                   const float *rope_cos, const float *rope_sin, float eps, float *ao);
void orc_prologue_matmul(const weight_t *w, int mode, const float *x, const float *x2, const float *norm_w, float eps,
                         int nt, float *out);

void orc_set_threads(int n);
/* 1: orc_matmul accumulates in double (float64 reference for the rounding
 * spread); 0: the host's float order (default). */
void orc_set_f64(int on);

#ifdef __cplusplus
}
#endif
#endif
