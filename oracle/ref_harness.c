/* ref_harness.c — TEST INFRASTRUCTURE: exposes the reference's own CPU path.
 *
 * Compiled by oracle/Makefile together with the reference sources where they
 * lie (REF=<reference checkout>); nothing of the reference is copied into this
 * repository.  This translation unit includes the reference's src/model.c so
 * it can drive the file-static forward pass (src/model.c:798-909) with token-id
 * prompts, which the reference's public API (text prompts only) cannot do.
 * The resulting library, oracle/_ref/libhymt2_ref.so, is used by the tests to
 * pin the C restatement in hy_oracle.c and by bench.py as the CPU baseline.
 */
#include "model.c"

/* Q8_K quantiser of the reference (src/kernels.c:128-165). */
HYMT2_API void refh_quantize_q8k(const float *x, int k, int nt, q8k_block *y) {
    kernels_init();
    for (int t = 0; t < nt; t++) quantize_q8k(x + (size_t)t * k, k, y + (size_t)t * (k / QK_K));
}

/* Panel repack of the reference (src/kernels.c:535-561). */
HYMT2_API int refh_panel_repack(unsigned ggml_type, const void *data, int rows, int k, uint8_t *pk, float *ps) {
    kernels_init();
    int t = type_from_ggml(ggml_type);
    if (!panel_supported(t)) return -1;
    weight_t w = {(const uint8_t *)data, t, k, rows, row_size(t, k), NULL, NULL, 0, 0, NULL};
    panel_repack_rows(&w, pk, ps, 0, rows);
    return 0;
}

/* Model geometry: [n_layer, hidden, ffn, heads, kv_heads, hdim, ctx, rope_half, vocab_out, outw_rows, batch]. */
HYMT2_API void refh_dims(const hymt2_model *m, int *out) {
    int v[11] = {m->n_layer, m->hidden, m->ffn, m->heads, m->kv_heads, m->hdim, m->ctx, m->rope_half,
                 m->vocab_out, m->outw.n, m->batch};
    memcpy(out, v, sizeof v);
}

/* Rope tables and eps as loaded (src/model.c:576-586). */
HYMT2_API const float *refh_rope_cos(const hymt2_model *m) { return m->rope_cos; }
HYMT2_API const float *refh_rope_sin(const hymt2_model *m) { return m->rope_sin; }
HYMT2_API float refh_eps(const hymt2_model *m) { return m->eps; }

/* forward_tokens from position pos0 (chunked by the model's batch size);
 * copies the residual rows of the last chunk and, if asked, the logits.
 * Returns the number of residual rows copied. */
HYMT2_API int refh_forward(hymt2_model *m, const int *toks, int nt, int pos0, float *h_out, float *logits) {
    forward_tokens(m, toks, nt, pos0, logits != NULL);
    const int last = nt - ((nt - 1) / m->batch) * m->batch;
    if (h_out) memcpy(h_out, m->h, sizeof(float) * (size_t)last * m->hidden);
    if (logits) memcpy(logits, m->logits, sizeof(float) * (size_t)m->vocab_out);
    return last;
}

/* Greedy decode from token ids: the prefill/argmax/feed-back loop of gen_ids
 * (src/model.c:930-954) without the chat template, tokenizer or stop check,
 * with the same longest-common-prefix reuse of the previous call's KV cache.
 * step_logits (optional) receives the logits each argmax was taken over. */
HYMT2_API int refh_greedy(hymt2_model *m, const int *ids, int n, int ngen, int *out, float *step_logits,
                          double *prefill_ms, double *decode_ms, int *cached) {
    if (n <= 0 || n + ngen > m->ctx) return -2;
    double t0 = now_ms();
    int keep = 0;
    while (keep < m->n_cache && keep < n - 1 && m->cache_tok[keep] == ids[keep]) keep++;
    m->n_cache = keep;
    forward_tokens(m, ids + keep, n - keep, keep, true);
    memcpy(m->cache_tok + keep, ids + keep, sizeof(int) * (size_t)(n - keep));
    m->n_cache = n;
    double t1 = now_ms();
    for (int i = 0; i < ngen; i++) {
        if (step_logits) memcpy(step_logits + (size_t)i * m->vocab_out, m->logits, sizeof(float) * (size_t)m->vocab_out);
        int best = 0;
        float bv = m->logits[0];
        for (int j = 1; j < m->vocab_out; j++)
            if (m->logits[j] > bv) {
                bv = m->logits[j];
                best = j;
            }
        out[i] = best;
        if (i + 1 == ngen) break;
        forward_tokens(m, &best, 1, m->n_cache, true);
        m->cache_tok[m->n_cache++] = best;
    }
    double t2 = now_ms();
    if (prefill_ms) *prefill_ms = t1 - t0;
    if (decode_ms) *decode_ms = t2 - t1;
    if (cached) *cached = keep;
    return ngen;
}

HYMT2_API void refh_reset_cache(hymt2_model *m) { m->n_cache = 0; }

/* bf16 KV cache rows [0, npos) of one layer. */
HYMT2_API void refh_kv(const hymt2_model *m, int layer, int npos, uint16_t *k_out, uint16_t *v_out) {
    memcpy(k_out, m->kc[layer], sizeof(uint16_t) * (size_t)npos * m->kvdim);
    memcpy(v_out, m->vc[layer], sizeof(uint16_t) * (size_t)npos * m->kvdim);
}

HYMT2_API int refh_threads(const hymt2_model *m) { return tp_threads(m->tp); }
HYMT2_API int refh_physical_cores(void) { return hy_physical_cpu_count(); }
HYMT2_API int refh_uses_device(const hymt2_model *m) { return m->use_gpu && m->use_fused; }
