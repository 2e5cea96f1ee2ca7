/* hysynth.h — seeded synthetic Hy-MT2-shaped GGUF writer (tests and benches). */
#ifndef HYSYNTH_H
#define HYSYNTH_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { HYSYNTH_REFTOOL = 0, HYSYNTH_SPEC = 1 };

typedef struct {
    int mode;           /* HYSYNTH_REFTOOL or HYSYNTH_SPEC */
    int n_layer, hidden, heads, kv_heads, hdim, ffn, vocab;
    int layer_type[7];  /* ggml types of q, k, v, o, gate, up, down (SPEC mode) */
    int embd_type;      /* token_embd type (SPEC mode) */
    int head_type;      /* separate output.weight type, -1 = tied to token_embd (SPEC mode) */
    float freq_base, rope_alpha, eps;
    uint64_t seed;
    /* SPEC-mode distributions:
     *  STQ1_0 / Q2_0C: codes uniform bytes, d = f16(|N(0, scale_sigma)|)
     *  Q4_K: d, dmin = f16(|N(0, kquant_sigma)|), scale/min bytes and codes uniform
     *  Q6_K (projections): codes uniform, sub-scales uniform int8, d = f16(|N(0, kquant_sigma)|)
     *  Q6_K (token_embd): the reference bench tool's ranges (sub-scales -20..20, d in f16 0x1400..0x14FF)
     *  Q8_0: codes clip(round(N(0, q8_code_sigma)), +-127), d = f16(|N(0, q8_scale_sigma)|)
     *  F16: N(0, f16_sigma);  norms: 1 + norm_jitter * N(0, 1) */
    double scale_sigma, kquant_sigma, q8_code_sigma, q8_scale_sigma, f16_sigma, norm_jitter;
} hysynth_spec;

void hysynth_default_spec(hysynth_spec *sp);
/* 0 on success, <0 on I/O error. */
int hysynth_write(const char *path, const hysynth_spec *sp);
int hysynth_block_weights(int type);

#ifdef __cplusplus
}
#endif
#endif
