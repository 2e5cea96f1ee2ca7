/* hysynth.c — seeded synthetic Hy-MT2-shaped GGUF files for tests and benches.
 *
 * There are no public model files on the machines this runs on, so every
 * parity test and benchmark uses random weights with the model's shapes.  Two
 * generators are provided:
 *
 *  - HYSYNTH_REFTOOL: reproduces, byte for byte, the file the reference's own
 *    benchmark tool writes (tools/make_bench_gguf.c): STQ1_0 layers, a Q6_K
 *    token embedding that doubles as the LM head, norms of 1.0, rope alpha
 *    1000, and a single xorshift64 stream (shifts 13/7/17, fixed start state)
 *    consumed in tensor order.  Only the layer count may be changed.
 *  - HYSYNTH_SPEC: any shape and per-projection type mix from a seeded
 *    splitmix64 stream, with the distributions chosen for each format
 *    (see hysynth.h).
 *
 * Files are GGUF v3 with 32-byte alignment and architecture "hunyuan-dense".
 */
#include "hysynth.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------ output */

typedef struct {
    FILE *f;
    int ok;
} wr;

static void put(wr *w, const void *p, size_t n) {
    if (w->ok && fwrite(p, 1, n, w->f) != n) w->ok = 0;
}
static void put_u32(wr *w, uint32_t v) { put(w, &v, 4); }
static void put_u64(wr *w, uint64_t v) { put(w, &v, 8); }
static void put_str(wr *w, const char *s) {
    put_u64(w, strlen(s));
    put(w, s, strlen(s));
}
static void kv_u32(wr *w, const char *k, uint32_t v) { put_str(w, k); put_u32(w, 4); put_u32(w, v); }
static void kv_f32(wr *w, const char *k, float v) { put_str(w, k); put_u32(w, 6); put(w, &v, 4); }
static void kv_str(wr *w, const char *k, const char *v) { put_str(w, k); put_u32(w, 8); put_str(w, v); }

/* ------------------------------------------------------------------ random streams */

typedef struct {
    int reftool;
    uint64_t s;
    int have_spare;
    double spare;
} rng_t;

/* Reference tool stream: xorshift64 (13, 7, 17), low 32 bits per draw. */
static uint32_t next32(rng_t *r) {
    if (r->reftool) {
        r->s ^= r->s << 13;
        r->s ^= r->s >> 7;
        r->s ^= r->s << 17;
        return (uint32_t)r->s;
    }
    /* splitmix64 */
    uint64_t z = (r->s += 0x9E3779B97F4A7C15ull);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return (uint32_t)((z ^ (z >> 31)) >> 32);
}

static double uniform01(rng_t *r) { return ((double)next32(r) + 0.5) / 4294967296.0; }

static double normal(rng_t *r) { /* Marsaglia polar method */
    if (r->have_spare) {
        r->have_spare = 0;
        return r->spare;
    }
    double u, v, s;
    do {
        u = 2.0 * uniform01(r) - 1.0;
        v = 2.0 * uniform01(r) - 1.0;
        s = u * u + v * v;
    } while (s >= 1.0 || s == 0.0);
    const double m = sqrt(-2.0 * log(s) / s);
    r->spare = v * m;
    r->have_spare = 1;
    return u * m;
}

static uint16_t to_f16(float x) {
    _Float16 h = (_Float16)x;
    uint16_t b;
    memcpy(&b, &h, 2);
    return b;
}

/* ------------------------------------------------------------------ tensors */

typedef struct {
    char name[64];
    int type; /* ggml type */
    uint64_t k, n; /* n == 0: vector of k */
    uint64_t bytes, off;
    int role; /* 0 weight, 1 norm, 2 embedding */
} tensor;

static uint64_t tensor_bytes(int type, uint64_t k, uint64_t n) {
    const uint64_t rows = n ? n : 1;
    switch (type) {
    case 0: return rows * k * 4;
    case 1: return rows * k * 2;
    case 8: return rows * (k / 32) * 34;
    case 12: return rows * (k / 256) * 144;
    case 14: return rows * (k / 256) * 210;
    case 40: return rows * (k / 512) * 130;
    case 43: return rows * (k / 256) * 42;
    }
    return 0;
}

static int block_weights(int type) {
    switch (type) {
    case 8: return 32;
    case 40: return 512;
    case 12: case 14: case 43: return 256;
    }
    return 1;
}

/* Fill one block of `type` into dst (block_bytes(type) bytes). */
static void fill_block(rng_t *r, int type, int role, const hysynth_spec *sp, uint8_t *dst) {
    switch (type) {
    case 43: /* STQ1_0: qs[32] slots, sign[8], f16 d */
        for (int j = 0; j < 40; j++) dst[j] = (uint8_t)next32(r);
        if (r->reftool) {
            uint16_t d = (uint16_t)(0x2000 + next32(r) % 256);
            memcpy(dst + 40, &d, 2);
        } else {
            uint16_t d = to_f16((float)fabs(normal(r) * sp->scale_sigma));
            memcpy(dst + 40, &d, 2);
        }
        break;
    case 14: /* Q6_K: ql[128] qh[64] scales[16] d */
        for (int j = 0; j < 192; j++) dst[j] = (uint8_t)next32(r);
        if (r->reftool || role == 2) {
            for (int j = 0; j < 16; j++) dst[192 + j] = (uint8_t)(int8_t)((int)(next32(r) % 41) - 20);
        } else {
            for (int j = 0; j < 16; j++) dst[192 + j] = (uint8_t)next32(r); /* full int8 code range */
        }
        {
            uint16_t d;
            if (r->reftool || role == 2) d = (uint16_t)(0x1400 + next32(r) % 256);
            else d = to_f16((float)fabs(normal(r) * sp->kquant_sigma));
            memcpy(dst + 208, &d, 2);
        }
        break;
    case 12: { /* Q4_K: d dmin scales[12] qs[128] */
        uint16_t d = to_f16((float)fabs(normal(r) * sp->kquant_sigma));
        uint16_t dm = to_f16((float)fabs(normal(r) * sp->kquant_sigma));
        memcpy(dst, &d, 2);
        memcpy(dst + 2, &dm, 2);
        for (int j = 4; j < 144; j++) dst[j] = (uint8_t)next32(r);
        break;
    }
    case 40: { /* Q2_0C: d qs[128] */
        uint16_t d = to_f16((float)fabs(normal(r) * sp->scale_sigma));
        memcpy(dst, &d, 2);
        for (int j = 2; j < 130; j++) dst[j] = (uint8_t)next32(r);
        break;
    }
    case 8: { /* Q8_0: d qs[32] */
        uint16_t d = to_f16((float)fabs(normal(r) * sp->q8_scale_sigma));
        memcpy(dst, &d, 2);
        for (int j = 0; j < 32; j++) {
            double v = nearbyint(normal(r) * sp->q8_code_sigma);
            if (v > 127) v = 127;
            if (v < -127) v = -127;
            dst[2 + j] = (uint8_t)(int8_t)v;
        }
        break;
    }
    case 1: { /* F16 */
        uint16_t h = to_f16((float)(normal(r) * sp->f16_sigma));
        memcpy(dst, &h, 2);
        break;
    }
    }
}

static size_t block_bytes(int type) {
    switch (type) {
    case 0: return 4;
    case 1: return 2;
    case 8: return 34;
    case 12: return 144;
    case 14: return 210;
    case 40: return 130;
    case 43: return 42;
    }
    return 0;
}

void hysynth_default_spec(hysynth_spec *sp) {
    memset(sp, 0, sizeof(*sp));
    sp->mode = HYSYNTH_REFTOOL;
    sp->n_layer = 32;
    sp->hidden = 2048;
    sp->heads = 16;
    sp->kv_heads = 4;
    sp->hdim = 128;
    sp->ffn = 6144;
    sp->vocab = 120818;
    for (int i = 0; i < 7; i++) sp->layer_type[i] = 43;
    sp->embd_type = 14;
    sp->head_type = -1;
    sp->freq_base = 10000.f;
    sp->rope_alpha = 1000.f;
    sp->eps = 1e-5f;
    sp->seed = 0;
    sp->scale_sigma = 0.02;
    sp->kquant_sigma = 0.01;
    sp->q8_code_sigma = 40.0;
    sp->q8_scale_sigma = 0.0005;
    sp->f16_sigma = 0.02;
    sp->norm_jitter = 0.0;
}

int hysynth_write(const char *path, const hysynth_spec *sp) {
    static const char *proj[7] = {"attn_q.weight", "attn_k.weight", "attn_v.weight", "attn_output.weight",
                                  "ffn_gate.weight", "ffn_up.weight", "ffn_down.weight"};
    const uint64_t H = (uint64_t)sp->hidden, QD = (uint64_t)sp->heads * sp->hdim, KD = (uint64_t)sp->kv_heads * sp->hdim;
    const uint64_t F = (uint64_t)sp->ffn, V = (uint64_t)sp->vocab;
    const uint64_t pk[7] = {H, H, H, QD, H, H, F}, pn[7] = {QD, KD, KD, H, F, F, H};
    const int reftool = sp->mode == HYSYNTH_REFTOOL;

    const int cap = 3 + sp->n_layer * 11;
    tensor *ts = (tensor *)calloc((size_t)cap, sizeof(tensor));
    int nt = 0;
    uint64_t cur = 0;
#define ADD(nm, ty, kk, nn, rl)                                             \
    do {                                                                    \
        snprintf(ts[nt].name, 64, "%s", nm);                                \
        ts[nt].type = ty; ts[nt].k = kk; ts[nt].n = nn; ts[nt].role = rl;   \
        ts[nt].bytes = tensor_bytes(ty, kk, nn); ts[nt].off = cur;          \
        cur += (ts[nt].bytes + 31) / 32 * 32; nt++;                         \
    } while (0)
    ADD("token_embd.weight", sp->embd_type, H, V, 2);
    ADD("output_norm.weight", 0, H, 0, 1);
    if (!reftool && sp->head_type >= 0) ADD("output.weight", sp->head_type, H, V, 0);
    char nm[64];
    for (int i = 0; i < sp->n_layer; i++) {
        static const char *norms[4] = {"attn_norm.weight", "ffn_norm.weight", "attn_q_norm.weight", "attn_k_norm.weight"};
        const uint64_t nlen[4] = {H, H, (uint64_t)sp->hdim, (uint64_t)sp->hdim};
        for (int j = 0; j < 4; j++) {
            snprintf(nm, 64, "blk.%d.%s", i, norms[j]);
            ADD(nm, 0, nlen[j], 0, 1);
        }
        for (int j = 0; j < 7; j++) {
            snprintf(nm, 64, "blk.%d.%s", i, proj[j]);
            ADD(nm, sp->layer_type[j], pk[j], pn[j], 0);
        }
    }
#undef ADD

    wr w = {fopen(path, "wb"), 1};
    if (!w.f) {
        free(ts);
        return -1;
    }
    const int n_kv = 19;
    put(&w, "GGUF", 4);
    put_u32(&w, 3);
    put_u64(&w, (uint64_t)nt);
    put_u64(&w, (uint64_t)n_kv);
    kv_str(&w, "general.architecture", "hunyuan-dense");
    kv_str(&w, "general.name", reftool ? "bench" : "hysynth");
    kv_u32(&w, "hunyuan-dense.embedding_length", (uint32_t)H);
    kv_u32(&w, "hunyuan-dense.block_count", (uint32_t)sp->n_layer);
    kv_u32(&w, "hunyuan-dense.feed_forward_length", (uint32_t)F);
    kv_u32(&w, "hunyuan-dense.attention.head_count", (uint32_t)sp->heads);
    kv_u32(&w, "hunyuan-dense.attention.head_count_kv", (uint32_t)sp->kv_heads);
    kv_u32(&w, "hunyuan-dense.attention.key_length", (uint32_t)sp->hdim);
    kv_u32(&w, "hunyuan-dense.rope.dimension_count", (uint32_t)sp->hdim);
    kv_f32(&w, "hunyuan-dense.rope.freq_base", sp->freq_base);
    kv_f32(&w, "hunyuan-dense.rope.scaling.alpha", sp->rope_alpha);
    kv_f32(&w, "hunyuan-dense.attention.layer_norm_rms_epsilon", sp->eps);
    kv_str(&w, "tokenizer.ggml.pre", "hunyuan-dense");
    kv_u32(&w, "tokenizer.ggml.bos_token_id", 1);
    kv_u32(&w, "tokenizer.ggml.eos_token_id", 2);
    kv_u32(&w, "tokenizer.ggml.unknown_token_id", 0);
    kv_str(&w, "tokenizer.ggml.model", "gpt2");
    kv_str(&w, "general.file_type", "x");
    put_str(&w, "tokenizer.ggml.tokens");
    put_u32(&w, 9);
    put_u32(&w, 8);
    put_u64(&w, V);
    for (uint64_t i = 0; i < V; i++) {
        char b[24];
        snprintf(b, sizeof b, "t%llu", (unsigned long long)i);
        put_str(&w, b);
    }
    for (int i = 0; i < nt; i++) {
        put_str(&w, ts[i].name);
        const uint32_t nd = ts[i].n ? 2 : 1;
        put_u32(&w, nd);
        put_u64(&w, ts[i].k);
        if (nd == 2) put_u64(&w, ts[i].n);
        put_u32(&w, (uint32_t)ts[i].type);
        put_u64(&w, ts[i].off);
    }
    long pos = ftell(w.f);
    while (pos % 32) {
        fputc(0, w.f);
        pos++;
    }

    rng_t r = {reftool, reftool ? 88172645463325252ull : (sp->seed * 0x2545F4914F6CDD1Dull + 0x1234567ull), 0, 0.0};
    const size_t chunk_cap = 1 << 20;
    uint8_t *buf = (uint8_t *)malloc(chunk_cap + 256);
    for (int i = 0; i < nt && w.ok; i++) {
        const tensor *t = &ts[i];
        if (t->type == 0) {
            /* norms: 1.0, optionally 1 + jitter*N(0,1) */
            for (uint64_t j = 0; j < t->bytes / 4; j++) {
                float v = 1.0f;
                if (!reftool && sp->norm_jitter > 0) v = (float)(1.0 + sp->norm_jitter * normal(&r));
                put(&w, &v, 4);
            }
        } else {
            const size_t bb = block_bytes(t->type);
            const uint64_t nblk = t->bytes / bb;
            size_t fill = 0;
            for (uint64_t b = 0; b < nblk; b++) {
                fill_block(&r, t->type, t->role, sp, buf + fill);
                fill += bb;
                if (fill + bb > chunk_cap) {
                    put(&w, buf, fill);
                    fill = 0;
                }
            }
            put(&w, buf, fill);
        }
        for (uint64_t p = t->bytes; p % 32; p++) fputc(0, w.f);
    }
    free(buf);
    free(ts);
    const int ok = w.ok && fclose(w.f) == 0;
    return ok ? 0 : -2;
}

int hysynth_block_weights(int type) { return block_weights(type); }
