/* hy_oracle.c — CPU restatement of the hymt2 hot path (TEST INFRASTRUCTURE).
 *
 * This file is the checker for the CUDA backend, nothing else: the product
 * library never links or loads it.  Each function states which reference
 * lines (zhangbo8418/hymt2, paths relative to the project root) it restates.
 * The restatement is scalar and deterministic: row loops run on several
 * threads but every output element is produced by one thread in a fixed
 * order, so results do not depend on the thread count.  Built with
 * -ffp-contract=off so no multiply-add is fused.
 */
#include "hy_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

/* ------------------------------------------------------------ parallel rows */

static int g_threads = 0;

void orc_set_threads(int n) { g_threads = n; }

static int nthreads(void) {
    if (g_threads > 0) return g_threads;
    long c = sysconf(_SC_NPROCESSORS_ONLN);
    return c < 1 ? 1 : (c > 64 ? 64 : (int)c);
}

typedef void (*range_fn)(void *ctx, int begin, int end);
typedef struct {
    range_fn fn;
    void *ctx;
    int begin, end;
} range_job;

static void *range_run(void *p) {
    range_job *j = (range_job *)p;
    j->fn(j->ctx, j->begin, j->end);
    return NULL;
}

/* Static split of [0, n) over threads; each index is handled by exactly one
 * thread, so the result never depends on the thread count. */
static void par_for(int n, range_fn fn, void *ctx) {
    int nt = nthreads();
    if (nt > n) nt = n;
    if (nt <= 1 || n < 64) {
        fn(ctx, 0, n);
        return;
    }
    pthread_t th[64];
    range_job jobs[64];
    for (int i = 0; i < nt; i++) {
        jobs[i].fn = fn;
        jobs[i].ctx = ctx;
        jobs[i].begin = (int)((long)n * i / nt);
        jobs[i].end = (int)((long)n * (i + 1) / nt);
    }
    for (int i = 1; i < nt; i++) pthread_create(&th[i], NULL, range_run, &jobs[i]);
    range_run(&jobs[0]);
    for (int i = 1; i < nt; i++) pthread_join(th[i], NULL);
}

/* ------------------------------------------------------------ conversions */

/* IEEE binary16 -> binary32 (exact).  Restates src/kernels.c:75-97. */
float orc_f16_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h >> 15) << 31;
    const uint32_t e = (h >> 10) & 0x1f, m = h & 0x3ff;
    uint32_t bits;
    if (e == 0x1f) {
        bits = sign | 0x7f800000u | (m << 13);
    } else if (e == 0) {
        /* zero or subnormal: m * 2^-24 is exact in binary32 */
        float v = ldexpf((float)m, -24);
        memcpy(&bits, &v, 4);
        bits |= sign;
    } else {
        bits = sign | ((e + 112u) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* Round-to-nearest-even to bfloat16.  Restates src/kernels.c:107-111. */
uint16_t orc_f32_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    const uint32_t lsb = (u >> 16) & 1u;
    return (uint16_t)((u + 0x7fffu + lsb) >> 16);
}

float orc_bf16_to_f32(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* ------------------------------------------------------------ Q8_K quantiser */

/* Lane-major copy order of the four 64-wide chunks (src/internal.h:33). */
static const int kPieceOrder[4] = {0, 2, 1, 3};

/* Restates src/kernels.c:128-165: signed value of the FIRST element of largest
 * magnitude, iscale = -127/max, d = 1/iscale, round-half-even, clip to +-127,
 * 16-wide partial sums, total sum, then the lane-major `qp` copy. */
void orc_quantize_q8k(const float *x, int k, q8k_block *y) {
    for (int b = 0; b < k / QK_K; b++) {
        const float *src = x + (size_t)b * QK_K;
        q8k_block *blk = &y[b];
        float best_abs = 0.f, best = 0.f;
        for (int j = 0; j < QK_K; j++) {
            const float a = fabsf(src[j]);
            if (a > best_abs) {
                best_abs = a;
                best = src[j];
            }
        }
        memset(blk, 0, sizeof(*blk));
        if (best_abs == 0.f) continue;
        const float iscale = -127.f / best;
        blk->d = 1.f / iscale;
        int total = 0;
        for (int s = 0; s < QK_K / 16; s++) {
            int part = 0;
            for (int j = s * 16; j < s * 16 + 16; j++) {
                /* the reference narrows lrintf's long to int before clipping
                 * (so a non-finite product becomes 0 on x86-64) */
                int v = (int)lrintf(iscale * src[j]);
                if (v > 127) v = 127;
                if (v < -127) v = -127;
                blk->qs[j] = (int8_t)v;
                part += v;
            }
            blk->bsums[s] = (int16_t)part;
            total += part;
        }
        blk->sum = total;
        for (int lane = 0; lane < 4; lane++)
            for (int p = 0; p < 4; p++)
                memcpy(blk->qp + lane * 64 + p * 16, blk->qs + kPieceOrder[p] * 64 + lane * 16, 16);
    }
}

void orc_quantize_rows(const float *x, int nt, int k, q8k_block *y) {
    for (int t = 0; t < nt; t++) orc_quantize_q8k(x + (size_t)t * k, k, y + (size_t)t * (k / QK_K));
}

/* ------------------------------------------------------------ formats */

/* Bytes per row of each GGUF encoding (src/kernels.c:113-125). */
size_t orc_row_size(int type, int k) {
    switch (type) {
    case GT_F32: return (size_t)k * 4;
    case GT_F16: return (size_t)k * 2;
    case GT_Q8_0: return (size_t)(k / 32) * 34;
    case GT_Q4_K: return (size_t)(k / QK_K) * 144;
    case GT_Q6_K: return (size_t)(k / QK_K) * 210;
    case GT_STQ1_0: return (size_t)(k / QK_K) * 42;
    case GT_Q2_0C: return (size_t)(k / 512) * 130;
    }
    return 0;
}

/* STQ1_0 4-weight group patterns, index (sign<<4)|slot, 2-bit lane codes
 * 0,1,2 = -1,0,+1.  This table is part of the file format; it must equal
 * src/kernels.c:178-181 entry for entry. */
static const uint8_t kStqPatterns[32] = {
    0xA9, 0x89, 0x29, 0x09, 0xA6, 0x86, 0x26, 0x06, 0x9A, 0x92, 0x1A, 0x12, 0x6A, 0x62, 0x4A, 0x42,
    0x01, 0x21, 0x81, 0xA1, 0x04, 0x24, 0x84, 0xA4, 0x10, 0x18, 0x90, 0x98, 0x40, 0x48, 0x60, 0x68,
};

/* STQ1_0 block: qs[32] 4-bit slots, sign[8] bits, f16 d (src/internal.h:22).
 * Group g's pattern (src/kernels.c:184-188). */
static uint8_t stq_group(const uint8_t *blk, int g) {
    const int slot = (blk[g >> 1] >> ((g & 1) * 4)) & 0x0f;
    const int sign = (blk[32 + (g >> 3)] >> (g & 7)) & 1;
    return kStqPatterns[(sign << 4) | slot];
}

static uint16_t rd16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }

/* Panel repack (src/kernels.c:535-561).  Byte `i` of piece `p` in a 64-byte
 * panel block holds lanes 0..3 (2 bits each) of 4-group i of chunk
 * kPieceOrder[p]; lane l is weight chunk*64 + i + 16*l. */
typedef struct {
    int type, nb;
    const uint8_t *data;
    size_t row_bytes;
    uint8_t *pk;
    float *ps;
} repack_ctx;

static void repack_range(void *c, int r0, int r1) {
    const repack_ctx *x = (const repack_ctx *)c;
    const int type = x->type, nb = x->nb;
    const uint8_t *data = x->data;
    const size_t row_bytes = x->row_bytes;
    uint8_t *pk = x->pk;
    float *ps = x->ps;
    for (int r = r0; r < r1; r++) {
        const uint8_t *row = data + (size_t)r * row_bytes;
        for (int b = 0; b < nb; b++) {
            uint8_t *dst = pk + ((size_t)r * nb + b) * 64;
            if (type == GT_STQ1_0) {
                const uint8_t *blk = row + (size_t)b * 42;
                ps[(size_t)r * nb + b] = orc_f16_to_f32(rd16(blk + 40));
                for (int g = 0; g < 64; g++) dst[kPieceOrder[g >> 4] * 16 + (g & 15)] = stq_group(blk, g);
            } else { /* Q2_0C: 512-weight block, two 256 halves share d */
                const uint8_t *blk = row + (size_t)(b >> 1) * 130;
                const int base = (b & 1) * 256;
                ps[(size_t)r * nb + b] = orc_f16_to_f32(rd16(blk));
                for (int g = 0; g < 64; g++) {
                    const int chunk = g >> 4, i = g & 15;
                    int byte = 0;
                    for (int l = 0; l < 4; l++) {
                        const int w = base + chunk * 64 + i + 16 * l;
                        byte |= ((blk[2 + (w >> 2)] >> ((w & 3) * 2)) & 3) << (2 * l);
                    }
                    dst[kPieceOrder[chunk] * 16 + i] = (uint8_t)byte;
                }
            }
        }
    }
}

void orc_panel_repack(int type, const uint8_t *data, size_t row_bytes, int n, int k, uint8_t *pk, float *ps) {
    repack_ctx c = {type, k / QK_K, data, row_bytes, pk, ps};
    par_for(n, repack_range, &c);
}

/* ------------------------------------------------------------ exact per-block integers */

/* Panel block: (enc << pshift) - poff*sum, enc = sum_l sum_i code_l(pk[i]) * qp[l*64+i]
 * (src/kernels.c:571-577). */
static int32_t panel_block_int(const uint8_t *pk, const q8k_block *y, int pshift, int poff) {
    int32_t enc = 0;
    for (int l = 0; l < 4; l++)
        for (int i = 0; i < 64; i++) enc += ((pk[i] >> (2 * l)) & 3) * (int32_t)y->qp[l * 64 + i];
    return enc * (1 << pshift) - poff * y->sum;
}

/* Q4_K 6-bit scale/min unpacking (src/kernels.c:839-842). */
static void q4k_scale_min(const uint8_t *s, int j, int *sc, int *mn) {
    if (j < 4) {
        *sc = s[j] & 63;
        *mn = s[j + 4] & 63;
    } else {
        *sc = (s[j + 4] & 0x0f) | ((s[j - 4] >> 6) << 4);
        *mn = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

/* Q4_K block (d, dmin, scales[12], qs[128]): sumi and summ of
 * src/kernels.c:861-877. */
static void q4k_block_ints(const uint8_t *blk, const q8k_block *y, int32_t *sumi, int32_t *summ) {
    const uint8_t *sc = blk + 4, *qs = blk + 16;
    int32_t si = 0, sm = 0;
    for (int g = 0; g < 4; g++) {
        int s_lo, m_lo, s_hi, m_hi;
        q4k_scale_min(sc, 2 * g, &s_lo, &m_lo);
        q4k_scale_min(sc, 2 * g + 1, &s_hi, &m_hi);
        int32_t a = 0, c = 0;
        for (int l = 0; l < 32; l++) {
            a += (qs[32 * g + l] & 0x0f) * (int32_t)y->qs[64 * g + l];
            c += (qs[32 * g + l] >> 4) * (int32_t)y->qs[64 * g + 32 + l];
        }
        si += s_lo * a + s_hi * c;
        sm += m_lo * (y->bsums[4 * g] + y->bsums[4 * g + 1]) + m_hi * (y->bsums[4 * g + 2] + y->bsums[4 * g + 3]);
    }
    *sumi = si;
    *summ = sm;
}

/* Q6_K 6-bit code of element e (0..255) of a block (ql[128], qh[64], sc[16], d):
 * layout of src/kernels.c:786-806. */
static int q6k_code(const uint8_t *blk, int e) {
    const uint8_t *ql = blk, *qh = blk + 128;
    const int half = e >> 7, w = e & 127, quarter = w >> 5, l = w & 31;
    const uint8_t lo_byte = ql[half * 64 + l + ((quarter & 1) ? 32 : 0)];
    const int lo = (quarter & 2) ? (lo_byte >> 4) : (lo_byte & 0x0f);
    const int hi = (qh[half * 32 + l] >> (2 * quarter)) & 3;
    return (lo | (hi << 4)) - 32;
}

/* Q6_K block: sum_j sc_j * sum_{16} q6*q8 (src/kernels.c:808-835). */
static int32_t q6k_block_int(const uint8_t *blk, const q8k_block *y) {
    const int8_t *sc = (const int8_t *)(blk + 192);
    int32_t acc = 0;
    for (int j = 0; j < 16; j++) {
        int32_t t = 0;
        for (int l = 0; l < 16; l++) t += q6k_code(blk, 16 * j + l) * (int32_t)y->qs[16 * j + l];
        acc += sc[j] * t;
    }
    return acc;
}

/* Q2_0C half block: sum_j (2c-3) * q8 over 256 (src/kernels.c:1222-1237). */
static int32_t q2c_half_int(const uint8_t *blk, int half, const q8k_block *y) {
    const uint8_t *qs = blk + 2;
    int32_t s = 0;
    for (int j = 0; j < 256; j++) {
        const int w = half * 256 + j;
        s += (2 * ((qs[w >> 2] >> ((w & 3) * 2)) & 3) - 3) * (int32_t)y->qs[j];
    }
    return s;
}

typedef struct {
    const weight_t *w;
    const q8k_block *y;
    int32_t *out;
    int t, per;
} ints_ctx;

static void ints_range(void *c, int r0, int r1) {
    const ints_ctx *x = (const ints_ctx *)c;
    const weight_t *w = x->w;
    const q8k_block *y = x->y;
    const int nb = w->k / QK_K, per = x->per, t = x->t;
    int32_t *out = x->out;
    {
        {
        for (int r = r0; r < r1; r++) {
            int32_t *o = out + ((size_t)t * w->n + r) * per;
            const uint8_t *row = w->data ? w->data + (size_t)r * w->row_bytes : NULL;
            for (int b = 0; b < nb; b++) {
                if (w->pk) o[b] = panel_block_int(w->pk + ((size_t)r * nb + b) * 64, y + b, w->pshift, w->poff);
                else if (w->type == GT_Q4_K) q4k_block_ints(row + (size_t)b * 144, y + b, &o[2 * b], &o[2 * b + 1]);
                else if (w->type == GT_Q6_K) o[b] = q6k_block_int(row + (size_t)b * 210, y + b);
                else if (w->type == GT_Q2_0C) o[b] = q2c_half_int(row + (size_t)(b >> 1) * 130, b & 1, y + b);
                else if (w->type == GT_STQ1_0) {
                    /* native STQ1_0: sum (code-1)*q8 (src/kernels.c:202-215) */
                    const uint8_t *blk = row + (size_t)b * 42;
                    int32_t s = 0;
                    for (int g = 0; g < 64; g++) {
                        const uint8_t p = stq_group(blk, g);
                        for (int l = 0; l < 4; l++) s += (((p >> (2 * l)) & 3) - 1) * (int32_t)y[b].qs[(g >> 4) * 64 + (g & 15) + 16 * l];
                    }
                    o[b] = s;
                } else o[b] = 0;
            }
        }
        }
    }
}

int orc_block_ints(const weight_t *w, const q8k_block *xq, int nt, int32_t *out) {
    const int nb = w->k / QK_K;
    const int per = (w->type == GT_Q4_K && !w->pk) ? 2 * nb : nb;
    for (int t = 0; t < nt; t++) {
        ints_ctx c = {w, xq + (size_t)t * nb, out, t, per};
        par_for(w->n, ints_range, &c);
    }
    return per;
}

/* ------------------------------------------------------------ fp32 row results */

/* out[t*n + r] as in src/kernels.c:1241-1302 (scalar combination order). */
typedef struct {
    const weight_t *w;
    const float *xf;
    const q8k_block *xq;
    int nt;
    float *out;
} mm_ctx;

/* Accumulation precision of orc_matmul: 0 = float (the host's order), 1 =
 * double (the float64 reference the reference's own model test compares
 * against to measure its rounding spread, tests/test_model.py:353-364). */
static int g_f64 = 0;
void orc_set_f64(int on) { g_f64 = on; }

static void matmul_range_f64(const mm_ctx *x, int r0, int r1);

static void matmul_range(void *c, int r0, int r1) {
    const mm_ctx *x = (const mm_ctx *)c;
    if (g_f64) {
        matmul_range_f64(x, r0, r1);
        return;
    }
    const weight_t *w = x->w;
    const float *xf = x->xf;
    const q8k_block *xq = x->xq;
    const int nt = x->nt, nb = w->k / QK_K;
    float *out = x->out;
    for (int r = r0; r < r1; r++) {
        const uint8_t *row = w->data ? w->data + (size_t)r * w->row_bytes : NULL;
        for (int t = 0; t < nt; t++) {
            float acc = 0.f;
            if (w->pk) {
                const q8k_block *y = xq + (size_t)t * nb;
                for (int b = 0; b < nb; b++)
                    acc += w->ps[(size_t)r * nb + b] * y[b].d *
                           (float)panel_block_int(w->pk + ((size_t)r * nb + b) * 64, y + b, w->pshift, w->poff);
            } else {
                switch (w->type) {
                case GT_Q4_K: {
                    const q8k_block *y = xq + (size_t)t * nb;
                    for (int b = 0; b < nb; b++) {
                        int32_t si, sm;
                        q4k_block_ints(row + (size_t)b * 144, y + b, &si, &sm);
                        acc += y[b].d * (orc_f16_to_f32(rd16(row + (size_t)b * 144)) * (float)si -
                                         orc_f16_to_f32(rd16(row + (size_t)b * 144 + 2)) * (float)sm);
                    }
                    break;
                }
                case GT_Q6_K: {
                    const q8k_block *y = xq + (size_t)t * nb;
                    for (int b = 0; b < nb; b++)
                        acc += orc_f16_to_f32(rd16(row + (size_t)b * 210 + 208)) * y[b].d *
                               (float)q6k_block_int(row + (size_t)b * 210, y + b);
                    break;
                }
                case GT_Q2_0C: {
                    const q8k_block *y = xq + (size_t)t * nb;
                    for (int b = 0; b < nb / 2; b++) {
                        const uint8_t *blk = row + (size_t)b * 130;
                        float part = 0.f;
                        for (int h = 0; h < 2; h++) part += (float)q2c_half_int(blk, h, y + 2 * b + h) * y[2 * b + h].d;
                        acc += orc_f16_to_f32(rd16(blk)) * part;
                    }
                    break;
                }
                case GT_STQ1_0: {
                    /* native STQ1_0 (src/kernels.c:202-215) */
                    const q8k_block *y = xq + (size_t)t * nb;
                    for (int b = 0; b < nb; b++) {
                        const uint8_t *blk = row + (size_t)b * 42;
                        int32_t s = 0;
                        for (int g = 0; g < 64; g++) {
                            const uint8_t p = stq_group(blk, g);
                            for (int l = 0; l < 4; l++)
                                s += (((p >> (2 * l)) & 3) - 1) * (int32_t)y[b].qs[(g >> 4) * 64 + (g & 15) + 16 * l];
                        }
                        acc += orc_f16_to_f32(rd16(blk + 40)) * y[b].d * (float)s;
                    }
                    break;
                }
                case GT_Q8_0: {
                    const float *x = xf + (size_t)t * w->k;
                    for (int b = 0; b < w->k / 32; b++) {
                        const uint8_t *blk = row + (size_t)b * 34;
                        float s = 0.f;
                        for (int j = 0; j < 32; j++) s += (float)(int8_t)blk[2 + j] * x[b * 32 + j];
                        acc += orc_f16_to_f32(rd16(blk)) * s;
                    }
                    break;
                }
                case GT_F16: {
                    const float *x = xf + (size_t)t * w->k;
                    for (int j = 0; j < w->k; j++) acc += orc_f16_to_f32(rd16(row + 2 * (size_t)j)) * x[j];
                    break;
                }
                case GT_F32: {
                    const float *x = xf + (size_t)t * w->k;
                    for (int j = 0; j < w->k; j++) {
                        float v;
                        memcpy(&v, row + 4 * (size_t)j, 4);
                        acc += v * x[j];
                    }
                    break;
                }
                }
            }
            out[(size_t)t * w->n + r] = acc;
        }
    }
}


/* The same rows with every product and sum in double; weights and Q8_K
 * activations enter exactly as in the float path. */
static void matmul_range_f64(const mm_ctx *x, int r0, int r1) {
    const weight_t *w = x->w;
    const int nt = x->nt, nb = w->k / QK_K;
    for (int r = r0; r < r1; r++) {
        const uint8_t *row = w->data ? w->data + (size_t)r * w->row_bytes : NULL;
        for (int t = 0; t < nt; t++) {
            double acc = 0.0;
            const q8k_block *y = x->xq + (size_t)t * nb;
            const float *xf = x->xf + (size_t)t * w->k;
            if (w->pk) {
                for (int b = 0; b < nb; b++)
                    acc += (double)w->ps[(size_t)r * nb + b] * (double)y[b].d *
                           (double)panel_block_int(w->pk + ((size_t)r * nb + b) * 64, y + b, w->pshift, w->poff);
            } else if (w->type == GT_Q4_K) {
                for (int b = 0; b < nb; b++) {
                    int32_t si, sm;
                    q4k_block_ints(row + (size_t)b * 144, y + b, &si, &sm);
                    acc += (double)y[b].d * ((double)orc_f16_to_f32(rd16(row + (size_t)b * 144)) * si -
                                             (double)orc_f16_to_f32(rd16(row + (size_t)b * 144 + 2)) * sm);
                }
            } else if (w->type == GT_Q6_K) {
                for (int b = 0; b < nb; b++)
                    acc += (double)orc_f16_to_f32(rd16(row + (size_t)b * 210 + 208)) * (double)y[b].d *
                           (double)q6k_block_int(row + (size_t)b * 210, y + b);
            } else if (w->type == GT_Q2_0C) {
                for (int b = 0; b < nb / 2; b++) {
                    const uint8_t *blk = row + (size_t)b * 130;
                    double part = 0.0;
                    for (int h = 0; h < 2; h++) part += (double)q2c_half_int(blk, h, y + 2 * b + h) * (double)y[2 * b + h].d;
                    acc += (double)orc_f16_to_f32(rd16(blk)) * part;
                }
            } else {
                float *deq = (float *)malloc(sizeof(float) * (size_t)w->k);
                orc_dequant_row(w, r, deq);
                if (w->type == GT_STQ1_0) {
                    for (int j = 0; j < w->k; j++)
                        acc += (double)deq[j] * (double)y[j / QK_K].qs[j % QK_K] * (double)y[j / QK_K].d;
                } else {
                    for (int j = 0; j < w->k; j++) acc += (double)deq[j] * (double)xf[j];
                }
                free(deq);
            }
            x->out[(size_t)t * w->n + r] = (float)acc;
        }
    }
}

void orc_matmul(const weight_t *w, const float *xf, const q8k_block *xq, int nt, float *out) {
    mm_ctx c = {w, xf, xq, nt, out};
    par_for(w->n, matmul_range, &c);
}

/* One row to fp32 (src/kernels.c:1304-1329). */
void orc_dequant_row(const weight_t *w, int row, float *dst) {
    const uint8_t *p = w->data + (size_t)row * w->row_bytes;
    switch (w->type) {
    case GT_F32: memcpy(dst, p, (size_t)w->k * 4); break;
    case GT_F16:
        for (int j = 0; j < w->k; j++) dst[j] = orc_f16_to_f32(rd16(p + 2 * (size_t)j));
        break;
    case GT_Q8_0:
        for (int b = 0; b < w->k / 32; b++) {
            const float d = orc_f16_to_f32(rd16(p + (size_t)b * 34));
            for (int j = 0; j < 32; j++) dst[b * 32 + j] = d * (float)(int8_t)p[(size_t)b * 34 + 2 + j];
        }
        break;
    case GT_Q4_K:
        for (int b = 0; b < w->k / QK_K; b++) {
            const uint8_t *blk = p + (size_t)b * 144;
            const float d = orc_f16_to_f32(rd16(blk)), dm = orc_f16_to_f32(rd16(blk + 2));
            for (int g = 0; g < 4; g++) {
                int s0, m0, s1, m1;
                q4k_scale_min(blk + 4, 2 * g, &s0, &m0);
                q4k_scale_min(blk + 4, 2 * g + 1, &s1, &m1);
                const float d0 = d * (float)s0, n0 = dm * (float)m0, d1 = d * (float)s1, n1 = dm * (float)m1;
                for (int l = 0; l < 32; l++) {
                    dst[b * 256 + 64 * g + l] = d0 * (float)(blk[16 + 32 * g + l] & 0x0f) - n0;
                    dst[b * 256 + 64 * g + 32 + l] = d1 * (float)(blk[16 + 32 * g + l] >> 4) - n1;
                }
            }
        }
        break;
    case GT_Q6_K:
        for (int b = 0; b < w->k / QK_K; b++) {
            const uint8_t *blk = p + (size_t)b * 210;
            const float d = orc_f16_to_f32(rd16(blk + 208));
            const int8_t *sc = (const int8_t *)(blk + 192);
            for (int e = 0; e < 256; e++) {
                /* d * sc * q, evaluated left to right as in src/kernels.c:800-803 */
                const int half = e >> 7, w128 = e & 127;
                const int sub = half * 8 + (w128 >> 5) * 2 + ((w128 & 31) >> 4);
                dst[b * 256 + e] = d * (float)sc[sub] * (float)q6k_code(blk, e);
            }
        }
        break;
    case GT_STQ1_0:
        for (int b = 0; b < w->k / QK_K; b++) {
            const uint8_t *blk = p + (size_t)b * 42;
            const float d = orc_f16_to_f32(rd16(blk + 40));
            for (int g = 0; g < 64; g++) {
                const uint8_t pat = stq_group(blk, g);
                for (int l = 0; l < 4; l++)
                    dst[b * 256 + (g >> 4) * 64 + (g & 15) + 16 * l] = (float)(((pat >> (2 * l)) & 3) - 1) * d;
            }
        }
        break;
    case GT_Q2_0C:
        for (int b = 0; b < w->k / 512; b++) {
            const uint8_t *blk = p + (size_t)b * 130;
            const float d = orc_f16_to_f32(rd16(blk));
            for (int j = 0; j < 512; j++)
                dst[b * 512 + j] = (float)(2 * ((blk[2 + (j >> 2)] >> ((j & 3) * 2)) & 3) - 3) * d;
        }
        break;
    }
}

/* ------------------------------------------------------------ model forward */

struct orc_model {
    orc_model_desc d;
    int qdim, kvdim, vocab_out, nb_max;
    float *rope_cos, *rope_sin;
    uint16_t **kc, **vc;
    float *h, *xn, *q, *k, *v, *ao, *g, *u, *tmp;
    q8k_block *xq;
};

orc_model *orc_model_create(const orc_model_desc *d) {
    orc_model *m = (orc_model *)calloc(1, sizeof(*m));
    m->d = *d;
    m->qdim = d->heads * d->hdim;
    m->kvdim = d->kv_heads * d->hdim;
    m->vocab_out = d->outw.n;
    const int half = d->rope_half;
    /* RoPE tables exactly as the loader builds them (src/model.c:576-586). */
    m->rope_cos = (float *)malloc(sizeof(float) * (size_t)d->ctx * half);
    m->rope_sin = (float *)malloc(sizeof(float) * (size_t)d->ctx * half);
    for (int i = 0; i < half; i++) {
        const float freq = 1.0f / powf(d->rope_base, (float)i / (float)half);
        for (int p = 0; p < d->ctx; p++) {
            const float a = (float)p * freq;
            m->rope_cos[(size_t)p * half + i] = cosf(a);
            m->rope_sin[(size_t)p * half + i] = sinf(a);
        }
    }
    m->kc = (uint16_t **)calloc((size_t)d->n_layer, sizeof(uint16_t *));
    m->vc = (uint16_t **)calloc((size_t)d->n_layer, sizeof(uint16_t *));
    for (int l = 0; l < d->n_layer; l++) {
        m->kc[l] = (uint16_t *)calloc((size_t)d->ctx * m->kvdim, 2);
        m->vc[l] = (uint16_t *)calloc((size_t)d->ctx * m->kvdim, 2);
    }
    const size_t B = 256;
    int maxk = d->hidden > d->ffn ? d->hidden : d->ffn;
    if (m->qdim > maxk) maxk = m->qdim;
    m->h = (float *)malloc(4 * B * d->hidden);
    m->xn = (float *)malloc(4 * B * maxk);
    m->q = (float *)malloc(4 * B * m->qdim);
    m->k = (float *)malloc(4 * B * m->kvdim);
    m->v = (float *)malloc(4 * B * m->kvdim);
    m->ao = (float *)malloc(4 * B * m->qdim);
    m->g = (float *)malloc(4 * B * d->ffn);
    m->u = (float *)malloc(4 * B * d->ffn);
    m->tmp = (float *)malloc(4 * B * d->hidden);
    m->xq = (q8k_block *)aligned_alloc(64, sizeof(q8k_block) * B * (maxk / QK_K));
    return m;
}

void orc_model_free(orc_model *m) {
    if (!m) return;
    for (int l = 0; l < m->d.n_layer; l++) {
        free(m->kc[l]);
        free(m->vc[l]);
    }
    free(m->kc); free(m->vc); free(m->rope_cos); free(m->rope_sin);
    free(m->h); free(m->xn); free(m->q); free(m->k); free(m->v); free(m->ao); free(m->g); free(m->u); free(m->tmp);
    free(m->xq);
    free(m);
}

void orc_model_reset(orc_model *m) {
    for (int l = 0; l < m->d.n_layer; l++) {
        memset(m->kc[l], 0, (size_t)m->d.ctx * m->kvdim * 2);
        memset(m->vc[l], 0, (size_t)m->d.ctx * m->kvdim * 2);
    }
}

int orc_vocab_out(const orc_model *m) { return m->vocab_out; }
const uint16_t *orc_kcache(const orc_model *m, int layer) { return m->kc[layer]; }
const uint16_t *orc_vcache(const orc_model *m, int layer) { return m->vc[layer]; }

/* RMSNorm, sequential fp32 sum (src/model.c:719-739, non-NEON branch). */
static void rmsnorm(const float *x, const float *w, float *y, int dim, float eps) {
    float ss = 0.f;
    for (int i = 0; i < dim; i++) ss += x[i] * x[i];
    const float scale = 1.0f / sqrtf(ss / (float)dim + eps);
    for (int i = 0; i < dim; i++) y[i] = x[i] * scale * w[i];
}

/* bf16 dot with four interleaved partial sums (src/kernels.c:1111-1121). */
static float dot_bf16(const float *q, const uint16_t *k, int n) {
    float a[4] = {0, 0, 0, 0};
    int d = 0;
    for (; d + 4 <= n; d += 4)
        for (int j = 0; j < 4; j++) a[j] += q[d + j] * orc_bf16_to_f32(k[d + j]);
    float s = (a[0] + a[1]) + (a[2] + a[3]);
    for (; d < n; d++) s += q[d] * orc_bf16_to_f32(k[d]);
    return s;
}

typedef struct {
    int heads, kv_heads, hd, pos0;
    const float *q;
    const uint16_t *kc, *vc;
    float *ao;
} attn_ctx;

static void attn_range(void *c, int i0, int i1) {
    const attn_ctx *a = (const attn_ctx *)c;
    const int QD = a->heads * a->hd, KD = a->kv_heads * a->hd, HD = a->hd;
    const int group = a->heads / a->kv_heads;
    const float scale = 1.0f / sqrtf((float)HD);
    for (int item = i0; item < i1; item++) {
        const int t = item / a->heads, h = item % a->heads, n = a->pos0 + t + 1, kvh = h / group;
        const float *qh = a->q + (size_t)t * QD + (size_t)h * HD;
        const uint16_t *K = a->kc + (size_t)kvh * HD, *V = a->vc + (size_t)kvh * HD;
        float *sc = (float *)malloc(sizeof(float) * (size_t)n);
        float mx = -INFINITY;
        for (int j = 0; j < n; j++) {
            sc[j] = dot_bf16(qh, K + (size_t)j * KD, HD) * scale;
            if (sc[j] > mx) mx = sc[j];
        }
        float sum = 0.f;
        for (int j = 0; j < n; j++) {
            sc[j] = expf(sc[j] - mx);
            sum += sc[j];
        }
        const float inv = 1.0f / sum;
        float *o = a->ao + (size_t)t * QD + (size_t)h * HD;
        for (int d = 0; d < HD; d++) o[d] = 0.f;
        for (int j = 0; j < n; j++) {
            const float p = sc[j] * inv;
            const uint16_t *vr = V + (size_t)j * KD;
            for (int d = 0; d < HD; d++) o[d] += p * orc_bf16_to_f32(vr[d]);
        }
        free(sc);
    }
}

/* Rope (NeoX halves, src/model.c:754-765) + per-head q/k RMSNorm + bf16 KV
 * store for tokens pos0.., then causal
 * GQA softmax attention (src/model.c:836-851 and :768-795).  q, k are
 * modified in place; kc/vc are one layer's [ctx][kvdim] caches. */
void orc_attention(int heads, int kv_heads, int hd, int rope_half, float *q, float *k, const float *v, int nt,
                   int pos0, uint16_t *kc, uint16_t *vc, const float *q_norm, const float *k_norm,
                   const float *rope_cos, const float *rope_sin, float eps, float *ao) {
    const int QD = heads * hd, KD = kv_heads * hd;
    for (int t = 0; t < nt; t++) {
        float *qt = q + (size_t)t * QD, *kt = k + (size_t)t * KD;
        const float *vt = v + (size_t)t * KD;
        const int pos = pos0 + t;
        const float *cs = rope_cos + (size_t)pos * rope_half, *sn = rope_sin + (size_t)pos * rope_half;
        for (int pass = 0; pass < 2; pass++) {
            float *x = pass ? kt : qt;
            const int nh = pass ? kv_heads : heads;
            for (int h = 0; h < nh; h++) {
                float *row = x + (size_t)h * hd;
                for (int i = 0; i < rope_half; i++) {
                    const float a = row[i], b = row[i + rope_half];
                    row[i] = a * cs[i] - b * sn[i];
                    row[i + rope_half] = a * sn[i] + b * cs[i];
                }
            }
        }
        for (int h = 0; h < heads; h++) rmsnorm(qt + h * hd, q_norm, qt + h * hd, hd, eps);
        for (int h = 0; h < kv_heads; h++) rmsnorm(kt + h * hd, k_norm, kt + h * hd, hd, eps);
        uint16_t *kd = kc + (size_t)pos * KD, *vd = vc + (size_t)pos * KD;
        for (int i = 0; i < KD; i++) {
            kd[i] = orc_f32_to_bf16(kt[i]);
            vd[i] = orc_f32_to_bf16(vt[i]);
        }
    }
    attn_ctx ac = {heads, kv_heads, hd, pos0, q, kc, vc, ao};
    par_for(nt * heads, attn_range, &ac);
}

/* The GEMV prologues: rmsnorm(x)*w (mode 2) or silu(x)*x2 (mode 3) per token,
 * then the matmul as the host runs it (src/model.c:824-881). */
void orc_prologue_matmul(const weight_t *w, int mode, const float *x, const float *x2, const float *norm_w, float eps,
                         int nt, float *out) {
    const int K = w->k;
    float *act = (float *)malloc(sizeof(float) * (size_t)nt * K);
    for (int t = 0; t < nt; t++) {
        const float *xt = x + (size_t)t * K;
        float *at = act + (size_t)t * K;
        if (mode == 2) rmsnorm(xt, norm_w, at, K, eps);
        else if (mode == 3)
            for (int i = 0; i < K; i++) {
                const float g = xt[i];
                at[i] = g / (1.0f + expf(-g)) * x2[(size_t)t * K + i];
            }
        else memcpy(at, xt, sizeof(float) * (size_t)K);
    }
    q8k_block *xq = (q8k_block *)aligned_alloc(64, sizeof(q8k_block) * (size_t)nt * (K / QK_K + 1));
    if (K % QK_K == 0) orc_quantize_rows(act, nt, K, xq);
    orc_matmul(w, act, xq, nt, out);
    free(xq);
    free(act);
}

void orc_forward(orc_model *m, const int *toks, int nt, int pos0, float *logits, float *h_out) {
    const orc_model_desc *D = &m->d;
    const int H = D->hidden, QD = m->qdim, F = D->ffn, HD = D->hdim;
    /* embedding (src/model.c:802) */
    for (int t = 0; t < nt; t++) orc_dequant_row(&D->embd, toks[t], m->h + (size_t)t * H);
    for (int li = 0; li < D->n_layer; li++) {
        /* attention block (src/model.c:824-858) */
        for (int t = 0; t < nt; t++) rmsnorm(m->h + (size_t)t * H, D->attn_norm[li], m->xn + (size_t)t * H, H, D->eps);
        orc_quantize_rows(m->xn, nt, H, m->xq);
        orc_matmul(&D->wq[li], m->xn, m->xq, nt, m->q);
        orc_matmul(&D->wk[li], m->xn, m->xq, nt, m->k);
        orc_matmul(&D->wv[li], m->xn, m->xq, nt, m->v);
        orc_attention(D->heads, D->kv_heads, HD, D->rope_half, m->q, m->k, m->v, nt, pos0, m->kc[li], m->vc[li],
                      D->q_norm[li], D->k_norm[li], m->rope_cos, m->rope_sin, D->eps, m->ao);
        orc_quantize_rows(m->ao, nt, QD, m->xq);
        orc_matmul(&D->wo[li], m->ao, m->xq, nt, m->tmp);
        for (size_t i = 0; i < (size_t)nt * H; i++) m->h[i] += m->tmp[i];
        /* feed-forward block (src/model.c:861-882) */
        for (int t = 0; t < nt; t++) rmsnorm(m->h + (size_t)t * H, D->ffn_norm[li], m->xn + (size_t)t * H, H, D->eps);
        orc_quantize_rows(m->xn, nt, H, m->xq);
        orc_matmul(&D->wg[li], m->xn, m->xq, nt, m->g);
        orc_matmul(&D->wu[li], m->xn, m->xq, nt, m->u);
        for (size_t i = 0; i < (size_t)nt * F; i++) {
            const float g = m->g[i];
            m->g[i] = g / (1.0f + expf(-g)) * m->u[i];
        }
        orc_quantize_rows(m->g, nt, F, m->xq);
        orc_matmul(&D->wd[li], m->g, m->xq, nt, m->tmp);
        for (size_t i = 0; i < (size_t)nt * H; i++) m->h[i] += m->tmp[i];
    }
    if (h_out) memcpy(h_out, m->h, sizeof(float) * (size_t)nt * H);
    if (logits) {
        /* head on the last token only (src/model.c:884-899) */
        rmsnorm(m->h + (size_t)(nt - 1) * H, D->out_norm, m->xn, H, D->eps);
        orc_quantize_rows(m->xn, 1, H, m->xq);
        orc_matmul(&D->outw, m->xn, m->xq, 1, logits);
    }
}

/* Prefill in chunks, then greedy argmax steps; first maximum wins
 * (src/model.c:904-909, 945-952). */
int orc_greedy(orc_model *m, const int *ids, int n, int ngen, int chunk, int *out, float *step_logits) {
    float *lg = (float *)malloc(sizeof(float) * (size_t)m->vocab_out);
    if (chunk < 1) chunk = 1;
    for (int i = 0; i < n; i += chunk) {
        const int nt = n - i < chunk ? n - i : chunk;
        orc_forward(m, ids + i, nt, i, i + nt == n ? lg : NULL, NULL);
    }
    int pos = n;
    for (int s = 0; s < ngen; s++) {
        if (step_logits) memcpy(step_logits + (size_t)s * m->vocab_out, lg, sizeof(float) * (size_t)m->vocab_out);
        int best = 0;
        float bv = lg[0];
        for (int j = 1; j < m->vocab_out; j++)
            if (lg[j] > bv) {
                bv = lg[j];
                best = j;
            }
        out[s] = best;
        if (s + 1 == ngen) break;
        orc_forward(m, &best, 1, pos, lg, NULL);
        pos++;
    }
    free(lg);
    return ngen;
}
