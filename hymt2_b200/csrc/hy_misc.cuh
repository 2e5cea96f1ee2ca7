// hy_misc.cuh — upload-time relayouts, embedding lookup and the decode-step
// bookkeeping kernel (sm_100a).
#pragma once
#include "hy_common.cuh"

namespace hyk {

// ---------------------------------------------------------------- upload relayouts

// Native STQ1_0 / Q2_0C rows -> panel blocks (same bytes the host's
// panel_repack_rows produces, reference src/kernels.c:535-561).  One thread
// per (row, 256-block).
__global__ void panel_from_native(const uint8_t *raw, long long row_bytes, int type, int n, int nb, uint8_t *pk,
                                  float *ps) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)n * nb) return;
    const int r = (int)(i / nb), b = (int)(i % nb);
    const uint8_t *row = raw + (size_t)r * row_bytes;
    uint8_t out[64];
    if (type == GT_STQ1_0) {
        const uint8_t *blk = row + (size_t)b * 42;
        ps[i] = h2f((uint16_t)(blk[40] | (blk[41] << 8)));
        for (int g = 0; g < 64; g++) {
            const int slot = (blk[g >> 1] >> ((g & 1) * 4)) & 0x0f;
            const int sign = (blk[32 + (g >> 3)] >> (g & 7)) & 1;
            out[piece_of_chunk(g >> 4) * 16 + (g & 15)] = (uint8_t)stq_pattern((sign << 4) | slot);
        }
    } else {
        const uint8_t *blk = row + (size_t)(b >> 1) * 130;
        const int base = (b & 1) * 256;
        ps[i] = h2f((uint16_t)(blk[0] | (blk[1] << 8)));
        for (int g = 0; g < 64; g++) {
            const int ch = g >> 4, gi = g & 15;
            int byte = 0;
            for (int l = 0; l < 4; l++) {
                const int wi = base + ch * 64 + gi + 16 * l;
                byte |= ((blk[2 + (wi >> 2)] >> ((wi & 3) * 2)) & 3) << (2 * l);
            }
            out[piece_of_chunk(ch) * 16 + gi] = (uint8_t)byte;
        }
    }
    uint4 *dst = (uint4 *)(pk + (size_t)i * 64);
    for (int j = 0; j < 4; j++) dst[j] = ((const uint4 *)out)[j];
}

// Native STQ1_0 rows (42-byte blocks qs[32] | sign[8] | d) -> the FMT_STQN
// planes: per row qs[nb*32] | sign[nb*8] | d[nb*2], the 8-byte qs chunks and
// 2-byte sign chunks of block b in panel piece order (unit 4b + p holds chunk
// piece_of_chunk(p)), the sign bits bit-sliced (stq_slice_signs).  The same
// 42 bytes per 256 weights.  One thread per (row, block).
__global__ void stqn_from_native(const uint8_t *raw, long long row_bytes, int n, int nb, uint8_t *dst,
                                 long long stride) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)n * nb) return;
    const int r = (int)(i / nb), b = (int)(i % nb);
    const uint8_t *blk = raw + (size_t)r * row_bytes + (size_t)b * 42;
    uint8_t *row = dst + (size_t)r * stride;
    for (int p = 0; p < 4; p++) {
        const int ch = piece_of_chunk(p);
        for (int j = 0; j < 8; j++) row[(size_t)b * 32 + p * 8 + j] = blk[ch * 8 + j];
        const uint32_t sg = stq_slice_signs((uint32_t)blk[32 + 2 * ch] | ((uint32_t)blk[33 + 2 * ch] << 8));
        row[(size_t)nb * 32 + (size_t)b * 8 + p * 2] = (uint8_t)sg;
        row[(size_t)nb * 32 + (size_t)b * 8 + p * 2 + 1] = (uint8_t)(sg >> 8);
    }
    row[(size_t)nb * 40 + (size_t)b * 2] = blk[40];
    row[(size_t)nb * 40 + (size_t)b * 2 + 1] = blk[41];
}

// Q6_K 210-byte blocks -> per-row planes ql | qh | scales | d.
__global__ void q6k_relayout(const uint8_t *raw, int n, int nb, uint8_t *dst, long long stride) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)n * nb) return;
    const int r = (int)(i / nb), b = (int)(i % nb);
    const uint8_t *blk = raw + (size_t)i * 210;
    uint8_t *row = dst + (size_t)r * stride;
    for (int j = 0; j < 128; j++) row[(size_t)b * 128 + j] = blk[j];
    for (int j = 0; j < 64; j++) row[(size_t)nb * 128 + (size_t)b * 64 + j] = blk[128 + j];
    for (int j = 0; j < 16; j++) row[(size_t)nb * 192 + (size_t)b * 16 + j] = blk[192 + j];
    row[(size_t)nb * 208 + 2 * b] = blk[208];
    row[(size_t)nb * 208 + 2 * b + 1] = blk[209];
}

// Q8_0 34-byte blocks -> per-row planes qs | d.
__global__ void q80_relayout(const uint8_t *raw, int n, int nblk, uint8_t *dst, long long stride) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)n * nblk) return;
    const int r = (int)(i / nblk), b = (int)(i % nblk);
    const uint8_t *blk = raw + (size_t)i * 34;
    uint8_t *row = dst + (size_t)r * stride;
    for (int j = 0; j < 32; j++) row[(size_t)b * 32 + j] = blk[2 + j];
    row[(size_t)nblk * 32 + 2 * b] = blk[0];
    row[(size_t)nblk * 32 + 2 * b + 1] = blk[1];
}

// ---------------------------------------------------------------- dequantisation (embedding rows)

// Element e of row r of a device weight, as fp32 (reference dequant_row,
// src/kernels.c:1304-1329, in each format's device layout).
__device__ inline float dequant_elem(const WDesc &w, int r, int e) {
    const uint8_t *row = w.w + (size_t)r * w.stride;
    const int nb = w.k / 256, b = e >> 8, x = e & 255;
    switch (w.fmt) {
    case FMT_PANEL: {
        const int ch = x >> 6, l = (x >> 4) & 3, i = x & 15;
        const uint8_t byte = row[(size_t)b * 64 + piece_of_chunk(ch) * 16 + i];
        const int code = (byte >> (2 * l)) & 3;
        return (float)(code * (1 << w.shift) - w.off) * w.s[(size_t)r * nb + b];
    }
    case FMT_STQN: {
        const int ch = x >> 6, l = (x >> 4) & 3, g = x & 15, u = b * 4 + piece_of_chunk(ch);
        const int slot = (row[(size_t)u * 8 + (g >> 1)] >> ((g & 1) * 4)) & 15;
        const uint32_t sg = row[(size_t)nb * 32 + u * 2] | ((uint32_t)row[(size_t)nb * 32 + u * 2 + 1] << 8);
        const int sign = (sg >> (4 * (g & 3) + (g >> 2))) & 1;
        const int code = (stq_pattern((sign << 4) | slot) >> (2 * l)) & 3;
        return (float)(code - 1) * h2f((uint16_t)(row[(size_t)nb * 40 + 2 * b] | (row[(size_t)nb * 40 + 2 * b + 1] << 8)));
    }
    case FMT_Q6K: {
        const int half = x >> 7, q = (x & 127) >> 5, l = x & 31;
        const uint8_t lb = row[(size_t)b * 128 + half * 64 + l + (q & 1) * 32];
        const int lo = (q & 2) ? (lb >> 4) : (lb & 15);
        const int hi = (row[(size_t)nb * 128 + (size_t)b * 64 + half * 32 + l] >> (2 * q)) & 3;
        const int8_t sc = (int8_t)row[(size_t)nb * 192 + (size_t)b * 16 + half * 8 + 2 * q + (l >> 4)];
        const float d = h2f((uint16_t)(row[(size_t)nb * 208 + 2 * b] | (row[(size_t)nb * 208 + 2 * b + 1] << 8)));
        return d * (float)sc * (float)((lo | (hi << 4)) - 32);
    }
    case FMT_Q4K: {
        const uint8_t *blk = row + (size_t)b * 144;
        const int g = x >> 6, hi = (x >> 5) & 1, l = x & 31;
        int sc, mn;
        const int j = 2 * g + hi;
        const uint8_t *q = blk + 4;
        if (j < 4) { sc = q[j] & 63; mn = q[j + 4] & 63; }
        else { sc = (q[j + 4] & 0x0f) | ((q[j - 4] >> 6) << 4); mn = (q[j + 4] >> 4) | ((q[j] >> 6) << 4); }
        const float d = h2f((uint16_t)(blk[0] | (blk[1] << 8))), dm = h2f((uint16_t)(blk[2] | (blk[3] << 8)));
        const uint8_t qb = blk[16 + 32 * g + l];
        const int v = hi ? (qb >> 4) : (qb & 15);
        return __fsub_rn(__fmul_rn(__fmul_rn(d, (float)sc), (float)v), __fmul_rn(dm, (float)mn));
    }
    case FMT_Q80: {
        const int blk = e >> 5;
        const float d = h2f((uint16_t)(row[w.k + 2 * blk] | (row[w.k + 2 * blk + 1] << 8)));
        return d * (float)(int8_t)row[e];
    }
    case FMT_F16:
        return h2f(((const uint16_t *)row)[e]);
    default:
        return ((const float *)row)[e];
    }
}

// h[t][:] = embedding row of tokens[t]; out-of-range ids read row 0.
__global__ void embed_rows(const __grid_constant__ WDesc w, const int *tokens, float *h, int trace) {
    trace_mark(trace, 0);
    pdl_trigger();
    pdl_wait();
    trace_mark(trace, 1);
    int tok = tokens[blockIdx.x];
    if (tok < 0 || tok >= w.n) tok = 0;
    for (int e = threadIdx.x; e < w.k; e += blockDim.x) h[(size_t)blockIdx.x * w.k + e] = dequant_elem(w, tok, e);
    trace_mark(trace, 3);
}

__global__ void dequant_row_kernel(const __grid_constant__ WDesc w, int r, float *dst) {
    for (int e = threadIdx.x; e < w.k; e += blockDim.x) dst[e] = dequant_elem(w, r, e);
}

// ---------------------------------------------------------------- decode-step bookkeeping

struct DecodeState {
    unsigned long long amax;  // argmax key of the last head launch (0 = none)
    int tok;                  // token to process next
    int pos;                  // its position
    int step;                 // tokens emitted so far
    int cap;                  // capacity of out_ids
    int stopped;              // a stop id was emitted
    int n_stop;
    int pos_fwd;              // first position of a prefill chunk / host forward
    int pad;
    int stop_ids[16];
};

// Consume the argmax: emit the token, advance the position, reset the key.
__global__ void decode_finalize(DecodeState *st, int *out_ids, int trace) {
    trace_mark(trace, 0);
    pdl_trigger();
    pdl_wait();
    trace_mark(trace, 1);
    if (threadIdx.x == 0) {
        const unsigned long long key = st->amax;
        const int idx = key ? (int)argmax_index(key) : 0;
        if (!st->stopped) {
            if (st->step < st->cap) out_ids[st->step] = idx;
            st->step++;
            for (int i = 0; i < st->n_stop; i++)
                if (st->stop_ids[i] == idx) st->stopped = 1;
        }
        st->tok = idx;
        st->pos = st->pos + 1;
        st->amax = 0ull;
    }
    trace_mark(trace, 3);
}

}  // namespace hyk
