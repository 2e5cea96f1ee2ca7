// hy_attn.cuh — GQA causal attention over the bf16 KV cache (sm_100a).
//
// Semantics of reference src/model.c:768-795 and :836-848: q and k are
// NeoX-rotated, then RMS-normalised per head (q_norm / k_norm, AFTER rope); k
// and v are rounded to bf16 into the cache; scores q.k/sqrt(hd) over positions
// 0..pos inclusive; softmax; output = sum p_j v_j.  Computed here with an
// online (running-max) softmax per 32-key tile, one warp per query head of a
// GQA group so each K/V row is read once per group, and split-KV over long
// contexts with a last-CTA log-sum-exp merge.
#pragma once
#include "hy_common.cuh"
#include "hy_pages.h"
#include "hy_tc.cuh"

namespace hyk {

struct AttnArgs {
    float *qkv;             // [nt][qkv_ld]: q | k | v (pre-rope); prefill rewrites q in place
    int qkv_ld;
    uint16_t *kc, *vc;      // this layer's cache, [ctx][kvdim] bf16
    const float *q_norm, *k_norm;
    const float *rope_cos, *rope_sin;  // [ctx][half]
    const int *pos_ptr;     // position of token 0
    int nt, heads, kv_heads, hd, kvdim, qdim, ctx, half;
    float eps, scale;
    float *ao;              // [nt][qdim]
    float *part;            // decode split partials [kv_heads][max_splits][G][HD+2]
    int *tickets;           // [kv_heads], zero between launches
    int split_len, max_splits;
    float *cpart;           // wide decode partials [heads][max_chunks][HD+kPartPad]
    int max_chunks, units;  // attn_max_chunks(ctx); units available (SMs)
    // all-decode passes whose o_proj runs on the tensor cores: attn_batch_dec
    // writes its Q8_K blocks straight into the GEMM's tiled activation (tca,
    // scales tcad, tc_nb blocks per token) instead of ao
    int8_t *tca;
    float *tcad;
    int tc_nb;
    int trace;              // timeline slot (< 0: off)
    // ragged batch of several sequences (prefill kernels only): token t sits
    // at position tok_pos[t] of sequence slot tok_slot[t], whose cache is
    // paged: row pos of a slot is row pos % kPageRows of page
    // pages[slot * page_max + pos / kPageRows], page_stride elements per page
    // (kc / vc: page 0's K / V rows of this layer)
    const int *tok_pos, *tok_slot;
    const int *pages;
    int page_max;
    long long page_stride;
    // query blocks of the tensor-core prefill kernel: (first token, count)
    // pairs of <= kFaQ consecutive positions of one slot; null: tokens
    // 16b .. 16b+15 of one sequence
    const int *qblk;
    int nqb;
};

// Position and sequence slot of token t, and the element offset (from kc /
// vc) of row pos of slot's cache: contiguous rows for the single-sequence
// cache, page-table rows for a batch.
__device__ __forceinline__ int attn_tok_pos(const AttnArgs &a, int t) { return a.tok_pos ? a.tok_pos[t] : *a.pos_ptr + t; }
__device__ __forceinline__ int attn_tok_slot(const AttnArgs &a, int t) { return a.tok_slot ? a.tok_slot[t] : 0; }
__device__ __forceinline__ long long attn_kv_row(const AttnArgs &a, int slot, int pos) {
    if (!a.pages) return (long long)pos * a.kvdim;
    return (long long)__ldg(a.pages + slot * a.page_max + (pos >> kPageShift)) * a.page_stride +
           (long long)(pos & (kPageRows - 1)) * a.kvdim;
}

// NeoX rotation + per-head RMSNorm of one head held as v[i] = x[lane + 32 i].
template <int HD>
__device__ __forceinline__ void rope_norm_warp(float (&v)[HD / 32], const float *cs, const float *sn, const float *nw,
                                               float eps) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int i = 0; i < HD / 64; i++) {
        const int e = lane + 32 * i;
        const float c = cs[e], s = sn[e];
        const float x0 = v[i], x1 = v[i + HD / 64];
        v[i] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
        v[i + HD / 64] = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
    }
    if (nw) {
        float ss = 0.f;
#pragma unroll
        for (int i = 0; i < HD / 32; i++) ss = __fadd_rn(ss, __fmul_rn(v[i], v[i]));
        ss = warp_sum(ss);
        const float scale = 1.0f / sqrtf(ss / (float)HD + eps);
#pragma unroll
        for (int i = 0; i < HD / 32; i++) v[i] = __fmul_rn(__fmul_rn(v[i], scale), nw[lane + 32 * i]);
    }
}

// Prefill prologue: rope + norm every q head in place, rope + norm + bf16
// store every k head, bf16 store every v head.  grid (nt), one warp per head.
template <int HD>
__global__ void rope_norm_store(const __grid_constant__ AttnArgs a) {
    pdl_trigger();
    pdl_wait();
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // the grid strides over the tokens (a few CTAs per SM, not one per token)
    for (int t = blockIdx.x; t < a.nt; t += gridDim.x) {
    const int pos = attn_tok_pos(a, t);
    const long long kvr = attn_kv_row(a, attn_tok_slot(a, t), pos);
    const float *cs = a.rope_cos + (size_t)pos * a.half, *sn = a.rope_sin + (size_t)pos * a.half;
    float *row = a.qkv + (size_t)t * a.qkv_ld;
    for (int hh = w; hh < a.heads + a.kv_heads; hh += blockDim.x >> 5) {
        float v[HD / 32];
        const bool is_q = hh < a.heads;
        float *src = is_q ? row + hh * HD : row + a.qdim + (hh - a.heads) * HD;
#pragma unroll
        for (int i = 0; i < HD / 32; i++) v[i] = src[lane + 32 * i];
        rope_norm_warp<HD>(v, cs, sn, is_q ? a.q_norm : a.k_norm, a.eps);
        if (is_q) {
#pragma unroll
            for (int i = 0; i < HD / 32; i++) src[lane + 32 * i] = v[i];
        } else {
            const int kvh = hh - a.heads;
            const float *vs = row + a.qdim + a.kvdim + kvh * HD;
            uint16_t *kd = a.kc + kvr + kvh * HD, *vd = a.vc + kvr + kvh * HD;
#pragma unroll
            for (int i = 0; i < HD / 32; i++) {
                kd[lane + 32 * i] = f32_to_bf16_bits(v[i]);
                vd[lane + 32 * i] = f32_to_bf16_bits(vs[lane + 32 * i]);
            }
        }
    }
    }
}

// Decode attention, one query token at position pos: grid (kv_heads, splits
// of kDecSplit keys).  Warps 0..G-1 are the query heads kvh*G + w, warp G
// rotates/normalises this KV head's k and stores k and v.  The split's cached
// K/V rows (positions < pos, written by earlier decode steps) are staged in
// shared memory by the caller; the current position comes from the prologue.
// The body is shared by the per-layer kernel (attn_decode2) and the
// persistent decode kernel, which differ only in how the rows are staged, so
// both produce bit-identical outputs.
constexpr int kDecSplit = 128;

template <int HD>
__host__ __device__ inline size_t attn_dec_smem() { return (size_t)2 * kDecSplit * HD * 2; }

// Per-position constants a warp needs for the prologue: rope row and the
// per-head norm weight (q_norm for the query warps, k_norm for the k/v warp).
template <int HD>
struct DecConsts {
    float rc[HD / 64], rs[HD / 64], nq[HD / 32];
};

template <int HD, int G>
__device__ __forceinline__ void attn_dec_consts(const AttnArgs &a, int pos, DecConsts<HD> &k) {
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const float *cs = a.rope_cos + (size_t)pos * a.half, *sn = a.rope_sin + (size_t)pos * a.half;
#pragma unroll
    for (int i = 0; i < HD / 64; i++) {
        k.rc[i] = __ldg(cs + lane + 32 * i);
        k.rs[i] = __ldg(sn + lane + 32 * i);
    }
    const float *nrm = w < G ? a.q_norm : a.k_norm;
#pragma unroll
    for (int i = 0; i < HD / 32; i++) k.nq[i] = __ldg(nrm + lane + 32 * i);
}

// Warps 0..G: rope + norm of the G query heads into sq, of k (and the bf16
// rounding of k and v) into skc/svc; when `store`, k and v go to the cache.
// q of the G heads (qs[G*HD]), k (ks[HD]) and v (vs[HD]) of this KV head,
// pre-rope, from any memory (the per-layer kernels pass the qkv row itself).
template <int HD, int G>
__device__ __forceinline__ void attn_dec_prologue(const AttnArgs &a, int kvh, int pos, bool store, const DecConsts<HD> &k,
                                                  float (*sq)[HD], float *skc, float *svc, const float *qs,
                                                  const float *ks, const float *vs) {
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float v[HD / 32], vraw[HD / 32];
    const float *src = w < G ? qs + w * HD : ks;
    const float *vr = vs;
#pragma unroll
    for (int i = 0; i < HD / 32; i++) {
        v[i] = src[lane + 32 * i];
        vraw[i] = w < G ? 0.f : vr[lane + 32 * i];  // the k/v warp loads v with k
    }
#pragma unroll
    for (int i = 0; i < HD / 64; i++) {
        const float x0 = v[i], x1 = v[i + HD / 64];
        v[i] = __fsub_rn(__fmul_rn(x0, k.rc[i]), __fmul_rn(x1, k.rs[i]));
        v[i + HD / 64] = __fadd_rn(__fmul_rn(x0, k.rs[i]), __fmul_rn(x1, k.rc[i]));
    }
    float ssq = 0.f;
#pragma unroll
    for (int i = 0; i < HD / 32; i++) ssq = __fadd_rn(ssq, __fmul_rn(v[i], v[i]));
    ssq = warp_sum(ssq);
    const float scale = 1.0f / sqrtf(ssq / (float)HD + a.eps);
#pragma unroll
    for (int i = 0; i < HD / 32; i++) v[i] = __fmul_rn(__fmul_rn(v[i], scale), k.nq[i]);
    if (w < G) {
#pragma unroll
        for (int i = 0; i < HD / 32; i++) sq[w][lane + 32 * i] = v[i];
    } else {
        uint16_t *kd = a.kc + (size_t)pos * a.kvdim + kvh * HD, *vd = a.vc + (size_t)pos * a.kvdim + kvh * HD;
#pragma unroll
        for (int i = 0; i < HD / 32; i++) {
            const int e = lane + 32 * i;
            const uint16_t kb = f32_to_bf16_bits(v[i]), vb = f32_to_bf16_bits(vraw[i]);
            skc[e] = bf16_bits_to_f32(kb);
            svc[e] = bf16_bits_to_f32(vb);
            if (store) {
                kd[e] = kb;
                vd[e] = vb;
            }
        }
    }
}

// Decode attention uses kDecWarps warps per (KV head, split): warp w takes
// query head kvh*G + (w % G) and the key subset sub = w / G, one key per lane
// (keys j0 + sub*32 + lane + k*32*NSUB), so every warp runs a short chain:
// one dot product per key, a warp softmax over its keys, and p.V over its 32
// (or 64) keys.  The NSUB partials of a head are then merged with the
// log-sum-exp rule, and splits of long contexts are merged by the last CTA
// of the KV head to finish.
constexpr int kDecWarps = 16;

template <int HD>
struct DecScratch {
    float pm[kDecWarps], pl[kDecWarps];
    float po[kDecWarps][HD];
    int last;
};

// All kDecWarps warps: scores over keys [j0, j1) of this split, softmax, p.V,
// warp partials merged per head, then either the final output (one split) or
// this split's partial and, in the last split CTA to finish, the merge.
// krow(j, c) is the 16-byte chunk c of cached K row j in shared memory,
// sV[j][HD] the V rows; key `pos` comes from skc/svc.  Synchronises the
// kDecWarps warps with named barrier `bar_id` and the G head warps with
// `bar_id + 1`.
template <int HD, int G, typename KRow>
__device__ __forceinline__ void attn_dec_main(const AttnArgs &a, int kvh, int split, int pos, KRow krow,
                                              const uint16_t *sV, const float (*sq)[HD], const float *skc,
                                              const float *svc, DecScratch<HD> &S, int bar_id) {
    constexpr int CH = HD / 8;    // 16-byte chunks per row
    constexpr int DPL = HD / 32;  // output dims per lane (contiguous)
    constexpr int NSUB = kDecWarps / G;
    constexpr int KPW = (kDecSplit + NSUB * 32 - 1) / (NSUB * 32);  // keys per lane
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int hh = w % G, sub = w / G;
    const int j0 = split * kDecSplit, j1 = min(pos + 1, j0 + kDecSplit), nk = j1 - j0;
    float s[KPW];
    float mx = -INFINITY;
#pragma unroll
    for (int k = 0; k < KPW; k++) {
        const int j = sub * 32 + lane + k * NSUB * 32;
        s[k] = -INFINITY;
        if (j < nk) {
            float dot = 0.f;
            if (j0 + j == pos) {
#pragma unroll 4
                for (int c = 0; c < CH; c++) {
                    const float4 qa = *(const float4 *)&sq[hh][c * 8], qb = *(const float4 *)&sq[hh][c * 8 + 4];
                    const float4 ka = *(const float4 *)&skc[c * 8], kb = *(const float4 *)&skc[c * 8 + 4];
                    dot = fmaf(qa.x, ka.x, dot);
                    dot = fmaf(qa.y, ka.y, dot);
                    dot = fmaf(qa.z, ka.z, dot);
                    dot = fmaf(qa.w, ka.w, dot);
                    dot = fmaf(qb.x, kb.x, dot);
                    dot = fmaf(qb.y, kb.y, dot);
                    dot = fmaf(qb.z, kb.z, dot);
                    dot = fmaf(qb.w, kb.w, dot);
                }
            } else {
#pragma unroll 4
                for (int c = 0; c < CH; c++) {
                    const float4 qa = *(const float4 *)&sq[hh][c * 8], qb = *(const float4 *)&sq[hh][c * 8 + 4];
                    const uint4 kk = *krow(j, c);
                    dot = fmaf(qa.x, bf16_bits_to_f32(kk.x & 0xffffu), dot);
                    dot = fmaf(qa.y, bf16_bits_to_f32(kk.x >> 16), dot);
                    dot = fmaf(qa.z, bf16_bits_to_f32(kk.y & 0xffffu), dot);
                    dot = fmaf(qa.w, bf16_bits_to_f32(kk.y >> 16), dot);
                    dot = fmaf(qb.x, bf16_bits_to_f32(kk.z & 0xffffu), dot);
                    dot = fmaf(qb.y, bf16_bits_to_f32(kk.z >> 16), dot);
                    dot = fmaf(qb.z, bf16_bits_to_f32(kk.w & 0xffffu), dot);
                    dot = fmaf(qb.w, bf16_bits_to_f32(kk.w >> 16), dot);
                }
            }
            s[k] = dot * a.scale;
        }
        mx = fmaxf(mx, s[k]);
    }
    mx = warp_max(mx);
    float l = 0.f;
#pragma unroll
    for (int k = 0; k < KPW; k++) {
        s[k] = (sub * 32 + lane + k * NSUB * 32 < nk) ? expf(s[k] - mx) : 0.f;
        l += s[k];
    }
    l = warp_sum(l);
    float o[DPL];
#pragma unroll
    for (int q = 0; q < DPL; q++) o[q] = 0.f;
#pragma unroll
    for (int k = 0; k < KPW; k++) {
        const int base = sub * 32 + k * NSUB * 32;
        const int lim = min(32, nk - base);
        int jj = 0;
        for (; jj + 4 <= lim; jj += 4) {
            float p[4], vv[4][DPL];
#pragma unroll
            for (int u = 0; u < 4; u++) {
                p[u] = __shfl_sync(0xffffffffu, s[k], jj + u);
                const int jr = base + jj + u;
                if (j0 + jr == pos) {
#pragma unroll
                    for (int q = 0; q < DPL; q++) vv[u][q] = svc[lane * DPL + q];
                } else {
                    const uint16_t *vr = sV + (size_t)jr * HD + lane * DPL;
                    if (DPL == 4) {
                        const uint2 x = *(const uint2 *)vr;
                        vv[u][0] = bf16_bits_to_f32(x.x & 0xffffu);
                        vv[u][1] = bf16_bits_to_f32(x.x >> 16);
                        vv[u][2] = bf16_bits_to_f32(x.y & 0xffffu);
                        vv[u][3] = bf16_bits_to_f32(x.y >> 16);
                    } else {
#pragma unroll
                        for (int q = 0; q < DPL; q++) vv[u][q] = bf16_bits_to_f32(vr[q]);
                    }
                }
            }
#pragma unroll
            for (int u = 0; u < 4; u++)
#pragma unroll
                for (int q = 0; q < DPL; q++) o[q] = fmaf(p[u], vv[u][q], o[q]);
        }
        for (; jj < lim; jj++) {
            const float p = __shfl_sync(0xffffffffu, s[k], jj);
            const int jr = base + jj;
#pragma unroll
            for (int q = 0; q < DPL; q++) {
                const float vq = j0 + jr == pos ? svc[lane * DPL + q] : bf16_bits_to_f32(sV[(size_t)jr * HD + lane * DPL + q]);
                o[q] = fmaf(p, vq, o[q]);
            }
        }
    }
    if (lane == 0) {
        S.pm[w] = sub * 32 < nk ? mx : -INFINITY;
        S.pl[w] = sub * 32 < nk ? l : 0.f;
    }
#pragma unroll
    for (int q = 0; q < DPL; q++) S.po[w][lane * DPL + q] = o[q];
    asm volatile("bar.sync %0, %1;" ::"r"(bar_id), "r"(kDecWarps * 32) : "memory");
    if (w >= G) return;
    // warp w < G: head kvh*G + w merges its NSUB key subsets
    float M = -INFINITY;
#pragma unroll
    for (int u = 0; u < NSUB; u++) M = fmaxf(M, S.pm[w + u * G]);
    float L = 0.f, O[DPL];
#pragma unroll
    for (int q = 0; q < DPL; q++) O[q] = 0.f;
#pragma unroll
    for (int u = 0; u < NSUB; u++) {
        const int src = w + u * G;
        const float f = S.pl[src] > 0.f ? expf(S.pm[src] - M) : 0.f;
        L = fmaf(S.pl[src], f, L);
#pragma unroll
        for (int q = 0; q < DPL; q++) O[q] = fmaf(S.po[src][lane * DPL + q], f, O[q]);
    }
    const int h = kvh * G + w;
    const int nsplit = (pos + kDecSplit) / kDecSplit;
    if (nsplit == 1) {
        const float inv = 1.0f / L;
#pragma unroll
        for (int q = 0; q < DPL; q++) a.ao[h * HD + lane * DPL + q] = O[q] * inv;
        return;
    }
    float *pp = a.part + (((size_t)kvh * a.max_splits + split) * G + w) * (HD + 2);
#pragma unroll
    for (int q = 0; q < DPL; q++) pp[2 + lane * DPL + q] = O[q];
    if (lane == 0) {
        pp[0] = M;
        pp[1] = L;
    }
    __threadfence();
    asm volatile("bar.sync %0, %1;" ::"r"(bar_id + 1), "r"(G * 32) : "memory");
    if (threadIdx.x == 0) S.last = atomicAdd(&a.tickets[kvh], 1) == nsplit - 1;
    asm volatile("bar.sync %0, %1;" ::"r"(bar_id + 1), "r"(G * 32) : "memory");
    if (!S.last) return;
    __threadfence();
    float MM = -INFINITY;
    for (int sp = 0; sp < nsplit; sp++)
        MM = fmaxf(MM, __ldcg(a.part + (((size_t)kvh * a.max_splits + sp) * G + w) * (HD + 2)));
    float LL = 0.f, OO[DPL];
#pragma unroll
    for (int q = 0; q < DPL; q++) OO[q] = 0.f;
    for (int sp = 0; sp < nsplit; sp++) {
        const float *pq = a.part + (((size_t)kvh * a.max_splits + sp) * G + w) * (HD + 2);
        const float f = expf(__ldcg(pq) - MM);
        LL = fmaf(__ldcg(pq + 1), f, LL);
#pragma unroll
        for (int q = 0; q < DPL; q++) OO[q] = fmaf(__ldcg(pq + 2 + lane * DPL + q), f, OO[q]);
    }
    const float inv = 1.0f / LL;
#pragma unroll
    for (int q = 0; q < DPL; q++) a.ao[h * HD + lane * DPL + q] = OO[q] * inv;
    if (threadIdx.x == 0) a.tickets[kvh] = 0;
}

// The per-layer kernel (kDecWarps warps): K rows are staged with their
// 16-byte chunks rotated by the row index so lanes reading different rows hit
// different banks; the copies are issued BEFORE griddepcontrol.wait (the
// cached rows were written at least two kernels back).
template <int HD, int G>
__global__ void __launch_bounds__(kDecWarps * 32) attn_decode2(const __grid_constant__ AttnArgs a) {
    extern __shared__ __align__(16) uint8_t dsm[];
    uint16_t *sK = (uint16_t *)dsm;                       // [kDecSplit][HD] rotated chunks
    uint16_t *sV = sK + (size_t)kDecSplit * HD;           // [kDecSplit][HD]
    __shared__ __align__(16) float sq[G][HD];
    __shared__ __align__(16) float skc[HD], svc[HD];
    __shared__ __align__(16) DecScratch<HD> S;
    constexpr int CH = HD / 8;
    trace_mark(a.trace, 0);
    pdl_trigger();
    const int kvh = blockIdx.x, split = blockIdx.y;
    const int w = threadIdx.x >> 5;
    const int pos = *a.pos_ptr;  // written before this graph / >= 2 kernels back
    const int j0 = split * kDecSplit;
    // the body's named barriers count kDecWarps warps: any other shape returns
    if (blockDim.x != kDecWarps * 32 || pos < 0 || pos >= a.ctx || j0 > pos) return;
    const int j1 = min(pos + 1, j0 + kDecSplit);
    const int ncache = min(j1, pos) - j0;  // rows already in the cache
    const uint16_t *Kg = a.kc + kvh * HD, *Vg = a.vc + kvh * HD;
    for (int idx = threadIdx.x; idx < ncache * CH; idx += blockDim.x) {
        const int j = idx / CH, c = idx - j * CH;
        const size_t g = (size_t)(j0 + j) * a.kvdim + c * 8;
        const unsigned dk = (unsigned)__cvta_generic_to_shared(sK + (size_t)j * HD + ((c + j) % CH) * 8);
        const unsigned dv = (unsigned)__cvta_generic_to_shared(sV + (size_t)j * HD + c * 8);
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dk), "l"(Kg + g) : "memory");
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dv), "l"(Vg + g) : "memory");
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
    DecConsts<HD> k;
    if (w <= G) attn_dec_consts<HD, G>(a, pos, k);
    pdl_wait();
    trace_mark(a.trace, 1);
    if (w <= G) attn_dec_prologue<HD, G>(a, kvh, pos, split == 0, k, sq, skc, svc, a.qkv + (kvh * G) * HD,
                                        a.qkv + a.qdim + kvh * HD, a.qkv + a.qdim + a.kvdim + kvh * HD);
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncthreads();
    trace_mark(a.trace, 2);
    const auto krow = [&](int j, int c) { return (const uint4 *)(sK + (size_t)j * HD + ((c + j) % CH) * 8); };
    attn_dec_main<HD, G>(a, kvh, split, pos, krow, sV, sq, skc, svc, S, 1);
    trace_mark(a.trace, 3);
}

// ---------------------------------------------------------------- wide decode attention
//
// Decode attention as many small units: unit (KV head g, chunk c) handles the
// G query heads of g over keys [c*cs, min((c+1)*cs, pos+1)), cs a multiple of
// 32 chosen so that kv_heads * chunks <= units (the SM count), and writes one
// partial (running max m, sum l, unnormalised p.V) per query head and chunk.
// attn_merge_head turns a head's partials into its output with the
// log-sum-exp rule.  Inside a unit (kDecWarps warps): warp w takes head
// w % G and the key subset sub = w / G; four lanes share a key, each
// multiplying HD/4 dimensions, so one warp scores 8 keys at once.  The
// per-layer path runs units as attn_chunk_kernel + attn_merge_kernel; the
// persistent kernel runs them as CTAs of its attention phase and merges in
// its o_proj staging, with the same arithmetic.
constexpr int kChunkMin = 32;   // smallest chunk (keys)
constexpr int kChunkKPad = 64;  // staged K rows padded by 64 bytes: two key groups hit disjoint banks
constexpr int kPartPad = 4;     // partial = (m, l, -, -, o[HD]): o 16-byte aligned
constexpr int kChunkMax = 128;  // largest chunk: the staging area holds kChunkMax rows

// Chunk length for position pos: the smallest multiple of 32 that keeps
// kv_heads * ceil((pos + 1) / cs) <= units; 0 if even kChunkMax does not.
constexpr int kMaxUnits = 64;   // attention units per position (two chunk weights per lane in the merge)
__host__ __device__ inline int attn_chunk_len(int pos, int kv_heads, int units) {
    if (units > kMaxUnits) units = kMaxUnits;
    for (int cs = kChunkMin; cs <= kChunkMax; cs += kChunkMin)
        if (kv_heads * ((pos + cs) / cs) <= units) return cs;
    return 0;
}

// The per-layer kernels' rule: attn_chunk_len where it has an answer (so the
// per-layer and persistent paths split a position identically), else the
// same search with up to kMaxUnitsWide units (long contexts: 4 KV heads x 37
// chunks of 128 keys on 148 SMs).  The per-layer merge holds kWideNR chunk
// weights per lane.
constexpr int kMaxUnitsWide = 160;
constexpr int kWideNR = kMaxUnitsWide / 32;
__host__ __device__ inline int attn_chunk_len_wide(int pos, int kv_heads, int units) {
    const int cs = attn_chunk_len(pos, kv_heads, units);
    if (cs || units <= kMaxUnits) return cs;
    if (units > kMaxUnitsWide) units = kMaxUnitsWide;
    for (int c = kChunkMin; c <= kChunkMax; c += kChunkMin)
        if (kv_heads * ((pos + c) / c) <= units) return c;
    return 0;
}
__host__ __device__ inline int attn_max_chunks(int ctx) { return (ctx + kChunkMin - 1) / kChunkMin; }

template <int HD>
struct ChunkScratch {
    float pm[kDecWarps], pl[kDecWarps];
    float po[kDecWarps][HD];
    float pw[kDecWarps][kChunkMax / 2];  // each warp's key probabilities (a warp holds <= cs/2 keys)
};

// All kDecWarps warps of a unit.  krow(j, c) is 16-byte chunk c of staged K
// row j (j relative to the chunk start), sV[j][HD] the staged V rows; key
// `pos` comes from skc/svc.  Writes part[(h * max_chunks + chunk) * (HD+2)]
// = (m, l, o[HD]) for h = kvh*G .. kvh*G+G-1.  Synchronises the kDecWarps
// warps with named barrier bar_id.
struct NoMark {
    __device__ __forceinline__ void operator()() const {}
};

template <int HD, int G, typename KRow, typename Mark = NoMark>
__device__ __forceinline__ void attn_chunk_main(const AttnArgs &a, int kvh, int chunk, int cs, int pos, KRow krow,
                                                const uint16_t *sV, const float (*sq)[HD], const float *skc,
                                                const float *svc, ChunkScratch<HD> &S, int bar_id,
                                                Mark mark = Mark()) {
    constexpr int DQ = HD / 4;            // dims per lane in a 4-lane key group
    constexpr int DPL = HD / 32;          // output dims per lane
    constexpr int NSUB = kDecWarps / G;   // warps per head
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31, grp = lane >> 2, qtr = lane & 3;
    const int hh = w % G, sub = w / G;
    const int j0 = chunk * cs, nk = min(pos + 1 - j0, cs);
    const int kw = (cs + NSUB - 1) / NSUB;  // keys of this warp: [sub*kw, sub*kw + kw)
    const int kb = sub * kw, ke = min(kb + kw, nk);
    constexpr int KMAX = (kChunkMax / NSUB + 7) / 8;  // keys per lane group (upper bound)
    float mloc = -INFINITY;
    float s[KMAX];
#pragma unroll
    for (int t = 0; t < KMAX; t++) {
        const int j = kb + grp + 8 * t;
        s[t] = -INFINITY;
        if (j < ke) {
            // lane quarter qtr takes the 8-dim chunks qtr + 4i (bank-spread q and K reads);
            // one accumulator per chunk (independent chains), then a fixed-order sum
            float dot = 0.f;
            float part[DQ / 8];
            if (j0 + j == pos) {
#pragma unroll
                for (int c = 0; c < DQ / 8; c++) {
                    const int d0 = (qtr + 4 * c) * 8;
                    const float4 qa = *(const float4 *)&sq[hh][d0], qb = *(const float4 *)&sq[hh][d0 + 4];
                    const float4 ka = *(const float4 *)&skc[d0], kb4 = *(const float4 *)&skc[d0 + 4];
                    float d = qa.x * ka.x;
                    d = fmaf(qa.y, ka.y, d);
                    d = fmaf(qa.z, ka.z, d);
                    d = fmaf(qa.w, ka.w, d);
                    d = fmaf(qb.x, kb4.x, d);
                    d = fmaf(qb.y, kb4.y, d);
                    d = fmaf(qb.z, kb4.z, d);
                    d = fmaf(qb.w, kb4.w, d);
                    part[c] = d;
                }
            } else {
                uint4 kk[DQ / 8];
#pragma unroll
                for (int c = 0; c < DQ / 8; c++) kk[c] = *krow(j, qtr + 4 * c);
#pragma unroll
                for (int c = 0; c < DQ / 8; c++) {
                    const int d0 = (qtr + 4 * c) * 8;
                    const float4 qa = *(const float4 *)&sq[hh][d0], qb = *(const float4 *)&sq[hh][d0 + 4];
                    float d = qa.x * bf16_bits_to_f32(kk[c].x & 0xffffu);
                    d = fmaf(qa.y, bf16_bits_to_f32(kk[c].x >> 16), d);
                    d = fmaf(qa.z, bf16_bits_to_f32(kk[c].y & 0xffffu), d);
                    d = fmaf(qa.w, bf16_bits_to_f32(kk[c].y >> 16), d);
                    d = fmaf(qb.x, bf16_bits_to_f32(kk[c].z & 0xffffu), d);
                    d = fmaf(qb.y, bf16_bits_to_f32(kk[c].z >> 16), d);
                    d = fmaf(qb.z, bf16_bits_to_f32(kk[c].w & 0xffffu), d);
                    d = fmaf(qb.w, bf16_bits_to_f32(kk[c].w >> 16), d);
                    part[c] = d;
                }
            }
#pragma unroll
            for (int c = 0; c < DQ / 8; c++) dot += part[c];
            s[t] = dot;  // partial over this lane's quarter of the dimensions
        }
    }
    // the 4 quarters of each key: fixed butterfly order
#pragma unroll
    for (int t = 0; t < KMAX; t++) {
        float v = s[t];
        v += __shfl_xor_sync(0xffffffffu, v, 1);
        v += __shfl_xor_sync(0xffffffffu, v, 2);
        const int j = kb + grp + 8 * t;
        s[t] = j < ke ? v * a.scale : -INFINITY;
        mloc = fmaxf(mloc, s[t]);
    }
    mark();
    mloc = warp_max(mloc);
    float lsum = 0.f;
#pragma unroll
    for (int t = 0; t < KMAX; t++) {
        const int j = kb + grp + 8 * t;
        s[t] = j < ke ? expf(s[t] - mloc) : 0.f;
        if (qtr == 0) lsum += s[t];
    }
    lsum = warp_sum(lsum);
    mark();
    float o[DPL];
#pragma unroll
    for (int q = 0; q < DPL; q++) o[q] = 0.f;
    // the warp's key probabilities go through shared memory, so p.V reads each
    // key's p with one broadcast load instead of a shuffle per candidate slot
    if (qtr == 0) {
#pragma unroll
        for (int t = 0; t < KMAX; t++) {
            const int j = kb + grp + 8 * t;
            if (j < ke) S.pw[w][j - kb] = s[t];
        }
    }
    __syncwarp();
    const auto p_of = [&](int j) { return S.pw[w][j - kb]; };
    const auto v_of = [&](int j, float (&vv)[DPL]) {
        if (j0 + j == pos) {
#pragma unroll
            for (int q = 0; q < DPL; q++) vv[q] = svc[lane * DPL + q];
        } else {
            const uint16_t *vr = sV + (size_t)j * HD + lane * DPL;
            if (DPL == 4) {
                const uint2 x = *(const uint2 *)vr;
                vv[0] = bf16_bits_to_f32(x.x & 0xffffu);
                vv[1] = bf16_bits_to_f32(x.x >> 16);
                vv[2] = bf16_bits_to_f32(x.y & 0xffffu);
                vv[3] = bf16_bits_to_f32(x.y >> 16);
            } else {
#pragma unroll
                for (int q = 0; q < DPL; q++) vv[q] = bf16_bits_to_f32(vr[q]);
            }
        }
    };
    int j = kb;
    for (; j + 4 <= ke; j += 4) {  // four keys' p and V rows fetched before any FMA
        float p[4], vv[4][DPL];
#pragma unroll
        for (int u = 0; u < 4; u++) {
            p[u] = p_of(j + u);
            v_of(j + u, vv[u]);
        }
#pragma unroll
        for (int u = 0; u < 4; u++)
#pragma unroll
            for (int q = 0; q < DPL; q++) o[q] = fmaf(p[u], vv[u][q], o[q]);
    }
    for (; j < ke; j++) {
        float vv[DPL];
        const float p = p_of(j);
        v_of(j, vv);
#pragma unroll
        for (int q = 0; q < DPL; q++) o[q] = fmaf(p, vv[q], o[q]);
    }
    mark();
    if (lane == 0) {
        S.pm[w] = kb < nk ? mloc : -INFINITY;
        S.pl[w] = kb < nk ? lsum : 0.f;
    }
#pragma unroll
    for (int q = 0; q < DPL; q++) S.po[w][lane * DPL + q] = o[q];
    asm volatile("bar.sync %0, %1;" ::"r"(bar_id), "r"(kDecWarps * 32) : "memory");
    mark();
    if (w >= G) return;
    float M = -INFINITY;
#pragma unroll
    for (int u = 0; u < NSUB; u++) M = fmaxf(M, S.pm[w + u * G]);
    float L = 0.f, O[DPL];
#pragma unroll
    for (int q = 0; q < DPL; q++) O[q] = 0.f;
#pragma unroll
    for (int u = 0; u < NSUB; u++) {
        const int src = w + u * G;
        const float f = S.pl[src] > 0.f ? expf(S.pm[src] - M) : 0.f;
        L = fmaf(S.pl[src], f, L);
#pragma unroll
        for (int q = 0; q < DPL; q++) O[q] = fmaf(S.po[src][lane * DPL + q], f, O[q]);
    }
    const size_t po = ((size_t)(kvh * G + w) * a.max_chunks + chunk) * (HD + kPartPad);
    float *pp = a.cpart + po;
#pragma unroll
    for (int q = 0; q < DPL; q++) pp[kPartPad + lane * DPL + q] = O[q];
    if (lane == 0) {
        pp[0] = M;
        pp[1] = L;
    }
}

// One warp: output of head h from its nchunks partials (log-sum-exp merge in
// chunk order), written to out[HD].
// Lane c holds chunk c's (m, l); M by warp max, L by warp sum of
// l_c e^(m_c - M) (lane order), O over chunks in chunk order with the chunk
// weights broadcast from their lanes.  Every load of the first four chunks is
// issued before any arithmetic.
// Partials of one head in plain memory: (m, l) of chunk c and its o slice.
template <int HD>
struct PlainPartLoader {
    const float *base;  // head's first chunk
    __device__ __forceinline__ float2 ml(int c) const { return __ldcg((const float2 *)(base + (size_t)c * (HD + kPartPad))); }
    template <int DPL>
    __device__ __forceinline__ void o(int c, int lane, float (&v)[DPL]) const {
        const float *p = base + (size_t)c * (HD + kPartPad) + kPartPad + lane * DPL;
        if constexpr (DPL == 4) {
            const float4 x = __ldcg((const float4 *)p);
            v[0] = x.x;
            v[1] = x.y;
            v[2] = x.z;
            v[3] = x.w;
        } else {
            const float2 x = __ldcg((const float2 *)p);
            v[0] = x.x;
            v[1] = x.y;
        }
    }
};

// One warp: output of a head from its nchunks partials.  Lane c holds chunk
// c's (m, l); M by warp max, L by warp sum of l_c e^(m_c - M) (lane order), O
// over chunks in chunk order with the chunk weights broadcast from their
// lanes; the first four chunks' rows are loaded before any arithmetic.  NR
// chunk weights per lane (nchunks <= 32 * NR); lanes past nchunks add exact
// zeros, so the result does not depend on NR.  Chunks past the fourth are
// loaded B at a time before their FMAs (B = 1: one load per FMA group, the
// persistent kernel's form); the FMA order, and so the result, is the same.
template <int HD, typename Loader, int NR = (kMaxUnits + 31) / 32, int B = 1>
__device__ __forceinline__ void attn_merge_head_with(const Loader &ld, int nchunks, float *out) {
    constexpr int DPL = HD / 32;
    const int lane = threadIdx.x & 31;
    float mc[NR], lc[NR];
#pragma unroll
    for (int r = 0; r < NR; r++) {
        const int c = lane + 32 * r;
        const float2 ml = c < nchunks ? ld.ml(c) : make_float2(-INFINITY, 0.f);
        mc[r] = ml.x;
        lc[r] = ml.y;
    }
    float ov0[4][DPL];
#pragma unroll
    for (int u = 0; u < 4; u++) {
        if (u < nchunks) {
            ld.template o<DPL>(u, lane, ov0[u]);
        } else {
#pragma unroll
            for (int q = 0; q < DPL; q++) ov0[u][q] = 0.f;
        }
    }
    float mm = mc[0];
#pragma unroll
    for (int r = 1; r < NR; r++) mm = fmaxf(mm, mc[r]);
    const float M = warp_max(mm);
    float f[NR], lf = 0.f;
#pragma unroll
    for (int r = 0; r < NR; r++) {
        f[r] = lane + 32 * r < nchunks ? expf(mc[r] - M) : 0.f;
        lf = fmaf(lc[r], f[r], lf);
    }
    const float L = warp_sum(lf);
    const auto f_of = [&](int cc) {  // weight of chunk cc, from lane cc % 32
        float v = 0.f;
#pragma unroll
        for (int r = 0; r < NR; r++)
            if ((cc >> 5) == r) v = __shfl_sync(0xffffffffu, f[r], cc & 31);
        return v;
    };
    float O[DPL];
#pragma unroll
    for (int q = 0; q < DPL; q++) O[q] = 0.f;
#pragma unroll
    for (int u = 0; u < 4; u++) {
        if (u < nchunks) {
            const float fw = f_of(u);
#pragma unroll
            for (int q = 0; q < DPL; q++) O[q] = fmaf(ov0[u][q], fw, O[q]);
        }
    }
    if constexpr (B == 1) {
        for (int c = 4; c < nchunks; c++) {
            const float fw = f_of(c);
            float vv[DPL];
            ld.template o<DPL>(c, lane, vv);
#pragma unroll
            for (int q = 0; q < DPL; q++) O[q] = fmaf(vv[q], fw, O[q]);
        }
    } else {
        for (int c0 = 4; c0 < nchunks; c0 += B) {
            float vv[B][DPL];
#pragma unroll
            for (int u = 0; u < B; u++)
                if (c0 + u < nchunks) ld.template o<DPL>(c0 + u, lane, vv[u]);
#pragma unroll
            for (int u = 0; u < B; u++) {
                if (c0 + u < nchunks) {
                    const float fw = f_of(c0 + u);
#pragma unroll
                    for (int q = 0; q < DPL; q++) O[q] = fmaf(vv[u][q], fw, O[q]);
                }
            }
        }
    }
    const float inv = 1.0f / L;
#pragma unroll
    for (int q = 0; q < DPL; q++) out[lane * DPL + q] = O[q] * inv;
}

template <int HD>
__device__ __forceinline__ void attn_merge_head(const float *part, int max_chunks, int nchunks, int h, float *out) {
    const PlainPartLoader<HD> ld{part + (size_t)h * max_chunks * (HD + kPartPad)};
    attn_merge_head_with<HD>(ld, nchunks, out);
}

// Per-layer form: grid (kv_heads, attn_max_chunks(ctx)), chunk length by
// attn_chunk_len_wide; units past the position's chunk count return.  Rows
// staged with cp.async (K rows padded by 64 bytes so the 8 key groups of a
// warp read different banks).
template <int HD, int G>
__global__ void __launch_bounds__(kDecWarps * 32) attn_chunk_kernel(const __grid_constant__ AttnArgs a) {
    constexpr int KROW = HD * 2 + kChunkKPad, CH = HD / 8;
    extern __shared__ __align__(16) uint8_t dsm[];
    uint8_t *sK = dsm;
    uint16_t *sV = (uint16_t *)(dsm + (size_t)kChunkMax * KROW);
    __shared__ __align__(16) float sq[G][HD];
    __shared__ __align__(16) float skc[HD], svc[HD];
    __shared__ __align__(16) ChunkScratch<HD> S;
    trace_mark(a.trace, 0);
    pdl_trigger();
    const int kvh = blockIdx.x, chunk = blockIdx.y, w = threadIdx.x >> 5;
    const int pos = *a.pos_ptr;  // written before this graph / >= 2 kernels back
    if (blockDim.x != kDecWarps * 32 || pos < 0 || pos >= a.ctx) return;
    const int cs = attn_chunk_len_wide(pos, a.kv_heads, a.units);
    if (cs == 0 || chunk * cs > pos) return;
    const int j0 = chunk * cs, ncache = max(0, min(pos, j0 + cs) - j0);
    const uint16_t *Kg = a.kc + kvh * HD, *Vg = a.vc + kvh * HD;
    for (int idx = threadIdx.x; idx < ncache * CH; idx += blockDim.x) {
        const int j = idx / CH, c = idx - j * CH;
        const size_t g = (size_t)(j0 + j) * a.kvdim + c * 8;
        const unsigned dk = (unsigned)__cvta_generic_to_shared(sK + (size_t)j * KROW + c * 16);
        const unsigned dv = (unsigned)__cvta_generic_to_shared(sV + (size_t)j * HD + c * 8);
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dk), "l"(Kg + g) : "memory");
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dv), "l"(Vg + g) : "memory");
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
    DecConsts<HD> k;
    if (w <= G) attn_dec_consts<HD, G>(a, pos, k);
    pdl_wait();
    trace_mark(a.trace, 1);
    if (w <= G)
        attn_dec_prologue<HD, G>(a, kvh, pos, chunk == 0, k, sq, skc, svc, a.qkv + (kvh * G) * HD,
                                 a.qkv + a.qdim + kvh * HD, a.qkv + a.qdim + a.kvdim + kvh * HD);
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncthreads();
    trace_mark(a.trace, 2);
    const auto krow = [&](int j, int c) { return (const uint4 *)(sK + (size_t)j * KROW + c * 16); };
    attn_chunk_main<HD, G>(a, kvh, chunk, cs, pos, krow, sV, sq, skc, svc, S, 1);
    trace_mark(a.trace, 3);
}

template <int HD>
__host__ __device__ inline size_t attn_chunk_smem() {
    return (size_t)kChunkMax * (HD * 2 + kChunkKPad) + (size_t)kChunkMax * HD * 2;
}

// grid (heads), one warp: ao[h] from the partials of attn_chunk_kernel.
template <int HD>
__global__ void __launch_bounds__(32) attn_merge_kernel(const __grid_constant__ AttnArgs a) {
    pdl_trigger();
    pdl_wait();
    const int pos = *a.pos_ptr;
    if (pos < 0 || pos >= a.ctx) return;
    const int cs = attn_chunk_len_wide(pos, a.kv_heads, a.units);
    if (cs == 0) return;
    const PlainPartLoader<HD> ld{a.cpart + (size_t)blockIdx.x * a.max_chunks * (HD + kPartPad)};
    attn_merge_head_with<HD, PlainPartLoader<HD>, kWideNR, 16>(ld, (pos + cs) / cs, a.ao + (size_t)blockIdx.x * HD);
}

// ---------------------------------------------------------------- batched decode attention
//
// A pass whose every token is the next token of its own sequence (the
// continuous-batching server's decode steps): token t attends to rows
// 0 .. pos of its slot, all already in the (paged) cache.  CTA = (KV head,
// token), kDbWarps warps taking groups of KG = 32 / G consecutive keys round
// robin.  Lane l owns head dims l * HD/32 .. of every head: the query of the
// G heads stays in registers, a key's K and V rows are read once and
// coalesced (HD * 2 bytes per warp per row), and the G x KG dot products of a
// group finish in one 31-step reduce-scatter that leaves lane l with the score
// of (key l / G, head l % G).  Online softmax per head (reference attn_task,
// src/model.c:768-795: q.k / sqrt(hd), max-subtracted expf, p.v over the sum
// of p), then the warps' (m, l, o) merge in shared memory.
constexpr int kDbWarps = 4;

template <int D>
struct BfRow;  // D consecutive bf16 of a row, as loaded by one lane
template <>
struct BfRow<4> {
    uint2 v;
    __device__ __forceinline__ void load(const uint16_t *p) { v = __ldg((const uint2 *)p); }
    __device__ __forceinline__ void zero() { v = make_uint2(0u, 0u); }
    __device__ __forceinline__ void get(float (&f)[4]) const {
        f[0] = __uint_as_float(v.x << 16);
        f[1] = __uint_as_float(v.x & 0xffff0000u);
        f[2] = __uint_as_float(v.y << 16);
        f[3] = __uint_as_float(v.y & 0xffff0000u);
    }
};
template <>
struct BfRow<2> {
    uint32_t v;
    __device__ __forceinline__ void load(const uint16_t *p) { v = __ldg((const uint32_t *)p); }
    __device__ __forceinline__ void zero() { v = 0u; }
    __device__ __forceinline__ void get(float (&f)[2]) const {
        f[0] = __uint_as_float(v << 16);
        f[1] = __uint_as_float(v & 0xffff0000u);
    }
};

template <int HD, int G>
__global__ void __launch_bounds__(kDbWarps * 32) attn_batch_dec(const __grid_constant__ AttnArgs a) {
    constexpr int D = HD / 32, KG = 32 / G;
    __shared__ float s_m[kDbWarps][G], s_l[kDbWarps][G], s_o[kDbWarps][G][HD];
    __shared__ __align__(16) float s_out[G * HD];  // the finished heads, for the fused quantiser
    pdl_trigger();
    const int kvh = blockIdx.x, t = blockIdx.y, w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    pdl_wait();
    const int pos = attn_tok_pos(a, t), slot = attn_tok_slot(a, t), nkeys = pos + 1;
    float q[G][D];
    const float *qr = a.qkv + (size_t)t * a.qkv_ld + (size_t)kvh * G * HD + lane * D;
#pragma unroll
    for (int h = 0; h < G; h++)
#pragma unroll
        for (int d = 0; d < D; d++) q[h][d] = qr[h * HD + d];
    // the slot's page numbers, lane j holding page j (tables of up to 32 pages)
    const bool reg_tab = a.pages && a.page_max <= 32;
    const int pg = reg_tab && lane < a.page_max ? __ldg(a.pages + slot * a.page_max + lane) : 0;
    const uint16_t *Kb = a.kc + kvh * HD + lane * D, *Vb = a.vc + kvh * HD + lane * D;
    float o[G][D];
#pragma unroll
    for (int h = 0; h < G; h++)
#pragma unroll
        for (int d = 0; d < D; d++) o[h][d] = 0.f;
    float mh = -INFINITY, lh = 0.f;  // running max and sum of head lane % G
    const int ngroups = (nkeys + KG - 1) / KG;
    // K and V rows of group g into registers (keys past pos read as zeros)
    auto load_group = [&](int g, BfRow<D> (&kr)[KG], BfRow<D> (&vr)[KG]) {
#pragma unroll
        for (int k = 0; k < KG; k++) {
            const int j = g * KG + k;
            if (j < nkeys) {
                const long long off = reg_tab ? (long long)__shfl_sync(0xffffffffu, pg, j >> kPageShift) * a.page_stride +
                                                    (long long)(j & (kPageRows - 1)) * a.kvdim
                                              : attn_kv_row(a, slot, j);
                kr[k].load(Kb + off);
                vr[k].load(Vb + off);
            } else {
                kr[k].zero();
                vr[k].zero();
            }
        }
    };
    BfRow<D> nkr[KG], nvr[KG];  // the next group's rows, in flight while this group computes
    if (w < ngroups) load_group(w, nkr, nvr);
    for (int g = w; g < ngroups; g += kDbWarps) {
        const int k0 = g * KG;
        BfRow<D> kr[KG], vr[KG];
#pragma unroll
        for (int k = 0; k < KG; k++) {
            kr[k] = nkr[k];
            vr[k] = nvr[k];
        }
        if (g + kDbWarps < ngroups) load_group(g + kDbWarps, nkr, nvr);
        // partial dots over this lane's dims: v[k * G + h]
        float v[32];
#pragma unroll
        for (int k = 0; k < KG; k++) {
            float kf[D];
            kr[k].get(kf);
#pragma unroll
            for (int h = 0; h < G; h++) {
                float acc = 0.f;
#pragma unroll
                for (int d = 0; d < D; d++) acc = fmaf(q[h][d], kf[d], acc);
                v[k * G + h] = acc;
            }
        }
        // reduce-scatter: after the stage of width sw, v[i] (i < sw) is the sum of
        // value i + (lane & -sw) over the lanes that differ from this one only in
        // bits >= sw; after sw = 1, v[0] is the warp's sum of value `lane`
#pragma unroll
        for (int sw = 16; sw >= 1; sw >>= 1) {
            const bool up = (lane & sw) != 0;
#pragma unroll
            for (int i = 0; i < sw; i++) {
                const float send = up ? v[i] : v[i + sw];
                const float keep = up ? v[i + sw] : v[i];
                v[i] = keep + __shfl_xor_sync(0xffffffffu, send, sw);
            }
        }
        const int mk = k0 + lane / G;
        const float sc = mk < nkeys ? v[0] * a.scale : -INFINITY;
        float gm = sc;
#pragma unroll
        for (int x = G; x < 32; x <<= 1) gm = fmaxf(gm, __shfl_xor_sync(0xffffffffu, gm, x));
        const float mn = fmaxf(mh, gm);
        const float corr = expf(mh - mn);
        const float p = mk < nkeys ? expf(sc - mn) : 0.f;
        float ps = p;
#pragma unroll
        for (int x = G; x < 32; x <<= 1) ps += __shfl_xor_sync(0xffffffffu, ps, x);
        lh = lh * corr + ps;
        mh = mn;
#pragma unroll
        for (int h = 0; h < G; h++) {
            const float ch = __shfl_sync(0xffffffffu, corr, h);  // lane h: head h
#pragma unroll
            for (int d = 0; d < D; d++) o[h][d] *= ch;
        }
#pragma unroll
        for (int k = 0; k < KG; k++) {
            float vf[D];
            vr[k].get(vf);
#pragma unroll
            for (int h = 0; h < G; h++) {
                const float pk = __shfl_sync(0xffffffffu, p, k * G + h);
#pragma unroll
                for (int d = 0; d < D; d++) o[h][d] = fmaf(pk, vf[d], o[h][d]);
            }
        }
    }
    if (lane < G) {
        s_m[w][lane] = mh;
        s_l[w][lane] = lh;
    }
#pragma unroll
    for (int h = 0; h < G; h++)
#pragma unroll
        for (int d = 0; d < D; d++) s_o[w][h][lane * D + d] = o[h][d];
    __syncthreads();
    for (int h = w; h < G; h += kDbWarps) {
        float M = -INFINITY;
#pragma unroll
        for (int x = 0; x < kDbWarps; x++) M = fmaxf(M, s_m[x][h]);
        float L = 0.f, O[D];
#pragma unroll
        for (int d = 0; d < D; d++) O[d] = 0.f;
#pragma unroll
        for (int x = 0; x < kDbWarps; x++) {
            const float f = s_l[x][h] > 0.f ? expf(s_m[x][h] - M) : 0.f;
            L = fmaf(s_l[x][h], f, L);
#pragma unroll
            for (int d = 0; d < D; d++) O[d] = fmaf(s_o[x][h][lane * D + d], f, O[d]);
        }
        const float inv = 1.0f / L;
        float *dst = a.tca ? s_out + h * HD + lane * D : a.ao + (size_t)t * a.qdim + (size_t)(kvh * G + h) * HD + lane * D;
#pragma unroll
        for (int d = 0; d < D; d++) dst[d] = O[d] * inv;
    }
    if (a.tca) {
        // the G heads are G * HD / 256 whole Q8_K blocks of the o_proj input:
        // warp j quantises block j exactly as tc_quantize_blocks would
        __syncthreads();
        constexpr int NBC = G * HD / 256;
        static_assert(NBC <= kDbWarps, "one warp per block");
        if (w < NBC) {
            const float4 v0 = *(const float4 *)&s_out[w * 256 + lane * 8], v1 = *(const float4 *)&s_out[w * 256 + lane * 8 + 4];
            const float v[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
            tc_quant_store(v, a.tca, a.tcad, t / kTcM, a.tc_nb, (kvh * G * HD) / 256 + w, t % kTcM);
        }
    }
}

// ---------------------------------------------------------------- prefill attention on tensor cores
//
// Causal GQA attention for multi-token passes (reference attn_task,
// src/model.c:768-795: scores q.k / sqrt(hd), max-subtracted expf, sum of
// p.v normalised by the sum of p), with q/k/v already rotated, normalised and
// stored by rope_norm_store.  CTA = one query block (<= 16 consecutive
// tokens of one sequence) x one KV head; warp w owns q head kvh*G + w, its
// 16 rows the block's tokens.  K/V tiles of 32 keys are staged with cp.async
// (double-buffered, rows padded by 8 elements so fragment loads hit distinct
// banks) and multiplied with mma.sync m16n8k16 bf16 into fp32 accumulators
// with an online softmax.  K and V are bf16 already; q and p are fp32 and
// enter the bf16 MMAs as three bf16 terms (x = x1 + x2 + x3, each the bf16
// rounding of what the previous ones leave), so every product keeps at
// least fp32's 24 bits and the sums stay fp32.
constexpr int kFaQ = 16;   // query tokens per block
constexpr int kFaK = 32;   // keys per tile (two CTAs of 4 warps fit an SM)

template <int HD>
__host__ __device__ constexpr int fa_row() { return HD + 8; }  // padded bf16 row
constexpr int kFaTerms = 3;  // bf16 terms of q and p
template <int HD, int G>
__host__ __device__ constexpr size_t fa_smem() {
    return (size_t)G * kFaQ * fa_row<HD>() * 2 * kFaTerms + (size_t)2 * 2 * kFaK * fa_row<HD>() * 2;
}

__device__ __forceinline__ uint32_t fa_pack(float lo, float hi) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *(const uint32_t *)&v;
}
// x = t[0] + t[1] + t[2] in bf16, packed pairs (element 0 in the low half);
// each remainder is exact in fp32
__device__ __forceinline__ void fa_split(float x0, float x1, uint32_t (&t)[kFaTerms]) {
#pragma unroll
    for (int i = 0; i < kFaTerms; i++) {
        const __nv_bfloat16 h0 = __float2bfloat16_rn(x0), h1 = __float2bfloat16_rn(x1);
        t[i] = (uint32_t)__bfloat16_as_ushort(h0) | ((uint32_t)__bfloat16_as_ushort(h1) << 16);
        x0 -= __bfloat162float(h0);
        x1 -= __bfloat162float(h1);
    }
}
__device__ __forceinline__ void fa_mma(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void fa_ldm4(uint32_t (&r)[4], const void *p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"((uint32_t)__cvta_generic_to_shared(p)));
}
__device__ __forceinline__ void fa_ldm4t(uint32_t (&r)[4], const void *p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"((uint32_t)__cvta_generic_to_shared(p)));
}

// Stage keys [k0, k0 + kFaK) (rows past kend zero-filled) of K and V.
template <int HD, int G>
__device__ __forceinline__ void fa_stage(const AttnArgs &a, const uint16_t *Kg, const uint16_t *Vg, int slot, int k0,
                                         int kend, uint16_t *sk, uint16_t *sv) {
    constexpr int CH = HD / 8;  // 16-byte chunks per row
    for (int i = threadIdx.x; i < kFaK * CH; i += G * 32) {
        const int r = i / CH, c = i % CH, key = k0 + r;
        uint16_t *dk = sk + r * fa_row<HD>() + c * 8, *dv = sv + r * fa_row<HD>() + c * 8;
        if (key < kend) {
            const long long ro = attn_kv_row(a, slot, key);
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dk)),
                         "l"(Kg + ro + c * 8)
                         : "memory");
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dv)),
                         "l"(Vg + ro + c * 8)
                         : "memory");
        } else {
            *(uint4 *)dk = make_uint4(0, 0, 0, 0);
            *(uint4 *)dv = make_uint4(0, 0, 0, 0);
        }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
}

// grid (query blocks, kv_heads), G warps.
template <int HD, int G>
__global__ void __launch_bounds__(G * 32) attn_fa(const __grid_constant__ AttnArgs a) {
    pdl_trigger();
    extern __shared__ __align__(16) uint8_t smem[];
    constexpr int R = fa_row<HD>(), NT = HD / 8;  // dim n-tiles of O
    uint16_t *qs = (uint16_t *)smem;                 // [term][G][16][R]
    uint16_t *sk0 = qs + kFaTerms * G * kFaQ * R;    // [2 stages][K | V][64][R]
    const int kvh = blockIdx.y, w = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, tq = lane & 3;
    pdl_wait();
    int t0, nq;
    if (a.qblk) {
        t0 = a.qblk[2 * blockIdx.x];
        nq = a.qblk[2 * blockIdx.x + 1];
    } else {
        t0 = blockIdx.x * kFaQ;
        nq = min(kFaQ, a.nt - t0);
    }
    const int pos0 = attn_tok_pos(a, t0);  // the block's positions are pos0 .. pos0 + nq - 1
    const int slot = attn_tok_slot(a, t0);
    const int kend = pos0 + nq;
    const int head = kvh * G + w;
    // q rows of this warp's head -> bf16 terms (rows past nq repeat the last token)
    for (int i = lane; i < kFaQ * HD / 2; i += 32) {
        const int r = i / (HD / 2), d = (i % (HD / 2)) * 2;
        const int t = t0 + min(r, nq - 1);
        const float2 v = *(const float2 *)(a.qkv + (size_t)t * a.qkv_ld + head * HD + d);
        uint32_t tt[kFaTerms];
        fa_split(v.x, v.y, tt);
#pragma unroll
        for (int x = 0; x < kFaTerms; x++) *(uint32_t *)(qs + ((size_t)(x * G + w) * kFaQ + r) * R + d) = tt[x];
    }
    const uint16_t *Kg = a.kc + kvh * HD, *Vg = a.vc + kvh * HD;
    const int ntiles = (kend + kFaK - 1) / kFaK;
    fa_stage<HD, G>(a, Kg, Vg, slot, 0, kend, sk0, sk0 + kFaK * R);
    const int qp0 = pos0 + min(g, nq - 1), qp1 = pos0 + min(g + 8, nq - 1);  // positions of rows g, g + 8
    float o[NT][4];
#pragma unroll
    for (int j = 0; j < NT; j++) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
    const float scale = a.scale;
    for (int kt = 0; kt < ntiles; kt++) {
        uint16_t *sk = sk0 + (size_t)(kt & 1) * 2 * kFaK * R, *sv = sk + kFaK * R;
        if (kt + 1 < ntiles) {
            uint16_t *nk = sk0 + (size_t)((kt + 1) & 1) * 2 * kFaK * R;
            fa_stage<HD, G>(a, Kg, Vg, slot, (kt + 1) * kFaK, kend, nk, nk + kFaK * R);
            asm volatile("cp.async.wait_group 1;" ::: "memory");
        } else {
            asm volatile("cp.async.wait_group 0;" ::: "memory");
        }
        __syncthreads();
        // S = q . K^T for kFaK keys: kFaK/8 key n-tiles x HD/16 k-steps, every q term
        constexpr int NS = kFaK / 8;
        float s[NS][4];
#pragma unroll
        for (int j = 0; j < NS; j++) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
        for (int kk = 0; kk < HD / 16; kk++) {
            const int ro = ((lane >> 3) & 1) * 8 + (lane & 7), co = kk * 16 + (lane >> 4) * 8;
            uint32_t aq[kFaTerms][4];
#pragma unroll
            for (int x = 0; x < kFaTerms; x++) fa_ldm4(aq[x], qs + ((size_t)(x * G + w) * kFaQ + ro) * R + co);
#pragma unroll
            for (int j = 0; j < NS; j++) {
                const uint16_t *kr = sk + (j * 8 + g) * R + kk * 16 + 2 * tq;
                const uint32_t b0 = *(const uint32_t *)kr, b1 = *(const uint32_t *)(kr + 8);
#pragma unroll
                for (int x = kFaTerms - 1; x >= 0; x--) fa_mma(s[j], aq[x], b0, b1);  // small terms first
            }
        }
        // online softmax over this tile (rows g and g + 8 of the warp)
        const int kb = kt * kFaK;
        float tm0 = -INFINITY, tm1 = -INFINITY;
#pragma unroll
        for (int j = 0; j < NS; j++) {
            const int key = kb + j * 8 + 2 * tq;
            s[j][0] = key <= qp0 ? s[j][0] * scale : -INFINITY;
            s[j][1] = key + 1 <= qp0 ? s[j][1] * scale : -INFINITY;
            s[j][2] = key <= qp1 ? s[j][2] * scale : -INFINITY;
            s[j][3] = key + 1 <= qp1 ? s[j][3] * scale : -INFINITY;
            tm0 = fmaxf(tm0, fmaxf(s[j][0], s[j][1]));
            tm1 = fmaxf(tm1, fmaxf(s[j][2], s[j][3]));
        }
        tm0 = fmaxf(tm0, __shfl_xor_sync(0xffffffffu, tm0, 1));
        tm0 = fmaxf(tm0, __shfl_xor_sync(0xffffffffu, tm0, 2));
        tm1 = fmaxf(tm1, __shfl_xor_sync(0xffffffffu, tm1, 1));
        tm1 = fmaxf(tm1, __shfl_xor_sync(0xffffffffu, tm1, 2));
        const float mn0 = fmaxf(m0, tm0), mn1 = fmaxf(m1, tm1);  // finite: key 0 is always visible
        const float c0 = expf(m0 - mn0), c1 = expf(m1 - mn1);
        m0 = mn0;
        m1 = mn1;
        l0 *= c0;
        l1 *= c1;
#pragma unroll
        for (int j = 0; j < NT; j++) {
            o[j][0] *= c0;
            o[j][1] *= c0;
            o[j][2] *= c1;
            o[j][3] *= c1;
        }
        // P (three bf16 terms) as A fragments, then O += P . V over kFaK/16 key k-steps
#pragma unroll
        for (int kk = 0; kk < kFaK / 16; kk++) {
            float p[8];
#pragma unroll
            for (int u = 0; u < 2; u++) {
                const int j = 2 * kk + u;
                p[4 * u + 0] = expf(s[j][0] - mn0);
                p[4 * u + 1] = expf(s[j][1] - mn0);
                p[4 * u + 2] = expf(s[j][2] - mn1);
                p[4 * u + 3] = expf(s[j][3] - mn1);
                l0 += p[4 * u + 0] + p[4 * u + 1];
                l1 += p[4 * u + 2] + p[4 * u + 3];
            }
            uint32_t pa[kFaTerms][4], tt[kFaTerms];
            // A fragment order: row g keys 2t | row g+8 keys 2t | row g keys 8+2t | row g+8 keys 8+2t
#pragma unroll
            for (int f = 0; f < 4; f++) {
                fa_split(p[2 * f], p[2 * f + 1], tt);
#pragma unroll
                for (int x = 0; x < kFaTerms; x++) pa[x][f] = tt[x];
            }
#pragma unroll
            for (int j = 0; j < NT; j += 2) {
                // V rows kk*16 .. +15, dims 8j .. 8j + 15: four transposed 8x8 matrices
                const int vr = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8, vc = j * 8 + (lane >> 4) * 8;
                uint32_t b[4];
                fa_ldm4t(b, sv + vr * R + vc);
#pragma unroll
                for (int x = kFaTerms - 1; x >= 0; x--) {
                    fa_mma(o[j], pa[x], b[0], b[1]);
                    fa_mma(o[j + 1], pa[x], b[2], b[3]);
                }
            }
        }
        __syncthreads();  // the stage is refilled next
    }
    l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
    l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
    const float i0 = 1.0f / l0, i1 = 1.0f / l1;
#pragma unroll
    for (int j = 0; j < NT; j++) {
        const int d = j * 8 + 2 * tq;
        if (g < nq) *(float2 *)(a.ao + (size_t)(t0 + g) * a.qdim + head * HD + d) = make_float2(o[j][0] * i0, o[j][1] * i0);
        if (g + 8 < nq)
            *(float2 *)(a.ao + (size_t)(t0 + g + 8) * a.qdim + head * HD + d) = make_float2(o[j][2] * i1, o[j][3] * i1);
    }
}

}  // namespace hyk
