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
};

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
    pdl_wait();
    const int t = blockIdx.x, w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int pos = *a.pos_ptr + t;
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
            uint16_t *kd = a.kc + (size_t)pos * a.kvdim + kvh * HD, *vd = a.vc + (size_t)pos * a.kvdim + kvh * HD;
#pragma unroll
            for (int i = 0; i < HD / 32; i++) {
                kd[lane + 32 * i] = f32_to_bf16_bits(v[i]);
                vd[lane + 32 * i] = f32_to_bf16_bits(vs[lane + 32 * i]);
            }
        }
    }
    pdl_trigger();
}

// Core loop shared by decode and prefill: keys [j0, j1) for the G heads of
// KV head kvh, query rows in sq[G][HD].  Key `cur` (if >= 0) is taken from
// sk/sv (values already bf16-rounded) instead of the cache.
template <int HD, int G>
__device__ __forceinline__ void attend_range(const AttnArgs &a, int kvh, int j0, int j1, int cur, const float (*sq)[HD],
                                             const float *sk, const float *sv, float (&m)[G], float (&l)[G],
                                             float (&o)[G][HD / 32]) {
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
    for (int h = 0; h < G; h++) {
        m[h] = -INFINITY;
        l[h] = 0.f;
#pragma unroll
        for (int i = 0; i < HD / 32; i++) o[h][i] = 0.f;
    }
    const uint16_t *Kb = a.kc + kvh * HD, *Vb = a.vc + kvh * HD;
    for (int tile = j0 + w * 32; tile < j1; tile += G * 32) {
        const int j = tile + lane;
        const bool valid = j < j1;
        float s[G];
#pragma unroll
        for (int h = 0; h < G; h++) s[h] = 0.f;
        if (valid) {
            if (j == cur) {
#pragma unroll 4
                for (int d = 0; d < HD; d++) {
                    const float kv = sk[d];
#pragma unroll
                    for (int h = 0; h < G; h++) s[h] = fmaf(sq[h][d], kv, s[h]);
                }
            } else {
                const uint16_t *kr = Kb + (size_t)j * a.kvdim;
#pragma unroll 2
                for (int d8 = 0; d8 < HD; d8 += 8) {
                    const uint4 kk = *(const uint4 *)(kr + d8);
                    const uint32_t kw[4] = {kk.x, kk.y, kk.z, kk.w};
#pragma unroll
                    for (int q = 0; q < 4; q++) {
                        const float k0 = bf16_bits_to_f32(kw[q] & 0xffffu), k1 = bf16_bits_to_f32(kw[q] >> 16);
#pragma unroll
                        for (int h = 0; h < G; h++) {
                            s[h] = fmaf(sq[h][d8 + 2 * q], k0, s[h]);
                            s[h] = fmaf(sq[h][d8 + 2 * q + 1], k1, s[h]);
                        }
                    }
                }
            }
        }
        float p[G];
#pragma unroll
        for (int h = 0; h < G; h++) {
            const float sc = valid ? s[h] * a.scale : -INFINITY;
            const float mt = warp_max(sc);
            const float mn = fmaxf(m[h], mt);
            const float corr = expf(m[h] - mn);
            p[h] = valid ? expf(sc - mn) : 0.f;
            l[h] = l[h] * corr + warp_sum(p[h]);
            m[h] = mn;
#pragma unroll
            for (int i = 0; i < HD / 32; i++) o[h][i] *= corr;
        }
        const int nk = min(32, j1 - tile);
        for (int jj = 0; jj < nk; jj++) {
            const int jk = tile + jj;
            float vv[HD / 32];
            if (jk == cur) {
#pragma unroll
                for (int i = 0; i < HD / 32; i++) vv[i] = sv[lane + 32 * i];
            } else {
                const uint16_t *vr = Vb + (size_t)jk * a.kvdim;
#pragma unroll
                for (int i = 0; i < HD / 32; i++) vv[i] = bf16_bits_to_f32(vr[lane + 32 * i]);
            }
#pragma unroll
            for (int h = 0; h < G; h++) {
                const float pj = __shfl_sync(0xffffffffu, p[h], jj);
#pragma unroll
                for (int i = 0; i < HD / 32; i++) o[h][i] = fmaf(pj, vv[i], o[h][i]);
            }
        }
    }
}

template <int HD, int G>
struct AttnSmem {
    float sq[G][HD];
    float sk[HD], sv[HD];
    float pm[G][G], pl[G][G];
    float po[G][G][HD];
    int last;
};

// Merge the G warps' partial (m, l, o) for head h = warp into (M, L, O).
template <int HD, int G>
__device__ __forceinline__ void merge_warps(AttnSmem<HD, G> &S, float &M, float &L, float (&O)[HD / 32]) {
    const int h = threadIdx.x >> 5, lane = threadIdx.x & 31;
    M = -INFINITY;
#pragma unroll
    for (int w = 0; w < G; w++) M = fmaxf(M, S.pm[w][h]);
    L = 0.f;
#pragma unroll
    for (int i = 0; i < HD / 32; i++) O[i] = 0.f;
#pragma unroll
    for (int w = 0; w < G; w++) {
        const float f = S.pl[w][h] > 0.f ? expf(S.pm[w][h] - M) : 0.f;
        L = fmaf(S.pl[w][h], f, L);
#pragma unroll
        for (int i = 0; i < HD / 32; i++) O[i] = fmaf(S.po[w][h][lane + 32 * i], f, O[i]);
    }
}

// Decode: one query token at *pos_ptr.  grid (kv_heads, max_splits), G warps.
// Prologue (each CTA): rope+norm of its G q heads and of k, bf16 k/v; split 0
// stores k/v into the cache.  Splits beyond the live context exit at once.
template <int HD, int G>
__global__ void __launch_bounds__(G * 32) attn_decode(const __grid_constant__ AttnArgs a) {
    __shared__ AttnSmem<HD, G> S;
    const int kvh = blockIdx.x, split = blockIdx.y;
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    pdl_wait();
    const int pos = *a.pos_ptr, n = pos + 1;
    const int j0 = split * a.split_len;
    // a position outside the cache (decode driven past ctx) writes nothing
    if (j0 >= n || pos < 0 || pos >= a.ctx) {
        pdl_trigger();
        return;
    }
    const int j1 = min(n, j0 + a.split_len);
    const int nsplit = (n + a.split_len - 1) / a.split_len;
    const float *cs = a.rope_cos + (size_t)pos * a.half, *sn = a.rope_sin + (size_t)pos * a.half;
    {
        const int h = kvh * G + w;
        float v[HD / 32];
#pragma unroll
        for (int i = 0; i < HD / 32; i++) v[i] = a.qkv[h * HD + lane + 32 * i];
        rope_norm_warp<HD>(v, cs, sn, a.q_norm, a.eps);
#pragma unroll
        for (int i = 0; i < HD / 32; i++) S.sq[w][lane + 32 * i] = v[i];
        if (w == 0) {
            float kv[HD / 32];
            const float *kr = a.qkv + a.qdim + kvh * HD, *vr = a.qkv + a.qdim + a.kvdim + kvh * HD;
#pragma unroll
            for (int i = 0; i < HD / 32; i++) kv[i] = kr[lane + 32 * i];
            rope_norm_warp<HD>(kv, cs, sn, a.k_norm, a.eps);
            uint16_t *kd = a.kc + (size_t)pos * a.kvdim + kvh * HD, *vd = a.vc + (size_t)pos * a.kvdim + kvh * HD;
#pragma unroll
            for (int i = 0; i < HD / 32; i++) {
                const int e = lane + 32 * i;
                const uint16_t kb = f32_to_bf16_bits(kv[i]), vb = f32_to_bf16_bits(vr[e]);
                S.sk[e] = bf16_bits_to_f32(kb);
                S.sv[e] = bf16_bits_to_f32(vb);
                if (split == 0) {
                    kd[e] = kb;
                    vd[e] = vb;
                }
            }
        }
    }
    __syncthreads();
    pdl_trigger();
    float m[G], l[G], o[G][HD / 32];
    attend_range<HD, G>(a, kvh, j0, j1, pos, S.sq, S.sk, S.sv, m, l, o);
#pragma unroll
    for (int h = 0; h < G; h++) {
        if (lane == 0) {
            S.pm[w][h] = m[h];
            S.pl[w][h] = l[h];
        }
#pragma unroll
        for (int i = 0; i < HD / 32; i++) S.po[w][h][lane + 32 * i] = o[h][i];
    }
    __syncthreads();
    float M, L, O[HD / 32];
    merge_warps<HD, G>(S, M, L, O);
    const int h = kvh * G + w;
    if (nsplit == 1) {
        const float inv = 1.0f / L;
#pragma unroll
        for (int i = 0; i < HD / 32; i++) a.ao[h * HD + lane + 32 * i] = O[i] * inv;
        return;
    }
    float *pp = a.part + (((size_t)kvh * a.max_splits + split) * G + w) * (HD + 2);
#pragma unroll
    for (int i = 0; i < HD / 32; i++) pp[2 + lane + 32 * i] = O[i];
    if (lane == 0) {
        pp[0] = M;
        pp[1] = L;
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) S.last = atomicAdd(&a.tickets[kvh], 1) == nsplit - 1;
    __syncthreads();
    if (!S.last) return;
    __threadfence();
    float MM = -INFINITY;
    for (int sp = 0; sp < nsplit; sp++)
        MM = fmaxf(MM, __ldcg(a.part + (((size_t)kvh * a.max_splits + sp) * G + w) * (HD + 2)));
    float LL = 0.f, OO[HD / 32];
#pragma unroll
    for (int i = 0; i < HD / 32; i++) OO[i] = 0.f;
    for (int sp = 0; sp < nsplit; sp++) {
        const float *q = a.part + (((size_t)kvh * a.max_splits + sp) * G + w) * (HD + 2);
        const float f = expf(__ldcg(q) - MM);
        LL = fmaf(__ldcg(q + 1), f, LL);
#pragma unroll
        for (int i = 0; i < HD / 32; i++) OO[i] = fmaf(__ldcg(q + 2 + lane + 32 * i), f, OO[i]);
    }
    const float inv = 1.0f / LL;
#pragma unroll
    for (int i = 0; i < HD / 32; i++) a.ao[h * HD + lane + 32 * i] = OO[i] * inv;
    if (threadIdx.x == 0) a.tickets[kvh] = 0;
}

// Prefill: token t (position *pos_ptr + t) attends to 0..pos inclusive; q
// already rotated/normalised and k/v already in the cache (rope_norm_store).
// grid (kv_heads, nt), G warps.
template <int HD, int G>
__global__ void __launch_bounds__(G * 32) attn_prefill(const __grid_constant__ AttnArgs a) {
    __shared__ AttnSmem<HD, G> S;
    const int kvh = blockIdx.x, t = blockIdx.y;
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    pdl_wait();
    const int pos = *a.pos_ptr + t;
    const float *qr = a.qkv + (size_t)t * a.qkv_ld + (kvh * G + w) * HD;
#pragma unroll
    for (int i = 0; i < HD / 32; i++) S.sq[w][lane + 32 * i] = qr[lane + 32 * i];
    __syncthreads();
    pdl_trigger();
    float m[G], l[G], o[G][HD / 32];
    attend_range<HD, G>(a, kvh, 0, pos + 1, -1, S.sq, S.sk, S.sv, m, l, o);
#pragma unroll
    for (int h = 0; h < G; h++) {
        if (lane == 0) {
            S.pm[w][h] = m[h];
            S.pl[w][h] = l[h];
        }
#pragma unroll
        for (int i = 0; i < HD / 32; i++) S.po[w][h][lane + 32 * i] = o[h][i];
    }
    __syncthreads();
    float M, L, O[HD / 32];
    merge_warps<HD, G>(S, M, L, O);
    const float inv = 1.0f / L;
    float *dst = a.ao + (size_t)t * a.qdim + (kvh * G + w) * HD;
#pragma unroll
    for (int i = 0; i < HD / 32; i++) dst[lane + 32 * i] = O[i] * inv;
}

}  // namespace hyk
