// hy_gemv.cuh — quantised GEMV / small-batch GEMM on CUDA cores (sm_100a).
//
// One launch computes out[t][row] = dot(W[row], act[t]) for up to three
// weights that share one activation (q/k/v, gate/up), t < nt <= NT.
//
// Prologue: every CTA builds the activation in shared memory itself —
// RMSNorm / SiLU*up / plain copy, then the Q8_K quantiser (bit-identical to
// reference src/kernels.c:128-165) — so no separate norm or quantise kernel
// and no grid-wide barrier sits between producer and GEMV.  Weights of the
// warp's first row are requested from HBM before griddepcontrol.wait, so the
// fetch overlaps the previous kernel's tail.
//
// Main loop: one warp per row; each lane streams 16-byte weight chunks,
// computes exact int32 per-256 block sums with dp4a, reduces each block
// across the lanes that share it (exact), applies the block's scales in the
// host's float order, then sums blocks across the warp.
#pragma once
#include "hy_common.cuh"

namespace hyk {

constexpr int kGemvWarps = 8;
constexpr int kFpInFlight = 8;  // gemv_fp: 16-byte weight units per lane loaded ahead
constexpr int kGemvThreads = kGemvWarps * 32;

struct GemvArgs {
    WDesc w[3];
    int nw;
    int rows_total;
    int nt;
    int k;
    // activation source
    int act;
    const q8k_block *xq;
    const float *x;
    const float *x2;
    int ldx;
    const float *norm_w;
    float eps;
    // epilogue
    int epi;
    unsigned long long *amax;
    int amax_rows;
    int amax_base;  // added to the row index in the argmax key (a vocabulary slice's first row)
    int32_t *ints;  // optional exact per-block integers [nt][rows][nblk]
    int trace;      // timeline slot (< 0: off)
    int interleave; // 2 weights of equal n: merged row m -> weight m & 1, row m >> 1
};

// ---------------------------------------------------------------- activation staging

// Shared-memory plan for the Q8_K activation of NT tokens and K inputs.
struct Q8Smem {
    float *x;        // [K] fp32 staging of one token
    int8_t *qp;      // [NT][4][K/4] plane-major codes
    float *d;        // [NT][nb]
    int *sum;        // [NT][nb]
    int16_t *bs;     // [NT][nb*16]
    float *red;      // [64]
};

__host__ __device__ inline size_t align16(size_t v) { return (v + 15) & ~(size_t)15; }

__host__ __device__ inline size_t q8_smem_bytes(int NT, int K) {
    const int nb = K / 256;
    return align16((size_t)K * 4) + align16((size_t)NT * K) + align16((size_t)NT * nb * 4) * 2 +
           align16((size_t)NT * nb * 32) + 64 * 4;
}

__device__ inline Q8Smem q8_smem(uint8_t *base, int NT, int K) {
    const int nb = K / 256;
    Q8Smem s;
    size_t o = 0;
    s.x = (float *)(base + o); o += align16((size_t)K * 4);
    s.qp = (int8_t *)(base + o); o += align16((size_t)NT * K);
    s.d = (float *)(base + o); o += align16((size_t)NT * nb * 4);
    s.sum = (int *)(base + o); o += align16((size_t)NT * nb * 4);
    s.bs = (int16_t *)(base + o); o += align16((size_t)NT * nb * 32);
    s.red = (float *)(base + o);
    return s;
}

// Block-wide sum over kGemvThreads threads.
__device__ inline float block_sum(float v, float *red) {
    v = warp_sum(v);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) red[w] = v;
    __syncthreads();
    float t = l < (int)(blockDim.x >> 5) ? red[l] : 0.f;
    return warp_sum(t);
}

// Fill dst[K] with token t's fp32 activation according to a.act.  Every
// thread issues all of its 16-byte loads (x, and norm weight or up) before
// using any of them, so the staging costs one L2 round trip, not K/blockDim.
// Needs K % 4 == 0 and K <= 4 * kStageVec * blockDim.x.
constexpr int kStageVec = 8;

// RMSNorm inputs are staged block-wise: warp w of nw holds the Q8_K blocks
// b = w, w + nw, ... (lane l: elements 256 b + 8 l .. 8 l + 7), so the sum of
// squares has one fixed order for any CTA size: each block's 8 squares per
// lane in element order, the warp butterfly per block, then the blocks in
// index order (norm_ss).  Float4 j of a thread is block w + (j >> 1) nw,
// half j & 1 of the lane's 8 elements.
__device__ __forceinline__ int norm_f4(int j, int warp, int lane, int nw) {
    return (warp + (j >> 1) * nw) * 64 + lane * 2 + (j & 1);
}

// The RMSNorm weight is a constant: load it before griddepcontrol.wait.
template <int SV = kStageVec>
__device__ inline void preload_norm(const GemvArgs &a, float4 (&nv)[SV], int K) {
    if (a.act != ACT_NORM) return;
    const float4 *y4 = (const float4 *)a.norm_w;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
#pragma unroll
    for (int j = 0; j < SV; j++) {
        const int i = norm_f4(j, warp, lane, nw);
        if (i < (K >> 2)) nv[j] = __ldg(y4 + i);
    }
}

// Sum of squares of the block-wise staged values xv (see norm_f4): per block
// the lane's 8 squares in element order and the warp butterfly, written to
// red[b]; then every thread adds red[0 .. nb-1] in order.  Needs nb <= 64
// and every thread of the CTA.
template <int SV>
__device__ __forceinline__ float norm_ss(const float4 (&xv)[SV], int K, float *red) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    const int nb = (K + 255) / 256, n4 = K >> 2;
#pragma unroll
    for (int j = 0; j < SV; j += 2) {
        const int b = warp + (j >> 1) * nw;
        float s = 0.f;
#pragma unroll
        for (int h = 0; h < 2; h++) {
            if (j + h < SV && norm_f4(j + h, warp, lane, nw) < n4) {
                const float4 v = xv[j + h];
                s = __fadd_rn(s, __fmul_rn(v.x, v.x));
                s = __fadd_rn(s, __fmul_rn(v.y, v.y));
                s = __fadd_rn(s, __fmul_rn(v.z, v.z));
                s = __fadd_rn(s, __fmul_rn(v.w, v.w));
            }
        }
        s = warp_sum(s);
        if (lane == 0 && b < nb) red[b] = s;
    }
    __syncthreads();
    float ss = 0.f;
    for (int b = 0; b < nb; b++) ss = __fadd_rn(ss, red[b]);
    return ss;
}

template <int SV = kStageVec>
__device__ inline void stage_fp32(const GemvArgs &a, int t, float *dst, float *red, int K,
                                  const float4 (*pre)[SV] = nullptr) {
    const float4 *x4 = (const float4 *)(a.x + (size_t)t * a.ldx);
    const float4 *y4 = a.act == ACT_NORM ? (const float4 *)a.norm_w
                                         : (a.act == ACT_SILU ? (const float4 *)(a.x2 + (size_t)t * a.ldx) : nullptr);
    const int n4 = K >> 2;
    const bool norm = a.act == ACT_NORM;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    float4 *d4 = (float4 *)dst;
    // one set of loads for every mode (RMSNorm inputs in the block-wise layout of norm_f4)
    float4 xv[SV], yv[SV];
#pragma unroll
    for (int j = 0; j < SV; j++) {
        const int i = norm ? norm_f4(j, warp, lane, nw) : (int)threadIdx.x + j * (int)blockDim.x;
        xv[j] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (i < n4) {
            xv[j] = x4[i];
            if (norm && pre) yv[j] = (*pre)[j];
            else if (y4) yv[j] = __ldg(y4 + i);
        }
    }
    if (norm) {
        __syncthreads();  // red and dst may still be read by the previous token's quantiser
        const float ss = norm_ss<SV>(xv, K, red);
        const float scale = 1.0f / sqrtf(ss / (float)K + a.eps);
#pragma unroll
        for (int j = 0; j < SV; j++) {
            const int i = norm_f4(j, warp, lane, nw);
            if (i < n4)
                d4[i] = make_float4(__fmul_rn(__fmul_rn(xv[j].x, scale), yv[j].x),
                                    __fmul_rn(__fmul_rn(xv[j].y, scale), yv[j].y),
                                    __fmul_rn(__fmul_rn(xv[j].z, scale), yv[j].z),
                                    __fmul_rn(__fmul_rn(xv[j].w, scale), yv[j].w));
        }
    } else if (a.act == ACT_SILU) {
#pragma unroll
        for (int j = 0; j < SV; j++) {
            const int i = threadIdx.x + j * blockDim.x;
            if (i < n4) {
                const float4 g = xv[j], u = yv[j];
                d4[i] = make_float4(__fmul_rn(g.x / (1.0f + expf(-g.x)), u.x), __fmul_rn(g.y / (1.0f + expf(-g.y)), u.y),
                                    __fmul_rn(g.z / (1.0f + expf(-g.z)), u.z), __fmul_rn(g.w / (1.0f + expf(-g.w)), u.w));
            }
        }
    } else {
#pragma unroll
        for (int j = 0; j < SV; j++) {
            const int i = threadIdx.x + j * blockDim.x;
            if (i < n4) d4[i] = xv[j];
        }
    }
}

// Q8_K quantisation of one 256 block held in smem `src`, by one warp; writes
// plane-major codes and block constants for token t.  Bit-identical to the
// host quantiser: first index of the largest |x|, iscale = -127/max,
// d = 1/iscale, round-half-even, clip +-127, non-finite products -> 0.
// The block's values are in registers: lane l holds elements 8 l .. 8 l + 7.
__device__ inline void quantize_vals_warp(const float (&v)[8], Q8Smem &s, int t, int b, int nb, int K) {
    const int lane = threadIdx.x & 31;
    // lane-local first maximum of |x|, then one redux for the max and one
    // for the smallest index holding it (finite |x| bit patterns order like
    // the values; NaN never qualifies, as in the host's strict '>')
    float ba = 0.f, lv = 0.f;
    int li = 0x7fffffff;
#pragma unroll
    for (int j = 0; j < 8; j++) {
        const float av = fabsf(v[j]);
        if (av > ba) { ba = av; lv = v[j]; li = lane * 8 + j; }
    }
    const unsigned mbits = __reduce_max_sync(0xffffffffu, __float_as_uint(ba));
    const unsigned cand = (__float_as_uint(ba) == mbits) ? (unsigned)li : 0x7fffffffu;
    const int bi = (int)__reduce_min_sync(0xffffffffu, cand);
    ba = __uint_as_float(mbits);
    const float bv = __shfl_sync(0xffffffffu, lv, (bi >> 3) & 31);
    int q[8];
    float d = 0.f;
    if (ba == 0.f) {
#pragma unroll
        for (int j = 0; j < 8; j++) q[j] = 0;
    } else {
        const float iscale = -127.f / bv;
        d = 1.f / iscale;
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const float f = __fmul_rn(iscale, v[j]);
            int r = isfinite(f) ? __float2int_rn(f) : 0;
            r = r > 127 ? 127 : (r < -127 ? -127 : r);
            q[j] = r;
        }
    }
    int part = 0;
#pragma unroll
    for (int j = 0; j < 8; j++) part += q[j];
    const int pair = part + __shfl_xor_sync(0xffffffffu, part, 1);
    const int total = __reduce_add_sync(0xffffffffu, part);
    // natural element e = lane*8 + j -> chunk ch = lane/8, plane l = (lane%8)/2, byte (lane&1)*8 + j
    const int ch = lane >> 3, l = (lane & 7) >> 1;
    const int pos = (b * 4 + piece_of_chunk(ch)) * 16 + (lane & 1) * 8;
    int8_t *dst = s.qp + (size_t)t * K + (size_t)l * (K / 4) + pos;
    uint32_t lo = (q[0] & 0xff) | ((q[1] & 0xff) << 8) | ((q[2] & 0xff) << 16) | ((uint32_t)(q[3] & 0xff) << 24);
    uint32_t hi = (q[4] & 0xff) | ((q[5] & 0xff) << 8) | ((q[6] & 0xff) << 16) | ((uint32_t)(q[7] & 0xff) << 24);
    *(uint2 *)dst = make_uint2(lo, hi);
    if ((lane & 1) == 0) s.bs[(size_t)t * nb * 16 + b * 16 + (lane >> 1)] = (int16_t)pair;
    if (lane == 0) {
        s.d[t * nb + b] = d;
        s.sum[t * nb + b] = total;
    }
}

__device__ inline void quantize_block_warp(const float *src, Q8Smem &s, int t, int b, int nb, int K) {
    const int lane = threadIdx.x & 31;
    const float *p = src + b * 256 + lane * 8;
    const float4 v0 = *(const float4 *)&p[0], v1 = *(const float4 *)&p[4];
    const float v[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
    quantize_vals_warp(v, s, t, b, nb, K);
}

// Build the Q8_K activation of all nt tokens in shared memory.
template <int SV = kStageVec>
__device__ inline void stage_q8k(const GemvArgs &a, Q8Smem &s, int K, const float4 (*pre)[SV] = nullptr) {
    const int nb = K / 256;
    const int warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    for (int t = 0; t < a.nt; t++) {
        if (a.act == ACT_Q8K) {
            // host-made blocks: qp is already lane-major per block
            const q8k_block *src = a.xq + (size_t)t * nb;
            for (int i = threadIdx.x; i < nb * 16; i += blockDim.x) {
                const int b = i >> 4, part = i & 15, l = part >> 2, piece = part & 3;
                const uint4 v = *(const uint4 *)&src[b].qp[l * 64 + piece * 16];
                *(uint4 *)&s.qp[(size_t)t * K + (size_t)l * (K / 4) + b * 64 + piece * 16] = v;
            }
            for (int i = threadIdx.x; i < nb * 16; i += blockDim.x)
                s.bs[(size_t)t * nb * 16 + i] = src[i >> 4].bsums[i & 15];
            for (int b = threadIdx.x; b < nb; b += blockDim.x) {
                s.d[t * nb + b] = src[b].d;
                s.sum[t * nb + b] = src[b].sum;
            }
        } else {
            stage_fp32<SV>(a, t, s.x, s.red, K, t == 0 ? pre : nullptr);
            __syncthreads();
            if (t == 0) trace_sub(a.trace, 0);
            for (int b = warp; b < nb; b += nwarps) quantize_block_warp(s.x, s, t, b, nb, K);
        }
        __syncthreads();
        if (t == 0) trace_sub(a.trace, 1);
    }
}

// ---------------------------------------------------------------- row bookkeeping

__device__ __forceinline__ void map_row(const GemvArgs &a, int r, int &wi, int &lr) {
    if (a.interleave) {
        wi = r & 1;
        lr = r >> 1;
        return;
    }
    wi = 0;
    lr = r;
    if (a.nw > 1 && lr >= a.w[0].n) {
        lr -= a.w[0].n;
        wi = 1;
        if (a.nw > 2 && lr >= a.w[1].n) {
            lr -= a.w[1].n;
            wi = 2;
        }
    }
}

__device__ __forceinline__ const WDesc &wsel(const GemvArgs &a, int wi) {
    return wi == 0 ? a.w[0] : (wi == 1 ? a.w[1] : a.w[2]);
}

// Lane 0 applies the row epilogue; `best` tracks the warp's argmax candidate.
template <int NT>
__device__ __forceinline__ void row_epilogue(const GemvArgs &a, const WDesc &w, int lr, int row, const float *res,
                                             unsigned long long &best) {
    if ((threadIdx.x & 31) != 0) return;
    if (a.epi == EPI_ARGMAX) {
        if (w.out) w.out[lr] = res[0];
        if (row < a.amax_rows) {
            const unsigned long long key = argmax_key(res[0], (uint32_t)(row + a.amax_base));
            if (key > best) best = key;
        }
        return;
    }
#pragma unroll
    for (int t = 0; t < NT; t++) {
        if (t >= a.nt) break;
        float *o = w.out + (size_t)t * w.ld + lr;
        if (a.epi == EPI_ADD) *o += res[t];
        else *o = res[t];
    }
}

__device__ inline void argmax_commit(const GemvArgs &a, unsigned long long best, float *red_area) {
    trace_mark(a.trace, 3);
    if (a.epi != EPI_ARGMAX) return;
    unsigned long long *sk = (unsigned long long *)red_area;
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) sk[w] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned long long m = 0;
        for (int i = 0; i < (int)(blockDim.x >> 5); i++) m = sk[i] > m ? sk[i] : m;
        if (m) atomicMax(a.amax, m);
    }
}

// ---------------------------------------------------------------- PANEL (STQ1_0 / Q2_0C)

// dp4a of unsigned weight bytes (0..255) with signed activation bytes.
__device__ __forceinline__ int dp4a_us(uint32_t a, int b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// Exact block integer of one 16-byte panel chunk against 64 activation bytes
// (4 planes x 16): sum_l sum_i code_l(w[i]) * a_l[i].  Plane l's codes are
// masked in place (bits 2l..2l+1 of every byte, no shift), so its dot product
// is 4^l times the plane's sum, an exact multiple that an arithmetic shift
// divides back out; four independent dp4a chains, one per plane.
__device__ __forceinline__ int panel_chunk_dot4(const uint4 wv, const int4 *act4) {
    const uint32_t wd[4] = {wv.x, wv.y, wv.z, wv.w};
    int e0 = 0, e1 = 0, e2 = 0, e3 = 0;
#pragma unroll
    for (int j = 0; j < 4; j++) {
        e0 = dp4a_us(wd[j] & 0x03030303u, ((const int *)&act4[0])[j], e0);
        e1 = dp4a_us(wd[j] & 0x0c0c0c0cu, ((const int *)&act4[1])[j], e1);
        e2 = dp4a_us(wd[j] & 0x30303030u, ((const int *)&act4[2])[j], e2);
        e3 = dp4a_us(wd[j] & 0xc0c0c0c0u, ((const int *)&act4[3])[j], e3);
    }
    return (e0 + (e1 >> 2)) + ((e2 >> 4) + (e3 >> 6));
}
__device__ __forceinline__ int panel_chunk_dot(const uint4 wv, const int4 *act4) { return panel_chunk_dot4(wv, act4); }

// One lane's 64-weight unit u of a row (u = 4 b + p: panel chunk u), as
// loaded from HBM, for the two 2-bit layouts.  PANEL: the 16-byte chunk of
// pre-decoded codes and the block's fp32 scale.  STQN (native STQ1_0, 42 B /
// 256): 8 bytes of slots, 16 sign bits and the f16 scale, decoded in
// registers (stq_decode_unit) into the identical chunk.
template <int FMT>
struct PUnit;
template <>
struct PUnit<FMT_PANEL> {
    uint4 w;
    float s;
    __device__ __forceinline__ void load(const WDesc &d, int r, int u, int nb) {
        w = ldg_stream(d.w + (size_t)r * d.stride + (size_t)u * 16);
        s = __ldg(d.s + (size_t)r * nb + (u >> 2));
    }
    __device__ __forceinline__ uint4 codes() const { return w; }
};
template <>
struct PUnit<FMT_STQN> {
    uint2 q;
    uint32_t sg, dh;
    __device__ __forceinline__ void load(const WDesc &d, int r, int u, int nb) {
        const uint8_t *row = d.w + (size_t)r * d.stride;
        q = ldg_stream8(row + (size_t)u * 8);
        sg = ldg_stream16(row + (size_t)nb * 32 + (size_t)u * 2);
        dh = ldg_stream16(row + (size_t)nb * 40 + (size_t)(u >> 2) * 2);
    }
    __device__ __forceinline__ uint4 codes() const { return stq_decode_unit(q, sg); }
    __device__ __forceinline__ float scale() const { return h2f((uint16_t)dh); }
};
__device__ __forceinline__ float punit_scale(const PUnit<FMT_PANEL> &u) { return u.s; }
__device__ __forceinline__ float punit_scale(const PUnit<FMT_STQN> &u) { return u.scale(); }

// Decode (nt == 1): the lane's activation chunks live in registers for the
// whole launch.  CPL = 16-byte chunks per lane per row (K <= 2048*CPL).
template <int CPL, int FMT = FMT_PANEL>
__global__ void __launch_bounds__(kGemvThreads) gemv_panel_nt1(const __grid_constant__ GemvArgs a) {
    trace_mark(a.trace, 0);
    pdl_trigger();
    extern __shared__ __align__(16) uint8_t smem[];
    const int K = a.k, nb = K / 256, nchunk = nb * 4;
    const int lane = threadIdx.x & 31;
    const int gw = blockIdx.x * kGemvWarps + (threadIdx.x >> 5), nw = gridDim.x * kGemvWarps;

    // prefetch the first row's weights before waiting on the producer
    PUnit<FMT> wcur[CPL];
    int r = gw, wi = 0, lr = 0;
    if (r < a.rows_total) {
        map_row(a, r, wi, lr);
        const WDesc &w = wsel(a, wi);
#pragma unroll
        for (int i = 0; i < CPL; i++) {
            const int c = lane + 32 * i;
            if (c < nchunk) wcur[i].load(w, lr, c, nb);
        }
    }
    pdl_wait();
    trace_mark(a.trace, 1);
    Q8Smem s = q8_smem(smem, 1, K);
    stage_q8k(a, s, K);
    trace_mark(a.trace, 2);

    int4 act[CPL][4];
    float dblk[CPL];
    int sblk[CPL];
#pragma unroll
    for (int i = 0; i < CPL; i++) {
        const int c = lane + 32 * i;
        if (c < nchunk) {
#pragma unroll
            for (int l = 0; l < 4; l++) act[i][l] = *(const int4 *)&s.qp[(size_t)l * (K / 4) + c * 16];
            dblk[i] = s.d[c >> 2];
            sblk[i] = s.sum[c >> 2];
        } else {
#pragma unroll
            for (int l = 0; l < 4; l++) act[i][l] = make_int4(0, 0, 0, 0);
            dblk[i] = 0.f;
            sblk[i] = 0;
        }
    }

    unsigned long long best = 0;
    for (; r < a.rows_total; r += nw) {
        // issue the next row's loads before computing this one
        const int rn = r + nw;
        int wn = 0, ln = 0;
        PUnit<FMT> wnext[CPL];
        if (rn < a.rows_total) {
            map_row(a, rn, wn, ln);
            const WDesc &w2 = wsel(a, wn);
#pragma unroll
            for (int i = 0; i < CPL; i++) {
                const int c = lane + 32 * i;
                if (c < nchunk) wnext[i].load(w2, ln, c, nb);
            }
        }
        const WDesc &w = wsel(a, wi);
        float acc = 0.f;
#pragma unroll
        for (int i = 0; i < CPL; i++) {
            const int c = lane + 32 * i;
            int e = c < nchunk ? panel_chunk_dot(wcur[i].codes(), act[i]) : 0;
            e += __shfl_xor_sync(0xffffffffu, e, 1);
            e += __shfl_xor_sync(0xffffffffu, e, 2);
            if (c < nchunk && (lane & 3) == 0) {
                const int v = e * (1 << w.shift) - w.off * sblk[i];
                if (a.ints) a.ints[(size_t)r * nb + (c >> 2)] = v;
                acc += punit_scale(wcur[i]) * dblk[i] * (float)v;
            }
        }
        acc = warp_sum(acc);
        row_epilogue<1>(a, w, lr, r, &acc, best);
#pragma unroll
        for (int i = 0; i < CPL; i++) wcur[i] = wnext[i];
        wi = wn;
        lr = ln;
    }
    argmax_commit(a, best, s.red);
}

// Decode (nt == 1) with the CTA's whole weight slice staged in shared memory.
// CTA c owns rows [c*rows_per_cta, ...) of the merged row space; before
// griddepcontrol.wait it issues cp.async copies of those rows' 64-byte panel
// blocks and scales (weights never depend on the previous kernel), so the
// HBM stream overlaps the producer kernel; after the wait it only builds the
// activation and computes from shared memory.
__host__ __device__ inline size_t panel_dec_smem(int rows_per_cta, int K, int fmt = FMT_PANEL) {
    const int nb = K / 256;
    if (fmt == FMT_STQN) return align16((size_t)rows_per_cta * align16((size_t)nb * 42)) + q8_smem_bytes(1, K);
    return align16((size_t)rows_per_cta * nb * 64) + align16((size_t)rows_per_cta * nb * 4) + q8_smem_bytes(1, K);
}

__device__ __forceinline__ void cp_async4(void *dst, const void *src) {
    const unsigned d = (unsigned)__cvta_generic_to_shared(dst);
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(d), "l"(src) : "memory");
}


// FMT_STQN stages each row's native bytes whole (qs | sign | d, the row
// stride) and decodes the patterns from shared memory (stq_decode_unit).
template <int CPL, int FMT = FMT_PANEL>
__global__ void __launch_bounds__(kGemvThreads) gemv_panel_dec(const __grid_constant__ GemvArgs a, int rows_per_cta) {
    constexpr int RG = CPL == 1 ? 4 : 2;  // rows per warp iteration (independent chains)
    constexpr bool NATIVE = FMT == FMT_STQN;
    extern __shared__ __align__(16) uint8_t smem[];
    trace_mark(a.trace, 0);
    pdl_trigger();
    const int K = a.k, nb = K / 256, nchunk = nb * 4;
    const int row_b = NATIVE ? (int)a.w[0].stride : nb * 64;  // merged weights share K, so the stride
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int r0 = blockIdx.x * rows_per_cta;
    const int r1 = min(r0 + rows_per_cta, a.rows_total);
    uint8_t *sw = smem;
    float *ss = (float *)(smem + align16((size_t)rows_per_cta * row_b));
    uint8_t *sact = smem + align16((size_t)rows_per_cta * row_b) + (NATIVE ? 0 : align16((size_t)rows_per_cta * nb * 4));
    // stage the weight slice (16-byte chunks) and scales (4-byte) asynchronously
    const int units = row_b / 16;
    for (int idx = threadIdx.x; idx < (r1 - r0) * units; idx += blockDim.x) {
        const int rr = idx / units, c = idx - rr * units;
        int wi, lr;
        map_row(a, r0 + rr, wi, lr);
        const WDesc &w = wsel(a, wi);
        cp_async16(sw + (size_t)rr * row_b + c * 16, w.w + (size_t)lr * w.stride + (size_t)c * 16);
    }
    if constexpr (!NATIVE) {
        for (int idx = threadIdx.x; idx < (r1 - r0) * nb; idx += blockDim.x) {
            const int rr = idx / nb, b = idx - rr * nb;
            int wi, lr;
            map_row(a, r0 + rr, wi, lr);
            const WDesc &w = wsel(a, wi);
            cp_async4(ss + (size_t)rr * nb + b, w.s + (size_t)lr * nb + b);
        }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
    constexpr int SV = 2 * CPL;  // K <= 2048*CPL: 2*CPL float4 per thread at 256 threads
    float4 nv[SV];
    preload_norm<SV>(a, nv, K);
    pdl_wait();
    trace_mark(a.trace, 1);
    Q8Smem s = q8_smem(sact, 1, K);
    stage_q8k<SV>(a, s, K, &nv);
    trace_mark(a.trace, 2);
    int4 act[CPL][4];
    float dblk[CPL];
    int sblk[CPL];
#pragma unroll
    for (int i = 0; i < CPL; i++) {
        const int c = lane + 32 * i;
        if (c < nchunk) {
#pragma unroll
            for (int l = 0; l < 4; l++) act[i][l] = *(const int4 *)&s.qp[(size_t)l * (K / 4) + c * 16];
            dblk[i] = s.d[c >> 2];
            sblk[i] = s.sum[c >> 2];
        } else {
#pragma unroll
            for (int l = 0; l < 4; l++) act[i][l] = make_int4(0, 0, 0, 0);
            dblk[i] = 0.f;
            sblk[i] = 0;
        }
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncthreads();
    trace_sub(a.trace, 2);
    const int shift = a.w[0].shift, off = a.w[0].off;  // merged weights share the format
    unsigned long long best = 0;
    for (int rb = r0 + warp * RG; rb < r1; rb += kGemvWarps * RG) {
        float acc[RG];
#pragma unroll
        for (int g = 0; g < RG; g++) acc[g] = 0.f;
#pragma unroll
        for (int i = 0; i < CPL; i++) {
            const int c = lane + 32 * i;
            int e[RG];
#pragma unroll
            for (int g = 0; g < RG; g++) {
                e[g] = 0;
                if (c < nchunk && rb + g < r1) {
                    const uint8_t *srow = sw + (size_t)(rb + g - r0) * row_b;
                    uint4 wv;
                    if constexpr (NATIVE)
                        wv = stq_decode_unit(*(const uint2 *)(srow + c * 8),
                                             *(const uint16_t *)(srow + nb * 32 + c * 2));
                    else
                        wv = *(const uint4 *)(srow + c * 16);
                    e[g] = panel_chunk_dot4(wv, act[i]);
                }
            }
#pragma unroll
            for (int g = 0; g < RG; g++) e[g] += __shfl_xor_sync(0xffffffffu, e[g], 1);
#pragma unroll
            for (int g = 0; g < RG; g++) e[g] += __shfl_xor_sync(0xffffffffu, e[g], 2);
            if (c < nchunk && (lane & 3) == 0) {
#pragma unroll
                for (int g = 0; g < RG; g++) {
                    if (rb + g >= r1) break;
                    const int v = e[g] * (1 << shift) - off * sblk[i];
                    if (a.ints) a.ints[(size_t)(rb + g) * nb + (c >> 2)] = v;
                    float sc;
                    if constexpr (NATIVE)
                        sc = h2f(*(const uint16_t *)(sw + (size_t)(rb + g - r0) * row_b + nb * 40 + (c >> 2) * 2));
                    else
                        sc = ss[(size_t)(rb + g - r0) * nb + (c >> 2)];
                    acc[g] += sc * dblk[i] * (float)v;
                }
            }
        }
        // only lanes 4k hold partial sums: three butterfly levels bring them to lane 0
#pragma unroll
        for (int o = 16; o >= 4; o >>= 1)
#pragma unroll
            for (int g = 0; g < RG; g++) acc[g] += __shfl_xor_sync(0xffffffffu, acc[g], o);
        if (a.epi == EPI_SILU) {
            // rows come in (gate, up) pairs of the same output index
            if (lane == 0) {
#pragma unroll
                for (int g = 0; g + 1 < RG; g += 2) {
                    if (rb + g + 1 >= r1) break;
                    const float gt = acc[g], up = acc[g + 1];
                    a.w[0].out[(rb + g) >> 1] = __fmul_rn(gt / (1.0f + expf(-gt)), up);
                }
            }
        } else {
#pragma unroll
            for (int g = 0; g < RG; g++) {
                if (rb + g >= r1) break;
                int wi, lr;
                map_row(a, rb + g, wi, lr);
                row_epilogue<1>(a, wsel(a, wi), lr, rb + g, &acc[g], best);
            }
        }
    }
    trace_sub(a.trace, 3);
    argmax_commit(a, best, s.red);
}

// Small batches (1 < nt <= NT): activations read from plane-major smem.
template <int NT, int FMT = FMT_PANEL>
__global__ void __launch_bounds__(kGemvThreads) gemv_panel_nt(const __grid_constant__ GemvArgs a) {
    trace_mark(a.trace, 0);
    pdl_trigger();
    extern __shared__ __align__(16) uint8_t smem[];
    const int K = a.k, nb = K / 256, nchunk = nb * 4;
    const int lane = threadIdx.x & 31;
    const int gw = blockIdx.x * kGemvWarps + (threadIdx.x >> 5), nw = gridDim.x * kGemvWarps;
    pdl_wait();
    trace_mark(a.trace, 1);
    Q8Smem s = q8_smem(smem, NT, K);
    stage_q8k(a, s, K);
    trace_mark(a.trace, 2);
    unsigned long long best = 0;
    for (int r = gw; r < a.rows_total; r += nw) {
        int wi, lr;
        map_row(a, r, wi, lr);
        const WDesc &w = wsel(a, wi);
        float acc[NT];
#pragma unroll
        for (int t = 0; t < NT; t++) acc[t] = 0.f;
        for (int c0 = 0; c0 < nchunk; c0 += 32) {
            const int c = c0 + lane;
            const bool ok = c < nchunk;
            uint4 wv = make_uint4(0, 0, 0, 0);
            float sc = 0.f;
            if (ok) {
                PUnit<FMT> pu;
                pu.load(w, lr, c, nb);
                wv = pu.codes();
                sc = punit_scale(pu);
            }
            const uint32_t wd[4] = {wv.x, wv.y, wv.z, wv.w};
            uint32_t code[4][4];
#pragma unroll
            for (int j = 0; j < 4; j++)
#pragma unroll
                for (int l = 0; l < 4; l++) code[l][j] = (wd[j] >> (2 * l)) & 0x03030303u;
#pragma unroll
            for (int t = 0; t < NT; t++) {
                if (t >= a.nt) break;
                int e = 0;
                if (ok) {
#pragma unroll
                    for (int l = 0; l < 4; l++) {
                        const int4 av = *(const int4 *)&s.qp[(size_t)t * K + (size_t)l * (K / 4) + c * 16];
                        e = dp4a((int)code[l][0], av.x, e);
                        e = dp4a((int)code[l][1], av.y, e);
                        e = dp4a((int)code[l][2], av.z, e);
                        e = dp4a((int)code[l][3], av.w, e);
                    }
                }
                e += __shfl_xor_sync(0xffffffffu, e, 1);
                e += __shfl_xor_sync(0xffffffffu, e, 2);
                if (ok && (lane & 3) == 0) {
                    const int b = c >> 2;
                    const int v = e * (1 << w.shift) - w.off * s.sum[t * nb + b];
                    if (a.ints) a.ints[((size_t)t * a.rows_total + r) * nb + b] = v;
                    acc[t] += sc * s.d[t * nb + b] * (float)v;
                }
            }
        }
#pragma unroll
        for (int t = 0; t < NT; t++) acc[t] = warp_sum(acc[t]);
        row_epilogue<NT>(a, w, lr, r, acc, best);
    }
    argmax_commit(a, best, s.red);
}

// ---------------------------------------------------------------- Q6_K

// Sub-scale `sub` (0..15) of a Q6_K block whose 16 int8 scales are held in
// scv.  Selecting the word and shifting keeps scv in registers; indexing it
// as a byte array with a lane-dependent index would go through local memory.
__device__ __forceinline__ int q6k_subscale(const uint4 &scv, int sub) { return (int)(int8_t)u4_byte(scv, sub); }

// Unit = (block b, half hf, 16-group s): ql[hf*64+s*16..+16], ql[..+32],
// qh[hf*32+s*16..+16] -> 64 codes in 4 quarters of 16; quarter q covers
// natural elements hf*128 + q*32 + s*16 + [0,16) with sub-scale index
// hf*8 + 2q + s (layout of reference src/kernels.c:786-806).
template <int NT>
__global__ void __launch_bounds__(kGemvThreads) gemv_q6k(const __grid_constant__ GemvArgs a) {
    trace_mark(a.trace, 0);
    pdl_trigger();
    extern __shared__ __align__(16) uint8_t smem[];
    const int K = a.k, nb = K / 256, nunit = nb * 4;
    const int lane = threadIdx.x & 31;
    const int gw = blockIdx.x * kGemvWarps + (threadIdx.x >> 5), nw = gridDim.x * kGemvWarps;
    pdl_wait();
    trace_mark(a.trace, 1);
    Q8Smem s = q8_smem(smem, NT, K);
    stage_q8k(a, s, K);
    trace_mark(a.trace, 2);
    unsigned long long best = 0;
    for (int r = gw; r < a.rows_total; r += nw) {
        int wi, lr;
        map_row(a, r, wi, lr);
        const WDesc &w = wsel(a, wi);
        const uint8_t *row = w.w + (size_t)lr * w.stride;
        float acc[NT];
#pragma unroll
        for (int t = 0; t < NT; t++) acc[t] = 0.f;
        for (int u0 = 0; u0 < nunit; u0 += 32) {
            const int u = u0 + lane;
            const bool ok = u < nunit;
            const int b = u >> 2, hf = (u >> 1) & 1, sg = u & 1;
            uint4 qa = make_uint4(0, 0, 0, 0), qb = qa, qh = qa, scv = qa;
            float dw = 0.f;
            if (ok) {
                qa = ldg_stream(row + (size_t)b * 128 + hf * 64 + sg * 16);
                qb = ldg_stream(row + (size_t)b * 128 + hf * 64 + 32 + sg * 16);
                qh = ldg_stream(row + (size_t)nb * 128 + (size_t)b * 64 + hf * 32 + sg * 16);
                scv = __ldg((const uint4 *)(row + (size_t)nb * 192 + (size_t)b * 16));
                dw = h2f(__ldg((const unsigned short *)(row + (size_t)nb * 208) + b));
            }
            const uint32_t A[4] = {qa.x, qa.y, qa.z, qa.w}, B[4] = {qb.x, qb.y, qb.z, qb.w};
            const uint32_t Hh[4] = {qh.x, qh.y, qh.z, qh.w};
            uint32_t code[4][4];
#pragma unroll
            for (int q = 0; q < 4; q++)
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const uint32_t src = (q & 1) ? B[j] : A[j];
                    const uint32_t lo = (src >> (4 * (q >> 1))) & 0x0f0f0f0fu;
                    const uint32_t hi = (Hh[j] >> (2 * q)) & 0x03030303u;
                    code[q][j] = lo | (hi << 4);
                }
#pragma unroll
            for (int t = 0; t < NT; t++) {
                if (t >= a.nt) break;
                int acc_i = 0;
                if (ok) {
#pragma unroll
                    for (int q = 0; q < 4; q++) {
                        // natural element base hf*128 + q*32 + sg*16 -> chunk hf*2 + q/2, plane (2q+sg)&3
                        const int ch = hf * 2 + (q >> 1), l = (2 * q + sg) & 3;
                        const int4 av = *(const int4 *)&s.qp[(size_t)t * K + (size_t)l * (K / 4) +
                                                            (b * 4 + piece_of_chunk(ch)) * 16];
                        int tq = dp4a((int)code[q][0], av.x, 0);
                        tq = dp4a((int)code[q][1], av.y, tq);
                        tq = dp4a((int)code[q][2], av.z, tq);
                        tq = dp4a((int)code[q][3], av.w, tq);
                        const int sub = hf * 8 + 2 * q + sg;
                        tq -= 32 * (int)s.bs[(size_t)t * nb * 16 + b * 16 + sub];
                        acc_i += q6k_subscale(scv, sub) * tq;
                    }
                }
                acc_i += __shfl_xor_sync(0xffffffffu, acc_i, 1);
                acc_i += __shfl_xor_sync(0xffffffffu, acc_i, 2);
                if (ok && (lane & 3) == 0) {
                    if (a.ints) a.ints[((size_t)t * a.rows_total + r) * nb + b] = acc_i;
                    acc[t] += dw * s.d[t * nb + b] * (float)acc_i;
                }
            }
        }
#pragma unroll
        for (int t = 0; t < NT; t++) acc[t] = warp_sum(acc[t]);
        row_epilogue<NT>(a, w, lr, r, acc, best);
    }
    argmax_commit(a, best, s.red);
}

// ---------------------------------------------------------------- Q4_K

// Scale and min of sub-block j from a Q4_K block header held in registers
// (hdr = d, dmin, scales[12]; the scales start at byte 4).
__device__ __forceinline__ void k4_scale_min(const uint4 &hdr, int j, int &sc, int &mn) {
    if (j < 4) {
        sc = (int)(u4_byte(hdr, 4 + j) & 63);
        mn = (int)(u4_byte(hdr, 8 + j) & 63);
    } else {
        sc = (int)((u4_byte(hdr, 8 + j) & 0x0f) | ((u4_byte(hdr, j) >> 6) << 4));
        mn = (int)((u4_byte(hdr, 8 + j) >> 4) | ((u4_byte(hdr, 4 + j) >> 6) << 4));
    }
}

// Unit = (block b, pair g, 16-half s): qs[32g + 16s .. +16]; low nibbles are
// elements 64g+16s+i (sub-block 2g), high nibbles 64g+32+16s+i (sub-block
// 2g+1) — reference src/kernels.c:861-877.
template <int NT>
__global__ void __launch_bounds__(kGemvThreads) gemv_q4k(const __grid_constant__ GemvArgs a) {
    trace_mark(a.trace, 0);
    pdl_trigger();
    extern __shared__ __align__(16) uint8_t smem[];
    const int K = a.k, nb = K / 256, nunit = nb * 8;
    const int lane = threadIdx.x & 31;
    const int gw = blockIdx.x * kGemvWarps + (threadIdx.x >> 5), nw = gridDim.x * kGemvWarps;
    pdl_wait();
    trace_mark(a.trace, 1);
    Q8Smem s = q8_smem(smem, NT, K);
    stage_q8k(a, s, K);
    trace_mark(a.trace, 2);
    unsigned long long best = 0;
    for (int r = gw; r < a.rows_total; r += nw) {
        int wi, lr;
        map_row(a, r, wi, lr);
        const WDesc &w = wsel(a, wi);
        const uint8_t *row = w.w + (size_t)lr * w.stride;
        float acc[NT];
#pragma unroll
        for (int t = 0; t < NT; t++) acc[t] = 0.f;
        for (int u0 = 0; u0 < nunit; u0 += 32) {
            const int u = u0 + lane;
            const bool ok = u < nunit;
            const int b = u >> 3, g = (u >> 1) & 3, sg = u & 1;
            uint4 qv = make_uint4(0, 0, 0, 0), hdr = qv;
            if (ok) {
                qv = ldg_stream(row + (size_t)b * 144 + 16 + g * 32 + sg * 16);
                hdr = __ldg((const uint4 *)(row + (size_t)b * 144));
            }
            int sc0, mn0, sc1, mn1;
            k4_scale_min(hdr, 2 * g, sc0, mn0);
            k4_scale_min(hdr, 2 * g + 1, sc1, mn1);
            const float dd = h2f((unsigned short)(hdr.x & 0xffffu)), dm = h2f((unsigned short)(hdr.x >> 16));
            const uint32_t Q[4] = {qv.x, qv.y, qv.z, qv.w};
#pragma unroll
            for (int t = 0; t < NT; t++) {
                if (t >= a.nt) break;
                int si = 0, sm = 0;
                if (ok) {
                    const int4 alo = *(const int4 *)&s.qp[(size_t)t * K + (size_t)sg * (K / 4) + (b * 4 + piece_of_chunk(g)) * 16];
                    const int4 ahi = *(const int4 *)&s.qp[(size_t)t * K + (size_t)(2 + sg) * (K / 4) + (b * 4 + piece_of_chunk(g)) * 16];
                    int s0 = dp4a((int)(Q[0] & 0x0f0f0f0fu), alo.x, 0);
                    s0 = dp4a((int)(Q[1] & 0x0f0f0f0fu), alo.y, s0);
                    s0 = dp4a((int)(Q[2] & 0x0f0f0f0fu), alo.z, s0);
                    s0 = dp4a((int)(Q[3] & 0x0f0f0f0fu), alo.w, s0);
                    int s1 = dp4a((int)((Q[0] >> 4) & 0x0f0f0f0fu), ahi.x, 0);
                    s1 = dp4a((int)((Q[1] >> 4) & 0x0f0f0f0fu), ahi.y, s1);
                    s1 = dp4a((int)((Q[2] >> 4) & 0x0f0f0f0fu), ahi.z, s1);
                    s1 = dp4a((int)((Q[3] >> 4) & 0x0f0f0f0fu), ahi.w, s1);
                    si = sc0 * s0 + sc1 * s1;
                    if (sg == 0) {
                        const int16_t *bs = s.bs + (size_t)t * nb * 16 + b * 16;
                        sm = mn0 * ((int)bs[4 * g] + (int)bs[4 * g + 1]) + mn1 * ((int)bs[4 * g + 2] + (int)bs[4 * g + 3]);
                    }
                }
#pragma unroll
                for (int o = 1; o < 8; o <<= 1) {
                    si += __shfl_xor_sync(0xffffffffu, si, o);
                    sm += __shfl_xor_sync(0xffffffffu, sm, o);
                }
                if (ok && (lane & 7) == 0) {
                    if (a.ints) {
                        a.ints[(((size_t)t * a.rows_total + r) * nb + b) * 2] = si;
                        a.ints[(((size_t)t * a.rows_total + r) * nb + b) * 2 + 1] = sm;
                    }
                    acc[t] += s.d[t * nb + b] * (dd * (float)si - dm * (float)sm);
                }
            }
        }
#pragma unroll
        for (int t = 0; t < NT; t++) acc[t] = warp_sum(acc[t]);
        row_epilogue<NT>(a, w, lr, r, acc, best);
    }
    argmax_commit(a, best, s.red);
}

// ---------------------------------------------------------------- fp32-activation formats

// Q8_0 / F16 / F32 use the fp32 activation itself (reference
// src/kernels.c:1272-1300), staged in shared memory as [t][quad][unit][4] so
// each lane's 16-byte reads are bank-conflict free.
template <int FMT>
struct FpFmt;
template <>
struct FpFmt<FMT_Q80> { static constexpr int kElems = 16; };  // 16 int8 per 16-byte unit
template <>
struct FpFmt<FMT_F16> { static constexpr int kElems = 8; };
template <>
struct FpFmt<FMT_F32> { static constexpr int kElems = 4; };

// [NT][K] permuted activations, then a [K] staging row and 64 floats of reduction space.
__host__ __device__ inline size_t fp_smem_bytes(int NT, int K) { return align16((size_t)NT * K * 4) + (size_t)K * 4 + 64 * 4; }

// One 16-byte weight unit u of a row at one token, folded into this lane's
// accumulator: gemv_fp's per-unit arithmetic for token 0 (Q8_0: the two
// 16-element halves of a 32-block are summed across the lane pair, then
// scaled once).
template <int FMT>
__device__ __forceinline__ void fp_unit1(const uint4 &v, unsigned short s16, bool ok, const float *sx, int nunit, int u,
                                         float &acc) {
    constexpr int E = FpFmt<FMT>::kElems, QPU = E / 4;
    const int lane = threadIdx.x & 31;
    float wf[E];
    float scale = 1.f;
    if (ok) {
        if (FMT == FMT_Q80) {
            const int8_t *q = (const int8_t *)&v;
#pragma unroll
            for (int j = 0; j < E; j++) wf[j] = (float)q[j];
            scale = h2f(s16);
        } else if (FMT == FMT_F16) {
            const __half *h = (const __half *)&v;
#pragma unroll
            for (int j = 0; j < E; j++) wf[j] = __half2float(h[j]);
        } else {
            const float *f = (const float *)&v;
#pragma unroll
            for (int j = 0; j < E; j++) wf[j] = f[j];
        }
    }
    float p = 0.f;
    if (ok) {
#pragma unroll
        for (int q = 0; q < QPU; q++) {
            const float4 xv = *(const float4 *)&sx[((size_t)q * nunit + u) * 4];
            p = fmaf(wf[4 * q + 0], xv.x, p);
            p = fmaf(wf[4 * q + 1], xv.y, p);
            p = fmaf(wf[4 * q + 2], xv.z, p);
            p = fmaf(wf[4 * q + 3], xv.w, p);
        }
    }
    if (FMT == FMT_Q80) {
        p += __shfl_xor_sync(0xffffffffu, p, 1);
        if ((lane & 1) == 0) acc += scale * p;
    } else {
        acc += p;
    }
}

template <int FMT, int NT>
__global__ void __launch_bounds__(kGemvThreads) gemv_fp(const __grid_constant__ GemvArgs a) {
    trace_mark(a.trace, 0);
    pdl_trigger();
    extern __shared__ __align__(16) uint8_t smem[];
    constexpr int E = FpFmt<FMT>::kElems, QPU = E / 4;
    const int K = a.k, nunit = K / E;
    const int lane = threadIdx.x & 31;
    const int gw = blockIdx.x * kGemvWarps + (threadIdx.x >> 5), nw = gridDim.x * kGemvWarps;
    float *sx = (float *)smem;                                   // [NT][QPU][nunit][4]
    float *stg = (float *)(smem + align16((size_t)NT * K * 4));  // [K] staging
    float *red = stg + K;
    pdl_wait();
    trace_mark(a.trace, 1);
    for (int t = 0; t < a.nt; t++) {
        stage_fp32(a, t, stg, red, K);
        __syncthreads();
        for (int e = threadIdx.x; e < K; e += blockDim.x) {
            const int u = e / E, q = (e % E) >> 2, j = e & 3;
            sx[(((size_t)t * QPU + q) * nunit + u) * 4 + j] = stg[e];
        }
        __syncthreads();
    }
    trace_mark(a.trace, 2);
    unsigned long long best = 0;
    if constexpr (NT == 1) {
        // one token: each warp streams two rows at once (rows r and r + nw), kFpInFlight / 2
        // units of each per lane loaded before the arithmetic, so a K = 2048 row (4 units per
        // lane) still keeps 8 loads in flight; per row the arithmetic is the loop's below
        constexpr int PF2 = kFpInFlight / 2;
        for (int r = gw; r < a.rows_total; r += 2 * nw) {
            const int rb = r + nw;
            const bool two = rb < a.rows_total;  // uniform across the warp
            int wa, la, wb = 0, lb = 0;
            map_row(a, r, wa, la);
            if (two) map_row(a, rb, wb, lb);
            const WDesc &WA = wsel(a, wa);
            const WDesc &WB = wsel(a, two ? wb : wa);
            const uint8_t *rowa = WA.w + (size_t)la * WA.stride;
            const uint8_t *rowb = two ? WB.w + (size_t)lb * WB.stride : rowa;
            float acca = 0.f, accb = 0.f;
            for (int c0 = 0; c0 < nunit; c0 += 32 * PF2) {
                uint4 va[PF2], vb[PF2];
                unsigned short sa[PF2], sb[PF2];
#pragma unroll
                for (int i = 0; i < PF2; i++) {
                    const int u = c0 + 32 * i + lane;
                    sa[i] = sb[i] = 0;
                    if (u < nunit) {
                        va[i] = ldg_stream(rowa + (size_t)u * 16);
                        if (two) vb[i] = ldg_stream(rowb + (size_t)u * 16);
                        if (FMT == FMT_Q80) {
                            sa[i] = __ldg((const unsigned short *)(rowa + K) + (u >> 1));
                            if (two) sb[i] = __ldg((const unsigned short *)(rowb + K) + (u >> 1));
                        }
                    }
                }
#pragma unroll
                for (int i = 0; i < PF2; i++) {
                    const int u0 = c0 + 32 * i;
                    if (u0 >= nunit) break;  // uniform across the warp
                    const int u = u0 + lane;
                    const bool ok = u < nunit;
                    fp_unit1<FMT>(va[i], sa[i], ok, sx, nunit, u, acca);
                    if (two) fp_unit1<FMT>(vb[i], sb[i], ok, sx, nunit, u, accb);
                }
            }
            float res[1] = {warp_sum(acca)};
            row_epilogue<1>(a, WA, la, r, res, best);
            if (two) {
                res[0] = warp_sum(accb);
                row_epilogue<1>(a, WB, lb, rb, res, best);
            }
        }
        argmax_commit(a, best, red);
        return;
    }
    for (int r = gw; r < a.rows_total; r += nw) {
        int wi, lr;
        map_row(a, r, wi, lr);
        const WDesc &w = wsel(a, wi);
        const uint8_t *row = w.w + (size_t)lr * w.stride;
        float acc[NT];

#pragma unroll
        for (int t = 0; t < NT; t++) acc[t] = 0.f;
        // kFpInFlight 16-byte units of the row per lane are loaded before any
        // arithmetic (enough bytes in flight to cover HBM latency); the
        // arithmetic and its order are per unit as before
        constexpr int PF = kFpInFlight;
        for (int c0 = 0; c0 < nunit; c0 += 32 * PF) {
        uint4 vv[PF];
        unsigned short sv[PF];
#pragma unroll
        for (int i = 0; i < PF; i++) {
            const int u = c0 + 32 * i + lane;
            if (u < nunit) {
                vv[i] = ldg_stream(row + (size_t)u * 16);
                if (FMT == FMT_Q80) sv[i] = __ldg((const unsigned short *)(row + K) + (u >> 1));
            }
        }
#pragma unroll
        for (int i = 0; i < PF; i++) {
            const int u0 = c0 + 32 * i;
            if (u0 >= nunit) break;  // uniform across the warp
            const int u = u0 + lane;
            const bool ok = u < nunit;
            float wf[E];
            float scale = 1.f;
            if (ok) {
                const uint4 v = vv[i];
                if (FMT == FMT_Q80) {
                    const int8_t *q = (const int8_t *)&v;
#pragma unroll
                    for (int j = 0; j < E; j++) wf[j] = (float)q[j];
                    scale = h2f(sv[i]);
                } else if (FMT == FMT_F16) {
                    const __half *h = (const __half *)&v;
#pragma unroll
                    for (int j = 0; j < E; j++) wf[j] = __half2float(h[j]);
                } else {
                    const float *f = (const float *)&v;
#pragma unroll
                    for (int j = 0; j < E; j++) wf[j] = f[j];
                }
            } else {
#pragma unroll
                for (int j = 0; j < E; j++) wf[j] = 0.f;
            }
#pragma unroll
            for (int t = 0; t < NT; t++) {
                if (t >= a.nt) break;
                float p = 0.f;
                if (ok) {
#pragma unroll
                    for (int q = 0; q < QPU; q++) {
                        const float4 xv = *(const float4 *)&sx[(((size_t)t * QPU + q) * nunit + u) * 4];
                        p = fmaf(wf[4 * q + 0], xv.x, p);
                        p = fmaf(wf[4 * q + 1], xv.y, p);
                        p = fmaf(wf[4 * q + 2], xv.z, p);
                        p = fmaf(wf[4 * q + 3], xv.w, p);
                    }
                }
                if (FMT == FMT_Q80) {
                    // two 16-wide halves form one 32-block: sum, then scale
                    p += __shfl_xor_sync(0xffffffffu, p, 1);
                    if ((lane & 1) == 0) acc[t] += scale * p;
                } else {
                    acc[t] += p;
                }
            }
        }
        }
#pragma unroll
        for (int t = 0; t < NT; t++) acc[t] = warp_sum(acc[t]);
        row_epilogue<NT>(a, w, lr, r, acc, best);
    }
    argmax_commit(a, best, red);
}

}  // namespace hyk
