// hy_mega.cuh — persistent single-launch greedy decode for panel (STQ1_0 /
// Q2_0C) models with a Q6_K LM head, on sm_100a.
//
// One cooperative launch, one 512-thread CTA per SM, runs `steps` decode
// steps (reference src/model.c:914-958 gen_ids loop over forward_tokens,
// :836-880 per layer).  Per layer the phases are separated by grid barriers:
//   q|k|v GEMV (RMSNorm + Q8_K prologue) | attention (rope, q/k norm, bf16
//   KV store, split-KV softmax) | o_proj GEMV (+residual) | gate|up GEMV
//   (interleaved rows, SiLU*up epilogue) | down GEMV (+residual)
// then the LM head with a fused argmax, the token bookkeeping of
// decode_finalize and the next token's embedding.
//
// Each CTA owns fixed row slices of every GEMV, so while layer l runs it
// streams its layer-(l+1) slices into four shared-memory slots with bulk
// async copies (cp.async.bulk, no multicast) completing on mbarriers; the
// attention CTAs stage the next layer's cached K/V rows with cp.async as soon
// as the current layer's attention is done.  Every arithmetic step (norm reduction order, quantiser, per-row dot
// products, attention body, head rows) is the one the per-layer kernels use,
// so this path is bit-identical to the graph of per-layer launches.
//
// All waits are bounded by %globaltimer: on a timeout the kernel raises the
// error word, every CTA leaves at its next barrier, and each CTA waits
// (bounded) for its own copies in flight before returning.
#pragma once
#include "hy_attn.cuh"
#include "hy_gemv.cuh"
#include "hy_misc.cuh"

namespace hyk {

constexpr int kMegaThreads = 512;
constexpr int kMegaWarps = kMegaThreads / 32;
constexpr int kMegaRowAlign = 8;                           // row slices in multiples of 8
constexpr unsigned long long kMegaWaitNs = 2000000000ull;  // 2 s bound on any wait
constexpr int kMegaKPad = kChunkKPad;                      // K rows padded in smem (bank spread)

enum MegaErr { MEGA_OK = 0, MEGA_ERR_BARRIER = 1, MEGA_ERR_POS = 2, MEGA_ERR_WEIGHTS = 3, MEGA_ERR_KV = 4 };

// Device-resident per-layer table.
struct MegaLayer {
    const uint8_t *w[7];  // panel codes: q k v o gate up down
    const float *s[7];    // panel scales
    const float *attn_norm, *ffn_norm, *q_norm, *k_norm;
    uint16_t *kc, *vc;
};

// Cross-CTA words; the host zeroes the whole struct before each launch.
struct MegaSync {
    unsigned long long amax[2];  // argmax key per step parity
    unsigned bar;                // grid barrier arrivals (monotonic within a launch)
    int err;                     // MegaErr of the first failure
    int tickets[64];             // attention split merge tickets per KV head
};

struct MegaArgs {
    const MegaLayer *layers;
    int L, H, F, kvh, qd, kvd, ctx;
    int shift, off;           // panel code transform shared by all layer weights
    float eps;
    int rpc[5];               // rows per CTA: q|k|v, o, gate|up (merged), down, head
    int slot_off[4];          // dynamic-smem offsets of the weight slots
    int stage_off, attn_off;  // dynamic-smem offsets of the Q8_K stage and the K/V area
    int kmax;                 // largest GEMV input length (stage plan)
    int head_ns;              // LM-head ring stages (kHeadRows rows each) and their smem offsets
    int head_off[4];
    int head_keep;            // rows of each CTA's head slice read with L2 evict-last (stay resident)
    AttnArgs attn;            // shape, rope tables, part buffer; per-layer fields set in-kernel
    WDesc head, embd;
    int vocab_out;
    const float *out_norm;
    float *h, *qkv, *ao, *act;
    unsigned long long *th, *tqkv, *tact, *tpart;  // tagged activations: h, q|k|v, silu*up, attention partials
    unsigned *done;  // per-CTA done words [4][grid]: o_proj rows, down rows, gate|up rows, attention unit
    unsigned tag0;   // first tag of this launch
    DecodeState *st;
    int *out_ids;
    MegaSync *sync;
    unsigned long long *tl;   // optional timeline (block 0): globaltimer per phase edge
    int tl_cap;
    int steps;
};

// ---------------------------------------------------------------- primitives

__device__ __forceinline__ unsigned smem_u32(const void *p) { return (unsigned)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void mbar_init(uint64_t *bar) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_expect(uint64_t *bar, unsigned tx) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(tx) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint64_t *bar, unsigned parity) {
    unsigned ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait for the completion of phase `parity`; false on timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, unsigned parity) {
    if (mbar_try(bar, parity)) return true;
    const unsigned long long t0 = gtimer();
    while (!mbar_try(bar, parity))
        if (gtimer() - t0 > kMegaWaitNs) return false;
    return true;
}
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, unsigned bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}
// The same copy with an L2 eviction policy (createpolicy): layer weights are
// read once per token (evict first); the part of the LM head kept resident
// across tokens is read with evict last.
__device__ __forceinline__ void bulk_g2s_hint(void *dst, const void *src, unsigned bytes, uint64_t *bar,
                                              uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ uint64_t l2_policy_evict_last() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ int ld_relaxed_s32(const int *p) {
    int v;
    asm volatile("ld.relaxed.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void raise_err(const MegaArgs &a, int code) { atomicCAS(&a.sync->err, 0, code); }

// Grid-wide barrier in two halves.  bar_arrive: once every thread's writes
// of the phase are done (__syncthreads), thread 0 publishes them
// (__threadfence) and adds 1 to the arrival counter.  Work that does not
// depend on other CTAs can run between the halves.  bar_wait: thread 0 polls
// until the counter reaches the running target; bounded, and a timeout or
// another CTA's error makes every CTA return false from here on.
__device__ __forceinline__ void bar_arrive(const MegaArgs &a, unsigned &target) {
    __syncthreads();
    target += gridDim.x;
    if (threadIdx.x == 0) {
        __threadfence();
        atomicAdd(&a.sync->bar, 1u);
    }
}
__device__ __forceinline__ bool bar_wait(const MegaArgs &a, unsigned target, int *s_flag) {
    if (threadIdx.x == 0) {
        int bad = 0;
        if ((int)(ld_acquire_u32(&a.sync->bar) - target) < 0) {
            const unsigned long long t0 = gtimer();
            unsigned it = 0;
            while ((int)(ld_acquire_u32(&a.sync->bar) - target) < 0) {
                if ((++it & 63) == 0) {
                    if (ld_relaxed_s32(&a.sync->err)) { bad = 1; break; }
                    if (gtimer() - t0 > kMegaWaitNs) { raise_err(a, MEGA_ERR_BARRIER); bad = 1; break; }
                }
            }
        }
        if (!bad && ld_relaxed_s32(&a.sync->err)) bad = 1;
        *s_flag = bad;
    }
    __syncthreads();
    return *s_flag == 0;
}

// Every thread of the CTA waits for slot `bar`; the outcome is made uniform
// across the CTA (a timeout seen by any thread fails the whole CTA), so no
// warp can diverge into a collective the others skip.
__device__ __forceinline__ bool mega_slot_ready(const MegaArgs &a, uint64_t *bar, unsigned parity) {
    const bool ready = __syncthreads_and(mbar_wait(bar, parity)) != 0;
    if (!ready && threadIdx.x == 0) raise_err(a, MEGA_ERR_WEIGHTS);
    return ready;
}

// Timeline (debug, a.tl non-null): [0, cap/2) phase edges of block 0;
// [cap/2, cap/2 + 8192) sub-phase marks of block 0; then per-CTA marks of
// one chosen (step, layer): 16 slots per CTA.
__device__ __forceinline__ void tl_mark(const MegaArgs &a, int &idx) {
    if (a.tl && blockIdx.x == 0 && threadIdx.x == 0 && idx < a.tl_cap / 2) a.tl[idx] = gtimer();
    idx++;
}
__device__ __forceinline__ void tl_sub(const MegaArgs &a, int &idx) {
    if (a.tl && blockIdx.x == 0 && threadIdx.x == 0 && idx < 8192) a.tl[a.tl_cap / 2 + idx] = gtimer();
    idx++;
}
__device__ __forceinline__ void tl_cta(const MegaArgs &a, bool on, int slot) {
    if (a.tl && on && threadIdx.x == 0) a.tl[a.tl_cap / 2 + 8192 + blockIdx.x * 16 + slot] = gtimer();
}

// ---------------------------------------------------------------- weight slots

__host__ __device__ inline int mega_slot_bytes(int rpc, int K) {
    return (int)align16((size_t)rpc * (K / 256) * 64) + (int)align16((size_t)rpc * (K / 256) * 4);
}
__host__ __device__ inline int mega_phase_k(int t, int H, int F, int qd) { return t == 1 ? qd : (t == 3 ? F : H); }
__host__ __device__ inline int mega_phase_rows(int t, int H, int F, int qd, int kvd) {
    return t == 0 ? qd + 2 * kvd : (t == 2 ? 2 * F : H);
}

// Thread 0: arm slot t's mbarrier and issue the bulk copies of this CTA's
// rows of GEMV t of layer l (codes, then scales after an aligned gap).
__device__ inline void mega_fill(const MegaArgs &a, const MegaLayer *tab, uint8_t *smem, uint64_t *bar, int t,
                                 int l) {
    const uint64_t pol = l2_policy_evict_first();
    const MegaLayer &ly = tab[l];
    const int K = mega_phase_k(t, a.H, a.F, a.qd);
    const int nb = K / 256, rb = nb * 64, rpc = a.rpc[t];
    uint8_t *sw = smem + a.slot_off[t];
    float *ss = (float *)(sw + align16((size_t)rpc * rb));
    const int total = mega_phase_rows(t, a.H, a.F, a.qd, a.kvd);
    const int r0 = blockIdx.x * rpc, r1 = min(r0 + rpc, total);
    if (r0 >= r1) {
        mbar_expect(bar, 0);
        return;
    }
    if (t == 2) {  // interleaved gate|up: gate rows at slot rows [0,n), up rows at [rpc/2, rpc/2+n)
        const int g0 = r0 >> 1, n = ((r1 + 1) >> 1) - g0;
        mbar_expect(bar, 2u * n * (rb + nb * 4));
        bulk_g2s_hint(sw, ly.w[4] + (size_t)g0 * rb, n * rb, bar, pol);
        bulk_g2s_hint(sw + (size_t)(rpc >> 1) * rb, ly.w[5] + (size_t)g0 * rb, n * rb, bar, pol);
        bulk_g2s_hint(ss, ly.s[4] + (size_t)g0 * nb, n * nb * 4, bar, pol);
        bulk_g2s_hint(ss + (size_t)(rpc >> 1) * nb, ly.s[5] + (size_t)g0 * nb, n * nb * 4, bar, pol);
        return;
    }
    mbar_expect(bar, (unsigned)(r1 - r0) * (rb + nb * 4));
    if (t == 0) {  // merged q|k|v rows
        const int lim[3] = {a.qd, a.qd + a.kvd, a.qd + 2 * a.kvd};
        int base = 0;
        for (int wi = 0; wi < 3; wi++) {
            const int s0 = max(r0, base), s1 = min(r1, lim[wi]);
            if (s0 < s1) {
                bulk_g2s_hint(sw + (size_t)(s0 - r0) * rb, ly.w[wi] + (size_t)(s0 - base) * rb, (s1 - s0) * rb, bar, pol);
                bulk_g2s_hint(ss + (size_t)(s0 - r0) * nb, ly.s[wi] + (size_t)(s0 - base) * nb, (s1 - s0) * nb * 4, bar, pol);
            }
            base = lim[wi];
        }
        return;
    }
    const int wi = t == 1 ? 3 : 6;
    bulk_g2s_hint(sw, ly.w[wi] + (size_t)r0 * rb, (r1 - r0) * rb, bar, pol);
    bulk_g2s_hint(ss, ly.s[wi] + (size_t)r0 * nb, (r1 - r0) * nb * 4, bar, pol);
}

// ---------------------------------------------------------------- activation staging

// RMSNorm weights of the next normalised phase, loaded before the barrier
// wait (they are constants): threads 0..255 hold elements t + 256 j.
template <int SV>
struct NormPre {
    float4 w[SV];
};
template <int SV>
__device__ __forceinline__ void norm_preload(const float *norm_w, int K, NormPre<SV> &p) {
    const int tid = threadIdx.x;
#pragma unroll
    for (int j = 0; j < SV; j++) {
        const int i = tid + j * kGemvThreads;
        if (tid < kGemvThreads && i < (K >> 2)) p.w[j] = __ldg((const float4 *)norm_w + i);
    }
}

// fp32 input (x, or the stage's own s.x when x == nullptr), optionally
// RMSNorm * (preloaded) weights, then Q8_K into shared memory.  With a norm,
// threads 0..255 hold elements i = t + 256 j exactly as the 256-thread
// per-layer kernels do, so the sum of squares (and everything after it) is
// bit-identical; the extra warps contribute zeros to the block reduction.
template <int SV>
__device__ inline void mega_stage(const float *x, const NormPre<SV> *pre, float eps, int K, Q8Smem &s) {
    const int n4 = K >> 2, tid = threadIdx.x;
    const float4 *src = x ? (const float4 *)x : (const float4 *)s.x;
    if (pre) {
        float4 xv[SV];
#pragma unroll
        for (int j = 0; j < SV; j++) {
            const int i = tid + j * kGemvThreads;
            if (tid < kGemvThreads && i < n4) xv[j] = src[i];
        }
        float ss = 0.f;
#pragma unroll
        for (int j = 0; j < SV; j++) {
            const int i = tid + j * kGemvThreads;
            if (tid < kGemvThreads && i < n4) {
                ss = __fadd_rn(ss, __fmul_rn(xv[j].x, xv[j].x));
                ss = __fadd_rn(ss, __fmul_rn(xv[j].y, xv[j].y));
                ss = __fadd_rn(ss, __fmul_rn(xv[j].z, xv[j].z));
                ss = __fadd_rn(ss, __fmul_rn(xv[j].w, xv[j].w));
            }
        }
        ss = block_sum(ss, s.red);  // also orders every read of s.x before the writes below
        const float scale = 1.0f / sqrtf(ss / (float)K + eps);
#pragma unroll
        for (int j = 0; j < SV; j++) {
            const int i = tid + j * kGemvThreads;
            if (tid < kGemvThreads && i < n4) {
                const float4 wv = pre->w[j];
                ((float4 *)s.x)[i] = make_float4(__fmul_rn(__fmul_rn(xv[j].x, scale), wv.x),
                                                 __fmul_rn(__fmul_rn(xv[j].y, scale), wv.y),
                                                 __fmul_rn(__fmul_rn(xv[j].z, scale), wv.z),
                                                 __fmul_rn(__fmul_rn(xv[j].w, scale), wv.w));
            }
        }
    } else if (x) {
        for (int i = tid; i < n4; i += kMegaThreads) ((float4 *)s.x)[i] = src[i];
    }
    __syncthreads();
    const int nb = K / 256;
    for (int b = tid >> 5; b < nb; b += kMegaWarps) quantize_block_warp(s.x, s, 0, b, nb, K);
    __syncthreads();
}

// o_proj staging: the attention output of every head, merged from the wide
// attention's chunk partials (attn_merge_head, one warp per head), then Q8_K.
template <int HD>
__device__ inline void mega_stage_attn(const MegaArgs &a, int pos, Q8Smem &s) {
    const int cs = attn_chunk_len(pos, a.kvh, gridDim.x), nch = (pos + cs) / cs, heads = a.qd / HD;
    for (int h = threadIdx.x >> 5; h < heads; h += kMegaWarps)
        attn_merge_head<HD>(a.attn.cpart, a.attn.max_chunks, nch, h, s.x + (size_t)h * HD);
    __syncthreads();
    const int nb = a.qd / 256;
    for (int b = threadIdx.x >> 5; b < nb; b += kMegaWarps) quantize_block_warp(s.x, s, 0, b, nb, a.qd);
    __syncthreads();
}

template <int CPL>
__device__ __forceinline__ void mega_act(const Q8Smem &s, int K, int4 (&act)[CPL][4], float (&dblk)[CPL],
                                         int (&sblk)[CPL]) {
    const int lane = threadIdx.x & 31, nchunk = K / 64;
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
}

// ---------------------------------------------------------------- panel rows from a slot

// Rows [r0, r1) of the phase's merged row space, weights from the slot (row
// rr = r - r0 at slot row srow(rr)), RG rows per warp iteration.  Same
// per-row arithmetic as gemv_panel_dec.  epi(r, acc[], r1) runs on lane 0.
template <int CPL, int RG, bool INTERLEAVED, typename Epi>
__device__ __forceinline__ void mega_rows(int shift, int off, int r0, int r1, int rpc, const uint8_t *sw,
                                         const float *ss, int K, const int4 (&act)[CPL][4], const float (&dblk)[CPL],
                                         const int (&sblk)[CPL], Epi epi) {
    const int nb = K / 256, nchunk = nb * 4, rb = nb * 64;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int rg = r0 + warp * RG; rg < r1; rg += kMegaWarps * RG) {
        float acc[RG];
        int srow[RG];
#pragma unroll
        for (int g = 0; g < RG; g++) {
            acc[g] = 0.f;
            const int rr = rg + g - r0;
            srow[g] = INTERLEAVED ? ((rr & 1) * (rpc >> 1) + (rr >> 1)) : rr;
        }
#pragma unroll
        for (int i = 0; i < CPL; i++) {
            const int c = lane + 32 * i;
            int e[RG];
#pragma unroll
            for (int g = 0; g < RG; g++) {
                e[g] = 0;
                if (c < nchunk && rg + g < r1)
                    e[g] = panel_chunk_dot4(*(const uint4 *)(sw + (size_t)srow[g] * rb + c * 16), act[i]);
            }
#pragma unroll
            for (int g = 0; g < RG; g++) e[g] += __shfl_xor_sync(0xffffffffu, e[g], 1);
#pragma unroll
            for (int g = 0; g < RG; g++) e[g] += __shfl_xor_sync(0xffffffffu, e[g], 2);
            if (c < nchunk && (lane & 3) == 0) {
#pragma unroll
                for (int g = 0; g < RG; g++) {
                    if (rg + g >= r1) break;
                    const int v = e[g] * (1 << shift) - off * sblk[i];
                    acc[g] += ss[(size_t)srow[g] * nb + (c >> 2)] * dblk[i] * (float)v;
                }
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
#pragma unroll
            for (int g = 0; g < RG; g++) acc[g] += __shfl_xor_sync(0xffffffffu, acc[g], o);
        if (lane == 0) epi(rg, acc, r1);
    }
}

// ---------------------------------------------------------------- LM head (Q6_K) with argmax

// The head streams through a ring of shared-memory stages of kHeadRows rows
// (one row per warp); each stage is one bulk copy of consecutive rows of the
// relayouted Q6_K head (ql | qh | scales | d planes per row).
constexpr int kHeadRows = kMegaWarps;

// One Q6_K row held in shared memory against the stage's Q8_K activation;
// the arithmetic (unit split, integer sums, float order, warp sum) is
// gemv_q6k's, so the logit is identical.  Returns the sum on every lane.
__device__ __forceinline__ float q6k_row_smem(const uint8_t *row, int nb, int K, const Q8Smem &s) {
    const int lane = threadIdx.x & 31, nunit = nb * 4;
    float acc = 0.f;
    for (int u0 = 0; u0 < nunit; u0 += 32) {
        const int u = u0 + lane;
        const bool ok = u < nunit;
        const int b = u >> 2, hf = (u >> 1) & 1, sg = u & 1;
        uint4 qa = make_uint4(0, 0, 0, 0), qb = qa, qh = qa, scv = qa;
        float dw = 0.f;
        if (ok) {
            qa = *(const uint4 *)(row + (size_t)b * 128 + hf * 64 + sg * 16);
            qb = *(const uint4 *)(row + (size_t)b * 128 + hf * 64 + 32 + sg * 16);
            qh = *(const uint4 *)(row + (size_t)nb * 128 + (size_t)b * 64 + hf * 32 + sg * 16);
            scv = *(const uint4 *)(row + (size_t)nb * 192 + (size_t)b * 16);
            dw = h2f(*(const unsigned short *)(row + (size_t)nb * 208 + 2 * b));
        }
        const uint32_t A[4] = {qa.x, qa.y, qa.z, qa.w}, B[4] = {qb.x, qb.y, qb.z, qb.w};
        const uint32_t Hh[4] = {qh.x, qh.y, qh.z, qh.w};
        int acc_i = 0;
        if (ok) {
#pragma unroll
            for (int q = 0; q < 4; q++) {
                const int ch = hf * 2 + (q >> 1), l = (2 * q + sg) & 3;
                const int4 av = *(const int4 *)&s.qp[(size_t)l * (K / 4) + (b * 4 + piece_of_chunk(ch)) * 16];
                uint32_t code[4];
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const uint32_t src = (q & 1) ? B[j] : A[j];
                    code[j] = ((src >> (4 * (q >> 1))) & 0x0f0f0f0fu) | (((Hh[j] >> (2 * q)) & 0x03030303u) << 4);
                }
                int tq = dp4a((int)code[0], av.x, 0);
                tq = dp4a((int)code[1], av.y, tq);
                tq = dp4a((int)code[2], av.z, tq);
                tq = dp4a((int)code[3], av.w, tq);
                const int sub = hf * 8 + 2 * q + sg;
                tq -= 32 * (int)s.bs[b * 16 + sub];
                acc_i += q6k_subscale(scv, sub) * tq;
            }
        }
        acc_i += __shfl_xor_sync(0xffffffffu, acc_i, 1);
        acc_i += __shfl_xor_sync(0xffffffffu, acc_i, 2);
        if (ok && (lane & 3) == 0) acc += dw * s.d[b] * (float)acc_i;
    }
    return warp_sum(acc);
}

// Thread 0: arm ring stage `si % ns` and copy rows [r0 + si*kHeadRows, ...)
// of this CTA's head slice into it.
__device__ __forceinline__ void head_fill(const MegaArgs &a, uint8_t *smem, uint64_t *hbar, int si, int r0, int r1) {
    const int k = si % a.head_ns, row = r0 + si * kHeadRows, n = min(kHeadRows, r1 - row);
    const unsigned bytes = (unsigned)n * (unsigned)a.head.stride;
    mbar_expect(&hbar[k], bytes);
    const uint64_t pol = si * kHeadRows < a.head_keep ? l2_policy_evict_last() : l2_policy_evict_first();
    bulk_g2s_hint(smem + a.head_off[k], a.head.w + (size_t)row * a.head.stride, bytes, &hbar[k], pol);
}

// ---------------------------------------------------------------- the kernel

constexpr int kMegaMaxLayers = 40;

// All threads: cp.async the cached K/V rows [j0, j0 + ncache) of KV head
// kvh of layer `ly` into the K/V area (K rows padded to HD*2 + kMegaKPad
// bytes) as one commit group.  cp.async is a generic-proxy copy, so rows
// that other CTAs stored before a grid barrier need no proxy fence.
template <int HD>
__device__ __forceinline__ void mega_kv_fill(const MegaArgs &a, const MegaLayer &ly, uint8_t *sK, uint16_t *sV,
                                             int kvh, int j0, int ncache) {
    constexpr int KROW = HD * 2 + kMegaKPad, CH = HD / 8;
    const uint16_t *Kg = ly.kc + kvh * HD, *Vg = ly.vc + kvh * HD;
    for (int idx = threadIdx.x; idx < ncache * CH; idx += kMegaThreads) {
        const int j = idx / CH, c = idx - j * CH;
        const size_t g = (size_t)(j0 + j) * a.kvd + c * 8;
        cp_async16(sK + (size_t)j * KROW + c * 16, Kg + g);
        cp_async16(sV + (size_t)j * HD + c * 8, Vg + g);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
}

// ---------------------------------------------------------------- tagged activations
//
// Between the phases of a step every activation value travels as one 64-bit
// word: the float's bits, and in the upper half a tag naming (launch, step,
// layer, phase).  A consumer polls exactly the words it needs until their tags
// match; a 64-bit access is single-copy atomic, so a matching tag implies the
// value beside it.  This replaces a grid barrier plus a load by the load.
// Reuse of a buffer is safe by the data flow itself: every rewrite of a
// buffer depends (through the values it is computed from) on every CTA that
// reads the buffer's previous contents having read them, because a CTA reads
// a phase's input only when it computes rows of that phase.

__device__ __forceinline__ unsigned long long tword(float v, unsigned tag) {
    return (unsigned long long)__float_as_uint(v) | ((unsigned long long)tag << 32);
}
__device__ __forceinline__ void tstore(unsigned long long *p, float v, unsigned tag) {
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(tword(v, tag)) : "memory");
}
__device__ __forceinline__ unsigned long long tload(const unsigned long long *p) {
    unsigned long long r;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(r) : "l"(p) : "memory");
    return r;
}
__device__ __forceinline__ ulonglong2 tload2(const unsigned long long *p) {  // 16-byte aligned
    ulonglong2 r;
    asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];" : "=l"(r.x), "=l"(r.y) : "l"(p) : "memory");
    return r;
}
__device__ __forceinline__ bool tag_is(unsigned long long w, unsigned tag) { return (unsigned)(w >> 32) == tag; }
__device__ __forceinline__ float tval(unsigned long long w) { return __uint_as_float((unsigned)w); }

// Poll n groups of four consecutive words (32-byte aligned) until every tag
// matches; all groups' loads are in flight together.  Bounded; false on
// timeout.
template <int NG>
__device__ __forceinline__ bool tpoll4(const unsigned long long *const (&p)[NG], const bool (&use)[NG], unsigned tag,
                                       float4 (&out)[NG]) {
    ulonglong2 lo[NG], hi[NG];
    bool done[NG];
    unsigned long long t0 = 0;
    for (int round = 0;; round++) {
#pragma unroll
        for (int g = 0; g < NG; g++)
            if (use[g] && (round == 0 || !done[g])) {
                lo[g] = tload2(p[g]);
                hi[g] = tload2(p[g] + 2);
            }
        bool all = true;
#pragma unroll
        for (int g = 0; g < NG; g++) {
            if (!use[g]) continue;
            done[g] = tag_is(lo[g].x, tag) && tag_is(lo[g].y, tag) && tag_is(hi[g].x, tag) && tag_is(hi[g].y, tag);
            all = all && done[g];
        }
        if (all) break;
        if (round == 0) t0 = gtimer();
        else if (gtimer() - t0 > kMegaWaitNs) return false;
    }
#pragma unroll
    for (int g = 0; g < NG; g++)
        if (use[g]) out[g] = make_float4(tval(lo[g].x), tval(lo[g].y), tval(hi[g].x), tval(hi[g].y));
    return true;
}
// One word; bounded; false on timeout.
__device__ __forceinline__ bool tpoll1(const unsigned long long *p, unsigned tag, float &v) {
    unsigned long long w = tload(p);
    if (!tag_is(w, tag)) {
        const unsigned long long t0 = gtimer();
        do {
            if (gtimer() - t0 > kMegaWaitNs) return false;
            w = tload(p);
        } while (!tag_is(w, tag));
    }
    v = tval(w);
    return true;
}

// Done words: after its rows of a phase a producer CTA stores the phase's
// tag into done[cta] (no fence).  A consumer first lets one warp poll the
// nprod producers' done words (a few hundred bytes instead of the whole
// vector, so 148 pollers do not flood the L2 lines of the data), then loads
// the tagged data, whose own tags still decide.  Bounded; false on timeout.
__device__ __forceinline__ void done_mark(unsigned *done, unsigned tag) {
    __syncthreads();
    if (threadIdx.x == 0) asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(done + blockIdx.x), "r"(tag) : "memory");
}
__device__ __forceinline__ bool done_wait(const unsigned *done, int nprod, unsigned tag) {
    bool good = true;
    if (threadIdx.x < 32) {
        const unsigned long long t0 = gtimer();
        for (int p = threadIdx.x; p < nprod; p += 32) {
            unsigned v;
            for (;;) {
                asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(done + p) : "memory");
                if (v == tag) break;
                if (gtimer() - t0 > kMegaWaitNs) {
                    good = false;
                    break;
                }
            }
            if (!good) break;
        }
    }
    return __syncthreads_and(good) != 0;
}

// Staging from tagged words: optional RMSNorm (threads 0..255 hold elements
// t + 256 j, as mega_stage), then Q8_K.  Returns false (uniformly) if a poll
// timed out.
template <int SV>
__device__ inline bool mega_stage_t(const unsigned long long *x, unsigned tag, const NormPre<SV> *pre, float eps, int K,
                                    Q8Smem &s) {
    const int n4 = K >> 2, tid = threadIdx.x;
    bool good = true;
    if (pre) {
        const unsigned long long *p[SV];
        bool use[SV];
        float4 xv[SV];
#pragma unroll
        for (int j = 0; j < SV; j++) {
            const int i = tid + j * kGemvThreads;
            use[j] = tid < kGemvThreads && i < n4;
            p[j] = x + 4 * (size_t)(use[j] ? i : 0);
        }
        good = tpoll4<SV>(p, use, tag, xv);
        float ss = 0.f;
#pragma unroll
        for (int j = 0; j < SV; j++) {
            if (use[j]) {
                ss = __fadd_rn(ss, __fmul_rn(xv[j].x, xv[j].x));
                ss = __fadd_rn(ss, __fmul_rn(xv[j].y, xv[j].y));
                ss = __fadd_rn(ss, __fmul_rn(xv[j].z, xv[j].z));
                ss = __fadd_rn(ss, __fmul_rn(xv[j].w, xv[j].w));
            }
        }
        if (!__syncthreads_and(good)) return false;
        ss = block_sum(ss, s.red);
        const float scale = 1.0f / sqrtf(ss / (float)K + eps);
#pragma unroll
        for (int j = 0; j < SV; j++) {
            const int i = tid + j * kGemvThreads;
            if (use[j]) {
                const float4 wv = pre->w[j];
                ((float4 *)s.x)[i] = make_float4(__fmul_rn(__fmul_rn(xv[j].x, scale), wv.x),
                                                 __fmul_rn(__fmul_rn(xv[j].y, scale), wv.y),
                                                 __fmul_rn(__fmul_rn(xv[j].z, scale), wv.z),
                                                 __fmul_rn(__fmul_rn(xv[j].w, scale), wv.w));
            }
        }
    } else {
        constexpr int NG = SV;  // groups of four per thread at kMegaThreads threads
        const unsigned long long *p[NG];
        bool use[NG];
        float4 xv[NG];
#pragma unroll
        for (int j = 0; j < NG; j++) {
            const int i = tid + j * kMegaThreads;
            use[j] = i < n4;
            p[j] = x + 4 * (size_t)(use[j] ? i : 0);
        }
        good = tpoll4<NG>(p, use, tag, xv);
#pragma unroll
        for (int j = 0; j < NG; j++)
            if (use[j]) ((float4 *)s.x)[tid + j * kMegaThreads] = xv[j];
        if (!__syncthreads_and(good)) return false;
    }
    __syncthreads();
    const int nb = K / 256;
    for (int b = tid >> 5; b < nb; b += kMegaWarps) quantize_block_warp(s.x, s, 0, b, nb, K);
    __syncthreads();
    return true;
}

// Partials of one head as tagged words (attn_chunk_main with a.tpart set).
template <int HD>
struct TaggedPartLoader {
    const unsigned long long *base;
    unsigned tag;
    bool *bad;
    __device__ __forceinline__ float2 ml(int c) const {
        const unsigned long long *p = base + (size_t)c * (HD + kPartPad);
        ulonglong2 w = tload2(p);
        if (!(tag_is(w.x, tag) && tag_is(w.y, tag))) {
            const unsigned long long t0 = gtimer();
            do {
                if (gtimer() - t0 > kMegaWaitNs) {
                    *bad = true;
                    return make_float2(0.f, 1.f);
                }
                w = tload2(p);
            } while (!(tag_is(w.x, tag) && tag_is(w.y, tag)));
        }
        return make_float2(tval(w.x), tval(w.y));
    }
    template <int DPL>
    __device__ __forceinline__ void o(int c, int lane, float (&v)[DPL]) const {
        const unsigned long long *p = base + (size_t)c * (HD + kPartPad) + kPartPad + lane * DPL;
#pragma unroll
        for (int q = 0; q < DPL; q += 2) {
            ulonglong2 w = tload2(p + q);
            if (!(tag_is(w.x, tag) && tag_is(w.y, tag))) {
                const unsigned long long t0 = gtimer();
                do {
                    if (gtimer() - t0 > kMegaWaitNs) {
                        *bad = true;
                        break;
                    }
                    w = tload2(p + q);
                } while (!(tag_is(w.x, tag) && tag_is(w.y, tag)));
            }
            v[q] = tval(w.x);
            v[q + 1] = tval(w.y);
        }
    }
};

// o_proj staging from tagged partials: every head merged (one warp per head)
// into the stage row, then Q8_K.  False (uniformly) on a poll timeout.
template <int HD>
__device__ inline bool mega_stage_attn_t(const MegaArgs &a, int pos, unsigned tag, Q8Smem &s) {
    const int cs = attn_chunk_len(pos, a.kvh, gridDim.x), nch = (pos + cs) / cs, heads = a.qd / HD;
    bool bad = false;
    for (int h = threadIdx.x >> 5; h < heads; h += kMegaWarps) {
        const TaggedPartLoader<HD> ld{a.tpart + (size_t)h * a.attn.max_chunks * (HD + kPartPad), tag, &bad};
        attn_merge_head_with<HD>(ld, nch, s.x + (size_t)h * HD);
    }
    if (!__syncthreads_and(!bad)) return false;
    const int nb = a.qd / 256;
    for (int b = threadIdx.x >> 5; b < nb; b += kMegaWarps) quantize_block_warp(s.x, s, 0, b, nb, a.qd);
    __syncthreads();
    return true;
}

// Launch shape contract (checked by the host): grid = number of SMs, all
// resident (cooperative launch); L <= kMegaMaxLayers; attention units of a
// position fit the grid (attn_chunk_len); every layer weight a panel with
// (shift, off); H, qd <= 2048 (one 64-element chunk per lane) and F <= 2048 *
// CF; head Q6_K with k == H.
//
// Per layer a CTA runs each phase it has rows in: it polls the phase's input
// words (tagged by the producing phase), stages and quantises them, waits for
// its weight slice in shared memory, computes its rows and stores them as
// tagged words, then refills the slot with the next layer's slice.  CTAs with
// no rows in a phase only keep the slot's mbarrier in step.  The LM head is
// the one grid-wide barrier per step (its argmax needs every CTA's rows).
template <int HD, int G, int CF>
__global__ void __launch_bounds__(kMegaThreads, 1) decode_mega(const __grid_constant__ MegaArgs a) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ __align__(8) uint64_t mbar[4];  // weight slots
    __shared__ __align__(8) uint64_t hbar[4];  // LM-head ring stages
    __shared__ int s_flag;
    __shared__ unsigned long long s_best[kMegaWarps];
    __shared__ __align__(16) float sq[G][HD];
    __shared__ __align__(16) float skc[HD], svc[HD];
    __shared__ __align__(16) float sqkv[(G + 2) * HD];  // this unit's q | k | v words, untagged
    __shared__ __align__(16) ChunkScratch<HD> S;
    __shared__ __align__(16) MegaLayer tab[kMegaMaxLayers];
    constexpr int KROW = HD * 2 + kMegaKPad;
    constexpr int RGQ = 2, RGO = 1, RGU = 6, RGD = 1;  // rows per warp iteration per phase
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    Q8Smem st = q8_smem(smem + a.stage_off, 1, a.kmax);
    uint8_t *sK = smem + a.attn_off;
    uint16_t *sV = (uint16_t *)(smem + a.attn_off + (size_t)kDecSplit * KROW);
    for (int i = tid; i < a.L * (int)(sizeof(MegaLayer) / 8); i += kMegaThreads)
        ((unsigned long long *)tab)[i] = ((const unsigned long long *)a.layers)[i];
    if (tid == 0) {
        for (int i = 0; i < 4; i++) {
            mbar_init(&mbar[i]);
            mbar_init(&hbar[i]);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    unsigned ph[4] = {0, 0, 0, 0};  // parity each mbarrier completes next
    unsigned hph[4] = {0, 0, 0, 0}, hpend = 0;  // head ring: parities, stages in flight
    unsigned pending = 0;              // bit i: a fill of mbarrier i is outstanding (same in every thread)
    unsigned target = 0;
    int tli = 0, tls = 0;
    int tok = a.st->tok, pos = a.st->pos;
    bool ok = true;
    // tags: h entering layer l = T(l,0); q|k|v and attention partials = T(l,1);
    // h after o_proj = T(l,2); silu(gate)*up = T(l,3); h entering the head = T(L,0)
    const auto T = [&](int step, int l, int ph_) {
        return a.tag0 + ((unsigned)(step * (a.L + 1) + l) << 2) + (unsigned)ph_;
    };
    // attention unit of this CTA: (KV head akvh, key chunk achunk) of the wide decode attention
    const int akvh = blockIdx.x % a.kvh, achunk = blockIdx.x / a.kvh;
    const auto cs_of = [&](int p) { return attn_chunk_len(p, a.kvh, gridDim.x); };
    const auto attn_cta = [&](int p) {
        const int cs = cs_of(p);
        return p >= 0 && p < a.ctx && cs > 0 && (int)blockIdx.x < a.kvh * ((p + cs) / cs);
    };
    const auto j0_of = [&](int p) { return achunk * cs_of(p); };
    const auto ncache_of = [&](int p) { return max(0, min(p, j0_of(p) + cs_of(p)) - j0_of(p)); };
    const int hr0 = blockIdx.x * a.rpc[4], hr1 = min(hr0 + a.rpc[4], a.head.n);
    const int hst = hr1 > hr0 ? (hr1 - hr0 + kHeadRows - 1) / kHeadRows : 0;  // head ring stages per step
    // row ranges of this CTA per phase (fixed for the launch)
    const int q0 = blockIdx.x * a.rpc[0], q1 = min(q0 + a.rpc[0], a.qd + 2 * a.kvd);
    const int o0 = blockIdx.x * a.rpc[1], o1 = min(o0 + a.rpc[1], a.H);
    const int u0 = blockIdx.x * a.rpc[2], u1 = min(u0 + a.rpc[2], 2 * a.F);
    const int d0 = blockIdx.x * a.rpc[3], d1 = min(d0 + a.rpc[3], a.H);
    // producer CTAs per phase (the CTAs that own rows) and their done words
    const int n_o = min((int)gridDim.x, (a.H + a.rpc[1] - 1) / a.rpc[1]);
    const int n_u = min((int)gridDim.x, (2 * a.F + a.rpc[2] - 1) / a.rpc[2]);
    const int n_d = min((int)gridDim.x, (a.H + a.rpc[3] - 1) / a.rpc[3]);
    unsigned *done_o = a.done, *done_d = a.done + gridDim.x, *done_u = a.done + 2 * gridDim.x,
             *done_a = a.done + 3 * gridDim.x;
    // prime: layer 0's weight slots and K/V rows, the first norm weights
    if (tid == 0)
        for (int t = 0; t < 4; t++) mega_fill(a, tab, smem, &mbar[t], t, 0);
    pending |= 0xfu;
    if (a.steps > 0 && attn_cta(pos)) mega_kv_fill<HD>(a, tab[0], sK, sV, akvh, j0_of(pos), ncache_of(pos));
    NormPre<2> npre;
    norm_preload<2>(tab[0].attn_norm, a.H, npre);
    // consume slot t's fill; uniform false (and error raised) on timeout
    const auto slot_take = [&](int t) {
        if (mega_slot_ready(a, &mbar[t], ph[t])) {
            ph[t] ^= 1;
            pending &= ~(1u << t);
            return true;
        }
        return false;
    };
    const auto slot_refill = [&](int t, int nl) {
        if (tid == 0) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            mega_fill(a, tab, smem, &mbar[t], t, nl);
        }
        pending |= 1u << t;
    };
    for (int step = 0; step < a.steps && ok; step++) {
        if (pos < 0 || pos >= a.ctx) {
            if (tid == 0) raise_err(a, MEGA_ERR_POS);
            ok = false;
            break;
        }
        const bool is_attn = attn_cta(pos);
        tl_mark(a, tli);
        // embedding of `tok` into the stage row; CTA b also publishes its slice of h
        {
            const int t0 = (tok < 0 || tok >= a.embd.n) ? 0 : tok;
            for (int e = tid; e < a.H; e += kMegaThreads) st.x[e] = dequant_elem(a.embd, t0, e);
            const int per = (a.H + gridDim.x - 1) / gridDim.x;
            const int e0 = blockIdx.x * per, e1 = min(a.H, e0 + per);
            for (int e = e0 + tid; e < e1; e += kMegaThreads) tstore(a.th + e, dequant_elem(a.embd, t0, e), T(step, 0, 0));
            __syncthreads();
        }
        for (int l = 0; l < a.L && ok; l++) {
            const MegaLayer &ly = tab[l];
            const bool more = !(l + 1 == a.L && step + 1 == a.steps);  // a following layer exists
            const int nl = l + 1 < a.L ? l + 1 : 0;
            const int npos = l + 1 < a.L ? pos : pos + 1;  // position the following layer runs at
            bool bad = false;
            // ---- q|k|v
            if (q0 < q1) {
                bool good = true;
                if (l == 0) mega_stage<2>(nullptr, &npre, a.eps, a.H, st);  // the stage row holds the embedding
                else good = done_wait(done_d, n_d, T(step, l, 0)) && mega_stage_t<2>(a.th, T(step, l, 0), &npre, a.eps, a.H, st);
                if (!good) { if (tid == 0) raise_err(a, MEGA_ERR_BARRIER); ok = false; break; }
                tl_sub(a, tls);
                int4 act[1][4];
                float dblk[1];
                int sblk[1];
                mega_act<1>(st, a.H, act, dblk, sblk);
                if (!slot_take(0)) { ok = false; break; }
                tl_sub(a, tls);
                const uint8_t *sw = smem + a.slot_off[0];
                const float *ss = (const float *)(sw + align16((size_t)a.rpc[0] * (a.H / 256) * 64));
                const unsigned tq = T(step, l, 1);
                unsigned long long *tqkv = a.tqkv;
                mega_rows<1, RGQ, false>(a.shift, a.off, q0, q1, a.rpc[0], sw, ss, a.H, act, dblk, sblk,
                                         [&](int rg, const float *acc, int rend) {
#pragma unroll
                                             for (int g = 0; g < RGQ; g++)
                                                 if (rg + g < rend) tstore(tqkv + rg + g, acc[g], tq);
                                         });
                tl_sub(a, tls);
            } else {
                if (!slot_take(0)) { ok = false; break; }
                tl_sub(a, tls); tl_sub(a, tls); tl_sub(a, tls);
            }
            __syncthreads();  // slot 0 consumed
            if (more) slot_refill(0, nl);
            tl_mark(a, tli);
            tl_mark(a, tli);
            // ---- attention (the units of this position)
            if (is_attn) {
                AttnArgs aa = a.attn;
                aa.kc = ly.kc;
                aa.vc = ly.vc;
                aa.q_norm = ly.q_norm;
                aa.k_norm = ly.k_norm;
                aa.tpart = a.tpart;
                aa.ptag = T(step, l, 1);
                DecConsts<HD> kcs;
                if (warp <= G) attn_dec_consts<HD, G>(aa, pos, kcs);
                // this unit's q (G heads), k and v words
                bool got = true;
                {
                    const unsigned tq = T(step, l, 1);
                    for (int i = tid; i < (G + 2) * HD; i += kMegaThreads) {
                        const size_t gi = i < G * HD ? (size_t)akvh * G * HD + i
                                                     : (i < (G + 1) * HD ? (size_t)a.qd + akvh * HD + (i - G * HD)
                                                                         : (size_t)a.qd + a.kvd + akvh * HD + (i - (G + 1) * HD));
                        float v = 0.f;
                        got = tpoll1(a.tqkv + gi, tq, v) && got;
                        sqkv[i] = v;
                    }
                }
                if (!__syncthreads_and(got)) { if (tid == 0) raise_err(a, MEGA_ERR_BARRIER); ok = false; break; }
                if (warp <= G)
                    attn_dec_prologue<HD, G>(aa, akvh, pos, achunk == 0, kcs, sq, skc, svc, sqkv, sqkv + G * HD,
                                             sqkv + (G + 1) * HD);
                tl_sub(a, tls);
                asm volatile("cp.async.wait_group 0;" ::: "memory");
                __syncthreads();  // K/V rows of every thread, and sq / skc / svc
                tl_sub(a, tls);
                const auto krow = [&](int j, int c) { return (const uint4 *)(sK + (size_t)j * KROW + c * 16); };
                attn_chunk_main<HD, G>(aa, akvh, achunk, cs_of(pos), pos, krow, sV, sq, skc, svc, S, 1);
                tl_sub(a, tls);
                done_mark(done_a, T(step, l, 1));  // partials published; every read of the K/V area is done
                // the next layer's K/V rows (after the last layer the area carries the LM-head
                // ring; the next step's rows follow the head)
                if (l + 1 < a.L && attn_cta(npos)) mega_kv_fill<HD>(a, tab[nl], sK, sV, akvh, j0_of(npos), ncache_of(npos));
            } else {
                tl_sub(a, tls); tl_sub(a, tls); tl_sub(a, tls);
            }
            tl_mark(a, tli);
            tl_mark(a, tli);
            // ---- o_proj (+ residual)
            if (o0 < o1) {
                const int cs = cs_of(pos);
                if (!done_wait(done_a, a.kvh * ((pos + cs) / cs), T(step, l, 1)) ||
                    !mega_stage_attn_t<HD>(a, pos, T(step, l, 1), st)) {
                    if (tid == 0) raise_err(a, MEGA_ERR_BARRIER);
                    ok = false;
                    break;
                }
                tl_sub(a, tls);
                int4 act[1][4];
                float dblk[1];
                int sblk[1];
                mega_act<1>(st, a.qd, act, dblk, sblk);
                if (!slot_take(1)) { ok = false; break; }
                tl_sub(a, tls);
                const uint8_t *sw = smem + a.slot_off[1];
                const float *ss = (const float *)(sw + align16((size_t)a.rpc[1] * (a.qd / 256) * 64));
                const unsigned tin = T(step, l, 0), tout = T(step, l, 2);
                unsigned long long *th = a.th;
                mega_rows<1, RGO, false>(a.shift, a.off, o0, o1, a.rpc[1], sw, ss, a.qd, act, dblk, sblk,
                                         [&](int rg, const float *acc, int rend) {
#pragma unroll
                                             for (int g = 0; g < RGO; g++)
                                                 if (rg + g < rend) {
                                                     float hv = 0.f;
                                                     bad |= !tpoll1(th + rg + g, tin, hv);
                                                     tstore(th + rg + g, hv + acc[g], tout);
                                                 }
                                         });
                tl_sub(a, tls);
            } else {
                if (!slot_take(1)) { ok = false; break; }
                tl_sub(a, tls); tl_sub(a, tls); tl_sub(a, tls);
            }
            if (__syncthreads_or(bad)) { if (tid == 0) raise_err(a, MEGA_ERR_BARRIER); ok = false; break; }
            if (o0 < o1) done_mark(done_o, T(step, l, 2));
            if (more) slot_refill(1, nl);
            norm_preload<2>(ly.ffn_norm, a.H, npre);
            tl_mark(a, tli);
            tl_mark(a, tli);
            // ---- gate|up (interleaved rows) -> silu(gate) * up
            if (u0 < u1) {
                if (!done_wait(done_o, n_o, T(step, l, 2)) || !mega_stage_t<2>(a.th, T(step, l, 2), &npre, a.eps, a.H, st)) {
                    if (tid == 0) raise_err(a, MEGA_ERR_BARRIER);
                    ok = false;
                    break;
                }
                tl_sub(a, tls);
                int4 act[1][4];
                float dblk[1];
                int sblk[1];
                mega_act<1>(st, a.H, act, dblk, sblk);
                if (!slot_take(2)) { ok = false; break; }
                tl_sub(a, tls);
                const uint8_t *sw = smem + a.slot_off[2];
                const float *ss = (const float *)(sw + align16((size_t)a.rpc[2] * (a.H / 256) * 64));
                const unsigned tout = T(step, l, 3);
                unsigned long long *tact = a.tact;
                mega_rows<1, RGU, true>(a.shift, a.off, u0, u1, a.rpc[2], sw, ss, a.H, act, dblk, sblk,
                                        [&](int rg, const float *acc, int rend) {
#pragma unroll
                                            for (int g = 0; g + 1 < RGU; g += 2) {
                                                if (rg + g + 1 >= rend) break;
                                                const float gt = acc[g], up = acc[g + 1];
                                                tstore(tact + ((rg + g) >> 1), __fmul_rn(gt / (1.0f + expf(-gt)), up), tout);
                                            }
                                        });
                tl_sub(a, tls);
            } else {
                if (!slot_take(2)) { ok = false; break; }
                tl_sub(a, tls); tl_sub(a, tls); tl_sub(a, tls);
            }
            if (u0 < u1) done_mark(done_u, T(step, l, 3));  // also: slot 2 consumed
            else __syncthreads();
            if (more && l + 1 < a.L) slot_refill(2, nl);  // after the last layer: once the head is done
            tl_mark(a, tli);
            tl_mark(a, tli);
            // ---- down (+ residual)
            if (d0 < d1) {
                if (!done_wait(done_u, n_u, T(step, l, 3)) ||
                    !mega_stage_t<CF>(a.tact, T(step, l, 3), (const NormPre<CF> *)nullptr, a.eps, a.F, st)) {
                    if (tid == 0) raise_err(a, MEGA_ERR_BARRIER);
                    ok = false;
                    break;
                }
                tl_sub(a, tls);
                int4 act[CF][4];
                float dblk[CF];
                int sblk[CF];
                mega_act<CF>(st, a.F, act, dblk, sblk);
                if (!slot_take(3)) { ok = false; break; }
                tl_sub(a, tls);
                const uint8_t *sw = smem + a.slot_off[3];
                const float *ss = (const float *)(sw + align16((size_t)a.rpc[3] * (a.F / 256) * 64));
                const unsigned tin = T(step, l, 2), tout = T(step, l + 1, 0);
                unsigned long long *th = a.th;
                mega_rows<CF, RGD, false>(a.shift, a.off, d0, d1, a.rpc[3], sw, ss, a.F, act, dblk, sblk,
                                          [&](int rg, const float *acc, int rend) {
#pragma unroll
                                              for (int g = 0; g < RGD; g++)
                                                  if (rg + g < rend) {
                                                      float hv = 0.f;
                                                      bad |= !tpoll1(th + rg + g, tin, hv);
                                                      tstore(th + rg + g, hv + acc[g], tout);
                                                  }
                                          });
                tl_sub(a, tls);
            } else {
                if (!slot_take(3)) { ok = false; break; }
                tl_sub(a, tls); tl_sub(a, tls); tl_sub(a, tls);
            }
            if (__syncthreads_or(bad)) { if (tid == 0) raise_err(a, MEGA_ERR_BARRIER); ok = false; break; }
            if (d0 < d1) done_mark(done_d, T(step, l + 1, 0));
            if (more && l + 1 < a.L) slot_refill(3, nl);  // after the last layer: once the head is done
            if (l + 1 == a.L) {
                // gate|up and down slots and the K/V area are free: start the LM-head ring
                if (tid == 0) {
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    for (int k = 0; k < a.head_ns && k < hst; k++) head_fill(a, smem, hbar, k, hr0, hr1);
                }
                for (int k = 0; k < a.head_ns && k < hst; k++) hpend |= 1u << k;
            }
            norm_preload<2>(l + 1 < a.L ? tab[l + 1].attn_norm : a.out_norm, a.H, npre);
            tl_mark(a, tli);
            tl_mark(a, tli);
        }
        if (!ok) break;
        // ---- LM head + argmax (rows < vocab_out compete), rows streamed through the ring
        {
            if (!done_wait(done_d, n_d, T(step, a.L, 0)) || !mega_stage_t<2>(a.th, T(step, a.L, 0), &npre, a.eps, a.H, st)) {
                if (tid == 0) raise_err(a, MEGA_ERR_BARRIER);
                ok = false;
                break;
            }
            const int nb = a.H / 256;
            unsigned long long best = 0;
            for (int si = 0; si < hst && ok; si++) {
                const int k = si % a.head_ns;
                if (__syncthreads_and(mbar_wait(&hbar[k], hph[k]))) {
                    hph[k] ^= 1;
                    hpend &= ~(1u << k);
                } else {
                    if (tid == 0) raise_err(a, MEGA_ERR_WEIGHTS);
                    ok = false;
                    break;
                }
                const int r = hr0 + si * kHeadRows + warp;
                if (r < hr1) {
                    const float v = q6k_row_smem(smem + a.head_off[k] + (size_t)warp * a.head.stride, nb, a.H, st);
                    if (lane == 0 && r < a.vocab_out) {
                        const unsigned long long key = argmax_key(v, (uint32_t)r);
                        if (key > best) best = key;
                    }
                }
                __syncthreads();  // stage k consumed
                if (si + a.head_ns < hst) {
                    if (tid == 0) {
                        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                        head_fill(a, smem, hbar, si + a.head_ns, hr0, hr1);
                    }
                    hpend |= 1u << k;
                }
            }
            if (lane == 0) s_best[warp] = best;
            __syncthreads();
            if (tid == 0) {
                unsigned long long m = 0;
                for (int i = 0; i < kMegaWarps; i++) m = s_best[i] > m ? s_best[i] : m;
                __threadfence();  // orders this step's max after the reset of its slot (block 0, last step)
                if (m) atomicMax(&a.sync->amax[step & 1], m);
            }
        }
        tl_mark(a, tli);
        bar_arrive(a, target);
        norm_preload<2>(tab[0].attn_norm, a.H, npre);
        if (ok && step + 1 < a.steps) {
            // the ring is drained: layer 0's gate|up and down slices and K/V rows for the next step
            if (tid == 0) {
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                mega_fill(a, tab, smem, &mbar[2], 2, 0);
                mega_fill(a, tab, smem, &mbar[3], 3, 0);
            }
            pending |= 4u | 8u;
            if (attn_cta(pos + 1)) mega_kv_fill<HD>(a, tab[0], sK, sV, akvh, j0_of(pos + 1), ncache_of(pos + 1));
        }
        if (!bar_wait(a, target, &s_flag)) { ok = false; break; }
        tl_mark(a, tli);
        // ---- token bookkeeping (decode_finalize's rules), in every CTA
        {
            const unsigned long long key = *(volatile unsigned long long *)&a.sync->amax[step & 1];
            const int idx = key ? (int)argmax_index(key) : 0;
            if (blockIdx.x == 0 && tid == 0) {
                // every CTA has read the previous step's slot (all passed this barrier): clear it for
                // the next step; the fence orders the clear before this CTA's next rows
                atomicExch(&a.sync->amax[(step + 1) & 1], 0ull);
                __threadfence();
                DecodeState *ds = a.st;
                if (!ds->stopped) {
                    if (ds->step < ds->cap) a.out_ids[ds->step] = idx;
                    ds->step++;
                    for (int i = 0; i < ds->n_stop; i++)
                        if (ds->stop_ids[i] == idx) ds->stopped = 1;
                }
            }
            tok = idx;
            pos += 1;
        }
    }
    if (blockIdx.x == 0 && tid == 0) {
        a.st->tok = tok;
        a.st->pos = pos;
        a.st->amax = 0ull;
    }
    // copies still in flight into this CTA's shared memory (error exits)
    if (tid == 0)
        for (int i = 0; i < 4; i++) {
            if (pending & (1u << i)) mbar_wait(&mbar[i], ph[i]);
            if (hpend & (1u << i)) mbar_wait(&hbar[i], hph[i]);
        }
    asm volatile("cp.async.wait_all;" ::: "memory");
    __syncthreads();
}

// Dynamic shared memory plan of decode_mega for a model shape.
struct MegaPlan {
    int rpc[5], slot_off[4], stage_off, attn_off, kmax;
    int head_ns, head_off[4];  // LM-head ring: stages placed in the gate|up + down slots and the K/V area
    size_t bytes;
};

inline MegaPlan mega_plan(int grid, int H, int F, int qd, int kvd, int vocab, int HD) {
    MegaPlan p;
    size_t off = 0;
    for (int t = 0; t < 4; t++) {
        const int rows = mega_phase_rows(t, H, F, qd, kvd);
        int r = (rows + grid - 1) / grid;
        r = (r + kMegaRowAlign - 1) / kMegaRowAlign * kMegaRowAlign;
        p.rpc[t] = r;
        p.slot_off[t] = (int)off;
        off += (size_t)mega_slot_bytes(r, mega_phase_k(t, H, F, qd));
    }
    p.rpc[4] = (vocab + grid - 1) / grid;
    p.kmax = H > F ? H : F;
    if (qd > p.kmax) p.kmax = qd;
    p.stage_off = (int)off;
    off += align16(q8_smem_bytes(1, p.kmax));
    p.attn_off = (int)off;
    off += (size_t)kDecSplit * (HD * 2 + kMegaKPad) + (size_t)kDecSplit * HD * 2;
    p.bytes = off;
    p.head_ns = 0;
    return p;
}

// Place up to four head-ring stages of kHeadRows rows of `head_stride` bytes
// in regions that are idle while the head runs; false if fewer than two fit.
inline bool mega_head_ring(MegaPlan &p, long long head_stride) {
    const size_t sb = (size_t)kHeadRows * (size_t)head_stride;
    p.head_ns = 0;
    for (size_t o = (size_t)p.slot_off[2]; o + sb <= (size_t)p.stage_off && p.head_ns < 4; o += sb)
        p.head_off[p.head_ns++] = (int)o;
    for (size_t o = (size_t)p.attn_off; o + sb <= p.bytes && p.head_ns < 4; o += sb) p.head_off[p.head_ns++] = (int)o;
    return p.head_ns >= 2;
}

}  // namespace hyk
