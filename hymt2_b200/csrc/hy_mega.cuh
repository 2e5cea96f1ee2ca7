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

enum MegaErr { MEGA_OK = 0, MEGA_ERR_BARRIER = 1, MEGA_ERR_POS = 2, MEGA_ERR_WEIGHTS = 3, MEGA_ERR_KV = 4, MEGA_ERR_HOST = 5 };

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
    int go, go_tok;              // resident host loop: the host's go for the next step (-1: stop), its token
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
    int head_reg[2], head_n1;  // LM-head row slots: head_n1 of them from head_reg[0], the rest from head_reg[1]
    AttnArgs attn;            // shape, rope tables, part buffer; per-layer fields set in-kernel
    WDesc head, embd;
    int vocab_out;
    const float *out_norm;
    float *h, *qkv, *ao, *act;
    DecodeState *st;
    int *out_ids;
    MegaSync *sync;
    unsigned long long *tl;   // optional timeline (block 0): globaltimer per phase edge
    int tl_cap;
    int steps;
    // resident host loop (null: off): mapped pinned ints [go, token in, done, token out].  Step s
    // starts once the host has set go >= s + 1 (go < 0: stop) and takes its input token from
    // token in; after it, token out holds its argmax and done = s + 1 (-1 after an error)
    int *host_io;
    unsigned long long host_limit_ns;  // bound on each wait for the host
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
// System-scope accesses of the mapped host words of the resident loop.
__device__ __forceinline__ int ld_acquire_sys_s32(const int *p) {
    int v;
    asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ int ld_relaxed_sys_s32(const int *p) {
    int v;
    asm volatile("ld.relaxed.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys_s32(int *p, int v) {
    asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void st_relaxed_sys_s32(int *p, int v) {
    asm volatile("st.relaxed.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void st_release_gpu_s32(int *p, int v) {
    asm volatile("st.release.gpu.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_gpu_s32(const int *p) {
    int v;
    asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Resident host loop, before step `step` (all threads): block 0's thread 0
// waits (bounded by host_limit_ns) for the host's go and reads its token,
// then publishes both in device memory, where every CTA's thread 0 waits for
// them (bounded).  Returns the token, or -1 when the host stopped the loop,
// did not answer (MEGA_ERR_HOST) or another CTA failed.
__device__ __forceinline__ int host_step_begin(const MegaArgs &a, int step, int *s_word) {
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        int v = ld_acquire_sys_s32(&a.host_io[0]);
        const unsigned long long t0 = gtimer();
        unsigned it = 0;
        while (v >= 0 && v < step + 1) {
            if ((++it & 63) == 0 && gtimer() - t0 > a.host_limit_ns) {
                raise_err(a, MEGA_ERR_HOST);
                v = -1;
                break;
            }
            v = ld_acquire_sys_s32(&a.host_io[0]);
        }
        const int t = v >= 0 ? ld_relaxed_sys_s32(&a.host_io[1]) : 0;
        a.sync->go_tok = t;
        st_release_gpu_s32(&a.sync->go, v >= 0 ? step + 1 : -1);
    }
    if (threadIdx.x == 0) {
        int g = ld_acquire_gpu_s32(&a.sync->go);
        const unsigned long long t0 = gtimer();
        unsigned it = 0;
        while (g >= 0 && g < step + 1) {
            if ((++it & 63) == 0) {
                if (ld_relaxed_s32(&a.sync->err)) { g = -1; break; }
                if (gtimer() - t0 > a.host_limit_ns + kMegaWaitNs) { raise_err(a, MEGA_ERR_BARRIER); g = -1; break; }
            }
            g = ld_acquire_gpu_s32(&a.sync->go);
        }
        *s_word = g < 0 ? -1 : *(volatile int *)&a.sync->go_tok;
    }
    __syncthreads();
    const int r = *s_word;
    __syncthreads();  // s_word is reused
    return r;
}


// Grid-wide barrier in two halves.  bar_arrive: once every thread's writes
// of the phase are done (__syncthreads), thread 0 adds 1 to the arrival
// counter with release semantics (publishing them).  Work that does not
// depend on other CTAs can run between the halves.  bar_wait: thread 0 polls
// until the counter reaches the running target; bounded, and a timeout or
// another CTA's error makes every CTA return false from here on.
__device__ __forceinline__ void bar_arrive(const MegaArgs &a, unsigned &target) {
    __syncthreads();
    target += gridDim.x;
    if (threadIdx.x == 0) asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(&a.sync->bar) : "memory");
}
__device__ __forceinline__ bool bar_wait(const MegaArgs &a, unsigned target, int *s_flag,
                                         unsigned long long limit_ns = kMegaWaitNs) {
    if (threadIdx.x == 0) {
        int bad = 0;
        if ((int)(ld_acquire_u32(&a.sync->bar) - target) < 0) {
            const unsigned long long t0 = gtimer();
            unsigned it = 0;
            while ((int)(ld_acquire_u32(&a.sync->bar) - target) < 0) {
                if ((++it & 63) == 0) {
                    if (ld_relaxed_s32(&a.sync->err)) { bad = 1; break; }
                    if (gtimer() - t0 > limit_ns) { raise_err(a, MEGA_ERR_BARRIER); bad = 1; break; }
                }
            }
        }
        if (!bad && ld_relaxed_s32(&a.sync->err)) bad = 1;
        *s_flag = bad;
    }
    __syncthreads();
    return *s_flag == 0;
}

// Each warp waits for slot `bar`; the outcome is uniform within the warp
// (its row loop uses warp shuffles).  A warp that times out raises the error
// word, skips its rows and still reaches every CTA barrier; the next grid
// barrier then stops every CTA.
__device__ __forceinline__ bool mega_slot_ready(const MegaArgs &a, uint64_t *bar, unsigned parity) {
    const bool ready = __all_sync(0xffffffffu, mbar_wait(bar, parity)) != 0;
    if (!ready && (threadIdx.x & 31) == 0) raise_err(a, MEGA_ERR_WEIGHTS);
    return ready;
}

// Timeline (measurement builds with -DHYK_TRACE and a.tl non-null): [0,
// cap/2) phase edges of block 0; [cap/2, cap/2 + 8192) sub-phase marks of
// block 0; then per-CTA marks of one chosen (step, layer): 16 slots per CTA.
#ifdef HYK_TRACE
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
#else
__device__ __forceinline__ void tl_mark(const MegaArgs &, int &) {}
__device__ __forceinline__ void tl_sub(const MegaArgs &, int &) {}
__device__ __forceinline__ void tl_cta(const MegaArgs &, bool, int) {}
#endif

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
// wait (they are constants), in the block-wise staging layout of norm_f4 with
// this CTA's warps: warp b < K/256 holds block b (lane l: elements 8l..8l+7).
struct NormPre {
    float4 w[2];
};
__device__ __forceinline__ void norm_preload(const float *norm_w, int K, NormPre &p) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (warp < K / 256) {
        p.w[0] = __ldg((const float4 *)norm_w + norm_f4(0, warp, lane, kMegaWarps));
        p.w[1] = __ldg((const float4 *)norm_w + norm_f4(1, warp, lane, kMegaWarps));
    }
}

// x (K <= 256 * kMegaWarps inputs, global or shared) -> RMSNorm * preloaded
// weights -> Q8_K in shared memory.  Warp b < K/256 loads, normalises and
// quantises block b in its registers; the sum of squares is norm_ss's fixed
// order, so codes and scales are those of the per-layer kernels (stage_fp32
// and quantize_block_warp).
__device__ inline void mega_stage_norm(const float *x, const NormPre &pre, float eps, int K, Q8Smem &s) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nb = K / 256;
    float4 xv[2] = {make_float4(0.f, 0.f, 0.f, 0.f), make_float4(0.f, 0.f, 0.f, 0.f)};
    if (warp < nb) {
        xv[0] = ((const float4 *)x)[norm_f4(0, warp, lane, kMegaWarps)];
        xv[1] = ((const float4 *)x)[norm_f4(1, warp, lane, kMegaWarps)];
    }
    const float ss = norm_ss<2>(xv, K, s.red);
    const float scale = 1.0f / sqrtf(ss / (float)K + eps);
    if (warp < nb) {
        const float v[8] = {__fmul_rn(__fmul_rn(xv[0].x, scale), pre.w[0].x),
                            __fmul_rn(__fmul_rn(xv[0].y, scale), pre.w[0].y),
                            __fmul_rn(__fmul_rn(xv[0].z, scale), pre.w[0].z),
                            __fmul_rn(__fmul_rn(xv[0].w, scale), pre.w[0].w),
                            __fmul_rn(__fmul_rn(xv[1].x, scale), pre.w[1].x),
                            __fmul_rn(__fmul_rn(xv[1].y, scale), pre.w[1].y),
                            __fmul_rn(__fmul_rn(xv[1].z, scale), pre.w[1].z),
                            __fmul_rn(__fmul_rn(xv[1].w, scale), pre.w[1].w)};
        quantize_vals_warp(v, s, 0, warp, nb, K);
    }
    __syncthreads();
}

// x (K inputs as they are) -> Q8_K: warp w quantises blocks w, w + 16, ...
// (NBW of them) in its registers, every load issued before any arithmetic;
// the values and element order of quantize_block_warp.
template <int NBW>
__device__ inline void mega_stage_plain(const float *x, int K, Q8Smem &s) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nb = K / 256;
    float4 xv[NBW][2];
#pragma unroll
    for (int i = 0; i < NBW; i++) {
        const int b = warp + kMegaWarps * i;
        if (b < nb) {
            xv[i][0] = ((const float4 *)x)[b * 64 + lane * 2];
            xv[i][1] = ((const float4 *)x)[b * 64 + lane * 2 + 1];
        }
    }
#pragma unroll
    for (int i = 0; i < NBW; i++) {
        const int b = warp + kMegaWarps * i;
        if (b < nb) {
            const float v[8] = {xv[i][0].x, xv[i][0].y, xv[i][0].z, xv[i][0].w,
                                xv[i][1].x, xv[i][1].y, xv[i][1].z, xv[i][1].w};
            quantize_vals_warp(v, s, 0, b, nb, K);
        }
    }
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
// per-row arithmetic as gemv_panel_dec.  After the butterfly every lane 4s
// holds all RG sums; epi(r, acc[], r1, s) runs on lanes 4s (s = 0..7), each
// finishing the rows (or row pairs) of its index s, so the epilogues of a
// group run side by side.
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
        // only lanes 4k hold partial sums: three butterfly levels bring them to lane 0
#pragma unroll
        for (int o = 16; o >= 4; o >>= 1)
#pragma unroll
            for (int g = 0; g < RG; g++) acc[g] += __shfl_xor_sync(0xffffffffu, acc[g], o);
        if ((lane & 3) == 0) epi(rg, acc, r1, lane >> 2);
    }
}

// ---------------------------------------------------------------- LM head (Q6_K) with argmax

// The head's native Q6_K rows (device layout ql | qh | scales | d per row)
// stream through a private ring of kHeadRing row slots per warp, filled with
// cp.async (16-byte copies spread over the lanes, one commit group per row),
// so each warp keeps kHeadRing rows in flight and no CTA barrier separates
// the rows.  Warp w takes rows r0 + w, r0 + w + 16, ... of its CTA's slice.
constexpr int kHeadRing = 5;

__device__ __forceinline__ uint8_t *head_slot(const MegaArgs &a, uint8_t *smem, int warp, int k) {
    const int i = warp * kHeadRing + k;
    const long long rb = a.head.stride;
    return smem + (i < a.head_n1 ? a.head_reg[0] + (long long)i * rb : a.head_reg[1] + (long long)(i - a.head_n1) * rb);
}

__device__ __forceinline__ void cp_async16_hint(void *dst, const void *src, uint64_t pol) {
    asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "l"(pol)
                 : "memory");
}

// Warp: copy head row `row` (if the warp has it) into slot k and commit one
// group per lane (empty when there is no row, so every lane's group count
// stays one per ring step).  Every head byte is read once per step.
__device__ __forceinline__ void head_row_issue(const MegaArgs &a, uint8_t *smem, int k, int row, int r0, int r1) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    (void)r0;
    if (row < r1) {
        const uint64_t pol = l2_policy_evict_first();
        const uint8_t *src = a.head.w + (size_t)row * a.head.stride;
        uint8_t *dst = head_slot(a, smem, warp, k);
        for (int c = lane * 16; c < (int)a.head.stride; c += 32 * 16) cp_async16_hint(dst + c, src + c, pol);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
}

// This lane's unit of the head activation (K <= 2048: one 64-element unit
// per lane), kept in registers for every row: the Q8_K codes each of its four
// 16-element groups meets, their bsums and the block scale.
struct HeadAct {
    int4 av[4];
    int bs[4];
    float d;
};
__device__ __forceinline__ void head_act_load(const Q8Smem &s, int K, HeadAct &h) {
    const int u = threadIdx.x & 31, b = u >> 2, hf = (u >> 1) & 1, sg = u & 1;
    const bool ok = u < K / 64;
#pragma unroll
    for (int q = 0; q < 4; q++) {
        const int ch = hf * 2 + (q >> 1), l = (2 * q + sg) & 3;
        h.av[q] = ok ? *(const int4 *)&s.qp[(size_t)l * (K / 4) + (b * 4 + piece_of_chunk(ch)) * 16] : make_int4(0, 0, 0, 0);
        h.bs[q] = ok ? (int)s.bs[b * 16 + hf * 8 + 2 * q + sg] : 0;
    }
    h.d = ok ? s.d[b] : 0.f;
}

// One native Q6_K row in shared memory against the register-held activation:
// the unit split, integer sums, float steps and warp sum of gemv_q6k (and
// q6k_row_smem) for K <= 2048, so the logit is the per-layer kernels' own.
__device__ __forceinline__ float q6k_row_regs(const uint8_t *row, int nb, const HeadAct &h) {
    const int u = threadIdx.x & 31, b = u >> 2, hf = (u >> 1) & 1, sg = u & 1;
    const bool ok = u < nb * 4;
    int acc_i = 0;
    float dw = 0.f;
    if (ok) {
        const uint4 qa = *(const uint4 *)(row + (size_t)b * 128 + hf * 64 + sg * 16);
        const uint4 qb = *(const uint4 *)(row + (size_t)b * 128 + hf * 64 + 32 + sg * 16);
        const uint4 qh = *(const uint4 *)(row + (size_t)nb * 128 + (size_t)b * 64 + hf * 32 + sg * 16);
        const uint4 scv = *(const uint4 *)(row + (size_t)nb * 192 + (size_t)b * 16);
        dw = h2f(*(const unsigned short *)(row + (size_t)nb * 208 + 2 * b));
        const uint32_t A[4] = {qa.x, qa.y, qa.z, qa.w}, B[4] = {qb.x, qb.y, qb.z, qb.w};
        const uint32_t Hh[4] = {qh.x, qh.y, qh.z, qh.w};
#pragma unroll
        for (int q = 0; q < 4; q++) {
            uint32_t code[4];
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const uint32_t src = (q & 1) ? B[j] : A[j];
                code[j] = ((src >> (4 * (q >> 1))) & 0x0f0f0f0fu) | (((Hh[j] >> (2 * q)) & 0x03030303u) << 4);
            }
            int tq = dp4a((int)code[0], h.av[q].x, 0);
            tq = dp4a((int)code[1], h.av[q].y, tq);
            tq = dp4a((int)code[2], h.av[q].z, tq);
            tq = dp4a((int)code[3], h.av[q].w, tq);
            tq -= 32 * h.bs[q];
            acc_i += q6k_subscale(scv, hf * 8 + 2 * q + sg) * tq;
        }
    }
    acc_i += __shfl_xor_sync(0xffffffffu, acc_i, 1);
    acc_i += __shfl_xor_sync(0xffffffffu, acc_i, 2);
    float acc = 0.f;
    if (ok && (u & 3) == 0) acc += dw * h.d * (float)acc_i;
    return warp_sum(acc);
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

// Launch shape contract (checked by the host): grid = number of SMs, all
// resident (cooperative launch); L <= kMegaMaxLayers; kvh * ceil(ctx /
// kDecSplit) <= grid; every layer weight a panel with (shift, off); H, qd <=
// 2048 (one 64-element chunk per lane) and F <= 2048 * CF; head Q6_K with
// k == H.
//
// Between bar_arrive and bar_wait each CTA does the work that needs nothing
// from other CTAs: it refills the weight slot it just consumed with the next
// layer's slice, stages the next layer's K/V rows (after this layer's
// attention), and loads the next phase's norm weights and rope constants.
template <int HD, int G, int CF>
__global__ void __launch_bounds__(kMegaThreads, 1) decode_mega(const __grid_constant__ MegaArgs a) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ __align__(8) uint64_t mbar[4];  // weight slots
    __shared__ int s_flag, s_hostw;
    __shared__ unsigned long long s_best[kMegaWarps];
    __shared__ __align__(16) float sq[G][HD];
    __shared__ __align__(16) float skc[HD], svc[HD];
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
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    unsigned ph[4] = {0, 0, 0, 0};  // parity each mbarrier completes next
    unsigned pending = 0;              // bit i: a fill of mbarrier i is outstanding (same in every thread)
    unsigned target = 0;
    int tli = 0, tls = 0;
    int tok = a.st->tok, pos = a.st->pos;
    bool ok = true;
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
    // prime: layer 0's weight slots and K/V rows, the first norm weights
    if (tid == 0)
        for (int t = 0; t < 4; t++) mega_fill(a, tab, smem, &mbar[t], t, 0);
    pending |= 0xfu;
    if (a.steps > 0 && attn_cta(pos)) mega_kv_fill<HD>(a, tab[0], sK, sV, akvh, j0_of(pos), ncache_of(pos));
    NormPre npre;
    norm_preload(tab[0].attn_norm, a.H, npre);
    bool host_early = false;  // the resident host loop ended before a.steps
    for (int step = 0; step < a.steps && ok; step++) {
        if (a.host_io) {
            const int t = host_step_begin(a, step, &s_hostw);
            if (t < 0) {
                host_early = true;
                break;
            }
            tok = t;
        }
        if (pos < 0 || pos >= a.ctx) {
            if (tid == 0) raise_err(a, MEGA_ERR_POS);
            ok = false;
            break;
        }
        const bool is_attn = attn_cta(pos);
        tl_mark(a, tli);
        // embedding of `tok` into the stage row; CTA b also writes its slice of h
        {
            const int t0 = (tok < 0 || tok >= a.embd.n) ? 0 : tok;
            for (int e = tid; e < a.H; e += kMegaThreads) st.x[e] = dequant_elem(a.embd, t0, e);
            const int per = (a.H + gridDim.x - 1) / gridDim.x;
            const int e0 = blockIdx.x * per, e1 = min(a.H, e0 + per);
            for (int e = e0 + tid; e < e1; e += kMegaThreads) a.h[e] = dequant_elem(a.embd, t0, e);
            __syncthreads();
        }
        for (int l = 0; l < a.L && ok; l++) {
            const MegaLayer &ly = tab[l];
            const bool more = !(l + 1 == a.L && step + 1 == a.steps);  // a following layer exists
            const int nl = l + 1 < a.L ? l + 1 : 0;
            const int npos = l + 1 < a.L ? pos : pos + 1;  // position the following layer runs at
            AttnArgs aa = a.attn;
            aa.kc = ly.kc;
            aa.vc = ly.vc;
            aa.q_norm = ly.q_norm;
            aa.k_norm = ly.k_norm;
            aa.tickets = a.sync->tickets;
            // ---- q|k|v
            {
                mega_stage_norm(l == 0 ? st.x : a.h, npre, a.eps, a.H, st);
                tl_sub(a, tls);
                int4 act[1][4];
                float dblk[1];
                int sblk[1];
                mega_act<1>(st, a.H, act, dblk, sblk);
                if (mega_slot_ready(a, &mbar[0], ph[0])) {
                    ph[0] ^= 1;
                    pending &= ~1u;
                } else {
                    ok = false;
                }
                tl_sub(a, tls);
                const int rpc = a.rpc[0], r0 = blockIdx.x * rpc, r1 = min(r0 + rpc, a.qd + 2 * a.kvd);
                const uint8_t *sw = smem + a.slot_off[0];
                const float *ss = (const float *)(sw + align16((size_t)rpc * (a.H / 256) * 64));
                float *qkv = a.qkv;
                if (ok)
                    mega_rows<1, RGQ, false>(a.shift, a.off, r0, r1, rpc, sw, ss, a.H, act, dblk, sblk,
                                             [&](int rg, const float *acc, int rend, int sel) {
#pragma unroll
                                                 for (int g = 0; g < RGQ; g++)
                                                     if (g == sel && rg + g < rend) qkv[rg + g] = acc[g];
                                             });
                tl_sub(a, tls);
            }
            tl_mark(a, tli);
            tl_cta(a, step == 1 && l == 5, 0);
            bar_arrive(a, target);
            if (more && ok) {
                if (tid == 0) {
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    mega_fill(a, tab, smem, &mbar[0], 0, nl);
                }
                pending |= 1u;
            }
            DecConsts<HD> kcs;
            if (is_attn && warp <= G) attn_dec_consts<HD, G>(aa, pos, kcs);
            if (!bar_wait(a, target, &s_flag)) { ok = false; break; }
            tl_cta(a, step == 1 && l == 5, 1);
            tl_mark(a, tli);
            if (l == 0 && blockIdx.x == 0 && tid == 0) a.sync->amax[(step + 1) & 1] = 0ull;
            // ---- attention (the CTAs of the splits that hold keys)
            if (is_attn) {
                if (warp <= G)
                    attn_dec_prologue<HD, G>(aa, akvh, pos, achunk == 0, kcs, sq, skc, svc, aa.qkv + (akvh * G) * HD,
                                             aa.qkv + aa.qdim + akvh * HD, aa.qkv + aa.qdim + aa.kvdim + akvh * HD);
                tl_sub(a, tls);
                asm volatile("cp.async.wait_group 0;" ::: "memory");
                __syncthreads();  // K/V rows of every thread, and sq / skc / svc
                tl_sub(a, tls);
                if (ok) {
                    const auto krow = [&](int j, int c) { return (const uint4 *)(sK + (size_t)j * KROW + c * 16); };
#ifdef HYK_TRACE
                    // attention sub-marks of block 0, layer 5 of step 1: [cap/2 + 7000 ..)
                    int am = 0;
                    const auto mark = [&]() {
                        if (a.tl && blockIdx.x == 0 && threadIdx.x == 0 && step == 1 && l == 5)
                            a.tl[a.tl_cap / 2 + 7000 + am] = gtimer();
                        am++;
                    };
                    if (a.tl && blockIdx.x == 0 && threadIdx.x == 0 && step == 1 && l == 5)
                        a.tl[a.tl_cap / 2 + 7010] = gtimer();
                    attn_chunk_main<HD, G>(aa, akvh, achunk, cs_of(pos), pos, krow, sV, sq, skc, svc, S, 1, mark);
                    if (a.tl && blockIdx.x == 0 && threadIdx.x == 0 && step == 1 && l == 5)
                        a.tl[a.tl_cap / 2 + 7011] = gtimer();
#else
                    attn_chunk_main<HD, G>(aa, akvh, achunk, cs_of(pos), pos, krow, sV, sq, skc, svc, S, 1);
#endif
                }
                tl_sub(a, tls);
            }
            tl_mark(a, tli);
            tl_cta(a, step == 1 && l == 5, 2);
            bar_arrive(a, target);
            if (!bar_wait(a, target, &s_flag)) { ok = false; break; }
            tl_cta(a, step == 1 && l == 5, 3);
            tl_mark(a, tli);
            // ---- o_proj (+ residual)
            {
                mega_stage_attn<HD>(a, pos, st);
                tl_sub(a, tls);
                int4 act[1][4];
                float dblk[1];
                int sblk[1];
                mega_act<1>(st, a.qd, act, dblk, sblk);
                if (mega_slot_ready(a, &mbar[1], ph[1])) {
                    ph[1] ^= 1;
                    pending &= ~2u;
                } else {
                    ok = false;
                }
                tl_sub(a, tls);
                const int rpc = a.rpc[1], r0 = blockIdx.x * rpc, r1 = min(r0 + rpc, a.H);
                const uint8_t *sw = smem + a.slot_off[1];
                const float *ss = (const float *)(sw + align16((size_t)rpc * (a.qd / 256) * 64));
                float *h = a.h;
                if (ok)
                    mega_rows<1, RGO, false>(a.shift, a.off, r0, r1, rpc, sw, ss, a.qd, act, dblk, sblk,
                                             [&](int rg, const float *acc, int rend, int sel) {
#pragma unroll
                                                 for (int g = 0; g < RGO; g++)
                                                     if (g == sel && rg + g < rend) h[rg + g] += acc[g];
                                             });
                tl_sub(a, tls);
            }
            tl_mark(a, tli);
            tl_cta(a, step == 1 && l == 5, 4);
            bar_arrive(a, target);
            if (more && ok && l + 1 < a.L) {  // after the last layer: once the head is done
                if (tid == 0) {
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    mega_fill(a, tab, smem, &mbar[1], 1, nl);
                }
                pending |= 2u;
            }
            if (more && ok) {
                // this layer's attention is done with the K/V area: stage the next layer's rows
                // (after the last layer the area carries the LM-head ring; the next step's rows
                // follow the head)
                if (l + 1 < a.L && attn_cta(npos)) mega_kv_fill<HD>(a, tab[nl], sK, sV, akvh, j0_of(npos), ncache_of(npos));
            }
            norm_preload(ly.ffn_norm, a.H, npre);
            if (!bar_wait(a, target, &s_flag)) { ok = false; break; }
            tl_cta(a, step == 1 && l == 5, 5);
            tl_mark(a, tli);
            // ---- gate|up (interleaved rows) -> silu(gate) * up
            {
                mega_stage_norm(a.h, npre, a.eps, a.H, st);
                tl_sub(a, tls);
                int4 act[1][4];
                float dblk[1];
                int sblk[1];
                mega_act<1>(st, a.H, act, dblk, sblk);
                if (mega_slot_ready(a, &mbar[2], ph[2])) {
                    ph[2] ^= 1;
                    pending &= ~4u;
                } else {
                    ok = false;
                }
                tl_sub(a, tls);
                const int rpc = a.rpc[2], r0 = blockIdx.x * rpc, r1 = min(r0 + rpc, 2 * a.F);
                const uint8_t *sw = smem + a.slot_off[2];
                const float *ss = (const float *)(sw + align16((size_t)rpc * (a.H / 256) * 64));
                float *out = a.act;
                if (ok)
                    mega_rows<1, RGU, true>(a.shift, a.off, r0, r1, rpc, sw, ss, a.H, act, dblk, sblk,
                                            [&](int rg, const float *acc, int rend, int sel) {
#pragma unroll
                                                for (int g = 0; g + 1 < RGU; g += 2) {
                                                    if (g != 2 * sel || rg + g + 1 >= rend) continue;
                                                    const float gt = acc[g], up = acc[g + 1];
                                                    out[(rg + g) >> 1] = __fmul_rn(gt / (1.0f + expf(-gt)), up);
                                                }
                                            });
                tl_sub(a, tls);
            }
            tl_mark(a, tli);
            tl_cta(a, step == 1 && l == 5, 6);
            bar_arrive(a, target);
            if (more && ok && l + 1 < a.L) {  // after the last layer: once the head is done
                if (tid == 0) {
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    mega_fill(a, tab, smem, &mbar[2], 2, nl);
                }
                pending |= 4u;
            }
            if (!bar_wait(a, target, &s_flag)) { ok = false; break; }
            tl_cta(a, step == 1 && l == 5, 7);
            tl_mark(a, tli);
            // ---- down (+ residual)
            {
                mega_stage_plain<(CF * 8 + kMegaWarps - 1) / kMegaWarps>(a.act, a.F, st);
                tl_sub(a, tls);
                int4 act[CF][4];
                float dblk[CF];
                int sblk[CF];
                mega_act<CF>(st, a.F, act, dblk, sblk);
                if (mega_slot_ready(a, &mbar[3], ph[3])) {
                    ph[3] ^= 1;
                    pending &= ~8u;
                } else {
                    ok = false;
                }
                tl_sub(a, tls);
                const int rpc = a.rpc[3], r0 = blockIdx.x * rpc, r1 = min(r0 + rpc, a.H);
                const uint8_t *sw = smem + a.slot_off[3];
                const float *ss = (const float *)(sw + align16((size_t)rpc * (a.F / 256) * 64));
                float *h = a.h;
                if (ok)
                    mega_rows<CF, RGD, false>(a.shift, a.off, r0, r1, rpc, sw, ss, a.F, act, dblk, sblk,
                                              [&](int rg, const float *acc, int rend, int sel) {
#pragma unroll
                                                  for (int g = 0; g < RGD; g++)
                                                      if (g == sel && rg + g < rend) h[rg + g] += acc[g];
                                              });
                tl_sub(a, tls);
            }
            tl_mark(a, tli);
            tl_cta(a, step == 1 && l == 5, 8);
            bar_arrive(a, target);
            if (more && ok && l + 1 < a.L) {  // after the last layer: once the head is done
                if (tid == 0) {
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    mega_fill(a, tab, smem, &mbar[3], 3, nl);
                }
                pending |= 8u;
            }
            if (l + 1 == a.L && ok) {
                // o_proj, gate|up and down slots and the K/V area are free: start every warp's
                // LM-head ring (no copy of this step's K/V rows is pending: the last layer stages none)
                for (int k = 0; k < kHeadRing; k++) head_row_issue(a, smem, k, hr0 + warp + k * kMegaWarps, hr0, hr1);
            }
            norm_preload(l + 1 < a.L ? tab[l + 1].attn_norm : a.out_norm, a.H, npre);
            if (!bar_wait(a, target, &s_flag)) { ok = false; break; }
            tl_cta(a, step == 1 && l == 5, 9);
            tl_mark(a, tli);
        }
        if (!ok) break;
        // ---- LM head + argmax (rows < vocab_out compete), rows streamed through the warp rings
        {
            mega_stage_norm(a.h, npre, a.eps, a.H, st);
            tl_sub(a, tls);
            HeadAct hact;
            head_act_load(st, a.H, hact);
            const int nb = a.H / 256;
            unsigned long long best = 0;
            int j = 0;
            for (int row = hr0 + warp; row < hr1; row += kMegaWarps, j++) {
                const int k = j % kHeadRing;
                // the oldest of this lane's kHeadRing groups (row j) has landed; then every lane's
                asm volatile("cp.async.wait_group %0;" ::"n"(kHeadRing - 1) : "memory");
                __syncwarp();
                const float v = q6k_row_regs(head_slot(a, smem, warp, k), nb, hact);
                if (lane == 0 && row < a.vocab_out) {
                    const unsigned long long key = argmax_key(v, (uint32_t)row);
                    if (key > best) best = key;
                }
                __syncwarp();  // slot k consumed by every lane
                head_row_issue(a, smem, k, row + kHeadRing * kMegaWarps, hr0, hr1);
            }
            asm volatile("cp.async.wait_all;" ::: "memory");
            tl_sub(a, tls);
            if (lane == 0) s_best[warp] = best;
            __syncthreads();
            if (tid == 0) {
                unsigned long long m = 0;
                for (int i = 0; i < kMegaWarps; i++) m = s_best[i] > m ? s_best[i] : m;
                if (m) atomicMax(&a.sync->amax[step & 1], m);
            }
        }
        tl_mark(a, tli);
        bar_arrive(a, target);
        norm_preload(tab[0].attn_norm, a.H, npre);
        if (ok && step + 1 < a.steps) {
            // the ring is drained: layer 0's o_proj, gate|up and down slices and K/V rows for the next step
            if (tid == 0) {
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                mega_fill(a, tab, smem, &mbar[1], 1, 0);
                mega_fill(a, tab, smem, &mbar[2], 2, 0);
                mega_fill(a, tab, smem, &mbar[3], 3, 0);
            }
            pending |= 2u | 4u | 8u;
            if (attn_cta(pos + 1)) mega_kv_fill<HD>(a, tab[0], sK, sV, akvh, j0_of(pos + 1), ncache_of(pos + 1));
        }
        if (!bar_wait(a, target, &s_flag)) { ok = false; break; }
        tl_mark(a, tli);
        // ---- token bookkeeping (decode_finalize's rules), in every CTA
        {
            const unsigned long long key = *(volatile unsigned long long *)&a.sync->amax[step & 1];
            const int idx = key ? (int)argmax_index(key) : 0;
            if (blockIdx.x == 0 && tid == 0) {
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
            if (a.host_io && blockIdx.x == 0 && tid == 0) {
                st_relaxed_sys_s32(&a.host_io[3], idx);
                __threadfence_system();
                st_release_sys_s32(&a.host_io[2], step + 1);
            }
        }
    }
    if (blockIdx.x == 0 && tid == 0) {
        a.st->tok = tok;
        a.st->pos = pos;
        a.st->amax = 0ull;
        if (a.host_io && (!ok || host_early)) st_release_sys_s32(&a.host_io[2], -1);
    }
    // copies still in flight into this CTA's shared memory (error exits)
    if (tid == 0)
        for (int i = 0; i < 4; i++)
            if (pending & (1u << i)) mbar_wait(&mbar[i], ph[i]);
    asm volatile("cp.async.wait_all;" ::: "memory");
    __syncthreads();
}

// Dynamic shared memory plan of decode_mega for a model shape.
struct MegaPlan {
    int rpc[5], slot_off[4], stage_off, attn_off, kmax;
    int head_reg[2], head_n1;  // LM-head row slots: in the o_proj, gate|up, down slots, then the K/V area
    size_t bytes;
};

inline MegaPlan mega_plan(int grid, int H, int F, int qd, int kvd, int vocab, int HD) {
    MegaPlan p;
    size_t off = 0;
    const int align = kMegaRowAlign;
    for (int t = 0; t < 4; t++) {
        const int rows = mega_phase_rows(t, H, F, qd, kvd);
        int r = (rows + grid - 1) / grid;
        r = (r + align - 1) / align * align;
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
    p.head_n1 = 0;
    return p;
}

// Place the kHeadRing row slots of every warp (rows of `head_stride` bytes, a
// multiple of 16) in the regions that are idle while the head runs: the
// o_proj, gate|up and down weight slots, then the K/V area.  False if they
// do not fit.
inline bool mega_head_ring(MegaPlan &p, long long head_stride) {
    if (head_stride <= 0 || head_stride % 16) return false;
    const long long n1 = ((long long)p.stage_off - p.slot_off[1]) / head_stride;
    const long long n2 = ((long long)p.bytes - p.attn_off) / head_stride;
    p.head_reg[0] = p.slot_off[1];
    p.head_reg[1] = p.attn_off;
    p.head_n1 = (int)n1;
    return n1 + n2 >= (long long)kMegaWarps * kHeadRing;
}

}  // namespace hyk
