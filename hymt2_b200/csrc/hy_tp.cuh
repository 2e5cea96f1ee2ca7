// hy_tp.cuh — tensor-parallel exchange kernels (sm_100a, one process per GPU).
//
// The tensor-parallel split of the decoder (heads and FFN columns per rank,
// o_proj and down row-parallel) needs two exchanges per layer: the residual
// stream after o_proj and after down is the sum over ranks of each rank's
// partial product.  The head is split by vocabulary rows, so the greedy token
// is the maximum over ranks of each rank's argmax key.
//
// Both exchanges are one-shot pushes over NVLink peer memory: every rank owns
// an exchange area (exported to its peers with CUDA IPC) and writes its
// contribution straight into every peer's area with plain stores, then
// raises a flag there; each rank waits for its peers' flags and reduces from
// its own area.  No TMA and no multicast: plain st/ld over the peer mapping.
//
// Sequencing.  A launch of the all-reduce uses CTAs 0..g-1; CTA c keeps its
// own counter seq[c] (the number of all-reduces it has taken part in), equal
// on every rank because every rank runs the same launches.  A collective with
// sequence number s uses buffer parity s & 1: the slot a rank writes for s was
// last read by its peer for s - 2, and the peer's flag for s - 1 (which the
// writer waited for) is only raised after that read.  Flags hold the full
// sequence number, so a flag is never mistaken for an older one.
//
// Every wait is bounded (%globaltimer, 2 s): a timeout sets the error word
// the host reads and the kernel returns.  Sums over ranks run in rank order,
// so every rank gets bit-identical results.
#pragma once
#include "hy_common.cuh"

namespace hyk {

constexpr int kTpMax = 8;        // ranks
constexpr int kTpMaxCtas = 64;   // CTAs of one all-reduce launch
constexpr int kTpThreads = 256;
constexpr int kTpSlice = 2048;   // floats per CTA of an all-reduce, until kTpMaxCtas CTAs are in use
constexpr unsigned long long kTpWaitNs = 2000000000ull;

// Byte layout of one rank's exchange area (cap floats per (parity, source)).
struct TpLayout {
    size_t recv_off, flag_off, key_off, kflag_off, seq_off, bytes;
};
__host__ __device__ inline TpLayout tp_layout(long long cap) {
    TpLayout l;
    l.recv_off = 0;
    l.flag_off = l.recv_off + (size_t)2 * kTpMax * cap * 4;
    l.key_off = l.flag_off + (size_t)2 * kTpMax * kTpMaxCtas * 4;
    l.kflag_off = l.key_off + (size_t)2 * kTpMax * 8;
    l.seq_off = l.kflag_off + (size_t)2 * kTpMax * 4;
    l.bytes = (l.seq_off + (size_t)(kTpMaxCtas + 1) * 4 + 255) & ~(size_t)255;
    return l;
}

struct TpArgs {
    uint8_t *area[kTpMax];  // every rank's exchange area (own one local, peers through IPC mappings)
    long long cap;          // floats per (parity, source) slot
    int rank, world;
    float *h;               // all-reduce: h[i] += sum over ranks of part[i], i < n
    const float *part;
    int n;                  // floats; n % 4 == 0
    int slice;              // floats per CTA (a multiple of 4)
    unsigned long long *key;  // argmax exchange: this rank's key in, the maximum over ranks out
    int *err;                 // set to 1 on a timed-out wait
};

__device__ __forceinline__ unsigned tp_ld_acquire_sys(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void tp_st_release_sys(unsigned *p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Thread 0..world-1 (except the own rank): wait until flag[src] == seq.
// Returns false (and raises the error word) on a timeout or a peer's error.
__device__ __forceinline__ bool tp_wait_flag(const unsigned *flag, unsigned seq, int *err) {
    if (tp_ld_acquire_sys(flag) == seq) return true;
    const unsigned long long t0 = gtimer();
    unsigned it = 0;
    while (tp_ld_acquire_sys(flag) != seq) {
        if ((++it & 255) == 0) {
            if (*(volatile int *)err) return false;
            if (gtimer() - t0 > kTpWaitNs) {
                atomicExch(err, 1);
                return false;
            }
        }
    }
    return true;
}

// h[i] += sum_q part_q[i] over the ranks q in order.  Grid: ceil(n / slice)
// CTAs (<= kTpMaxCtas) of kTpThreads.
__global__ void __launch_bounds__(kTpThreads) tp_allreduce_add(const __grid_constant__ TpArgs a) {
    __shared__ unsigned s_seq;
    __shared__ int s_bad;
    const int c = blockIdx.x, tid = threadIdx.x;
    const TpLayout L = tp_layout(a.cap);
    unsigned *my_seq = (unsigned *)(a.area[a.rank] + L.seq_off);
    if (tid == 0) {
        s_seq = my_seq[c] + 1;
        s_bad = 0;
    }
    __syncthreads();
    const unsigned seq = s_seq, par = seq & 1;
    const int i0 = c * a.slice, i1 = min(a.n, i0 + a.slice);
    // 1. this rank's slice into every peer's slot (par, rank)
    for (int p = 0; p < a.world; p++) {
        if (p == a.rank) continue;
        float *dst = (float *)(a.area[p] + L.recv_off) + ((size_t)par * kTpMax + a.rank) * a.cap;
        for (int i = i0 + tid * 4; i < i1; i += kTpThreads * 4)
            *(float4 *)(dst + i) = *(const float4 *)(a.part + i);
    }
    __syncthreads();
    // 2. publish: the stores above (every thread's, ordered by the barrier) before the flags
    if (tid == 0) {
        asm volatile("fence.acq_rel.sys;" ::: "memory");
        for (int p = 0; p < a.world; p++)
            if (p != a.rank)
                tp_st_release_sys((unsigned *)(a.area[p] + L.flag_off) + ((size_t)par * kTpMax + a.rank) * kTpMaxCtas + c,
                                  seq);
    }
    // 3. the peers' slices of this CTA
    if (tid < a.world && tid != a.rank) {
        const unsigned *f = (const unsigned *)(a.area[a.rank] + L.flag_off) + ((size_t)par * kTpMax + tid) * kTpMaxCtas + c;
        if (!tp_wait_flag(f, seq, a.err)) s_bad = 1;
    }
    __syncthreads();
    if (s_bad) return;
    // 4. reduce in rank order (L2 loads: peers wrote this memory over NVLink)
    const float *recv = (const float *)(a.area[a.rank] + L.recv_off) + (size_t)par * kTpMax * a.cap;
    for (int i = i0 + tid * 4; i < i1; i += kTpThreads * 4) {
        float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int q = 0; q < a.world; q++) {
            const float4 v = q == a.rank ? *(const float4 *)(a.part + i) : __ldcg((const float4 *)(recv + (size_t)q * a.cap + i));
            s.x += v.x;
            s.y += v.y;
            s.z += v.z;
            s.w += v.w;
        }
        float4 hv = *(float4 *)(a.h + i);
        hv.x += s.x;
        hv.y += s.y;
        hv.z += s.z;
        hv.w += s.w;
        *(float4 *)(a.h + i) = hv;
    }
    if (tid == 0) my_seq[c] = seq;
}

// *key = max over ranks of each rank's key (one warp).
__global__ void __launch_bounds__(32) tp_argmax_exchange(const __grid_constant__ TpArgs a) {
    const int lane = threadIdx.x;
    const TpLayout L = tp_layout(a.cap);
    unsigned *my_seq = (unsigned *)(a.area[a.rank] + L.seq_off) + kTpMaxCtas;
    const unsigned seq = *my_seq + 1, par = seq & 1;
    const unsigned long long mine = *a.key;
    if (lane < a.world && lane != a.rank) {
        unsigned long long *dst = (unsigned long long *)(a.area[lane] + L.key_off) + (size_t)par * kTpMax + a.rank;
        asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(dst), "l"(mine) : "memory");
        asm volatile("fence.acq_rel.sys;" ::: "memory");
        tp_st_release_sys((unsigned *)(a.area[lane] + L.kflag_off) + (size_t)par * kTpMax + a.rank, seq);
    }
    unsigned long long k = 0;
    int bad = 0;
    if (lane < a.world && lane != a.rank) {
        const unsigned *f = (const unsigned *)(a.area[a.rank] + L.kflag_off) + (size_t)par * kTpMax + lane;
        if (tp_wait_flag(f, seq, a.err)) {
            const unsigned long long *src = (const unsigned long long *)(a.area[a.rank] + L.key_off) + (size_t)par * kTpMax + lane;
            asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(k) : "l"(src) : "memory");
        } else {
            bad = 1;
        }
    } else if (lane == a.rank) {
        k = mine;
    }
    if (__any_sync(0xffffffffu, bad)) return;
    // the maximum over lanes (keys are unsigned and larger wins)
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, k, o);
        k = other > k ? other : k;
    }
    __syncwarp();
    if (lane == 0) {
        *a.key = k;
        *my_seq = seq;
    }
}

}  // namespace hyk
