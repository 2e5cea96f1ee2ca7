// hy_common.cuh — shared device helpers for the hymt2 sm_100a backend.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/hy_device_abi.h"

namespace hyk {

// Device weight layouts (chosen at upload; see hy_backend.cu):
//   PANEL  n x nb x 64 B of 2-bit codes (host panel order) + float scale [n*nb]
//   Q4K    native 144-byte blocks, rows of nb*144 B
//   Q6K    per row: ql[nb*128] | qh[nb*64] | scales[nb*16] | d f16[nb] padded to 16 B
//   Q80    per row: qs[k] int8 | d f16[k/32] padded to 16 B
//   F16    native half rows;  F32 native float rows
enum Fmt { FMT_PANEL = 0, FMT_Q4K = 1, FMT_Q6K = 2, FMT_Q80 = 3, FMT_F16 = 4, FMT_F32 = 5 };

// How a GEMV launch builds its activation in shared memory.
enum ActMode {
    ACT_Q8K = 0,   // copy host-made q8k_block[nt][nb] from global memory
    ACT_VEC = 1,   // quantise x[t*ldx + i]
    ACT_NORM = 2,  // quantise rmsnorm(x[t]) * norm_w
    ACT_SILU = 3,  // quantise silu(x[t]) * x2[t]
};

// What happens to each output row.
// EPI_SILU: interleaved gate|up pair -> w[0].out[row] = silu(gate) * up.
enum Epi { EPI_STORE = 0, EPI_ADD = 1, EPI_ARGMAX = 2, EPI_SILU = 3 };

constexpr int kPieceOrder[4] = {0, 2, 1, 3};

__device__ __forceinline__ int piece_of_chunk(int ch) { return ch == 1 ? 2 : (ch == 2 ? 1 : ch); }

// Programmatic dependent launch: wait for the previous kernel in the stream
// (its memory becomes visible) / allow the next one to start its prologue.
// Both are no-ops when the launch did not opt into PDL.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ int warp_sum_i(int v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__device__ __forceinline__ int dp4a(int a, int b, int c) { return __dp4a(a, b, c); }

// Byte i (0..15) of a 16-byte register vector.  Selecting the word and
// shifting keeps the vector in registers; indexing it as a byte array with a
// lane-dependent index would place it in local memory.
__device__ __forceinline__ uint32_t u4_byte(const uint4 &v, int i) {
    const int ws = i >> 2;
    const uint32_t w = ws == 0 ? v.x : (ws == 1 ? v.y : (ws == 2 ? v.z : v.w));
    return (w >> (8 * (i & 3))) & 0xffu;
}

__device__ __forceinline__ float bf16_bits_to_f32(uint32_t h16) { return __uint_as_float(h16 << 16); }

// Round-to-nearest-even fp32 -> bf16 bits, identical to the host's integer
// formula (reference src/kernels.c:107-111), NaN included.
__device__ __forceinline__ uint16_t f32_to_bf16_bits(float f) {
    const uint32_t u = __float_as_uint(f);
    return (uint16_t)((u + 0x7fffu + ((u >> 16) & 1u)) >> 16);
}

__device__ __forceinline__ float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }

// 16-byte streaming load of weights (read-only, not kept in L1).
__device__ __forceinline__ uint4 ldg_stream(const void *p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

__device__ __forceinline__ unsigned long long gtimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

// Optional per-kernel timeline, compiled in only with -DHYK_TRACE (the
// measurement build; the product library has none of it): slot s holds
// [launch of CTA 0, CTA 0 past griddepcontrol.wait, CTA 0 past its prologue,
// last CTA end] in %globaltimer nanoseconds.  Slot < 0 disables recording.
constexpr int kTraceSlots = 1024;
#ifdef HYK_TRACE
__device__ unsigned long long g_trace[kTraceSlots][4];
__device__ unsigned long long g_trace2[kTraceSlots][4];  // sub-phases of CTA 0
__device__ unsigned long long g_trace3[kTraceSlots][4];  // CTA 0: clock64 and globaltimer at wait / end

__device__ __forceinline__ void trace_mark(int slot, int which) {
    if (slot >= 0 && slot < kTraceSlots && threadIdx.x == 0) {
        const unsigned long long t = gtimer();
        if (which == 3) atomicMax(&g_trace[slot][3], t);
        else if (blockIdx.x == 0 && blockIdx.y == 0) g_trace[slot][which] = t;
        if (blockIdx.x == 0 && blockIdx.y == 0 && (which == 1 || which == 3)) {
            g_trace3[slot][which == 1 ? 0 : 2] = clock64();
            g_trace3[slot][which == 1 ? 1 : 3] = t;
        }
    }
}

__device__ __forceinline__ void trace_sub(int slot, int which) {
    if (slot >= 0 && slot < kTraceSlots && threadIdx.x == 0 && blockIdx.x == 0 && blockIdx.y == 0)
        g_trace2[slot][which] = gtimer();
}
#else
__device__ __forceinline__ void trace_mark(int, int) {}
__device__ __forceinline__ void trace_sub(int, int) {}
#endif

// Monotone 64-bit argmax key: larger value wins, equal values -> smaller index
// wins (the host loop keeps the first maximum with a strict '>').  NaN never
// wins (ranked as -inf).
__device__ __forceinline__ unsigned long long argmax_key(float v, uint32_t idx) {
    if (v != v) v = -INFINITY;
    uint32_t u = __float_as_uint(v);
    u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((unsigned long long)u << 32) | (unsigned long long)(0xffffffffu - idx);
}
__device__ __forceinline__ uint32_t argmax_index(unsigned long long key) {
    return 0xffffffffu - (uint32_t)(key & 0xffffffffull);
}

// Descriptor of one device weight, passed by value in kernel arguments.
struct WDesc {
    const uint8_t *w;   // device bytes in the format's layout
    const float *s;     // PANEL: per-block fp32 scales [n*nb]
    float *out;         // EPI_STORE / EPI_ADD target: out[t*ld + row]
    long long stride;   // bytes per row in `w`
    int fmt, n, k, shift, off, ld;
};

// 16-byte asynchronous global -> shared copy (L2 only), one commit group per caller.
__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    const unsigned d = (unsigned)__cvta_generic_to_shared(dst);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d), "l"(src) : "memory");
}

}  // namespace hyk
