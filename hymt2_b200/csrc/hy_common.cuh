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
//   STQN   native STQ1_0, 42 B per 256 weights, per row: qs[nb*32] | sign[nb*8] |
//          d f16[nb] padded to 16 B (chunk order and sign bits: stq_decode_unit)
//   Q4K    native 144-byte blocks, rows of nb*144 B
//   Q6K    per row: ql[nb*128] | qh[nb*64] | scales[nb*16] | d f16[nb] padded to 16 B
//   Q80    per row: qs[k] int8 | d f16[k/32] padded to 16 B
//   F16    native half rows;  F32 native float rows
enum Fmt { FMT_PANEL = 0, FMT_Q4K = 1, FMT_Q6K = 2, FMT_Q80 = 3, FMT_F16 = 4, FMT_F32 = 5, FMT_STQN = 6 };

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

// ---------------------------------------------------------------- STQ1_0 patterns

// The STQ1_0 pattern table, a constant of the file format (reference
// src/kernels.c:178-181): entry (sign << 4) | slot holds four 2-bit codes,
// code - 1 in {-1, 0, +1}, lane l at bits 2l .. 2l+1, exactly one zero.
struct StqPatterns { uint8_t v[32]; };
constexpr StqPatterns kStqPatterns = {{
    0xA9, 0x89, 0x29, 0x09, 0xA6, 0x86, 0x26, 0x06, 0x9A, 0x92, 0x1A, 0x12, 0x6A, 0x62, 0x4A, 0x42,
    0x01, 0x21, 0x81, 0xA1, 0x04, 0x24, 0x84, 0xA4, 0x10, 0x18, 0x90, 0x98, 0x40, 0x48, 0x60, 0x68,
}};
// Entries 4m .. 4m+3 as one little-endian word.
__host__ __device__ constexpr uint32_t stq_word(int m) {
    return (uint32_t)kStqPatterns.v[4 * m] | ((uint32_t)kStqPatterns.v[4 * m + 1] << 8) |
           ((uint32_t)kStqPatterns.v[4 * m + 2] << 16) | ((uint32_t)kStqPatterns.v[4 * m + 3] << 24);
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}

// Patterns of four groups at once, from registers (no table memory): nibble i
// of `slots` (bits 0..15; higher bits ignored) is group i's 4-bit slot, and
// bit 2 of nibble i of `sel_sign` its sign, the other bits of sel_sign being
// 0x3210.  Byte permutes over the table words: the slot's low 3 bits pick a
// byte of each 8-entry quarter, its bit 3 picks the quarter within a sign
// half, the sign picks the half.  Byte i of the result = group i's pattern.
__device__ __forceinline__ uint32_t stq_decode_quad(uint32_t slots, uint32_t sel_sign) {
    const uint32_t s1 = slots & 0x7777u;
    const uint32_t q0 = prmt(stq_word(0), stq_word(1), s1), q1 = prmt(stq_word(2), stq_word(3), s1);
    const uint32_t q2 = prmt(stq_word(4), stq_word(5), s1), q3 = prmt(stq_word(6), stq_word(7), s1);
    const uint32_t s2 = ((slots >> 1) & 0x4444u) | 0x3210u;
    return prmt(prmt(q0, q1, s2), prmt(q2, q3, s2), sel_sign);
}

// One pattern: (sign << 4) | slot -> its byte.
__device__ __forceinline__ uint32_t stq_pattern(int idx) {
    return stq_decode_quad((uint32_t)(idx & 15), 0x3210u | (uint32_t)((idx >> 4) & 1) << 2) & 0xffu;
}

// One 64-weight unit of a native row (see FMT_STQN): the 16 slots of one
// 16-group chunk of a block (8 qs bytes, group m at nibble m) and its 16 sign
// bits stored bit-sliced (bit 4i + j = sign of group 4j + i).  Returns the
// unit's patterns as a 16-byte panel chunk: word j, byte i = group 4j + i.
__device__ __forceinline__ uint4 stq_decode_unit(uint2 qs, uint32_t sg) {
    uint4 w;
    w.x = stq_decode_quad(qs.x, ((sg << 2) & 0x4444u) | 0x3210u);
    w.y = stq_decode_quad(qs.x >> 16, ((sg << 1) & 0x4444u) | 0x3210u);
    w.z = stq_decode_quad(qs.y, (sg & 0x4444u) | 0x3210u);
    w.w = stq_decode_quad(qs.y >> 16, ((sg >> 1) & 0x4444u) | 0x3210u);
    return w;
}

// Bit-sliced form of a chunk's 16 natural sign bits (bit m = group m):
// bit 4i + j <- bit 4j + i (a 4 x 4 bit transpose).
__host__ __device__ inline uint32_t stq_slice_signs(uint32_t s) {
    uint32_t o = 0;
    for (int i = 0; i < 4; i++)
        for (int j = 0; j < 4; j++) o |= ((s >> (4 * j + i)) & 1u) << (4 * i + j);
    return o;
}

// 16-byte streaming load of weights (read-only, not kept in L1).
__device__ __forceinline__ uint4 ldg_stream(const void *p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}
__device__ __forceinline__ uint2 ldg_stream8(const void *p) {
    uint2 r;
    asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(p));
    return r;
}
__device__ __forceinline__ uint32_t ldg_stream16(const void *p) {
    unsigned short r;
    asm volatile("ld.global.nc.L1::no_allocate.u16 %0, [%1];" : "=h"(r) : "l"(p));
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
