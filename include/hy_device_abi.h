/* hy_device_abi.h — binary layouts shared with the hymt2 host library.
 *
 * The hymt2 host (model loader, generation loop, device dispatcher) talks to an
 * accelerator through one vtable of plain C function pointers.  A CUDA backend
 * that wants to be a drop-in for `HYMT2_DEVICE=cuda` must therefore agree with
 * the host on the exact byte layout of every struct that crosses that vtable.
 * This header restates those layouts; field order, types and alignment are
 * fixed by the host and must not be changed here:
 *
 *   q8k_block       — reference src/internal.h:34-41 (576 B, 64-B aligned)
 *   weight_t        — reference src/internal.h:48-61
 *   GT_* type ids   — reference src/internal.h:46
 *   hy_fused_layer  — reference src/device.h:44-47
 *   hy_fused_args   — reference src/device.h:49-59
 *   hy_device_ops   — reference src/device.h:70-79
 *
 * Only these layouts are shared.  Everything behind the vtable (device memory
 * layout, kernels, graphs) is this library's own.
 */
#ifndef HY_DEVICE_ABI_H
#define HY_DEVICE_ABI_H

#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#ifndef QK_K
#define QK_K 256
#endif
/* Largest token count the host passes to one fused_forward / matmul call
 * (reference src/internal.h:12). */
#ifndef MAX_BATCH
#define MAX_BATCH 16
#endif

/* Q8_K activation block: 256 int8 codes for one 256-wide slice of an fp32
 * activation row.  `qp` is a lane-major copy of `qs` (piece order 0,2,1,3 per
 * lane, see reference src/internal.h:26-33); `qs` is natural order. */
#if defined(__CUDACC__) || defined(__GNUC__)
#define HY_ABI_ALIGN64 __attribute__((aligned(64)))
#else
#define HY_ABI_ALIGN64
#endif
typedef struct HY_ABI_ALIGN64 {
    int8_t qp[QK_K];
    float d;
    int32_t sum;
    int16_t bsums[QK_K / 16];
    uint8_t _pad[64 - 8 - 32];
    int8_t qs[QK_K];
} q8k_block;

/* ggml type numbers accepted by the host (reference src/internal.h:46). */
enum {
    GT_F32 = 0,
    GT_F16 = 1,
    GT_Q8_0 = 8,
    GT_Q4_K = 12,
    GT_Q6_K = 14,
    GT_Q2_0C = 40,
    GT_STQ1_0 = 43,
    GT_UNSUPPORTED = -1
};

/* One weight matrix as the host holds it: `n` rows of `k` inputs, row-major,
 * `row_bytes` per row of the native GGUF encoding.  For STQ1_0 / Q2_0C the host
 * has also built the "panel" form: `pk` = n*(k/256) blocks of 64 B of 2-bit
 * codes, `ps` = one fp32 scale per block, and the per-block result is
 * ps * y.d * ((enc << pshift) - poff * y.sum). */
typedef struct {
    const uint8_t *data;
    int type;
    int k;
    int n;
    size_t row_bytes;
    const uint8_t *pk;
    const float *ps;
    int pshift, poff;
    void *gpu;
} weight_t;

typedef struct hy_device hy_device;     /* host-side wrapper, opaque here */
typedef struct hy_dweight hy_dweight;   /* device weight handle, owned by the backend */

typedef enum {
    HY_DEV_NONE = 0,
    HY_DEV_VULKAN = 1,
    HY_DEV_CUDA = 2,
    HY_DEV_METAL = 3,
    HY_DEV_NPU = 4
} hy_dev_kind;

typedef struct hy_fused_layer {
    hy_dweight *wq, *wk, *wv, *wo, *wg, *wu, *wd;
    const float *attn_norm, *ffn_norm, *q_norm, *k_norm;
} hy_fused_layer;

typedef struct hy_fused_args {
    int n_layer, hidden, ffn, heads, kv_heads, hdim, qdim, kvdim, ctx, rope_half, nt, pos0;
    float eps;
    int want_logits;
    hy_fused_layer *layers;
    hy_dweight *outw;
    const float *out_norm;
    const float *rope_cos, *rope_sin; /* [ctx * rope_half] */
    float *h;      /* in/out [nt * hidden], host memory, already embedded */
    float *logits; /* out [outw rows] when want_logits */
} hy_fused_args;

typedef struct hy_device_ops {
    void (*destroy_impl)(void *impl);
    hy_dweight *(*upload)(void *impl, const weight_t *w);
    void (*release)(hy_dweight *w);
    bool (*matmul)(void *impl, hy_dweight *const *ws, float *const *outs, int cnt, const q8k_block *xq, int nt);
    bool (*is_software)(const void *impl);
    float *(*weight_out)(hy_dweight *w);
    bool (*fused_prepare)(void *impl, const hy_fused_args *shape);
    bool (*fused_forward)(void *impl, hy_fused_args *a);
} hy_device_ops;

#ifdef __cplusplus
}
#endif
#endif
