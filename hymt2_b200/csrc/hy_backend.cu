// hy_backend.cu — the hymt2 device backend for B200 (sm_100a).
//
// Implements the host's hy_device_ops vtable (reference src/device.h:70-79)
// and the additive decode API of include/hymt2_cuda.h.  Everything the host
// hands over is resident in HBM after upload/fused_prepare; a decode step is
// one CUDA graph of programmatic-dependent launches:
//   embed -> L x [qkv GEMV | attention | o_proj GEMV (+residual) |
//                 gate/up GEMV | down GEMV (SiLU*up prologue, +residual)]
//         -> LM-head GEMV with fused argmax -> token feedback
// and never synchronises with the host.  For panel models with a Q6_K head
// the decode loop can instead run as one persistent cooperative kernel for
// any number of steps (hy_mega.cuh), bit-identical to the graph.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <algorithm>
#include <atomic>
#include <chrono>
#include <cstring>
#include <mutex>
#include <vector>

#include "../../include/hymt2_cuda.h"
#include "hy_attn.cuh"
#include "hy_gemv.cuh"
#include "hy_mega.cuh"
#include "hy_misc.cuh"
#include "hy_tc.cuh"
#include "hy_tp.cuh"

using namespace hyk;

// Provided by the host's device layer (reference src/device.c:25) when this
// backend is linked into the host library; absent in the standalone .so.
extern "C" hy_device *hy_device_wrap(hy_dev_kind kind, const char *name, void *impl, const hy_device_ops *ops,
                                     bool software) __attribute__((weak));

namespace {

constexpr int kMaxChunk = 256;     // tokens per device prefill / forward chunk
constexpr int kSplitLen = kDecSplit;  // keys per decode attention split
constexpr size_t kMaxDynSmem = 200 * 1024;

struct HyCtx;

struct HyWeight {
    int gtype, fmt, n, k, nb, shift, off;
    uint8_t *w;
    float *s;
    long long stride;
    float *d_out;   // matmul op output [MAX_BATCH][n] (lazy)
    float *h_out;   // pinned alias returned by weight_out (lazy)
    HyCtx *c;
    int8_t *tc_w;   // tensor-core tiles of a panel weight (lazy, hy_tc.cuh layout)
    float *tc_ws;   // their block scales
    int8_t *tc_w64; // the tiles 64-row slices first (lazy: launches of 64-row slices of wider tiles)
};

struct Layer {
    HyWeight *q, *k, *v, *o, *g, *u, *d;
    float *attn_norm, *ffn_norm, *q_norm, *k_norm;  // device
};

struct Graph {
    cudaGraphExec_t exec = nullptr;
    long long kernels = 0;
};

struct Batch;

struct HyCtx {
    int dev = 0;
    cudaStream_t st = nullptr;
    int nsm = 148;
    bool broken = false;
    char err[256] = {0};
    long long launches = 0;
    long long capture_kernels = 0;
    // matmul-op staging
    q8k_block *d_xq = nullptr;
    size_t xq_cap = 0;
    float *d_x32 = nullptr;
    size_t x32_cap = 0;
    int32_t *d_ints = nullptr;
    size_t ints_cap = 0;
    // fused model state
    bool fused = false;
    int L = 0, H = 0, F = 0, heads = 0, kvh = 0, hd = 0, qd = 0, kvd = 0, ctx = 0, half = 0;
    float eps = 0.f;
    std::vector<Layer> layers;
    float *d_norms = nullptr;
    HyWeight *outw = nullptr, *embd = nullptr;
    float *d_out_norm = nullptr, *d_cos = nullptr, *d_sin = nullptr;
    uint16_t *d_kv = nullptr;
    float *d_h = nullptr, *d_qkv = nullptr, *d_ao = nullptr, *d_g = nullptr, *d_u = nullptr, *d_logits = nullptr;
    float *d_part = nullptr;
    float *d_cpart = nullptr;       // wide decode attention partials [heads][max_chunks][hd+2]
    int max_chunks = 0;
    int *d_tickets = nullptr;
    int max_splits = 0;
    DecodeState *d_state = nullptr;
    int *d_out_ids = nullptr, *d_tokens = nullptr, *d_chunk_pos = nullptr;
    float *d_tmp_h() { return d_h + (size_t)(kMaxChunk - 1) * H; }  // scratch row for timing runs
    int *h_pinned_int = nullptr;  // small pinned staging: [0] forward position, [2..1001] rewind ring
    unsigned rewind_slot = 0;
    int vocab_out = 0;
    Graph g_fwd1, g_fwd1_logits, g_dec;
    int g_dec_vocab = -1;
    bool trace_on = false;  // assign timeline slots to launches (debug)
    int trace_next = 0;
    // persistent decode kernel
    int decode_mode = 0;            // 0: persistent kernel when supported, 1: graph of per-layer launches
    int *host_io = nullptr;         // device view of the resident host loop's words (hyc_decode_resident)
    unsigned long long host_limit_ns = 0;
    int mega_state = -1;            // -1 unchecked, 0 unsupported, 1 ready
    char mega_why[128] = {0};       // why unsupported
    MegaLayer *d_mega_layers = nullptr;
    MegaSync *d_mega_sync = nullptr;
    unsigned long long *d_tl = nullptr;
    int tl_cap = 0;
    MegaPlan mega_plan_v{};
    // STQ1_0 weights: panels (default) or the native 42 B / 256 layout
    // (FMT_STQN), from HYMT2_STQ_LAYOUT=native or hyc_set_stq_layout
    bool stq_native = false;
    // tensor-core path for multi-token chunks (hy_tc.cuh)
    bool tc_on = true;
    int max_tokens = kMaxChunk;     // tokens per forward pass (the batch engine raises it)
    int8_t *d_tca = nullptr;        // tiled Q8_K codes of up to max_tokens tokens
    float *d_tcad = nullptr;        // their block scales
    int *d_tcerr = nullptr;         // set by tc_gemm on a bounded-wait timeout
    size_t tca_bytes = 0;
    size_t l2_bytes = 0;
    void *mega_kernel = nullptr;
    Batch *bat = nullptr;           // ragged multi-sequence batches (hy_batch.cuh)
    // weight upload: a pinned staging ring (the host's mmap'd GGUF bytes are copied through it, so
    // every device copy is an asynchronous DMA from pinned memory) and a reusable buffer for the raw
    // bytes the device repacks
    uint8_t *h_stage[2] = {nullptr, nullptr};
    cudaEvent_t stage_ev[2] = {nullptr, nullptr};
    uint8_t *d_raw = nullptr;
    size_t raw_cap = 0;
    // tensor parallelism: this handle holds one rank's share of a split model (hy_tp.cuh)
    int tp_rank = 0, tp_world = 1, tp_vocab0 = 0;
    bool tp_on = false;             // connected to its peers: o_proj / down / head exchange
    uint8_t *d_tp_area = nullptr;   // own exchange area, exported to the peers
    float *d_tp_part = nullptr;     // partial o_proj / down products [kMaxChunk][H]
    int *d_tp_err = nullptr;
    long long tp_cap = 0;
    TpArgs tp{};
};

int trace_slot(HyCtx *c) { return c->trace_on && c->trace_next < kTraceSlots ? c->trace_next++ : -1; }

bool fail(HyCtx *c, const char *what, cudaError_t e) {
    c->broken = true;
    snprintf(c->err, sizeof c->err, "%s: %s", what, e == cudaSuccess ? "invalid request" : cudaGetErrorString(e));
    return false;
}
#define CK(c, call)                                          \
    do {                                                     \
        cudaError_t _e = (call);                             \
        if (_e != cudaSuccess) return fail((c), #call, _e); \
    } while (0)
#define REQ(c, cond, msg)                                             \
    do {                                                              \
        if (!(cond)) {                                                \
            snprintf((c)->err, sizeof (c)->err, "%s", (msg));          \
            return false;                                             \
        }                                                             \
    } while (0)

// All host<->device copies go through the handle's stream: a plain cudaMemcpy
// from pageable memory may return before its DMA lands, and the stream is
// non-blocking, so only stream order makes the data visible to our kernels.
cudaError_t h2d(HyCtx *c, void *dst, const void *src, size_t bytes) {
    return cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, c->st);
}
cudaError_t d2h(HyCtx *c, void *dst, const void *src, size_t bytes) {
    cudaError_t e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, c->st);
    return e == cudaSuccess ? cudaStreamSynchronize(c->st) : e;
}

// Host bytes (pageable, e.g. the mmap'd GGUF) -> device, through two pinned
// staging slots: the host copy of one chunk overlaps the DMA of the previous
// one.  Returns when every copy is enqueued; stream order makes them visible.
constexpr size_t kStageBytes = 16u << 20;
cudaError_t h2d_staged(HyCtx *c, void *dst, const void *src, size_t bytes) {
    if (!c->h_stage[0]) {
        for (int i = 0; i < 2; i++) {
            cudaError_t e = cudaHostAlloc((void **)&c->h_stage[i], kStageBytes, cudaHostAllocDefault);
            if (e == cudaSuccess) e = cudaEventCreateWithFlags(&c->stage_ev[i], cudaEventDisableTiming);
            if (e != cudaSuccess) return e;
        }
    }
    size_t o = 0;
    for (int i = 0; o < bytes; i++, o += kStageBytes) {
        const int k = i & 1;
        const size_t n = bytes - o < kStageBytes ? bytes - o : kStageBytes;
        cudaError_t e = cudaEventSynchronize(c->stage_ev[k]);  // the slot's previous DMA is done
        if (e != cudaSuccess) return e;
        memcpy(c->h_stage[k], (const uint8_t *)src + o, n);
        e = cudaMemcpyAsync((uint8_t *)dst + o, c->h_stage[k], n, cudaMemcpyHostToDevice, c->st);
        if (e == cudaSuccess) e = cudaEventRecord(c->stage_ev[k], c->st);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

// The reusable device buffer for raw bytes the device repacks (grown as needed).
uint8_t *raw_buf(HyCtx *c, size_t bytes) {
    if (bytes > c->raw_cap) {
        if (c->d_raw) {
            cudaStreamSynchronize(c->st);
            cudaFree(c->d_raw);
        }
        c->d_raw = nullptr;
        c->raw_cap = 0;
        if (cudaMalloc(&c->d_raw, bytes) != cudaSuccess) return nullptr;
        c->raw_cap = bytes;
    }
    return c->d_raw;
}

template <typename... KArgs, typename... Args>
bool launch(HyCtx *c, void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, bool pdl, Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = c->st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
    if (e != cudaSuccess) {
        fail(c, "kernel launch", e);
        if (e == cudaErrorLaunchOutOfResources) {  // say which limit
            cudaFuncAttributes fa;
            int optin = 0;
            cudaFuncGetAttributes(&fa, (const void *)kern);
            cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, c->dev);
            const size_t used = strlen(c->err);
            snprintf(c->err + used, sizeof c->err - used,
                     " (block %u, dyn smem %zu of max %d, static %zu, opt-in %d, regs %d, max threads %d)",
                     block.x * block.y * block.z, smem, fa.maxDynamicSharedSizeBytes, fa.sharedSizeBytes, optin,
                     fa.numRegs, fa.maxThreadsPerBlock);
        }
        return false;
    }
    c->launches++;
    c->capture_kernels++;
    return true;
}

template <typename... KArgs, typename... Args>
cudaError_t cudaLaunchKernelEx_compat(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                                      Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cfg.numAttrs = 0;
    return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

WDesc desc(const HyWeight *w, float *out, int ld) {
    WDesc d;
    d.w = w->w;
    d.s = w->s;
    d.out = out;
    d.stride = w->stride;
    d.fmt = w->fmt;
    d.n = w->n;
    d.k = w->k;
    d.shift = w->shift;
    d.off = w->off;
    d.ld = ld;
    return d;
}

bool is_q8_fmt(int fmt) { return fmt == FMT_PANEL || fmt == FMT_STQN || fmt == FMT_Q4K || fmt == FMT_Q6K; }

// ---------------------------------------------------------------- GEMV dispatch

template <typename K>
void set_smem(K kern, size_t bytes = kMaxDynSmem) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
}

void init_kernel_attrs_current();

// Dynamic shared-memory limits are a per-device property of each kernel:
// raise them once for every device this process uses, with that device
// current (hyc_create, and the first allocation-free call on a device).
constexpr int kMaxDevices = 128;
std::mutex g_attr_mu;
bool g_attr_done[kMaxDevices] = {false};

bool init_kernel_attrs(int dev) {
    if (dev < 0 || dev >= kMaxDevices) return false;
    std::lock_guard<std::mutex> lock(g_attr_mu);
    if (g_attr_done[dev]) return true;
    init_kernel_attrs_current();
    g_attr_done[dev] = cudaGetLastError() == cudaSuccess;
    return g_attr_done[dev];
}

void init_kernel_attrs_current() {
    set_smem(gemv_panel_nt1<1>);
    set_smem(gemv_panel_nt1<2>);
    set_smem(gemv_panel_nt1<3>);
    set_smem(gemv_panel_nt1<4>);
    set_smem(gemv_panel_nt<4>);
    set_smem(gemv_panel_nt<16>);
    set_smem(gemv_panel_nt1<1, FMT_STQN>);
    set_smem(gemv_panel_nt1<2, FMT_STQN>);
    set_smem(gemv_panel_nt1<3, FMT_STQN>);
    set_smem(gemv_panel_nt1<4, FMT_STQN>);
    set_smem(gemv_panel_nt<4, FMT_STQN>);
    set_smem(gemv_panel_nt<16, FMT_STQN>);
    set_smem(gemv_panel_dec<1, FMT_STQN>);
    set_smem(gemv_panel_dec<2, FMT_STQN>);
    set_smem(gemv_panel_dec<3, FMT_STQN>);
    set_smem(gemv_panel_dec<4, FMT_STQN>);
    set_smem(gemv_q6k<1>);
    set_smem(gemv_q6k<4>);
    set_smem(gemv_q6k<16>);
    set_smem(gemv_q4k<1>);
    set_smem(gemv_q4k<4>);
    set_smem(gemv_q4k<16>);
    set_smem(gemv_fp<FMT_Q80, 1>);
    set_smem(gemv_fp<FMT_Q80, 4>);
    set_smem(gemv_fp<FMT_F16, 1>);
    set_smem(gemv_fp<FMT_F16, 4>);
    set_smem(gemv_fp<FMT_F32, 1>);
    set_smem(gemv_fp<FMT_F32, 4>);
    set_smem(gemv_panel_dec<1>);
    set_smem(gemv_panel_dec<2>);
    set_smem(gemv_panel_dec<3>);
    set_smem(gemv_panel_dec<4>);
    set_smem(attn_decode2<128, 1>);
    set_smem(attn_decode2<128, 2>);
    set_smem(attn_decode2<128, 4>);
    set_smem(attn_decode2<128, 8>);
    set_smem(attn_decode2<64, 1>);
    set_smem(attn_decode2<64, 2>);
    set_smem(attn_decode2<64, 4>);
    set_smem(attn_decode2<64, 8>);
    set_smem(attn_chunk_kernel<128, 1>);
    set_smem(attn_chunk_kernel<128, 2>);
    set_smem(attn_chunk_kernel<128, 4>);
    set_smem(attn_chunk_kernel<128, 8>);
    set_smem(attn_chunk_kernel<64, 1>);
    set_smem(attn_chunk_kernel<64, 2>);
    set_smem(attn_chunk_kernel<64, 4>);
    set_smem(attn_chunk_kernel<64, 8>);
    set_smem(attn_fa<128, 1>, fa_smem<128, 1>());
    set_smem(attn_fa<128, 2>, fa_smem<128, 2>());
    set_smem(attn_fa<128, 4>, fa_smem<128, 4>());
    set_smem(attn_fa<128, 8>, fa_smem<128, 8>());
    set_smem(attn_fa<64, 1>, fa_smem<64, 1>());
    set_smem(attn_fa<64, 2>, fa_smem<64, 2>());
    set_smem(attn_fa<64, 4>, fa_smem<64, 4>());
    set_smem(attn_fa<64, 8>, fa_smem<64, 8>());
    set_smem(tc_gemm<1, 256>, tc_smem_bytes(1, 256));
    set_smem(tc_gemm<1, 64>, tc_smem_bytes(1, 64));
    set_smem(tc_gemm<2, 128>, tc_smem_bytes(2, 128));
    set_smem(tc_gemm<2, 64>, tc_smem_bytes(2, 64));
    set_smem(tc_gemm<3, 64>, tc_smem_bytes(3, 64));
    set_smem(tc_gemm<1, 256, true>, tc_smem_bytes(1, 256));
    set_smem(tc_gemm<1, 64, true>, tc_smem_bytes(1, 64));
    set_smem(tc_gemm<2, 128, true>, tc_smem_bytes(2, 128));
    set_smem(tc_gemm<2, 64, true>, tc_smem_bytes(2, 64));
    set_smem(tc_gemm<3, 64, true>, tc_smem_bytes(3, 64));
}

// One launch for nt <= NT tokens.
bool gemv_launch(HyCtx *c, const GemvArgs &a_in, bool pdl, int ctas_per_sm) {
    GemvArgs a = a_in;
    a.trace = trace_slot(c);
    const int fmt = a.w[0].fmt;
    int grid = (a.rows_total + kGemvWarps - 1) / kGemvWarps;
    if (grid > c->nsm * ctas_per_sm) grid = c->nsm * ctas_per_sm;
    const dim3 blk(kGemvThreads);
    if (is_q8_fmt(fmt)) {
        const int NT = a.nt == 1 ? 1 : (a.nt <= 4 ? 4 : 16);
        const size_t smem = q8_smem_bytes(NT, a.k);
        if (fmt == FMT_PANEL) {
            const int cpl = (a.k + 2047) / 2048;
            if (NT == 1 && cpl <= 4 && a.epi != EPI_ARGMAX) {
                // whole weight slice of each CTA staged in shared memory
                // row slices in multiples of 4 (the kernel's row groups; keeps
                // interleaved gate/up pairs inside one warp)
                const int rpc = ((a.rows_total + grid - 1) / grid + 3) & ~3;
                const size_t sm = panel_dec_smem(rpc, a.k);
                if (sm <= kMaxDynSmem) {
                    switch (cpl) {
                    case 1: return launch(c, gemv_panel_dec<1>, grid, blk, sm, pdl, a, rpc);
                    case 2: return launch(c, gemv_panel_dec<2>, grid, blk, sm, pdl, a, rpc);
                    case 3: return launch(c, gemv_panel_dec<3>, grid, blk, sm, pdl, a, rpc);
                    default: return launch(c, gemv_panel_dec<4>, grid, blk, sm, pdl, a, rpc);
                    }
                }
            }
            REQ(c, a.epi != EPI_SILU, "interleaved gate|up pair needs the staged decode GEMV");
            if (NT == 1 && cpl <= 4) {
                switch (cpl) {
                case 1: return launch(c, gemv_panel_nt1<1>, grid, blk, smem, pdl, a);
                case 2: return launch(c, gemv_panel_nt1<2>, grid, blk, smem, pdl, a);
                case 3: return launch(c, gemv_panel_nt1<3>, grid, blk, smem, pdl, a);
                default: return launch(c, gemv_panel_nt1<4>, grid, blk, smem, pdl, a);
                }
            }
            if (NT <= 4) return launch(c, gemv_panel_nt<4>, grid, blk, q8_smem_bytes(4, a.k), pdl, a);
            return launch(c, gemv_panel_nt<16>, grid, blk, smem, pdl, a);
        }
        if (fmt == FMT_STQN) {
            const int cpl = (a.k + 2047) / 2048;
            if (NT == 1 && cpl <= 4 && a.epi != EPI_ARGMAX) {
                const int rpc = ((a.rows_total + grid - 1) / grid + 3) & ~3;
                const size_t sm = panel_dec_smem(rpc, a.k, FMT_STQN);
                if (sm <= kMaxDynSmem) {
                    switch (cpl) {
                    case 1: return launch(c, gemv_panel_dec<1, FMT_STQN>, grid, blk, sm, pdl, a, rpc);
                    case 2: return launch(c, gemv_panel_dec<2, FMT_STQN>, grid, blk, sm, pdl, a, rpc);
                    case 3: return launch(c, gemv_panel_dec<3, FMT_STQN>, grid, blk, sm, pdl, a, rpc);
                    default: return launch(c, gemv_panel_dec<4, FMT_STQN>, grid, blk, sm, pdl, a, rpc);
                    }
                }
            }
            REQ(c, a.epi != EPI_SILU, "interleaved gate|up pair needs the staged decode GEMV");
            if (NT == 1 && cpl <= 4) {
                switch (cpl) {
                case 1: return launch(c, gemv_panel_nt1<1, FMT_STQN>, grid, blk, smem, pdl, a);
                case 2: return launch(c, gemv_panel_nt1<2, FMT_STQN>, grid, blk, smem, pdl, a);
                case 3: return launch(c, gemv_panel_nt1<3, FMT_STQN>, grid, blk, smem, pdl, a);
                default: return launch(c, gemv_panel_nt1<4, FMT_STQN>, grid, blk, smem, pdl, a);
                }
            }
            if (NT <= 4) return launch(c, gemv_panel_nt<4, FMT_STQN>, grid, blk, q8_smem_bytes(4, a.k), pdl, a);
            return launch(c, gemv_panel_nt<16, FMT_STQN>, grid, blk, smem, pdl, a);
        }
        if (fmt == FMT_Q6K) {
            if (NT == 1) return launch(c, gemv_q6k<1>, grid, blk, smem, pdl, a);
            if (NT == 4) return launch(c, gemv_q6k<4>, grid, blk, smem, pdl, a);
            return launch(c, gemv_q6k<16>, grid, blk, smem, pdl, a);
        }
        if (NT == 1) return launch(c, gemv_q4k<1>, grid, blk, smem, pdl, a);
        if (NT == 4) return launch(c, gemv_q4k<4>, grid, blk, smem, pdl, a);
        return launch(c, gemv_q4k<16>, grid, blk, smem, pdl, a);
    }
    const int NT = a.nt == 1 ? 1 : 4;
    const size_t smem = fp_smem_bytes(NT, a.k);
    if (NT == 1) {
        // one token: the rows stream from HBM, so up to 2 CTAs per SM keep more loads in flight
        const int cap = c->nsm * (ctas_per_sm > 2 ? ctas_per_sm : 2);
        grid = (a.rows_total + kGemvWarps - 1) / kGemvWarps;
        if (grid > cap) grid = cap;
    }
    if (fmt == FMT_Q80) return NT == 1 ? launch(c, gemv_fp<FMT_Q80, 1>, grid, blk, smem, pdl, a)
                                       : launch(c, gemv_fp<FMT_Q80, 4>, grid, blk, smem, pdl, a);
    if (fmt == FMT_F16) return NT == 1 ? launch(c, gemv_fp<FMT_F16, 1>, grid, blk, smem, pdl, a)
                                       : launch(c, gemv_fp<FMT_F16, 4>, grid, blk, smem, pdl, a);
    return NT == 1 ? launch(c, gemv_fp<FMT_F32, 1>, grid, blk, smem, pdl, a)
                   : launch(c, gemv_fp<FMT_F32, 4>, grid, blk, smem, pdl, a);
}

// Any nt: split into token groups the kernels take (16 for Q8_K formats,
// 4 for fp32-activation formats).
bool run_gemv(HyCtx *c, GemvArgs a, bool pdl, int ctas_per_sm = 1) {
    const int group = is_q8_fmt(a.w[0].fmt) ? 16 : 4;
    const int nt = a.nt;
    if (nt <= group) return gemv_launch(c, a, pdl, ctas_per_sm);
    REQ(c, a.epi != EPI_ARGMAX && a.ints == nullptr, "token groups need a plain epilogue");
    for (int t0 = 0; t0 < nt; t0 += group) {
        GemvArgs b = a;
        b.nt = nt - t0 < group ? nt - t0 : group;
        if (b.xq) b.xq += (size_t)t0 * (a.k / 256);
        if (b.x) b.x += (size_t)t0 * a.ldx;
        if (b.x2) b.x2 += (size_t)t0 * a.ldx;
        for (int i = 0; i < a.nw; i++) b.w[i].out += (size_t)t0 * a.w[i].ld;
        if (!gemv_launch(c, b, pdl, ctas_per_sm)) return false;
    }
    return true;
}

GemvArgs gemv_args(int nt, int k) {
    GemvArgs a;
    memset(&a, 0, sizeof a);
    a.nt = nt;
    a.k = k;
    a.trace = -1;
    return a;
}

// Launch GEMVs for up to three weights sharing one activation, merging the
// ones with the same device format into a single launch.
bool run_multi(HyCtx *c, HyWeight *const *ws, float *const *outs, const int *lds, int cnt, const GemvArgs &tmpl,
               bool pdl) {
    bool done[3] = {false, false, false};
    for (int i = 0; i < cnt; i++) {
        if (done[i]) continue;
        GemvArgs a = tmpl;
        a.nw = 0;
        a.rows_total = 0;
        for (int j = i; j < cnt; j++) {
            if (done[j] || ws[j]->fmt != ws[i]->fmt || ws[j]->k != ws[i]->k) continue;
            a.w[a.nw++] = desc(ws[j], outs[j], lds[j]);
            a.rows_total += ws[j]->n;
            done[j] = true;
        }
        if (!run_gemv(c, a, pdl)) return false;
    }
    return true;
}

// ---------------------------------------------------------------- tensor-core chunks

constexpr int kTcMinTokens = 32;  // chunks at least this long use the tensor-core GEMM

bool tc_usable(HyCtx *c, int nt, HyWeight *const *ws, int cnt) {
    if (!c->tc_on || nt < kTcMinTokens || nt > c->max_tokens) return false;
    for (int i = 0; i < cnt; i++)
        if (!tc_planes(ws[i]->fmt) || ws[i]->k % 256) return false;
    return true;
}

// Tensor-core planes and scales of a weight, built on first use.
bool tc_weight(HyCtx *c, HyWeight *w) {
    if (w->tc_w) return true;
    const int P = tc_planes(w->fmt), N = tc_n(P);
    REQ(c, P > 0, "weight format has no tensor-core form");
    const int ntiles = (w->n + N - 1) / N;
    CK(c, cudaMalloc(&w->tc_w, (size_t)ntiles * w->nb * tc_bbytes(P)));
    CK(c, cudaMalloc(&w->tc_ws, (size_t)ntiles * w->nb * tc_sbytes(P)));
    const long long total = (long long)ntiles * N * w->nb * 16;
    const unsigned grid = (unsigned)((total + 255) / 256);
    const WDesc d = desc(w, nullptr, 0);
    if (P == 1) tc_weight_to_tiled<1><<<grid, 256, 0, c->st>>>(d, w->tc_w, w->tc_ws);
    else if (P == 2) tc_weight_to_tiled<2><<<grid, 256, 0, c->st>>>(d, w->tc_w, w->tc_ws);
    else tc_weight_to_tiled<3><<<grid, 256, 0, c->st>>>(d, w->tc_w, w->tc_ws);
    CK(c, cudaGetLastError());
    return true;
}

// The slice-first copy of a weight's tiles, built on first use.
bool tc_slices(HyCtx *c, HyWeight *w) {
    if (w->tc_w64) return true;
    const int P = tc_planes(w->fmt), N = tc_n(P);
    const size_t bytes = (size_t)((w->n + N - 1) / N) * w->nb * tc_bbytes(P);
    CK(c, cudaMalloc(&w->tc_w64, bytes));
    const long long units = (long long)(bytes / 16);
    const unsigned grid = (unsigned)((units + 255) / 256);
    if (P == 1) tc_tiles_to_slices<1><<<grid, 256, 0, c->st>>>(w->tc_w, w->tc_w64, units);
    else tc_tiles_to_slices<2><<<grid, 256, 0, c->st>>>(w->tc_w, w->tc_w64, units);
    CK(c, cudaGetLastError());
    return true;
}

bool tc_scratch(HyCtx *c, int K) {
    const size_t nbmax = (size_t)(K / 256), tmax = (size_t)(c->max_tokens + kTcM - 1) / kTcM * kTcM;
    const size_t bytes = tmax * nbmax * kTcKB;
    if (bytes <= c->tca_bytes) return true;
    if (c->d_tca) cudaFree(c->d_tca);
    if (c->d_tcad) cudaFree(c->d_tcad);
    c->d_tca = nullptr;
    c->d_tcad = nullptr;
    c->tca_bytes = 0;
    CK(c, cudaMalloc(&c->d_tca, bytes));
    CK(c, cudaMalloc(&c->d_tcad, tmax * nbmax * 4));
    if (!c->d_tcerr) {
        CK(c, cudaMalloc(&c->d_tcerr, 4));
        CK(c, cudaMemsetAsync(c->d_tcerr, 0, 4, c->st));
    }
    c->tca_bytes = bytes;
    return true;
}

// One tensor-core GEMM launch over the weights in `ta` (all P planes).  MMA
// rows: the whole weight tile, or 64-row slices of it when the whole tiles
// would leave SMs idle (read from the slice-first copy, built on first use).
// INTS: the test instantiation that also stores the per-block integers.
template <bool INTS = false>
bool tc_gemm_launch(HyCtx *c, TcArgs &ta, int P, HyWeight *const *ws, int cnt, bool pdl) {
    const int NM = tc_tiles_all(P, tc_n(P), ta) >= c->nsm ? tc_n(P) : 64;
    const int ntiles = tc_tiles_all(P, NM, ta);
    if (NM < tc_n(P))
        for (int j = 0; j < cnt; j++)
            if (tc_planes(ws[j]->fmt) == P) {
                if (!tc_slices(c, ws[j])) return false;
                for (int q = 0; q < ta.nw; q++)
                    if (ta.w[q] == ws[j]->tc_w) ta.w64[q] = ws[j]->tc_w64;
            }
    const dim3 grid(ntiles < c->nsm ? ntiles : c->nsm), blk(kTcThreads);
    if (P == 1 && NM == 256) return launch(c, tc_gemm<1, 256, INTS>, grid, blk, tc_smem_bytes(1, 256), pdl, ta);
    if (P == 1) return launch(c, tc_gemm<1, 64, INTS>, grid, blk, tc_smem_bytes(1, 64), pdl, ta);
    if (P == 2 && NM == 128) return launch(c, tc_gemm<2, 128, INTS>, grid, blk, tc_smem_bytes(2, 128), pdl, ta);
    if (P == 2) return launch(c, tc_gemm<2, 64, INTS>, grid, blk, tc_smem_bytes(2, 64), pdl, ta);
    return launch(c, tc_gemm<3, 64, INTS>, grid, blk, tc_smem_bytes(3, 64), pdl, ta);
}

// nt tokens through up to three weights sharing one activation
// prologue (pro.act / x / x2 / norm_w / eps, pro.k = K): one quantise launch
// writing tiled Q8_K codes, then one tensor-core GEMM per weight format; outs[i] is
// [nt][lds[i]], stored (epi 0) or accumulated (epi 1).
// act_ready: the tiled Q8_K activation of the nt tokens is in place already
// (written by the kernel before, e.g. attn_batch_dec), so no quantiser runs.
bool tc_linear(HyCtx *c, const GemvArgs &pro, int nt, HyWeight *const *ws, float *const *outs, const int *lds,
               int cnt, int epi, bool pdl, bool act_ready = false) {
    const int K = pro.k, nb = K / 256, tpad = (nt + kTcM - 1) / kTcM * kTcM;
    if (!tc_scratch(c, K)) return false;
    for (int i = 0; i < cnt; i++)
        if (!tc_weight(c, ws[i])) return false;
    if (!act_ready) {
        const dim3 g(tpad), b(kGemvThreads);
        const size_t sm = (size_t)(K + 64) * 4;
        const int sv = (K / 4 + kGemvThreads - 1) / kGemvThreads;
        bool ok;
        if ((pro.act == ACT_VEC || pro.act == ACT_SILU) && pro.ldx % 8 == 0) {
            const long long ctas = ((long long)tpad * nb + 7) / 8;
            const unsigned grid = (unsigned)(ctas < 32LL * c->nsm ? ctas : 32LL * c->nsm);
            ok = launch(c, tc_quantize_blocks, dim3(grid), dim3(256), 0, pdl, pro, nt, tpad, c->d_tca, c->d_tcad);
        } else if (sv <= 2) ok = launch(c, tc_quantize<2>, g, b, sm, pdl, pro, nt, c->d_tca, c->d_tcad);
        else if (sv <= 4) ok = launch(c, tc_quantize<4>, g, b, sm, pdl, pro, nt, c->d_tca, c->d_tcad);
        else if (sv <= 6) ok = launch(c, tc_quantize<6>, g, b, sm, pdl, pro, nt, c->d_tca, c->d_tcad);
        else ok = launch(c, tc_quantize<kStageVec>, g, b, sm, pdl, pro, nt, c->d_tca, c->d_tcad);
        if (!ok) return false;
    }
    // one persistent launch per weight format (the weights of a launch share the activation tiles)
    bool done[kTcMaxW] = {false, false, false};
    for (int i = 0; i < cnt; i++) {
        if (done[i]) continue;
        const int P = tc_planes(ws[i]->fmt);
        TcArgs ta;
        memset(&ta, 0, sizeof ta);
        ta.a = c->d_tca;
        ta.ad = c->d_tcad;
        ta.T = nt;
        ta.nb = nb;
        ta.epi = epi;
        ta.err = c->d_tcerr;
        for (int j = i; j < cnt; j++) {
            if (done[j] || tc_planes(ws[j]->fmt) != P) continue;
            ta.w[ta.nw] = ws[j]->tc_w;
            ta.ws[ta.nw] = ws[j]->tc_ws;
            ta.out[ta.nw] = outs[j];
            ta.ldo[ta.nw] = lds[j];
            ta.N[ta.nw] = ws[j]->n;
            ta.nw++;
            done[j] = true;
        }
        if (!tc_gemm_launch(c, ta, P, ws, cnt, pdl)) return false;
    }
    return true;
}

// The tensor-core GEMM reports a timed-out wait through its error word.
bool tc_status(HyCtx *c) {
    if (!c->d_tcerr) return true;
    int err = 0;
    CK(c, cudaMemcpyAsync(&err, c->d_tcerr, 4, cudaMemcpyDeviceToHost, c->st));
    CK(c, cudaStreamSynchronize(c->st));
    if (!err) return true;
    c->broken = true;
    snprintf(c->err, sizeof c->err, "tensor-core GEMM: a pipeline wait timed out");
    return false;
}

// Tensor-parallel exchanges report a timed-out wait through their error word.
bool tp_status(HyCtx *c) {
    if (!c->d_tp_err) return true;
    int err = 0;
    CK(c, cudaMemcpyAsync(&err, c->d_tp_err, 4, cudaMemcpyDeviceToHost, c->st));
    CK(c, cudaStreamSynchronize(c->st));
    if (!err) return true;
    c->broken = true;
    snprintf(c->err, sizeof c->err, "tensor-parallel exchange: a wait for a peer timed out");
    return false;
}

// ---------------------------------------------------------------- fused layer loop

template <int HD, int G>
bool attn_launch(HyCtx *c, const AttnArgs &aa, int nt, bool pdl) {
    if (nt == 1 && !aa.tok_pos && aa.cpart && attn_chunk_len_wide(aa.ctx - 1, aa.kv_heads, aa.units) > 0) {
        // wide decode attention: units of (KV head, key chunk), then the per-head merge.  The chunk
        // rule keeps kv_heads * chunks <= min(units, kMaxUnitsWide) at every position, so no more
        // chunk rows are launched than that (one wave of CTAs).
        const int ych = std::min(aa.max_chunks, std::min(aa.units, kMaxUnitsWide) / aa.kv_heads);
        if (!launch(c, attn_chunk_kernel<HD, G>, dim3(aa.kv_heads, ych), dim3(kDecWarps * 32),
                    attn_chunk_smem<HD>(), pdl, aa))
            return false;
        return launch(c, attn_merge_kernel<HD>, dim3(aa.heads), dim3(32), 0, pdl, aa);
    }
    if (nt == 1 && !aa.tok_pos)
        return launch(c, attn_decode2<HD, G>, dim3(aa.kv_heads, aa.max_splits), dim3(kDecWarps * 32), attn_dec_smem<HD>(),
                      pdl, aa);
    int warps = aa.heads + aa.kv_heads;
    if (warps > 32) warps = 32;
    const int rgrid = nt < 16 * c->nsm ? nt : 16 * c->nsm;
    if (!launch(c, rope_norm_store<HD>, dim3(rgrid), dim3(warps * 32), 0, pdl, aa)) return false;
    const int nqb = aa.qblk ? aa.nqb : (nt + kFaQ - 1) / kFaQ;
    if (nqb == nt && aa.tok_slot)  // one token per sequence (a batch of decode steps)
        return launch(c, attn_batch_dec<HD, G>, dim3(aa.kv_heads, nt), dim3(kDbWarps * 32), 0, pdl, aa);
    return launch(c, attn_fa<HD, G>, dim3(nqb, aa.kv_heads), dim3(G * 32), fa_smem<HD, G>(), pdl, aa);
}

bool attention(HyCtx *c, const AttnArgs &aa_in, int nt, bool pdl) {
    AttnArgs aa = aa_in;
    aa.trace = trace_slot(c);
    const int G = aa.heads / aa.kv_heads;
#define HY_ATT(HD_, G_) \
    if (aa.hd == HD_ && G == G_) return attn_launch<HD_, G_>(c, aa, nt, pdl);
    HY_ATT(128, 4) HY_ATT(128, 1) HY_ATT(128, 2) HY_ATT(128, 8)
    HY_ATT(64, 4) HY_ATT(64, 1) HY_ATT(64, 2) HY_ATT(64, 8)
#undef HY_ATT
    REQ(c, false, "unsupported head geometry");
}

// gate|up then down.  Single-token steps with two panel weights of the same
// shape use one interleaved launch whose warps own (gate_r, up_r) pairs and
// write silu(gate)*up once (reference src/model.c:873-876); down then only
// quantises that vector.  Otherwise gate and up land in separate buffers and
// down applies SiLU*up in its prologue.
bool ffn_pair_ok(const Layer &L, int nt) {
    return nt == 1 && (L.g->fmt == FMT_PANEL || L.g->fmt == FMT_STQN) && L.u->fmt == L.g->fmt && L.g->n == L.u->n &&
           L.g->k == L.u->k &&
           L.g->shift == L.u->shift && L.g->off == L.u->off;
}

// Activation buffers and cache addressing of one forward pass: either the
// single sequence of the fused ops (token t at *pos_ptr + t of one cache) or
// a ragged batch (token t at tok_pos[t] of sequence slot tok_slot[t]).
struct Fwd {
    float *h, *qkv, *ao, *g, *u;  // [tokens][H | qd + 2 kvd | qd | F | F]
    uint16_t *kv;                 // layer li's K cache at kv + li * layer_stride, V v_rows rows later
    size_t layer_stride;
    const int *pages;             // batch: page table [slot][page_max] (hy_pages.h), page_stride elements a page
    int page_max;
    long long page_stride;
    int kv_ctx, v_rows;
    const int *pos_ptr;
    const int *tok_pos, *tok_slot;
    const int *qblk;              // batch: attention query blocks (first token, count)
    int nqb;
};

Fwd fwd_single(HyCtx *c, const int *pos_ptr) {
    Fwd f;
    memset(&f, 0, sizeof f);
    f.h = c->d_h;
    f.qkv = c->d_qkv;
    f.ao = c->d_ao;
    f.g = c->d_g;
    f.u = c->d_u;
    f.kv = c->d_kv;
    f.layer_stride = (size_t)2 * c->ctx * c->kvd;
    f.kv_ctx = c->ctx;
    f.v_rows = c->ctx;
    f.pos_ptr = pos_ptr;
    return f;
}

bool gateup_forward(HyCtx *c, const Fwd &f, const Layer &L, int nt, bool pdl) {
    GemvArgs a = gemv_args(nt, c->H);
    a.act = ACT_NORM;
    a.x = f.h;
    a.ldx = c->H;
    a.norm_w = L.ffn_norm;
    a.eps = c->eps;
    if (ffn_pair_ok(L, nt)) {
        a.epi = EPI_SILU;
        a.nw = 2;
        a.interleave = 1;
        a.rows_total = 2 * L.g->n;
        a.w[0] = desc(L.g, f.g, c->F);
        a.w[1] = desc(L.u, nullptr, c->F);
        return run_gemv(c, a, pdl);
    }
    HyWeight *ws[2] = {L.g, L.u};
    float *outs[2] = {f.g, f.u};
    const int lds[2] = {c->F, c->F};
    if (tc_usable(c, nt, ws, 2)) return tc_linear(c, a, nt, ws, outs, lds, 2, 0, pdl);
    a.epi = EPI_STORE;
    return run_multi(c, ws, outs, lds, 2, a, pdl);
}

// dst += down(act) (store instead when !accumulate: a tensor-parallel partial)
bool down_forward(HyCtx *c, const Fwd &f, const Layer &L, int nt, bool pdl, float *dst, bool accumulate = true) {
    GemvArgs a = gemv_args(nt, c->F);
    if (ffn_pair_ok(L, nt)) {
        a.act = ACT_VEC;  // g already holds silu(gate)*up
        a.x = f.g;
    } else {
        a.act = ACT_SILU;
        a.x = f.g;
        a.x2 = f.u;
    }
    a.ldx = c->F;
    {
        HyWeight *ws[1] = {L.d};
        float *outs[1] = {dst};
        const int lds[1] = {c->H};
        if (tc_usable(c, nt, ws, 1)) return tc_linear(c, a, nt, ws, outs, lds, 1, accumulate ? 1 : 0, pdl);
    }
    a.epi = accumulate ? EPI_ADD : EPI_STORE;
    a.nw = 1;
    a.rows_total = L.d->n;
    a.w[0] = desc(L.d, dst, c->H);
    return run_gemv(c, a, pdl);
}

// Tensor parallelism: h[0 .. nt*H) += the sum over ranks of their partial
// products in d_tp_part (one-shot push over peer memory, hy_tp.cuh).
bool tp_reduce(HyCtx *c, float *h, int nt) {
    TpArgs a = c->tp;
    a.h = h;
    a.part = c->d_tp_part;
    a.n = nt * c->H;
    const int ctas = std::min(kTpMaxCtas, (a.n + kTpSlice - 1) / kTpSlice);
    a.slice = ((a.n + ctas - 1) / ctas + 3) & ~3;
    return launch(c, tp_allreduce_add, dim3(ctas), dim3(kTpThreads), 0, false, a);
}

bool ffn_forward(HyCtx *c, const Fwd &f, const Layer &L, int nt, bool pdl) {
    if (!c->tp_on) return gateup_forward(c, f, L, nt, pdl) && down_forward(c, f, L, nt, pdl, f.h);
    // tensor parallelism: the rank's partial down product, then h += the sum over ranks
    return gateup_forward(c, f, L, nt, pdl) && down_forward(c, f, L, nt, pdl, c->d_tp_part, false) &&
           tp_reduce(c, f.h, nt);
}

bool layer_forward(HyCtx *c, const Fwd &f, int li, int nt, bool pdl) {
    const Layer &L = c->layers[li];
    const int qkv_ld = c->qd + 2 * c->kvd;
    // an all-decode batch pass (one token per query block: attn_batch_dec)
    // whose o_proj runs on the tensor cores: the attention kernel writes the
    // GEMM's tiled Q8_K input itself (whole blocks: G * hd a multiple of 256)
    HyWeight *wo[1] = {L.o};
    const bool fuse_oq = f.tok_slot && f.qblk && f.nqb == nt && L.o->k == c->qd &&
                         ((c->heads / c->kvh) * c->hd) % 256 == 0 && tc_usable(c, nt, wo, 1);
    {
        HyWeight *ws[3] = {L.q, L.k, L.v};
        float *outs[3] = {f.qkv, f.qkv + c->qd, f.qkv + c->qd + c->kvd};
        const int lds[3] = {qkv_ld, qkv_ld, qkv_ld};
        GemvArgs a = gemv_args(nt, c->H);
        a.act = ACT_NORM;
        a.x = f.h;
        a.ldx = c->H;
        a.norm_w = L.attn_norm;
        a.eps = c->eps;
        if (tc_usable(c, nt, ws, 3)) {
            if (!tc_linear(c, a, nt, ws, outs, lds, 3, 0, pdl)) return false;
        } else {
            a.epi = EPI_STORE;
            if (!run_multi(c, ws, outs, lds, 3, a, pdl)) return false;
        }
    }
    {
        AttnArgs aa;
        memset(&aa, 0, sizeof aa);
        aa.qkv = f.qkv;
        aa.qkv_ld = qkv_ld;
        aa.kc = f.kv + (size_t)li * f.layer_stride;
        aa.vc = aa.kc + (size_t)f.v_rows * c->kvd;
        aa.q_norm = L.q_norm;
        aa.k_norm = L.k_norm;
        aa.rope_cos = c->d_cos;
        aa.rope_sin = c->d_sin;
        aa.pos_ptr = f.pos_ptr;
        aa.tok_pos = f.tok_pos;
        aa.tok_slot = f.tok_slot;
        aa.pages = f.pages;
        aa.page_max = f.page_max;
        aa.page_stride = f.page_stride;
        aa.qblk = f.qblk;
        aa.nqb = f.nqb;
        aa.nt = nt;
        aa.heads = c->heads;
        aa.kv_heads = c->kvh;
        aa.hd = c->hd;
        aa.kvdim = c->kvd;
        aa.qdim = c->qd;
        aa.ctx = f.kv_ctx;
        aa.half = c->half;
        aa.eps = c->eps;
        aa.scale = 1.0f / sqrtf((float)c->hd);
        aa.ao = f.ao;
        aa.part = c->d_part;
        aa.cpart = c->d_cpart;
        aa.max_chunks = c->max_chunks;
        aa.units = c->nsm;
        aa.tickets = c->d_tickets;
        aa.split_len = kSplitLen;
        aa.max_splits = c->max_splits;
        if (fuse_oq) {
            if (!tc_scratch(c, c->qd)) return false;
            aa.tca = c->d_tca;
            aa.tcad = c->d_tcad;
            aa.tc_nb = c->qd / 256;
        }
        if (!attention(c, aa, nt, pdl)) return false;
    }
    {
        // tensor parallelism: the rank's partial product, then h += the sum over ranks
        float *dst = c->tp_on ? c->d_tp_part : f.h;
        const int epi = c->tp_on ? 0 : 1;
        GemvArgs a = gemv_args(nt, c->qd);
        a.act = ACT_VEC;
        a.x = f.ao;
        a.ldx = c->qd;
        HyWeight *ws[1] = {L.o};
        float *outs[1] = {dst};
        const int lds[1] = {c->H};
        if (tc_usable(c, nt, ws, 1)) {
            if (!tc_linear(c, a, nt, ws, outs, lds, 1, epi, pdl, fuse_oq)) return false;
        } else {
            a.epi = epi ? EPI_ADD : EPI_STORE;
            a.nw = 1;
            a.rows_total = L.o->n;
            a.w[0] = desc(L.o, dst, c->H);
            if (!run_gemv(c, a, pdl)) return false;
        }
        if (c->tp_on && !tp_reduce(c, f.h, nt)) return false;
    }
    return ffn_forward(c, f, L, nt, pdl);
}

// LM head on one token's residual x (RMSNorm with out_norm first).
bool head_forward(HyCtx *c, const float *x, bool store_logits, bool argmax, bool pdl) {
    REQ(c, c->outw != nullptr, "no LM head uploaded");
    GemvArgs a = gemv_args(1, c->H);
    a.act = ACT_NORM;
    a.x = x;
    a.ldx = c->H;
    a.norm_w = c->d_out_norm;
    a.eps = c->eps;
    a.nw = 1;
    a.rows_total = c->outw->n;
    a.w[0] = desc(c->outw, store_logits ? c->d_logits : nullptr, c->outw->n);
    if (argmax) {
        // rows below vocab_out compete; a tensor-parallel rank holds rows tp_vocab0 .. of the vocabulary
        const int lim = (c->vocab_out > 0 ? c->vocab_out : c->outw->n + c->tp_vocab0) - c->tp_vocab0;
        a.epi = EPI_ARGMAX;
        a.amax = &c->d_state->amax;
        a.amax_rows = std::max(0, std::min(lim, c->outw->n));
        a.amax_base = c->tp_vocab0;
    } else {
        a.epi = EPI_STORE;
    }
    if (!run_gemv(c, a, pdl, 2)) return false;
    if (argmax && c->tp_on) {  // the greedy token: the largest key over the ranks' vocabulary slices
        TpArgs t = c->tp;
        t.key = &c->d_state->amax;
        return launch(c, tp_argmax_exchange, dim3(1), dim3(32), 0, false, t);
    }
    return true;
}

bool layers_forward(HyCtx *c, const Fwd &f, int nt, bool pdl) {
    for (int li = 0; li < c->L; li++)
        if (!layer_forward(c, f, li, nt, pdl)) return false;
    return true;
}

bool layers_forward(HyCtx *c, int nt, const int *pos_ptr, bool pdl) {
    return layers_forward(c, fwd_single(c, pos_ptr), nt, pdl);
}

// ---------------------------------------------------------------- graphs

void graph_reset(Graph &g) {
    if (g.exec) cudaGraphExecDestroy(g.exec);
    g.exec = nullptr;
    g.kernels = 0;
}

template <typename F>
bool capture(HyCtx *c, Graph &g, F body) {
    graph_reset(g);
    CK(c, cudaStreamBeginCapture(c->st, cudaStreamCaptureModeThreadLocal));
    c->capture_kernels = 0;
    const long long before = c->launches;
    const bool ok = body();
    cudaGraph_t graph = nullptr;
    cudaError_t e = cudaStreamEndCapture(c->st, &graph);
    c->launches = before;
    if (!ok) {
        if (graph) cudaGraphDestroy(graph);
        return false;
    }
    if (e != cudaSuccess) return fail(c, "cudaStreamEndCapture", e);
    e = cudaGraphInstantiate(&g.exec, graph, 0);
    cudaGraphDestroy(graph);
    if (e != cudaSuccess) return fail(c, "cudaGraphInstantiate", e);
    g.kernels = c->capture_kernels;
    return true;
}

bool graph_launch(HyCtx *c, Graph &g) {
    CK(c, cudaGraphLaunch(g.exec, c->st));
    c->launches += g.kernels;
    return true;
}

bool build_decode_graph(HyCtx *c) {
    if (c->g_dec.exec && c->g_dec_vocab == c->vocab_out) return true;
    REQ(c, c->embd != nullptr, "no embedding weight set (hyc_set_embedding)");
    const bool ok = capture(c, c->g_dec, [&]() {
        if (!launch(c, embed_rows, dim3(1), dim3(256), 0, true, desc(c->embd, nullptr, 0),
                    (const int *)&c->d_state->tok, c->d_h, trace_slot(c)))
            return false;
        if (!layers_forward(c, 1, &c->d_state->pos, true)) return false;
        if (!head_forward(c, c->d_h, false, true, true)) return false;
        return launch(c, decode_finalize, dim3(1), dim3(32), 0, true, c->d_state, c->d_out_ids, trace_slot(c));
    });
    if (ok) c->g_dec_vocab = c->vocab_out;
    return ok;
}

// ---------------------------------------------------------------- persistent decode

template <int HD, int G, int CF>
void *mega_kernel_for() {
    return (void *)decode_mega<HD, G, CF>;
}

// Decide once per prepared model whether the persistent kernel can run it,
// and build its device tables.  Unsupported shapes keep the graph path.
bool mega_check(HyCtx *c) {
    if (c->mega_state >= 0) return c->mega_state == 1;
    c->mega_state = 0;
    auto no = [&](const char *why) {
        snprintf(c->mega_why, sizeof c->mega_why, "%s", why);
        return false;
    };
    if (!c->fused || !c->outw || !c->embd) return no("model not prepared");
    if (c->tp_world > 1) return no("tensor-parallel rank (the per-layer graph carries the exchanges)");
    const int G = c->heads / c->kvh;
    int CF = (c->F + 2047) / 2048;
    if (CF == 2) CF = 3;
    if (c->hd == 128 && G == 4 && CF == 3) c->mega_kernel = mega_kernel_for<128, 4, 3>();
    else if (c->hd == 64 && G == 2 && CF == 1) c->mega_kernel = mega_kernel_for<64, 2, 1>();
    else if (c->hd == 64 && G == 4 && CF == 1) c->mega_kernel = mega_kernel_for<64, 4, 1>();
    else return no("head geometry / FFN width without a persistent-kernel instance");
    if (c->H > 2048 || c->qd > 2048) return no("hidden or q width above 2048");
    if (c->L > kMegaMaxLayers) return no("more layers than the persistent kernel's table holds");
    if (c->outw->fmt != FMT_Q6K || c->outw->k != c->H) return no("LM head is not Q6_K");
    if (c->kvh > 64 || attn_chunk_len(c->ctx - 1, c->kvh, c->nsm) == 0)
        return no("context too long for the attention units of one launch");
    const HyWeight *w0 = c->layers[0].q;
    for (const Layer &L : c->layers) {
        const HyWeight *ws[7] = {L.q, L.k, L.v, L.o, L.g, L.u, L.d};
        for (const HyWeight *w : ws)
            if (w->fmt != FMT_PANEL || w->shift != w0->shift || w->off != w0->off) return no("layer weights not all panels");
        if (L.g->n != c->F || L.u->n != c->F || L.d->n != c->H || L.o->n != c->H || L.q->n != c->qd ||
            L.k->n != c->kvd || L.v->n != c->kvd)
            return no("layer weight rows do not match the model");
    }
    int coop = 0;
    if (cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, c->dev) != cudaSuccess || !coop)
        return no("no cooperative launch");
    c->mega_plan_v = mega_plan(c->nsm, c->H, c->F, c->qd, c->kvd, c->outw->n, c->hd);
    if (!mega_head_ring(c->mega_plan_v, c->outw->stride))
        return no("LM-head rows do not fit the shared-memory rings");
    // about three quarters of L2 holds the first rows of every CTA's head slice
    // across tokens (the layer weights, read once per token, are evict-first)
    if (cudaFuncSetAttribute(c->mega_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)c->mega_plan_v.bytes) != cudaSuccess) {
        cudaGetLastError();
        return no("shared-memory plan too large");
    }
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, c->mega_kernel, kMegaThreads, c->mega_plan_v.bytes) !=
            cudaSuccess ||
        per_sm < 1) {
        cudaGetLastError();
        return no("persistent kernel does not fit on an SM");
    }
    std::vector<MegaLayer> tab(c->L);
    for (int i = 0; i < c->L; i++) {
        const Layer &L = c->layers[i];
        const HyWeight *ws[7] = {L.q, L.k, L.v, L.o, L.g, L.u, L.d};
        for (int j = 0; j < 7; j++) {
            tab[i].w[j] = ws[j]->w;
            tab[i].s[j] = ws[j]->s;
        }
        tab[i].attn_norm = L.attn_norm;
        tab[i].ffn_norm = L.ffn_norm;
        tab[i].q_norm = L.q_norm;
        tab[i].k_norm = L.k_norm;
        tab[i].kc = c->d_kv + (size_t)i * 2 * c->ctx * c->kvd;
        tab[i].vc = tab[i].kc + (size_t)c->ctx * c->kvd;
    }
    if (!c->d_mega_layers) CK(c, cudaMalloc(&c->d_mega_layers, (size_t)c->L * sizeof(MegaLayer)));
    if (!c->d_mega_sync) CK(c, cudaMalloc(&c->d_mega_sync, sizeof(MegaSync)));
    CK(c, h2d(c, c->d_mega_layers, tab.data(), (size_t)c->L * sizeof(MegaLayer)));
    CK(c, cudaMemsetAsync(c->d_mega_sync, 0, sizeof(MegaSync), c->st));
    CK(c, cudaStreamSynchronize(c->st));  // the host table is a local
    c->mega_state = 1;
    return true;
}

bool use_mega(HyCtx *c) { return c->decode_mode == 0 && mega_check(c); }

// `steps` greedy decode steps from the DecodeState's (tok, pos) in one launch.
bool mega_launch(HyCtx *c, int steps) {
    MegaArgs a;
    memset(&a, 0, sizeof a);
    const MegaPlan &p = c->mega_plan_v;
    a.layers = c->d_mega_layers;
    a.L = c->L;
    a.H = c->H;
    a.F = c->F;
    a.kvh = c->kvh;
    a.qd = c->qd;
    a.kvd = c->kvd;
    a.ctx = c->ctx;
    a.shift = c->layers[0].q->shift;
    a.off = c->layers[0].q->off;
    a.eps = c->eps;
    for (int i = 0; i < 5; i++) a.rpc[i] = p.rpc[i];
    for (int i = 0; i < 4; i++) a.slot_off[i] = p.slot_off[i];
    a.stage_off = p.stage_off;
    a.attn_off = p.attn_off;
    a.kmax = p.kmax;
    a.head_reg[0] = p.head_reg[0];
    a.head_reg[1] = p.head_reg[1];
    a.head_n1 = p.head_n1;
    AttnArgs &aa = a.attn;
    aa.qkv = c->d_qkv;
    aa.qkv_ld = c->qd + 2 * c->kvd;
    aa.rope_cos = c->d_cos;
    aa.rope_sin = c->d_sin;
    aa.pos_ptr = &c->d_state->pos;
    aa.nt = 1;
    aa.heads = c->heads;
    aa.kv_heads = c->kvh;
    aa.hd = c->hd;
    aa.kvdim = c->kvd;
    aa.qdim = c->qd;
    aa.ctx = c->ctx;
    aa.half = c->half;
    aa.eps = c->eps;
    aa.scale = 1.0f / sqrtf((float)c->hd);
    aa.ao = c->d_ao;
    aa.part = c->d_part;
        aa.cpart = c->d_cpart;
        aa.max_chunks = c->max_chunks;
        aa.units = c->nsm;
    aa.split_len = kSplitLen;
    aa.max_splits = c->max_splits;
    aa.trace = -1;
    a.head = desc(c->outw, nullptr, c->outw->n);
    a.embd = desc(c->embd, nullptr, 0);
    a.vocab_out = c->vocab_out > 0 ? c->vocab_out : c->outw->n;
    a.out_norm = c->d_out_norm;
    a.h = c->d_h;
    a.qkv = c->d_qkv;
    a.ao = c->d_ao;
    a.act = c->d_g;
    a.st = c->d_state;
    a.out_ids = c->d_out_ids;
    a.sync = c->d_mega_sync;
    a.tl = c->trace_on ? c->d_tl : nullptr;
    a.tl_cap = c->tl_cap;
    a.steps = steps;
    a.host_io = c->host_io;
    a.host_limit_ns = c->host_limit_ns;
    CK(c, cudaMemsetAsync(c->d_mega_sync, 0, sizeof(MegaSync), c->st));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(c->nsm);
    cfg.blockDim = dim3(kMegaThreads);
    cfg.dynamicSmemBytes = p.bytes;
    cfg.stream = c->st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    void *args[] = {&a};
    CK(c, cudaLaunchKernelExC(&cfg, c->mega_kernel, args));
    c->launches++;
    return true;
}

// The persistent kernel reports failures through its error word.
bool mega_status(HyCtx *c) {
    if (c->mega_state != 1 || !c->d_mega_sync) return true;
    int err = 0;
    CK(c, cudaMemcpyAsync(&err, &c->d_mega_sync->err, 4, cudaMemcpyDeviceToHost, c->st));
    CK(c, cudaStreamSynchronize(c->st));
    if (err == MEGA_OK) return true;
    if (err == MEGA_ERR_HOST) {
        // the resident loop ended cleanly (state written, copies drained): the handle stays usable
        snprintf(c->err, sizeof c->err, "persistent decode kernel: the host did not answer within the limit");
        CK(c, cudaMemsetAsync(&c->d_mega_sync->err, 0, 4, c->st));
        return false;
    }
    static const char *what[] = {"", "grid barrier timed out", "position outside the context",
                                 "weight slice copy timed out", "K/V row copy timed out"};
    c->broken = true;
    snprintf(c->err, sizeof c->err, "persistent decode kernel: %s", err > 0 && err < 5 ? what[err] : "unknown error");
    return false;
}

// Decode steps through whichever path the model uses.
bool decode_run(HyCtx *c, int steps) {
    if (steps <= 0) return true;
    if (use_mega(c)) return mega_launch(c, steps);
    if (!build_decode_graph(c)) return false;
    for (int i = 0; i < steps; i++)
        if (!graph_launch(c, c->g_dec)) return false;
    return true;
}

// ---------------------------------------------------------------- test hooks

// Runs the GEMV prologue's quantiser (stage_q8k) and writes full host-layout
// blocks: natural qs, lane-major qp, d, sum, bsums.
__global__ void __launch_bounds__(kGemvThreads) quantize_export(const __grid_constant__ GemvArgs a, q8k_block *y) {
    extern __shared__ __align__(16) uint8_t smem[];
    const int K = a.k, nb = K / 256;
    Q8Smem s = q8_smem(smem, 16, K);
    stage_q8k(a, s, K);
    for (int t = 0; t < a.nt; t++) {
        for (int i = threadIdx.x; i < nb * 256; i += blockDim.x) {
            const int b = i >> 8, e = i & 255, ch = e >> 6, l = (e >> 4) & 3, j = e & 15;
            const int8_t v = s.qp[(size_t)t * K + (size_t)l * (K / 4) + (b * 4 + piece_of_chunk(ch)) * 16 + j];
            q8k_block &blk = y[(size_t)t * nb + b];
            blk.qs[e] = v;
            // qp[l*64 + p*16 + j] holds natural chunk kPieceOrder[p], plane l
            blk.qp[l * 64 + piece_of_chunk(ch) * 16 + j] = v;
        }
        for (int i = threadIdx.x; i < nb; i += blockDim.x) {
            q8k_block &blk = y[(size_t)t * nb + i];
            blk.d = s.d[t * nb + i];
            blk.sum = s.sum[t * nb + i];
            for (int j = 0; j < 16; j++) blk.bsums[j] = s.bs[(size_t)t * nb * 16 + i * 16 + j];
            for (int j = 0; j < (int)sizeof(blk._pad); j++) blk._pad[j] = 0;
        }
    }
}

// ---------------------------------------------------------------- vtable ops

void batch_free(HyCtx *c);

void free_fused(HyCtx *c) {
    batch_free(c);
    graph_reset(c->g_fwd1);
    graph_reset(c->g_fwd1_logits);
    graph_reset(c->g_dec);
    c->g_dec_vocab = -1;
    void *ptrs[] = {c->d_norms, c->d_out_norm, c->d_cos, c->d_sin, c->d_kv, c->d_h, c->d_qkv, c->d_ao,
                    c->d_g, c->d_u, c->d_logits, c->d_part, c->d_cpart, c->d_tickets, c->d_state, c->d_out_ids,
                    c->d_tokens, c->d_chunk_pos};
    for (void *p : ptrs)
        if (p) cudaFree(p);
    c->d_norms = c->d_out_norm = c->d_cos = c->d_sin = nullptr;
    c->d_kv = nullptr;
    c->d_h = c->d_qkv = c->d_ao = c->d_g = c->d_u = c->d_logits = c->d_part = c->d_cpart = nullptr;
    c->d_tickets = nullptr;
    c->d_state = nullptr;
    c->d_out_ids = c->d_tokens = c->d_chunk_pos = nullptr;
    c->layers.clear();
    c->fused = false;
    if (c->d_mega_layers) cudaFree(c->d_mega_layers);
    if (c->d_mega_sync) cudaFree(c->d_mega_sync);
    if (c->d_tl) cudaFree(c->d_tl);
    c->d_mega_layers = nullptr;
    c->d_mega_sync = nullptr;
    c->d_tl = nullptr;
    c->tl_cap = 0;
    c->mega_state = -1;
}

void tp_free(HyCtx *c) {
    for (int q = 0; q < c->tp_world && q < kTpMax; q++)
        if (q != c->tp_rank && c->tp.area[q]) cudaIpcCloseMemHandle(c->tp.area[q]);
    if (c->d_tp_area) cudaFree(c->d_tp_area);
    if (c->d_tp_part) cudaFree(c->d_tp_part);
    if (c->d_tp_err) cudaFree(c->d_tp_err);
    c->d_tp_area = nullptr;
    c->d_tp_part = nullptr;
    c->d_tp_err = nullptr;
    memset(&c->tp, 0, sizeof c->tp);
    c->tp_on = false;
    c->tp_world = 1;
    c->tp_rank = 0;
    c->tp_vocab0 = 0;
}

void destroy_impl(void *impl) {
    HyCtx *c = (HyCtx *)impl;
    if (!c) return;
    cudaSetDevice(c->dev);
    tp_free(c);
    free_fused(c);
    if (c->d_xq) cudaFree(c->d_xq);
    if (c->d_x32) cudaFree(c->d_x32);
    if (c->d_ints) cudaFree(c->d_ints);
    if (c->d_tca) cudaFree(c->d_tca);
    if (c->d_tcad) cudaFree(c->d_tcad);
    if (c->d_tcerr) cudaFree(c->d_tcerr);
    if (c->h_pinned_int) cudaFreeHost(c->h_pinned_int);
    for (int i = 0; i < 2; i++) {
        if (c->h_stage[i]) cudaFreeHost(c->h_stage[i]);
        if (c->stage_ev[i]) cudaEventDestroy(c->stage_ev[i]);
    }
    if (c->d_raw) cudaFree(c->d_raw);
    if (c->st) cudaStreamDestroy(c->st);
    delete c;
}

void release(hy_dweight *hw) {
    HyWeight *w = (HyWeight *)hw;
    if (!w) return;
    if (w->w) cudaFree(w->w);
    if (w->s) cudaFree(w->s);
    if (w->d_out) cudaFree(w->d_out);
    if (w->h_out) cudaFreeHost(w->h_out);
    if (w->tc_w) cudaFree(w->tc_w);
    if (w->tc_ws) cudaFree(w->tc_ws);
    if (w->tc_w64) cudaFree(w->tc_w64);
    delete w;
}

// Device copy of one host weight (reference contract src/device.h:32,
// src/model.c:384-406).  STQ1_0 / Q2_0C arrive with the host-built panel
// (pk/ps); when they do not, the panel is built here on the device.
hy_dweight *upload(void *impl, const weight_t *w) {
    HyCtx *c = (HyCtx *)impl;
    if (!c || c->broken || !w || w->n <= 0 || w->k <= 0) return nullptr;
    if (cudaSetDevice(c->dev) != cudaSuccess) return nullptr;
    HyWeight *d = new HyWeight();
    memset(d, 0, sizeof *d);
    d->c = c;
    d->gtype = w->type;
    d->n = w->n;
    d->k = w->k;
    d->nb = w->k / 256;
    bool ok = true;
    auto bail = [&](const char *why) {
        snprintf(c->err, sizeof c->err, "upload: %s", why);
        release((hy_dweight *)d);
        return (hy_dweight *)nullptr;
    };
    switch (w->type) {
    case GT_STQ1_0:
        if (c->stq_native) {
            // the file's 42-byte blocks, relaid per row into qs | sign | d planes
            if (w->k % 256) return bail("inner dimension not a block multiple");
            if (!w->data || w->row_bytes != (size_t)d->nb * 42) return bail("native STQ1_0 rows needed");
            d->fmt = FMT_STQN;
            d->shift = 0;
            d->off = 1;
            d->stride = (long long)align16((size_t)d->nb * 42);
            const size_t rb = (size_t)d->n * w->row_bytes;
            ok = cudaMalloc(&d->w, (size_t)d->n * d->stride) == cudaSuccess;
            uint8_t *raw = ok ? raw_buf(c, rb) : nullptr;
            ok = raw && h2d_staged(c, raw, w->data, rb) == cudaSuccess;
            if (ok) {
                const long long tot = (long long)d->n * d->nb;
                stqn_from_native<<<(unsigned)((tot + 255) / 256), 256, 0, c->st>>>(raw, (long long)w->row_bytes, d->n,
                                                                                 d->nb, d->w, d->stride);
                ok = cudaGetLastError() == cudaSuccess;
            }
            break;
        }
        [[fallthrough]];
    case GT_Q2_0C: {
        if (w->k % (w->type == GT_Q2_0C ? 512 : 256)) return bail("inner dimension not a block multiple");
        d->fmt = FMT_PANEL;
        d->shift = w->type == GT_Q2_0C ? 1 : 0;
        d->off = w->type == GT_Q2_0C ? 3 : 1;
        if (w->pk) {
            d->shift = w->pshift;
            d->off = w->poff;
        }
        d->stride = (long long)d->nb * 64;
        const size_t pk_bytes = (size_t)d->n * d->nb * 64, ps_bytes = (size_t)d->n * d->nb * 4;
        ok = cudaMalloc(&d->w, pk_bytes) == cudaSuccess && cudaMalloc(&d->s, ps_bytes) == cudaSuccess;
        if (!ok) return bail("out of device memory");
        if (w->pk) {
            ok = h2d_staged(c, d->w, w->pk, pk_bytes) == cudaSuccess &&
                 h2d_staged(c, d->s, w->ps, ps_bytes) == cudaSuccess;
        } else {
            // the file's native rows, repacked to panels on the device
            const size_t rb = (size_t)d->n * w->row_bytes;
            uint8_t *raw = raw_buf(c, rb);
            ok = raw && h2d_staged(c, raw, w->data, rb) == cudaSuccess;
            if (ok) {
                const long long tot = (long long)d->n * d->nb;
                panel_from_native<<<(unsigned)((tot + 255) / 256), 256, 0, c->st>>>(raw, (long long)w->row_bytes, w->type,
                                                                                  d->n, d->nb, d->w, d->s);
                ok = cudaGetLastError() == cudaSuccess;
            }
        }
        break;
    }
    case GT_Q4_K:
        if (w->k % 256) return bail("inner dimension not a block multiple");
        d->fmt = FMT_Q4K;
        d->stride = (long long)d->nb * 144;
        ok = cudaMalloc(&d->w, (size_t)d->n * d->stride) == cudaSuccess &&
             h2d_staged(c, d->w, w->data, (size_t)d->n * d->stride) == cudaSuccess;
        break;
    case GT_Q6_K: {
        if (w->k % 256) return bail("inner dimension not a block multiple");
        d->fmt = FMT_Q6K;
        d->stride = (long long)align16((size_t)d->nb * 208 + (size_t)d->nb * 2);
        const size_t rb = (size_t)d->n * d->nb * 210;
        ok = cudaMalloc(&d->w, (size_t)d->n * d->stride) == cudaSuccess;
        uint8_t *raw = ok ? raw_buf(c, rb) : nullptr;
        ok = raw && h2d_staged(c, raw, w->data, rb) == cudaSuccess;
        if (ok) {
            const long long tot = (long long)d->n * d->nb;
            q6k_relayout<<<(unsigned)((tot + 255) / 256), 256, 0, c->st>>>(raw, d->n, d->nb, d->w, d->stride);
            ok = cudaGetLastError() == cudaSuccess;
        }
        break;
    }
    case GT_Q8_0: {
        if (w->k % 32) return bail("inner dimension not a block multiple");
        d->fmt = FMT_Q80;
        const int nblk = w->k / 32;
        d->stride = (long long)align16((size_t)w->k + (size_t)nblk * 2);
        const size_t rb = (size_t)d->n * nblk * 34;
        ok = cudaMalloc(&d->w, (size_t)d->n * d->stride) == cudaSuccess;
        uint8_t *raw = ok ? raw_buf(c, rb) : nullptr;
        ok = raw && h2d_staged(c, raw, w->data, rb) == cudaSuccess;
        if (ok) {
            const long long tot = (long long)d->n * nblk;
            q80_relayout<<<(unsigned)((tot + 255) / 256), 256, 0, c->st>>>(raw, d->n, nblk, d->w, d->stride);
            ok = cudaGetLastError() == cudaSuccess;
        }
        break;
    }
    case GT_F16:
    case GT_F32: {
        const int es = w->type == GT_F16 ? 2 : 4;
        if ((w->k * es) % 16) return bail("row length not a multiple of 16 bytes");
        d->fmt = w->type == GT_F16 ? FMT_F16 : FMT_F32;
        d->stride = (long long)w->k * es;
        ok = cudaMalloc(&d->w, (size_t)d->n * d->stride) == cudaSuccess &&
             h2d_staged(c, d->w, w->data, (size_t)d->n * d->stride) == cudaSuccess;
        break;
    }
    default:
        return bail("unsupported weight type");
    }
    if (ok) ok = cudaStreamSynchronize(c->st) == cudaSuccess;
    if (!ok) {
        c->broken = true;
        return bail("device copy failed");
    }
    return (hy_dweight *)d;
}

bool ensure_out(HyWeight *w) {
    if (w->d_out) return true;
    const size_t bytes = (size_t)MAX_BATCH * w->n * sizeof(float);
    if (cudaMalloc(&w->d_out, bytes) != cudaSuccess) return false;
    if (cudaHostAlloc((void **)&w->h_out, bytes, cudaHostAllocDefault) != cudaSuccess) return false;
    return true;
}

float *weight_out(hy_dweight *hw) {
    HyWeight *w = (HyWeight *)hw;
    if (!w || !ensure_out(w)) return nullptr;
    return w->h_out;
}

bool is_software(const void *) { return false; }

bool ensure_buf(HyCtx *c, void **p, size_t *cap, size_t need) {
    if (need <= *cap) return true;
    if (*p) cudaFree(*p);
    *p = nullptr;
    *cap = 0;
    CK(c, cudaMalloc(p, need));
    *cap = need;
    return true;
}

// Synchronous batched GEMV over host Q8_K activations (reference contract:
// src/device.h:35-38, host blocks xq[nt][nb], outputs out[t*n + r]).
bool matmul(void *impl, hy_dweight *const *ws, float *const *outs, int cnt, const q8k_block *xq, int nt) {
    HyCtx *c = (HyCtx *)impl;
    if (!c || c->broken || cnt < 1 || nt < 1 || nt > MAX_BATCH || !xq) return false;
    if (cudaSetDevice(c->dev) != cudaSuccess) return false;
    const int nb = ((HyWeight *)ws[0])->nb;
    for (int i = 0; i < cnt; i++) {
        HyWeight *w = (HyWeight *)ws[i];
        if (!w || w->nb != nb || !is_q8_fmt(w->fmt)) return false;  // fp32 formats need fp32 activations
        if (!ensure_out(w)) return fail(c, "matmul output", cudaErrorMemoryAllocation);
    }
    const size_t bytes = (size_t)nt * nb * sizeof(q8k_block);
    if (!ensure_buf(c, (void **)&c->d_xq, &c->xq_cap, bytes)) return false;
    CK(c, cudaMemcpyAsync(c->d_xq, xq, bytes, cudaMemcpyHostToDevice, c->st));
    for (int i = 0; i < cnt; i++) {
        HyWeight *w = (HyWeight *)ws[i];
        GemvArgs a = gemv_args(nt, w->k);
        a.act = ACT_Q8K;
        a.xq = c->d_xq;
        a.epi = EPI_STORE;
        a.nw = 1;
        a.rows_total = w->n;
        a.w[0] = desc(w, w->d_out, w->n);
        if (!run_gemv(c, a, false)) return false;
    }
    for (int i = 0; i < cnt; i++) {
        HyWeight *w = (HyWeight *)ws[i];
        float *dst = outs[i] ? outs[i] : w->h_out;
        CK(c, cudaMemcpyAsync(dst, w->d_out, (size_t)nt * w->n * sizeof(float), cudaMemcpyDeviceToHost, c->st));
    }
    CK(c, cudaStreamSynchronize(c->st));
    return true;
}

// Allocate KV cache, scratch and constants for the model shape (reference
// contract src/device.h:61-64, src/cuda.c:282-337; idempotent per shape).
bool fused_prepare(void *impl, const hy_fused_args *sh) {
    HyCtx *c = (HyCtx *)impl;
    if (!c || c->broken || !sh || !sh->layers) return false;
    if (cudaSetDevice(c->dev) != cudaSuccess) return false;
    REQ(c, sh->heads > 0 && sh->kv_heads > 0 && sh->heads % sh->kv_heads == 0, "bad head counts");
    const int G = sh->heads / sh->kv_heads;
    REQ(c, (sh->hdim == 64 || sh->hdim == 128) && (G == 1 || G == 2 || G == 4 || G == 8), "unsupported head geometry");
    REQ(c, sh->rope_half * 2 == sh->hdim, "partial rotary dimension not supported");
    REQ(c, sh->hidden % 256 == 0 && sh->ffn % 256 == 0 && sh->qdim % 256 == 0, "dims must be multiples of 256");
    REQ(c, sh->qdim == sh->heads * sh->hdim && sh->kvdim == sh->kv_heads * sh->hdim, "inconsistent dims");
    REQ(c, sh->ctx > 0, "ctx must be positive");
    const bool same = c->fused && c->L == sh->n_layer && c->H == sh->hidden && c->F == sh->ffn &&
                      c->heads == sh->heads && c->kvh == sh->kv_heads && c->hd == sh->hdim && c->ctx == sh->ctx;
    if (!same) {
        free_fused(c);
        c->L = sh->n_layer;
        c->H = sh->hidden;
        c->F = sh->ffn;
        c->heads = sh->heads;
        c->kvh = sh->kv_heads;
        c->hd = sh->hdim;
        c->qd = sh->qdim;
        c->kvd = sh->kvdim;
        c->ctx = sh->ctx;
        c->half = sh->rope_half;
        c->eps = sh->eps;
        c->max_splits = (c->ctx + kSplitLen - 1) / kSplitLen;
        const size_t T = kMaxChunk;
        const size_t vocab = sh->outw ? (size_t)((HyWeight *)sh->outw)->n : 1;
        CK(c, cudaMalloc(&c->d_kv, (size_t)c->L * 2 * c->ctx * c->kvd * sizeof(uint16_t)));
        CK(c, cudaMemsetAsync(c->d_kv, 0, (size_t)c->L * 2 * c->ctx * c->kvd * sizeof(uint16_t), c->st));
        CK(c, cudaMalloc(&c->d_h, T * c->H * 4));
        CK(c, cudaMalloc(&c->d_qkv, T * (c->qd + 2 * c->kvd) * 4));
        CK(c, cudaMalloc(&c->d_ao, T * c->qd * 4));
        CK(c, cudaMalloc(&c->d_g, T * c->F * 4));
        CK(c, cudaMalloc(&c->d_u, T * c->F * 4));
        CK(c, cudaMalloc(&c->d_logits, vocab * 4));
        CK(c, cudaMalloc(&c->d_part, (size_t)c->kvh * c->max_splits * G * (c->hd + 2) * 4));
        c->max_chunks = attn_max_chunks(c->ctx);
        CK(c, cudaMalloc(&c->d_cpart, (size_t)c->heads * c->max_chunks * (c->hd + kPartPad) * 4));
        CK(c, cudaMalloc(&c->d_tickets, (size_t)c->kvh * 4));
        CK(c, cudaMemsetAsync(c->d_tickets, 0, (size_t)c->kvh * 4, c->st));
        CK(c, cudaMalloc(&c->d_state, sizeof(DecodeState)));
        CK(c, cudaMemsetAsync(c->d_state, 0, sizeof(DecodeState), c->st));
        CK(c, cudaMalloc(&c->d_out_ids, (size_t)(c->ctx + 1) * 4));
        CK(c, cudaMalloc(&c->d_tokens, (size_t)(c->ctx + 1) * 4));
        CK(c, cudaMalloc(&c->d_chunk_pos, (size_t)(c->ctx / kMaxChunk + 2) * 4));
        const size_t half_tab = (size_t)c->ctx * c->half * 4;
        CK(c, cudaMalloc(&c->d_cos, half_tab));
        CK(c, cudaMalloc(&c->d_sin, half_tab));
        CK(c, cudaMalloc(&c->d_out_norm, (size_t)c->H * 4));
        CK(c, cudaMalloc(&c->d_norms, (size_t)c->L * (2 * c->H + 2 * c->hd) * 4));
    }
    const size_t half_tab = (size_t)c->ctx * c->half * 4;
    CK(c, h2d(c, c->d_cos, sh->rope_cos, half_tab));
    CK(c, h2d(c, c->d_sin, sh->rope_sin, half_tab));
    if (sh->out_norm) CK(c, h2d(c, c->d_out_norm, sh->out_norm, (size_t)c->H * 4));
    c->layers.assign(c->L, Layer());
    for (int i = 0; i < c->L; i++) {
        const hy_fused_layer &fl = sh->layers[i];
        Layer &L = c->layers[i];
        L.q = (HyWeight *)fl.wq; L.k = (HyWeight *)fl.wk; L.v = (HyWeight *)fl.wv; L.o = (HyWeight *)fl.wo;
        L.g = (HyWeight *)fl.wg; L.u = (HyWeight *)fl.wu; L.d = (HyWeight *)fl.wd;
        REQ(c, L.q && L.k && L.v && L.o && L.g && L.u && L.d, "missing layer weight");
        REQ(c, L.q->k == c->H && L.k->k == c->H && L.v->k == c->H && L.o->k == c->qd && L.g->k == c->H &&
                   L.u->k == c->H && L.d->k == c->F,
            "layer weight shapes do not match the model");
        float *base = c->d_norms + (size_t)i * (2 * c->H + 2 * c->hd);
        L.attn_norm = base;
        L.ffn_norm = base + c->H;
        L.q_norm = base + 2 * c->H;
        L.k_norm = base + 2 * c->H + c->hd;
        CK(c, h2d(c, L.attn_norm, fl.attn_norm, (size_t)c->H * 4));
        CK(c, h2d(c, L.ffn_norm, fl.ffn_norm, (size_t)c->H * 4));
        CK(c, h2d(c, L.q_norm, fl.q_norm, (size_t)c->hd * 4));
        CK(c, h2d(c, L.k_norm, fl.k_norm, (size_t)c->hd * 4));
    }
    c->outw = (HyWeight *)sh->outw;
    if (c->outw) REQ(c, c->outw->k == c->H, "LM head shape does not match the model");
    graph_reset(c->g_fwd1);
    graph_reset(c->g_fwd1_logits);
    graph_reset(c->g_dec);
    c->g_dec_vocab = -1;
    c->mega_state = -1;
    CK(c, cudaStreamSynchronize(c->st));
    c->fused = true;
    return true;
}

// Whole-network forward for nt tokens at pos0.. with host h in/out and host
// logits of the last token (reference contract src/device.h:65,
// src/cuda.c:339-421): one H2D, device-resident layers, one D2H, one sync.
bool fused_forward(void *impl, hy_fused_args *a) {
    HyCtx *c = (HyCtx *)impl;
    if (!c || c->broken || !c->fused || !a || !a->h || a->nt < 1 || a->nt > kMaxChunk) return false;
    if (a->pos0 < 0 || a->pos0 + a->nt > c->ctx) return false;
    if (a->want_logits && (!c->outw || !a->logits)) return false;
    REQ(c, c->tp_world == 1, "fused_forward: a tensor-parallel rank holds only a slice of the logits");
    if (cudaSetDevice(c->dev) != cudaSuccess) return false;
    const int nt = a->nt;
    for (int i = 0; i < c->L; i++) {  // the host may pass a fresh layer array; handles must match
        const hy_fused_layer &fl = a->layers[i];
        if ((HyWeight *)fl.wq != c->layers[i].q || (HyWeight *)fl.wd != c->layers[i].d) return false;
    }
    CK(c, cudaMemcpyAsync(c->d_h, a->h, (size_t)nt * c->H * 4, cudaMemcpyHostToDevice, c->st));
    *c->h_pinned_int = a->pos0;
    CK(c, cudaMemcpyAsync(&c->d_state->pos_fwd, c->h_pinned_int, 4, cudaMemcpyHostToDevice, c->st));
    const int *pos_ptr = &c->d_state->pos_fwd;
    if (nt == 1) {
        Graph &g = a->want_logits ? c->g_fwd1_logits : c->g_fwd1;
        if (!g.exec) {
            const bool logits = a->want_logits != 0;
            if (!capture(c, g, [&]() {
                    if (!layers_forward(c, 1, pos_ptr, true)) return false;
                    return !logits || head_forward(c, c->d_h, true, false, true);
                }))
                return false;
        }
        if (!graph_launch(c, g)) return false;
    } else {
        if (!layers_forward(c, nt, pos_ptr, false)) return false;
        if (a->want_logits && !head_forward(c, c->d_h + (size_t)(nt - 1) * c->H, true, false, false)) return false;
    }
    CK(c, cudaMemcpyAsync(a->h, c->d_h, (size_t)nt * c->H * 4, cudaMemcpyDeviceToHost, c->st));
    if (a->want_logits)
        CK(c, cudaMemcpyAsync(a->logits, c->d_logits, (size_t)c->outw->n * 4, cudaMemcpyDeviceToHost, c->st));
    CK(c, cudaStreamSynchronize(c->st));
    return tc_status(c);
}

#include "hy_batch.cuh"

// Failure-detection probe: the bounded waits of the persistent decode kernel
// (grid barrier on its arrival counter) and of the tensor-core GEMM (an
// mbarrier phase) given targets that nothing reaches and a limit of
// limit_ns.  out[0] = what the grid-barrier wait returned (0: gave up),
// out[1] = the error word it raised, out[2] = what the mbarrier wait
// returned.  Nothing traps, faults or hangs: each wait gives up after the
// limit and the kernel returns.
__global__ void wait_probe(MegaSync *sync, unsigned long long limit_ns, int *out) {
    __shared__ __align__(8) uint64_t mb;
    __shared__ int flag;
    MegaArgs a;
    memset(&a, 0, sizeof a);
    a.sync = sync;
    const bool passed = bar_wait(a, gridDim.x + 1, &flag, limit_ns);  // one arrival more than the grid makes
    if (threadIdx.x == 0) {
        out[0] = passed;
        out[1] = ld_relaxed_s32(&sync->err);
        tc_mbar_init(&mb, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    const bool done = tc_mbar_wait(&mb, 0, limit_ns);  // nothing arrives: phase 0 never completes
    if (threadIdx.x == 0) out[2] = done;
}

const hy_device_ops kOps = {destroy_impl, upload, release, matmul, is_software, weight_out, fused_prepare,
                            fused_forward};

}  // namespace

// ==================================================================== C ABI

extern "C" {

HYC_API int hy_cuda_probe(char *out, int cap) {
    int n = 0;
    const int ok = cudaGetDeviceCount(&n) == cudaSuccess && n > 0;
    if (!ok) cudaGetLastError();
    if (out && cap > 0) snprintf(out, (size_t)cap, "%d", ok);
    return ok;
}

HYC_API void *hyc_create(int device, char *info, size_t cap) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n < 1) {
        cudaGetLastError();
        if (info && cap) snprintf(info, cap, "no CUDA device");
        return nullptr;
    }
    if (device < 0 || device >= n) {
        if (info && cap) snprintf(info, cap, "CUDA device %d out of range (%d present)", device, n);
        return nullptr;
    }
    cudaDeviceProp p;
    if (cudaGetDeviceProperties(&p, device) != cudaSuccess || p.major != 10) {
        if (info && cap) snprintf(info, cap, "device %d is not sm_100 (this build targets B200 / sm_100a)", device);
        return nullptr;
    }
    if (cudaSetDevice(device) != cudaSuccess) {
        if (info && cap) snprintf(info, cap, "cudaSetDevice(%d) failed", device);
        return nullptr;
    }
    HyCtx *c = new HyCtx();
    c->dev = device;
    const char *lay = getenv("HYMT2_STQ_LAYOUT");
    c->stq_native = lay && strcmp(lay, "native") == 0;
    c->nsm = p.multiProcessorCount;
    c->l2_bytes = (size_t)p.l2CacheSize;
    if (!init_kernel_attrs(device)) {
        if (info && cap) snprintf(info, cap, "setting kernel shared-memory limits on device %d failed", device);
        delete c;
        return nullptr;
    }
    set_smem(quantize_export);
    if (cudaStreamCreateWithFlags(&c->st, cudaStreamNonBlocking) != cudaSuccess ||
        cudaHostAlloc((void **)&c->h_pinned_int, 4096, cudaHostAllocDefault) != cudaSuccess) {
        if (info && cap) snprintf(info, cap, "stream / pinned allocation failed");
        destroy_impl(c);
        return nullptr;
    }
    if (info && cap) snprintf(info, cap, "%s (sm_%d%d, %d SMs, %.0f GB)", p.name, p.major, p.minor, p.multiProcessorCount,
                              (double)p.totalGlobalMem / 1e9);
    return c;
}

HYC_API const hy_device_ops *hyc_device_ops(void) { return &kOps; }

HYC_API hy_device *hy_cuda_create(const char *pref, char *info, size_t cap) {
    int dev = 0;
    if (pref && pref[0] >= '0' && pref[0] <= '9') dev = atoi(pref);
    if (!hy_device_wrap) {
        if (info && cap) snprintf(info, cap, "host device layer not linked (standalone library: use hyc_create)");
        return nullptr;
    }
    void *impl = hyc_create(dev, info, cap);
    if (!impl) return nullptr;
    hy_device *d = hy_device_wrap(HY_DEV_CUDA, "cuda", impl, &kOps, false);
    if (!d) destroy_impl(impl);
    return d;
}

HYC_API int hyc_last_error(void *impl, char *out, int cap) {
    HyCtx *c = (HyCtx *)impl;
    if (!out || cap <= 0) return 0;
    snprintf(out, (size_t)cap, "%s", c ? c->err : "null handle");
    return (int)strlen(out);
}

HYC_API void *hyc_stream(void *impl) { return impl ? (void *)((HyCtx *)impl)->st : nullptr; }

HYC_API int hyc_sync(void *impl) {
    HyCtx *c = (HyCtx *)impl;
    if (!c) return -1;
    cudaError_t e = cudaStreamSynchronize(c->st);
    if (e != cudaSuccess) {
        fail(c, "cudaStreamSynchronize", e);
        return -1;
    }
    return mega_status(c) && tc_status(c) && tp_status(c) ? 0 : -1;
}

HYC_API int hyc_set_embedding(void *impl, hy_dweight *embd) {
    HyCtx *c = (HyCtx *)impl;
    if (!c || !embd) return -1;
    c->embd = (HyWeight *)embd;
    graph_reset(c->g_dec);
    c->g_dec_vocab = -1;
    c->mega_state = -1;
    return 0;
}

HYC_API int hyc_set_stq_layout(void *impl, int native) {
    HyCtx *c = (HyCtx *)impl;
    if (!c) return -1;
    c->stq_native = native != 0;
    return 0;
}

HYC_API int hyc_set_tc(void *impl, int on) {
    HyCtx *c = (HyCtx *)impl;
    if (!c) return -1;
    c->tc_on = on != 0;
    return 0;
}

HYC_API int hyc_tc_test(void *impl, hy_dweight *hw, int act, const float *x, const float *x2, const float *norm_w,
                        float eps, int nt, float *out) {
    HyCtx *c = (HyCtx *)impl;
    HyWeight *w = (HyWeight *)hw;
    if (!c || c->broken || !w || !tc_planes(w->fmt) || nt < 1 || nt > kMaxChunk || act < ACT_VEC || act > ACT_SILU ||
        (act == ACT_NORM && !norm_w) || (act == ACT_SILU && !x2))
        return -1;
    if (cudaSetDevice(c->dev) != cudaSuccess) return -1;
    const int K = w->k;
    float *dx = nullptr, *dx2 = nullptr, *dn = nullptr, *dout = nullptr;
    bool ok = cudaMalloc(&dx, (size_t)nt * K * 4) == cudaSuccess && cudaMalloc(&dx2, (size_t)nt * K * 4) == cudaSuccess &&
              cudaMalloc(&dn, (size_t)K * 4) == cudaSuccess && cudaMalloc(&dout, (size_t)nt * w->n * 4) == cudaSuccess &&
              h2d(c, dx, x, (size_t)nt * K * 4) == cudaSuccess &&
              (!x2 || h2d(c, dx2, x2, (size_t)nt * K * 4) == cudaSuccess) &&
              (!norm_w || h2d(c, dn, norm_w, (size_t)K * 4) == cudaSuccess);
    if (ok) {
        GemvArgs pro = gemv_args(nt, K);
        pro.act = act;
        pro.x = dx;
        pro.x2 = dx2;
        pro.ldx = K;
        pro.norm_w = dn;
        pro.eps = eps;
        HyWeight *ws[1] = {w};
        float *outs[1] = {dout};
        const int lds[1] = {w->n};
        ok = tc_linear(c, pro, nt, ws, outs, lds, 1, 0, false) &&
             cudaMemcpyAsync(out, dout, (size_t)nt * w->n * 4, cudaMemcpyDeviceToHost, c->st) == cudaSuccess &&
             cudaStreamSynchronize(c->st) == cudaSuccess && tc_status(c);
    }
    cudaFree(dx);
    cudaFree(dx2);
    cudaFree(dn);
    cudaFree(dout);
    return ok ? 0 : -1;
}

HYC_API int hyc_tc_block_ints(void *impl, hy_dweight *hw, const q8k_block *xq, int nt, int32_t *out) {
    HyCtx *c = (HyCtx *)impl;
    HyWeight *w = (HyWeight *)hw;
    if (!c || c->broken || !w || !xq || !out || !tc_planes(w->fmt) || w->k % 256 || nt < 1 || nt > 65536) return -1;
    if (cudaSetDevice(c->dev) != cudaSuccess) return -1;
    const int P = tc_planes(w->fmt), nb = w->nb, per = P == 3 ? 2 * nb : nb, tpad = (nt + kTcM - 1) / kTcM * kTcM;
    if (nt > c->max_tokens) c->max_tokens = nt;  // the tiled activation scratch grows to nt tokens
    if (!tc_scratch(c, w->k) || !tc_weight(c, w)) return -1;
    q8k_block *dxq = nullptr;
    int32_t *dints = nullptr;
    float *dout = nullptr;
    const size_t xb = (size_t)nt * nb * sizeof(q8k_block), ib = (size_t)nt * w->n * per * 4;
    bool ok = cudaMalloc(&dxq, xb) == cudaSuccess && cudaMalloc(&dints, ib) == cudaSuccess &&
              cudaMalloc(&dout, (size_t)nt * w->n * 4) == cudaSuccess && h2d(c, dxq, xq, xb) == cudaSuccess;
    if (ok) {
        const long long units = (long long)tpad * nb * 16;
        tc_from_q8k<<<(unsigned)((units + 255) / 256), 256, 0, c->st>>>(dxq, nt, tpad, nb, c->d_tca, c->d_tcad);
        ok = cudaGetLastError() == cudaSuccess;
    }
    if (ok) {
        TcArgs ta;
        memset(&ta, 0, sizeof ta);
        ta.a = c->d_tca;
        ta.ad = c->d_tcad;
        ta.T = nt;
        ta.nb = nb;
        ta.err = c->d_tcerr;
        ta.nw = 1;
        ta.w[0] = w->tc_w;
        ta.ws[0] = w->tc_ws;
        ta.out[0] = dout;
        ta.ldo[0] = w->n;
        ta.N[0] = w->n;
        ta.ints = dints;
        HyWeight *ws[1] = {w};
        ok = tc_gemm_launch<true>(c, ta, P, ws, 1, false) &&
             cudaMemcpyAsync(out, dints, ib, cudaMemcpyDeviceToHost, c->st) == cudaSuccess &&
             cudaStreamSynchronize(c->st) == cudaSuccess && tc_status(c);
    }
    cudaFree(dxq);
    cudaFree(dints);
    cudaFree(dout);
    return ok ? per : -1;
}

HYC_API int hyc_batch_prepare(void *impl, int slots, int slot_ctx, int max_tokens, int max_out) {
    HyCtx *c = (HyCtx *)impl;
    if (!c || c->broken || c->tp_world > 1 || cudaSetDevice(c->dev) != cudaSuccess) return -1;
    return batch_prepare(c, slots, slot_ctx, max_tokens, max_out) ? 0 : -1;
}

HYC_API int hyc_batch_forward(void *impl, const int *tokens, const int *tok_slot, const int *tok_pos, int nt,
                              const int *out_rows, int nout, int vocab_out, int *out_ids, float *logits) {
    HyCtx *c = (HyCtx *)impl;
    if (!c || c->broken || !c->bat || !tokens || !tok_slot || !tok_pos || cudaSetDevice(c->dev) != cudaSuccess)
        return -1;
    Batch &b = *c->bat;
    if (nt < 1 || nt > b.max_tokens || nout < 0 || nout > b.max_out || (nout > 0 && (!out_rows || !out_ids))) return -1;
    for (int t = 0; t < nt; t++)
        if (tok_slot[t] < 0 || tok_slot[t] >= b.slots || tok_pos[t] < 0 || tok_pos[t] >= b.slot_ctx) return -1;
    for (int i = 0; i < nout; i++)
        if (out_rows[i] < 0 || out_rows[i] >= nt) return -1;
    const int vo = vocab_out > 0 && vocab_out <= c->outw->n ? vocab_out : c->outw->n;
    const size_t T = (size_t)b.max_tokens;
    memcpy(b.h_in, tokens, (size_t)nt * 4);
    memcpy(b.h_in + T, tok_slot, (size_t)nt * 4);
    memcpy(b.h_in + 2 * T, tok_pos, (size_t)nt * 4);
    if (nout > 0) memcpy(b.h_in + 3 * T, out_rows, (size_t)nout * 4);
    if (!batch_upload(c, nt, nout) || !batch_run(c, nt, nout, vo)) return -1;
    if (nout > 0) {
        if (cudaMemcpyAsync(b.h_ids, b.d_ids, (size_t)nout * 4, cudaMemcpyDeviceToHost, c->st) != cudaSuccess) return -1;
        if (logits && cudaMemcpyAsync(logits, b.logits, (size_t)nout * c->outw->n * 4, cudaMemcpyDeviceToHost, c->st) !=
                          cudaSuccess)
            return -1;
    }
    if (cudaStreamSynchronize(c->st) != cudaSuccess) {
        fail(c, "batch_forward", cudaGetLastError());
        return -1;
    }
    if (!tc_status(c)) return -1;
    if (nout > 0) memcpy(out_ids, b.h_ids, (size_t)nout * 4);
    return 0;
}

HYC_API int hyc_batch_kv_copy(void *impl, int src_slot, int dst_slot, int npos) {
    HyCtx *c = (HyCtx *)impl;
    if (!c || c->broken || !c->bat || cudaSetDevice(c->dev) != cudaSuccess) return -1;
    const Batch &b = *c->bat;
    if (src_slot < 0 || src_slot >= b.slots || dst_slot < 0 || dst_slot >= b.slots || npos < 0 || npos > b.slot_ctx)
        return -1;
    return kv_copy(c, src_slot, dst_slot, npos) && cudaStreamSynchronize(c->st) == cudaSuccess ? 0 : -1;
}

HYC_API int hyc_batch_kv_read(void *impl, int slot, int layer, int npos, uint16_t *k, uint16_t *v) {
    HyCtx *c = (HyCtx *)impl;
    if (!c || c->broken || !c->bat || !k || !v || cudaSetDevice(c->dev) != cudaSuccess) return -1;
    const Batch &b = *c->bat;
    if (slot < 0 || slot >= b.slots || layer < 0 || layer >= c->L || npos < 1 || npos > b.slot_ctx) return -1;
    // page by page through the slot's row of the page table
    for (int j = 0; j * kPageRows < npos; j++) {
        const int n = npos - j * kPageRows < kPageRows ? npos - j * kPageRows : kPageRows;
        const uint16_t *kc = b.kv + (size_t)layer * b.layer_stride(c) +
                             (size_t)b.h_pages[slot * b.page_max + j] * b.page_stride(c);
        const uint16_t *vc = kc + (size_t)kPageRows * c->kvd;
        const size_t o = (size_t)j * kPageRows * c->kvd, bytes = (size_t)n * c->kvd * 2;
        if (cudaMemcpyAsync(k + o, kc, bytes, cudaMemcpyDeviceToHost, c->st) != cudaSuccess ||
            cudaMemcpyAsync(v + o, vc, bytes, cudaMemcpyDeviceToHost, c->st) != cudaSuccess)
            return -1;
    }
    return cudaStreamSynchronize(c->st) == cudaSuccess ? 0 : -1;
}

HYC_API int hyc_serve(void *impl, const int *prompts, const int *prompt_off, int nreq, int max_new,
                      const int *stop_ids, int n_stop, int vocab_out, int step_tokens, int *out_ids, int *out_len,
                      hyc_serve_stats *stats) {
    HyCtx *c = (HyCtx *)impl;
    if (!c || c->broken || !c->bat || !prompts || !prompt_off || nreq < 0 || !out_ids || !out_len || n_stop < 0 ||
        n_stop > 16 || (n_stop > 0 && !stop_ids) || cudaSetDevice(c->dev) != cudaSuccess)
        return -1;
    hyc_serve_stats local;
    const int vo = vocab_out > 0 && vocab_out <= c->outw->n ? vocab_out : c->outw->n;
    return serve_run(c, prompts, prompt_off, nreq, max_new, stop_ids, n_stop, vo, step_tokens, out_ids, out_len,
                     stats ? stats : &local)
               ? 0
               : -1;
}

HYC_API int hyc_wait_probe(void *impl, unsigned long long limit_ns, int *out) {
    HyCtx *c = (HyCtx *)impl;
    if (!c || c->broken || !out || limit_ns == 0 || limit_ns > 1000000000ull || cudaSetDevice(c->dev) != cudaSuccess)
        return -1;
    MegaSync *d_sync = nullptr;
    int *d_out = nullptr;
    bool ok = cudaMalloc(&d_sync, sizeof(MegaSync)) == cudaSuccess && cudaMalloc(&d_out, 3 * sizeof(int)) == cudaSuccess &&
              cudaMemsetAsync(d_sync, 0, sizeof(MegaSync), c->st) == cudaSuccess &&
              launch(c, wait_probe, dim3(1), dim3(32), 0, false, d_sync, limit_ns, d_out) &&
              cudaMemcpyAsync(out, d_out, 3 * sizeof(int), cudaMemcpyDeviceToHost, c->st) == cudaSuccess &&
              cudaStreamSynchronize(c->st) == cudaSuccess;
    cudaFree(d_sync);
    cudaFree(d_out);
    return ok ? 0 : -1;
}

HYC_API int hyc_set_decode_mode(void *impl, int mode) {
    HyCtx *c = (HyCtx *)impl;
    if (!c || mode < 0 || mode > 1) return -1;
    c->decode_mode = mode;
    return 0;
}

HYC_API int hyc_decode_path(void *impl, char *why, int cap) {
    HyCtx *c = (HyCtx *)impl;
    if (!c || c->broken || !c->fused) return -1;
    const int mega = use_mega(c) ? 1 : 0;
    if (why && cap > 0)
        snprintf(why, (size_t)cap, "%s", mega ? "persistent kernel"
                                              : (c->decode_mode == 1 ? "graph (requested)" : c->mega_why));
    return mega;
}

HYC_API long long hyc_launch_count(void *impl) { return impl ? ((HyCtx *)impl)->launches : 0; }

HYC_API void *hyc_host_alloc(size_t bytes) {
    void *p = nullptr;
    return cudaHostAlloc(&p, bytes, cudaHostAllocDefault) == cudaSuccess ? p : nullptr;
}
HYC_API void hyc_host_free(void *p) {
    if (p) cudaFreeHost(p);
}

HYC_API int hyc_decode_begin(void *impl, const int *prompt, int n, int keep, int max_new, const int *stop_ids,
                             int n_stop, int vocab_out) {
    HyCtx *c = (HyCtx *)impl;
    if (!c || c->broken || !c->fused || !c->embd || !c->outw || !prompt) return -1;
    if (n < 1 || keep < 0 || keep >= n || max_new < 1 || n + max_new > c->ctx || n_stop < 0 || n_stop > 16) return -1;
    if (cudaSetDevice(c->dev) != cudaSuccess) return -1;
    // rows below vocab_out (of the whole vocabulary: a tensor-parallel rank's head holds rows tp_vocab0 ..)
    // compete for the argmax
    c->vocab_out = vocab_out > 0 ? vocab_out : c->outw->n + c->tp_vocab0;
    DecodeState s;
    memset(&s, 0, sizeof s);
    s.pos = n - 1;
    s.cap = max_new;
    s.n_stop = n_stop;
    for (int i = 0; i < n_stop; i++) s.stop_ids[i] = stop_ids[i];
    std::vector<int> cp;
    for (int p0 = keep; p0 < n; p0 += kMaxChunk) cp.push_back(p0);
    if (cudaMemcpyAsync(c->d_state, &s, sizeof s, cudaMemcpyHostToDevice, c->st) != cudaSuccess ||
        cudaMemcpyAsync(c->d_tokens, prompt + keep, (size_t)(n - keep) * 4, cudaMemcpyHostToDevice, c->st) != cudaSuccess ||
        cudaMemcpyAsync(c->d_chunk_pos, cp.data(), cp.size() * 4, cudaMemcpyHostToDevice, c->st) != cudaSuccess) {
        fail(c, "decode_begin copies", cudaErrorUnknown);
        return -1;
    }
    for (size_t i = 0; i < cp.size(); i++) {
        const int p0 = cp[i], nt = (n - p0) < kMaxChunk ? (n - p0) : kMaxChunk;
        if (!launch(c, embed_rows, dim3(nt), dim3(256), 0, false, desc(c->embd, nullptr, 0),
                    (const int *)(c->d_tokens + (p0 - keep)), c->d_h, -1))
            return -1;
        if (!layers_forward(c, nt, c->d_chunk_pos + i, false)) return -1;
        if (i + 1 == cp.size()) {
            if (!head_forward(c, c->d_h + (size_t)(nt - 1) * c->H, false, true, false)) return -1;
            if (!launch(c, decode_finalize, dim3(1), dim3(32), 0, false, c->d_state, c->d_out_ids, -1)) return -1;
        }
    }
    // the copies above were ordered before the launches; the graph for
    // single-token steps is built once per vocab_out when it is the decode path
    if (!use_mega(c) && !build_decode_graph(c)) return -1;
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        fail(c, "decode_begin", e);
        return -1;
    }
    return 0;
}

HYC_API int hyc_decode_steps(void *impl, int steps) {
    HyCtx *c = (HyCtx *)impl;
    if (!c || c->broken || !c->fused || steps < 0) return -1;
    return decode_run(c, steps) ? 0 : -1;
}

HYC_API int hyc_decode_steps_host(void *impl, int steps, int *tok_io) {
    HyCtx *c = (HyCtx *)impl;
    if (!c || c->broken || !c->fused || !tok_io || steps < 0) return -1;
    if (cudaMemcpyAsync(&tok_io[0], &c->d_state->tok, 4, cudaMemcpyDeviceToHost, c->st) != cudaSuccess) return -1;
    for (int i = 0; i < steps; i++) {
        if (cudaMemcpyAsync(&c->d_state->tok, &tok_io[i], 4, cudaMemcpyHostToDevice, c->st) != cudaSuccess) return -1;
        if (!decode_run(c, 1)) return -1;
        if (cudaMemcpyAsync(&tok_io[i + 1], &c->d_state->tok, 4, cudaMemcpyDeviceToHost, c->st) != cudaSuccess) return -1;
    }
    return 0;
}

HYC_API int hyc_decode_resident(void *impl, int max_steps, int *io, unsigned long long limit_ns) {
    HyCtx *c = (HyCtx *)impl;
    if (!c || c->broken || !c->fused || !io || max_steps < 1) return -1;
    if (cudaSetDevice(c->dev) != cudaSuccess) return -1;
    if (!use_mega(c)) {
        snprintf(c->err, sizeof c->err, "resident decode needs the persistent kernel: %s",
                 c->decode_mode == 1 ? "graph requested" : c->mega_why);
        return -1;
    }
    int *dio = nullptr;
    if (cudaHostGetDevicePointer((void **)&dio, io, 0) != cudaSuccess || !dio) {
        cudaGetLastError();
        snprintf(c->err, sizeof c->err, "resident decode: io is not pinned host memory (hyc_host_alloc)");
        return -1;
    }
    ((volatile int *)io)[2] = 0;
    std::atomic_thread_fence(std::memory_order_seq_cst);
    c->host_io = dio;
    c->host_limit_ns = limit_ns == 0 ? kMegaWaitNs : (limit_ns < 10000000000ull ? limit_ns : 10000000000ull);
    const bool ok = mega_launch(c, max_steps);
    c->host_io = nullptr;
    return ok ? 0 : -1;
}

HYC_API int hyc_resident_go(int *io, int step, int tok) {
    if (!io) return -1;
    volatile int *v = io;
    v[1] = tok;
    std::atomic_thread_fence(std::memory_order_seq_cst);
    v[0] = step < 0 ? -1 : step + 1;
    return 0;
}

HYC_API int hyc_resident_wait(const int *io, int step, int *tok, unsigned long long limit_ns) {
    if (!io || !tok || step < 0) return -1;
    const volatile int *v = io;
    const auto t0 = std::chrono::steady_clock::now();
    for (unsigned it = 0;; it++) {
        const int d = v[2];
        if (d < 0) return -1;
        if (d >= step + 1) break;
        if ((it & 1023) == 1023 &&
            (unsigned long long)std::chrono::duration_cast<std::chrono::nanoseconds>(
                std::chrono::steady_clock::now() - t0).count() > limit_ns)
            return -2;
    }
    std::atomic_thread_fence(std::memory_order_seq_cst);
    *tok = v[3];
    return 0;
}

HYC_API int hyc_decode_read(void *impl, int *out_ids, int cap) {
    HyCtx *c = (HyCtx *)impl;
    if (!c || c->broken || !c->fused) return -1;
    if (!mega_status(c) || !tc_status(c) || !tp_status(c)) return -1;
    DecodeState s;
    if (cudaMemcpyAsync(&s, c->d_state, sizeof s, cudaMemcpyDeviceToHost, c->st) != cudaSuccess ||
        cudaStreamSynchronize(c->st) != cudaSuccess) {
        fail(c, "decode_read", cudaErrorUnknown);
        return -1;
    }
    int n = s.step < s.cap ? s.step : s.cap;
    if (n > cap) n = cap;
    if (n > 0 && out_ids) {
        if (d2h(c, out_ids, c->d_out_ids, (size_t)n * 4) != cudaSuccess) return -1;
        // truncate after the first stop id, as the host loop breaks there
        for (int i = 0; i < n; i++)
            for (int j = 0; j < s.n_stop; j++)
                if (out_ids[i] == s.stop_ids[j]) return i;
    }
    return n;
}

HYC_API int hyc_decode_rewind(void *impl, int pos, int tok) {
    HyCtx *c = (HyCtx *)impl;
    if (!c || c->broken || !c->fused || pos < 0 || pos >= c->ctx) return -1;
    // tok and pos are adjacent ints in DecodeState; the values go through a
    // ring of pinned slots so the copy can stay asynchronous
    int *slot = c->h_pinned_int + 2 + 2 * (c->rewind_slot++ % 500);
    slot[0] = tok;
    slot[1] = pos;
    if (cudaMemcpyAsync(&c->d_state->tok, slot, 8, cudaMemcpyHostToDevice, c->st) != cudaSuccess) return -1;
    return 0;
}

HYC_API int hyc_generate(void *impl, const int *prompt, int n, int keep, int max_new, const int *stop_ids, int n_stop,
                         int vocab_out, int *out_ids) {
    if (hyc_decode_begin(impl, prompt, n, keep, max_new, stop_ids, n_stop, vocab_out) != 0) return -1;
    if (max_new > 1 && hyc_decode_steps(impl, max_new - 1) != 0) return -1;
    return hyc_decode_read(impl, out_ids, max_new);
}

HYC_API int hyc_quantize_q8k(void *impl, const float *x, int k, int nt, q8k_block *y) {
    HyCtx *c = (HyCtx *)impl;
    if (!c || c->broken || !x || !y || k <= 0 || k % 256 || nt < 1 || nt > 16) return -1;
    if (cudaSetDevice(c->dev) != cudaSuccess) return -1;
    const size_t xb = (size_t)nt * k * 4, yb = (size_t)nt * (k / 256) * sizeof(q8k_block);
    if (!ensure_buf(c, (void **)&c->d_x32, &c->x32_cap, xb) || !ensure_buf(c, (void **)&c->d_xq, &c->xq_cap, yb)) return -1;
    if (cudaMemcpyAsync(c->d_x32, x, xb, cudaMemcpyHostToDevice, c->st) != cudaSuccess) return -1;
    GemvArgs a = gemv_args(nt, k);
    a.act = ACT_VEC;
    a.x = c->d_x32;
    a.ldx = k;
    if (!launch(c, quantize_export, dim3(1), dim3(kGemvThreads), q8_smem_bytes(16, k), false, a, c->d_xq)) return -1;
    if (cudaMemcpyAsync(y, c->d_xq, yb, cudaMemcpyDeviceToHost, c->st) != cudaSuccess ||
        cudaStreamSynchronize(c->st) != cudaSuccess)
        return fail(c, "quantize", cudaErrorUnknown) ? 0 : -1;
    return 0;
}

HYC_API int hyc_block_ints(void *impl, hy_dweight *hw, const q8k_block *xq, int nt, int32_t *out) {
    HyCtx *c = (HyCtx *)impl;
    HyWeight *w = (HyWeight *)hw;
    if (!c || c->broken || !w || !xq || !out || nt < 1 || nt > 16 || !is_q8_fmt(w->fmt)) return -1;
    if (cudaSetDevice(c->dev) != cudaSuccess || !ensure_out(w)) return -1;
    const int per = w->fmt == FMT_Q4K ? 2 * w->nb : w->nb;
    const size_t xb = (size_t)nt * w->nb * sizeof(q8k_block), ib = (size_t)nt * w->n * per * 4;
    if (!ensure_buf(c, (void **)&c->d_xq, &c->xq_cap, xb) || !ensure_buf(c, (void **)&c->d_ints, &c->ints_cap, ib))
        return -1;
    if (cudaMemcpyAsync(c->d_xq, xq, xb, cudaMemcpyHostToDevice, c->st) != cudaSuccess) return -1;
    GemvArgs a = gemv_args(nt, w->k);
    a.act = ACT_Q8K;
    a.xq = c->d_xq;
    a.epi = EPI_STORE;
    a.nw = 1;
    a.rows_total = w->n;
    a.w[0] = desc(w, w->d_out, w->n);
    a.ints = c->d_ints;
    if (!gemv_launch(c, a, false, 1)) return -1;
    if (cudaMemcpyAsync(out, c->d_ints, ib, cudaMemcpyDeviceToHost, c->st) != cudaSuccess ||
        cudaStreamSynchronize(c->st) != cudaSuccess)
        return -1;
    return per;
}

HYC_API int hyc_matmul_f32(void *impl, hy_dweight *hw, const float *x, int nt, float *out) {
    HyCtx *c = (HyCtx *)impl;
    HyWeight *w = (HyWeight *)hw;
    if (!c || c->broken || !w || !x || !out || nt < 1 || nt > MAX_BATCH) return -1;
    if (cudaSetDevice(c->dev) != cudaSuccess || !ensure_out(w)) return -1;
    const size_t xb = (size_t)nt * w->k * 4;
    if (!ensure_buf(c, (void **)&c->d_x32, &c->x32_cap, xb)) return -1;
    if (cudaMemcpyAsync(c->d_x32, x, xb, cudaMemcpyHostToDevice, c->st) != cudaSuccess) return -1;
    GemvArgs a = gemv_args(nt, w->k);
    a.act = ACT_VEC;  // Q8_K formats quantise on the device, fp32 formats use x as is
    a.x = c->d_x32;
    a.ldx = w->k;
    a.epi = EPI_STORE;
    a.nw = 1;
    a.rows_total = w->n;
    a.w[0] = desc(w, w->d_out, w->n);
    if (!run_gemv(c, a, false)) return -1;
    if (cudaMemcpyAsync(out, w->d_out, (size_t)nt * w->n * 4, cudaMemcpyDeviceToHost, c->st) != cudaSuccess ||
        cudaStreamSynchronize(c->st) != cudaSuccess)
        return -1;
    return 0;
}

HYC_API int hyc_dequant_row(void *impl, hy_dweight *hw, int row, float *dst) {
    HyCtx *c = (HyCtx *)impl;
    HyWeight *w = (HyWeight *)hw;
    if (!c || c->broken || !w || !dst || row < 0 || row >= w->n) return -1;
    if (cudaSetDevice(c->dev) != cudaSuccess) return -1;
    if (!ensure_buf(c, (void **)&c->d_x32, &c->x32_cap, (size_t)w->k * 4)) return -1;
    if (!launch(c, dequant_row_kernel, dim3(1), dim3(256), 0, false, desc(w, nullptr, 0), row, c->d_x32)) return -1;
    if (cudaMemcpyAsync(dst, c->d_x32, (size_t)w->k * 4, cudaMemcpyDeviceToHost, c->st) != cudaSuccess ||
        cudaStreamSynchronize(c->st) != cudaSuccess)
        return -1;
    return 0;
}

HYC_API int hyc_kv_read(void *impl, int layer, int npos, uint16_t *k, uint16_t *v) {
    HyCtx *c = (HyCtx *)impl;
    if (!c || c->broken || !c->fused || layer < 0 || layer >= c->L || npos < 0 || npos > c->ctx) return -1;
    const uint16_t *kc = c->d_kv + (size_t)layer * 2 * c->ctx * c->kvd, *vc = kc + (size_t)c->ctx * c->kvd;
    if (cudaMemcpyAsync(k, kc, (size_t)npos * c->kvd * 2, cudaMemcpyDeviceToHost, c->st) != cudaSuccess ||
        cudaMemcpyAsync(v, vc, (size_t)npos * c->kvd * 2, cudaMemcpyDeviceToHost, c->st) != cudaSuccess ||
        cudaStreamSynchronize(c->st) != cudaSuccess)
        return -1;
    return 0;
}

// Enqueue `iters` launches of one hot operation of the fused decode step
// (no synchronisation) so a caller can time it with events on hyc_stream:
//   0 LM-head GEMV + argmax    1 q|k|v GEMV     2 gate|up GEMV
//   3 down GEMV (+SiLU prologue, +residual)     4 o_proj GEMV (+residual)
//   5 decode attention at the current decode position
// Layer weights rotate over all layers so they stream from HBM, not L2.
HYC_API int hyc_bench_op(void *impl, int op, int iters) {
    HyCtx *c = (HyCtx *)impl;
    if (!c || c->broken || !c->fused || iters < 1) return -1;
    if (op == 0 && c->d_state && c->outw) {
        for (int i = 0; i < iters; i++)
            if (!head_forward(c, c->d_h, false, true, true)) return -1;
        return 0;
    }
    for (int i = 0; i < iters; i++) {
        const Layer &L = c->layers[i % c->L];
        const int qkv_ld = c->qd + 2 * c->kvd;
        bool ok = true;
        if (op == 1) {
            HyWeight *ws[3] = {L.q, L.k, L.v};
            float *outs[3] = {c->d_qkv, c->d_qkv + c->qd, c->d_qkv + c->qd + c->kvd};
            int lds[3] = {qkv_ld, qkv_ld, qkv_ld};
            GemvArgs a = gemv_args(1, c->H);
            a.act = ACT_NORM;
            a.x = c->d_h;
            a.ldx = c->H;
            a.norm_w = L.attn_norm;
            a.eps = c->eps;
            a.epi = EPI_STORE;
            ok = run_multi(c, ws, outs, lds, 3, a, true);
        } else if (op == 2) {
            ok = gateup_forward(c, fwd_single(c, &c->d_state->pos), L, 1, true);
        } else if (op == 3) {
            ok = down_forward(c, fwd_single(c, &c->d_state->pos), L, 1, true, c->d_tmp_h());
        } else if (op == 4) {
            GemvArgs a = gemv_args(1, L.o->k);
            a.act = ACT_VEC;
            a.x = c->d_ao;
            a.ldx = L.o->k;
            a.epi = EPI_ADD;
            a.nw = 1;
            a.rows_total = L.o->n;
            a.w[0] = desc(L.o, c->d_tmp_h(), c->H);
            ok = run_gemv(c, a, true);
        } else if (op == 5) {
            AttnArgs aa;
            memset(&aa, 0, sizeof aa);
            aa.qkv = c->d_qkv;
            aa.qkv_ld = qkv_ld;
            aa.kc = c->d_kv + (size_t)(i % c->L) * 2 * c->ctx * c->kvd;
            aa.vc = aa.kc + (size_t)c->ctx * c->kvd;
            aa.q_norm = L.q_norm;
            aa.k_norm = L.k_norm;
            aa.rope_cos = c->d_cos;
            aa.rope_sin = c->d_sin;
            aa.pos_ptr = &c->d_state->pos;
            aa.nt = 1;
            aa.heads = c->heads;
            aa.kv_heads = c->kvh;
            aa.hd = c->hd;
            aa.kvdim = c->kvd;
            aa.qdim = c->qd;
            aa.ctx = c->ctx;
            aa.half = c->half;
            aa.eps = c->eps;
            aa.scale = 1.0f / sqrtf((float)c->hd);
            aa.ao = c->d_ao;
            aa.part = c->d_part;
        aa.cpart = c->d_cpart;
        aa.max_chunks = c->max_chunks;
        aa.units = c->nsm;
            aa.tickets = c->d_tickets;
            aa.split_len = kSplitLen;
            aa.max_splits = c->max_splits;
            ok = attention(c, aa, 1, true);
        } else {
            return -1;
        }
        if (!ok) return -1;
    }
    return 0;
}

// One GEMV with a fused prologue on host inputs (act 1 copy, 2 RMSNorm*w,
// 3 SiLU(x)*x2); epi_add != 0 adds into the host `out` it is given.
HYC_API int hyc_gemv_test(void *impl, hy_dweight *hw, int act, const float *x, const float *x2, const float *norm_w,
                          float eps, int nt, int epi_add, float *out) {
    HyCtx *c = (HyCtx *)impl;
    HyWeight *w = (HyWeight *)hw;
    if (!c || c->broken || !w || !x || !out || nt < 1 || nt > MAX_BATCH || act < 1 || act > 3) return -1;
    if ((act == 2 && !norm_w) || (act == 3 && !x2)) return -1;
    if (cudaSetDevice(c->dev) != cudaSuccess || !ensure_out(w)) return -1;
    const size_t xb = (size_t)nt * w->k * 4;
    float *dx = nullptr, *dx2 = nullptr, *dn = nullptr;
    bool ok = cudaMalloc(&dx, xb) == cudaSuccess && cudaMalloc(&dx2, xb) == cudaSuccess &&
              cudaMalloc(&dn, (size_t)w->k * 4) == cudaSuccess &&
              h2d(c, dx, x, xb) == cudaSuccess &&
              (!x2 || h2d(c, dx2, x2, xb) == cudaSuccess) &&
              (!norm_w || h2d(c, dn, norm_w, (size_t)w->k * 4) == cudaSuccess) &&
              (!epi_add || h2d(c, w->d_out, out, (size_t)nt * w->n * 4) == cudaSuccess);
    if (ok) {
        GemvArgs a = gemv_args(nt, w->k);
        a.act = act;
        a.x = dx;
        a.x2 = dx2;
        a.ldx = w->k;
        a.norm_w = dn;
        a.eps = eps;
        a.epi = epi_add ? EPI_ADD : EPI_STORE;
        a.nw = 1;
        a.rows_total = w->n;
        a.w[0] = desc(w, w->d_out, w->n);
        ok = run_gemv(c, a, false) &&
             cudaMemcpyAsync(out, w->d_out, (size_t)nt * w->n * 4, cudaMemcpyDeviceToHost, c->st) == cudaSuccess &&
             cudaStreamSynchronize(c->st) == cudaSuccess;
    }
    cudaFree(dx);
    cudaFree(dx2);
    cudaFree(dn);
    return ok ? 0 : -1;
}

// Up to three weights sharing one activation, merged into launches the way
// the fused layer merges q|k|v and gate|up; outs[i] receive [nt][n_i].
HYC_API int hyc_gemv_multi_test(void *impl, hy_dweight *const *hws, int cnt, int act, const float *x,
                                const float *norm_w, float eps, int nt, float *const *outs) {
    HyCtx *c = (HyCtx *)impl;
    if (!c || c->broken || !hws || cnt < 1 || cnt > 3 || !x || nt < 1 || nt > MAX_BATCH || act < 1 || act > 2) return -1;
    if (act == 2 && !norm_w) return -1;
    HyWeight *ws[3];
    float *douts[3] = {nullptr, nullptr, nullptr};
    int lds[3];
    for (int i = 0; i < cnt; i++) {
        ws[i] = (HyWeight *)hws[i];
        if (!ws[i] || ws[i]->k != ws[0]->k || !ensure_out(ws[i])) return -1;
        douts[i] = ws[i]->d_out;
        lds[i] = ws[i]->n;
    }
    const int K = ws[0]->k;
    float *dx = nullptr, *dn = nullptr;
    bool ok = cudaMalloc(&dx, (size_t)nt * K * 4) == cudaSuccess && cudaMalloc(&dn, (size_t)K * 4) == cudaSuccess &&
              h2d(c, dx, x, (size_t)nt * K * 4) == cudaSuccess &&
              (!norm_w || h2d(c, dn, norm_w, (size_t)K * 4) == cudaSuccess);
    if (ok) {
        GemvArgs a = gemv_args(nt, K);
        a.act = act;
        a.x = dx;
        a.ldx = K;
        a.norm_w = dn;
        a.eps = eps;
        a.epi = EPI_STORE;
        ok = run_multi(c, ws, douts, lds, cnt, a, false);
        for (int i = 0; ok && i < cnt; i++)
            ok = cudaMemcpyAsync(outs[i], douts[i], (size_t)nt * ws[i]->n * 4, cudaMemcpyDeviceToHost, c->st) ==
                 cudaSuccess;
        ok = ok && cudaStreamSynchronize(c->st) == cudaSuccess;
    }
    cudaFree(dx);
    cudaFree(dn);
    return ok ? 0 : -1;
}

// Attention with its fused rope / q-k norm / bf16 KV-store prologue on host
// buffers: qkv [nt][q|k|v] pre-rope, kc/vc [ctx][kvdim] in/out, ao [nt][qdim].
// nt == 1 runs the decode kernel (split-KV), nt > 1 the prefill pair.
HYC_API int hyc_attention_test(void *impl, int heads, int kv_heads, int hdim, int ctx, int nt, int pos0, float eps,
                               const float *qkv, uint16_t *kc, uint16_t *vc, const float *q_norm,
                               const float *k_norm, const float *rope_cos, const float *rope_sin, float *ao) {
    HyCtx *c = (HyCtx *)impl;
    if (!c || c->broken || heads < 1 || kv_heads < 1 || heads % kv_heads || nt < 1 || nt > kMaxChunk || pos0 < 0 ||
        pos0 + nt > ctx)
        return -1;
    if (cudaSetDevice(c->dev) != cudaSuccess) return -1;
    const int G = heads / kv_heads, qd = heads * hdim, kvd = kv_heads * hdim, half = hdim / 2;
    const int splits = (ctx + kSplitLen - 1) / kSplitLen;
    const size_t qkv_b = (size_t)nt * (qd + 2 * kvd) * 4, kv_b = (size_t)ctx * kvd * 2, tab_b = (size_t)ctx * half * 4;
    float *dqkv = nullptr, *dqn = nullptr, *dkn = nullptr, *dcos = nullptr, *dsin = nullptr, *dao = nullptr,
          *dpart = nullptr, *dcpart = nullptr;
    const int max_chunks = attn_max_chunks(ctx);
    uint16_t *dkc = nullptr, *dvc = nullptr;
    int *dtick = nullptr, *dpos = nullptr;
    bool ok = cudaMalloc(&dqkv, qkv_b) == cudaSuccess && cudaMalloc(&dkc, kv_b) == cudaSuccess &&
              cudaMalloc(&dvc, kv_b) == cudaSuccess && cudaMalloc(&dqn, hdim * 4) == cudaSuccess &&
              cudaMalloc(&dkn, hdim * 4) == cudaSuccess && cudaMalloc(&dcos, tab_b) == cudaSuccess &&
              cudaMalloc(&dsin, tab_b) == cudaSuccess && cudaMalloc(&dao, (size_t)nt * qd * 4) == cudaSuccess &&
              cudaMalloc(&dpart, (size_t)kv_heads * splits * G * (hdim + 2) * 4) == cudaSuccess &&
              cudaMalloc(&dcpart, (size_t)heads * max_chunks * (hdim + kPartPad) * 4) == cudaSuccess &&
              cudaMalloc(&dtick, kv_heads * 4) == cudaSuccess && cudaMalloc(&dpos, 4) == cudaSuccess &&
              cudaMemsetAsync(dtick, 0, kv_heads * 4, c->st) == cudaSuccess &&
              h2d(c, dpos, &pos0, 4) == cudaSuccess &&
              h2d(c, dqkv, qkv, qkv_b) == cudaSuccess &&
              h2d(c, dkc, kc, kv_b) == cudaSuccess &&
              h2d(c, dvc, vc, kv_b) == cudaSuccess &&
              h2d(c, dqn, q_norm, hdim * 4) == cudaSuccess &&
              h2d(c, dkn, k_norm, hdim * 4) == cudaSuccess &&
              h2d(c, dcos, rope_cos, tab_b) == cudaSuccess &&
              h2d(c, dsin, rope_sin, tab_b) == cudaSuccess;
    if (ok) {
        AttnArgs aa;
        memset(&aa, 0, sizeof aa);
        aa.qkv = dqkv;
        aa.qkv_ld = qd + 2 * kvd;
        aa.kc = dkc;
        aa.vc = dvc;
        aa.q_norm = dqn;
        aa.k_norm = dkn;
        aa.rope_cos = dcos;
        aa.rope_sin = dsin;
        aa.pos_ptr = dpos;
        aa.nt = nt;
        aa.heads = heads;
        aa.kv_heads = kv_heads;
        aa.hd = hdim;
        aa.kvdim = kvd;
        aa.qdim = qd;
        aa.ctx = ctx;
        aa.half = half;
        aa.eps = eps;
        aa.scale = 1.0f / sqrtf((float)hdim);
        aa.ao = dao;
        aa.part = dpart;
        aa.tickets = dtick;
        aa.split_len = kSplitLen;
        aa.max_splits = splits;
        aa.cpart = dcpart;
        aa.max_chunks = max_chunks;
        aa.units = c->nsm;
        ok = attention(c, aa, nt, false) &&
             cudaMemcpyAsync(ao, dao, (size_t)nt * qd * 4, cudaMemcpyDeviceToHost, c->st) == cudaSuccess &&
             cudaMemcpyAsync(kc, dkc, kv_b, cudaMemcpyDeviceToHost, c->st) == cudaSuccess &&
             cudaMemcpyAsync(vc, dvc, kv_b, cudaMemcpyDeviceToHost, c->st) == cudaSuccess &&
             cudaStreamSynchronize(c->st) == cudaSuccess;
    }
    void *ptrs[] = {dqkv, dqn, dkn, dcos, dsin, dao, dpart, dcpart, dkc, dvc, dtick, dpos};
    for (void *p : ptrs) cudaFree(p);
    return ok ? 0 : -1;
}

// Copy one internal activation buffer of the fused state to the host:
// 0 h [256][hidden], 1 qkv [256][q|k|v], 2 ao [256][qdim], 3 gate, 4 up [256][ffn].
HYC_API int hyc_debug_buffer(void *impl, int which, float *out, size_t count) {
    HyCtx *c = (HyCtx *)impl;
    if (!c || !c->fused || !out) return -1;
    const float *src[5] = {c->d_h, c->d_qkv, c->d_ao, c->d_g, c->d_u};
    const size_t cap[5] = {(size_t)kMaxChunk * c->H, (size_t)kMaxChunk * (c->qd + 2 * c->kvd), (size_t)kMaxChunk * c->qd,
                           (size_t)kMaxChunk * c->F, (size_t)kMaxChunk * c->F};
    if (which < 0 || which > 4 || count > cap[which]) return -1;
    if (cudaStreamSynchronize(c->st) != cudaSuccess ||
        d2h(c, out, src[which], count * 4) != cudaSuccess)
        return -1;
    return 0;
}

// Debug timeline: on != 0 rebuilds the graphs with one slot per kernel launch
// (launch / past-wait / past-prologue / end in %globaltimer ns).
HYC_API int hyc_trace(void *impl, int on) {
#ifdef HYK_TRACE
    HyCtx *c = (HyCtx *)impl;
    if (!c) return -1;
    c->trace_on = on != 0;
    c->trace_next = 0;
    if (c->trace_on && c->fused && !c->d_tl) {
        c->tl_cap = 1 << 16;
        if (cudaMalloc(&c->d_tl, (size_t)c->tl_cap * 8) != cudaSuccess) return -1;
    }
    if (c->d_tl && cudaMemsetAsync(c->d_tl, 0, (size_t)c->tl_cap * 8, c->st) != cudaSuccess) return -1;
    graph_reset(c->g_fwd1);
    graph_reset(c->g_fwd1_logits);
    graph_reset(c->g_dec);
    c->g_dec_vocab = -1;
    static unsigned long long zeros[kTraceSlots][4];
    return cudaMemcpyToSymbolAsync(g_trace, zeros, sizeof zeros, 0, cudaMemcpyHostToDevice, c->st) == cudaSuccess &&
                   cudaMemcpyToSymbolAsync(g_trace2, zeros, sizeof zeros, 0, cudaMemcpyHostToDevice, c->st) ==
                       cudaSuccess &&
                   cudaMemcpyToSymbolAsync(g_trace3, zeros, sizeof zeros, 0, cudaMemcpyHostToDevice, c->st) ==
                       cudaSuccess &&
                   cudaStreamSynchronize(c->st) == cudaSuccess
               ? 0
               : -1;
#else
    (void)impl;
    (void)on;
    return -1;  // this library was built without the timeline (HYK_TRACE)
#endif
}

// Copy the timeline (slots * 4 values) and return the number of slots in use.
HYC_API int hyc_trace_read(void *impl, unsigned long long *out, int max_slots) {
#ifdef HYK_TRACE
    HyCtx *c = (HyCtx *)impl;
    if (!c || !out) return -1;
    const int n = c->trace_next < max_slots ? c->trace_next : max_slots;
    // out holds [max_slots][4] main stamps followed by [max_slots][4] sub-phase stamps
    if (cudaStreamSynchronize(c->st) != cudaSuccess ||
        cudaMemcpyFromSymbol(out, g_trace, (size_t)n * 4 * sizeof(unsigned long long)) != cudaSuccess ||
        cudaMemcpyFromSymbol(out + (size_t)max_slots * 4, g_trace2, (size_t)n * 4 * sizeof(unsigned long long)) !=
            cudaSuccess ||
        cudaMemcpyFromSymbol(out + (size_t)max_slots * 8, g_trace3, (size_t)n * 4 * sizeof(unsigned long long)) !=
            cudaSuccess)
        return -1;
    return n;
#else
    (void)impl;
    (void)out;
    (void)max_slots;
    return -1;  // this library was built without the timeline (HYK_TRACE)
#endif
}

// Persistent-kernel timeline of the last traced launch: %globaltimer at every
// phase edge of block 0 (step start, then before/after each grid barrier).
HYC_API int hyc_mega_timeline(void *impl, unsigned long long *out, int cap) {
#ifdef HYK_TRACE
    HyCtx *c = (HyCtx *)impl;
    if (!c || !out || !c->d_tl) return -1;
    const int n = cap < c->tl_cap ? cap : c->tl_cap;
    if (cudaStreamSynchronize(c->st) != cudaSuccess ||
        cudaMemcpy(out, c->d_tl, (size_t)n * 8, cudaMemcpyDeviceToHost) != cudaSuccess)
        return -1;
    return n;
#else
    (void)impl;
    (void)out;
    (void)cap;
    return -1;  // this library was built without the timeline (HYK_TRACE)
#endif
}

// ---------------------------------------------------------------- tensor parallelism

// This handle holds rank `rank` of `world` of a tensor-parallel split (its
// fused_prepare shape is the rank's share: heads, KV heads and FFN columns
// per rank; o_proj and down with the rank's K columns; the head with
// vocabulary rows vocab0 ..).  Allocates and zeroes the exchange area and
// writes its CUDA IPC handle (64 bytes) to handle_out.
HYC_API int hyc_tp_init(void *impl, int rank, int world, int vocab0, unsigned char *handle_out) {
    HyCtx *c = (HyCtx *)impl;
    if (!c || c->broken || !c->fused || !handle_out || world < 1 || world > kTpMax || rank < 0 || rank >= world ||
        vocab0 < 0)
        return -1;
    if (cudaSetDevice(c->dev) != cudaSuccess) return -1;
    tp_free(c);
    c->tp_cap = (long long)kMaxChunk * c->H;
    const TpLayout L = tp_layout(c->tp_cap);
    cudaIpcMemHandle_t hdl;
    const bool ok = cudaMalloc(&c->d_tp_area, L.bytes) == cudaSuccess &&
                    cudaMalloc(&c->d_tp_part, (size_t)c->tp_cap * 4) == cudaSuccess &&
                    cudaMalloc(&c->d_tp_err, 4) == cudaSuccess &&
                    cudaMemsetAsync(c->d_tp_area, 0, L.bytes, c->st) == cudaSuccess &&
                    cudaMemsetAsync(c->d_tp_err, 0, 4, c->st) == cudaSuccess &&
                    cudaStreamSynchronize(c->st) == cudaSuccess &&
                    cudaIpcGetMemHandle(&hdl, c->d_tp_area) == cudaSuccess;
    if (!ok) {
        cudaGetLastError();
        tp_free(c);
        snprintf(c->err, sizeof c->err, "tensor-parallel exchange area: allocation or IPC export failed");
        return -1;
    }
    memcpy(handle_out, &hdl, sizeof hdl);
    c->tp_rank = rank;
    c->tp_world = world;
    c->tp_vocab0 = vocab0;
    c->mega_state = -1;
    return (int)sizeof hdl;
}

// Map the peers' exchange areas (handles[q * 64 ..] from every rank's
// hyc_tp_init, the own one ignored) and switch the layer loop and the head
// to the exchanges.  Every rank must have finished hyc_tp_init (its area
// zeroed) before any rank connects: a host barrier between the two calls.
HYC_API int hyc_tp_connect(void *impl, const unsigned char *handles) {
    HyCtx *c = (HyCtx *)impl;
    if (!c || c->broken || !c->d_tp_area || !handles) return -1;
    if (cudaSetDevice(c->dev) != cudaSuccess) return -1;
    TpArgs t;
    memset(&t, 0, sizeof t);
    t.cap = c->tp_cap;
    t.rank = c->tp_rank;
    t.world = c->tp_world;
    t.err = c->d_tp_err;
    for (int q = 0; q < c->tp_world; q++) {
        if (q == c->tp_rank) {
            t.area[q] = c->d_tp_area;
            continue;
        }
        cudaIpcMemHandle_t hdl;
        memcpy(&hdl, handles + (size_t)q * sizeof hdl, sizeof hdl);
        void *p = nullptr;
        if (cudaIpcOpenMemHandle(&p, hdl, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
            cudaGetLastError();
            for (int j = 0; j < q; j++)
                if (j != c->tp_rank && t.area[j]) cudaIpcCloseMemHandle(t.area[j]);
            snprintf(c->err, sizeof c->err, "tensor-parallel exchange: mapping rank %d's area failed", q);
            return -1;
        }
        t.area[q] = (uint8_t *)p;
    }
    c->tp = t;
    c->tp_on = c->tp_world > 1;
    graph_reset(c->g_fwd1);
    graph_reset(c->g_fwd1_logits);
    graph_reset(c->g_dec);
    c->g_dec_vocab = -1;
    return 0;
}

// ---------------------------------------------------------------- allocation-free decode attention
//
// For callers that cannot allocate device memory themselves at the point of
// the call (a host that has handed all free memory to its own arena or
// caching allocator, or a latency-critical serving loop where cudaMalloc /
// cudaFree would synchronise the device and stall other streams), the
// split-KV decode attention can run with its scratch — the per-split
// partial softmax states and the per-KV-head completion tickets — in a
// fixed file-scope device array instead of memory from fused_prepare.
// Every GPU that loads this library holds these 512 KiB + 256 B until the
// process exits.
constexpr size_t kNoAllocPartFloats = 131072;  // 512 KiB of split partials
constexpr int kNoAllocTickets = 64;
static __device__ __align__(256) float g_noalloc_part[kNoAllocPartFloats];
static __device__ __align__(256) int g_noalloc_tickets[kNoAllocTickets];

struct NoAllocScratch {
    float *part = nullptr;
    int *tickets = nullptr;
    bool ready = false;
};
static NoAllocScratch g_noalloc[128];  // per device ordinal, filled on first use
static std::mutex g_noalloc_mu;

static int noalloc_fail(char *err, int cap, int code, const char *msg) {
    if (err && cap > 0) snprintf(err, (size_t)cap, "%s", msg);
    return code;
}

// The host loader's RoPE tables (reference src/model.c:537 and :576-586),
// evaluated with the same single-precision libm calls.
HYC_API int hyc_rope_tables(float freq_base, float alpha, int hdim, int rope_dim, int ctx, float *cos_out,
                            float *sin_out) {
    if (hdim <= 0 || rope_dim <= 0 || (rope_dim & 1) || ctx <= 0 || !cos_out || !sin_out) return -1;
    float base = freq_base;
    if (alpha > 0 && hdim > 2) base *= powf(alpha, (float)hdim / (float)(hdim - 2));
    const int half = rope_dim / 2;
    for (int i = 0; i < half; i++) {
        const float freq = 1.0f / powf(base, (float)i / (float)half);
        for (int p = 0; p < ctx; p++) {
            const float ang = (float)p * freq;
            cos_out[(size_t)p * half + i] = cosf(ang);
            sin_out[(size_t)p * half + i] = sinf(ang);
        }
    }
    return 0;
}


// Decode attention for one token (rope -> q/k RMSNorm -> bf16 K/V store at
// *d_pos -> causal GQA softmax over 0..*d_pos) on caller-provided device
// buffers, with no device allocation: the split-KV scratch lives in
// g_noalloc_part / g_noalloc_tickets.  See include/hymt2_cuda.h.
HYC_API int hyc_attention_decode_noalloc(void *stream, int heads, int kv_heads, int hdim, int ctx, const int *d_pos,
                                         float eps, float *d_qkv, uint16_t *d_kc, uint16_t *d_vc,
                                         const float *d_q_norm, const float *d_k_norm, const float *d_rope_cos,
                                         const float *d_rope_sin, float *d_ao, char *err, int err_cap) {
    if (heads < 1 || kv_heads < 1 || heads % kv_heads || ctx < 1 || !d_pos || !d_qkv || !d_kc || !d_vc ||
        !d_q_norm || !d_k_norm || !d_rope_cos || !d_rope_sin || !d_ao)
        return noalloc_fail(err, err_cap, -1, "invalid argument");
    const int G = heads / kv_heads;
    if ((hdim != 64 && hdim != 128) || (G != 1 && G != 2 && G != 4 && G != 8))
        return noalloc_fail(err, err_cap, -1, "unsupported head geometry (hdim 64/128, group 1/2/4/8)");
    const int splits = (ctx + kDecSplit - 1) / kDecSplit;
    const size_t need = (size_t)kv_heads * splits * G * (hdim + 2);
    if (need > kNoAllocPartFloats || kv_heads > kNoAllocTickets) {
        char msg[192];
        snprintf(msg, sizeof msg,
                 "scratch limit exceeded: kv_heads*ceil(ctx/%d)*group*(hdim+2) = %zu floats > %zu, or kv_heads %d > %d",
                 kDecSplit, need, kNoAllocPartFloats, kv_heads, kNoAllocTickets);
        return noalloc_fail(err, err_cap, -2, msg);
    }
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 128)
        return noalloc_fail(err, err_cap, -3, "no current CUDA device");
    NoAllocScratch &sc = g_noalloc[dev];
    {
        // once per device, with that device current: the symbols' device
        // addresses (the host-side names are only stand-ins)
        std::lock_guard<std::mutex> lock(g_noalloc_mu);
        if (!sc.ready) {
            void *p = nullptr, *t = nullptr;
            if (cudaGetSymbolAddress(&p, g_noalloc_part) != cudaSuccess ||
                cudaGetSymbolAddress(&t, g_noalloc_tickets) != cudaSuccess) {
                cudaGetLastError();
                return noalloc_fail(err, err_cap, -3, "cudaGetSymbolAddress failed for the scratch array");
            }
            if (!init_kernel_attrs(dev))
                return noalloc_fail(err, err_cap, -3, "setting kernel shared-memory limits failed");
            sc.part = (float *)p;
            sc.tickets = (int *)t;
            sc.ready = true;
        }
    }
    cudaStream_t st = (cudaStream_t)stream;
    // the array keeps the previous call's contents: tickets must start at zero
    if (cudaMemsetAsync(sc.tickets, 0, (size_t)kv_heads * sizeof(int), st) != cudaSuccess)
        return noalloc_fail(err, err_cap, -3, "clearing the ticket scratch failed");
    AttnArgs aa;
    memset(&aa, 0, sizeof aa);
    aa.qkv = d_qkv;
    aa.qkv_ld = heads * hdim + 2 * kv_heads * hdim;
    aa.kc = d_kc;
    aa.vc = d_vc;
    aa.q_norm = d_q_norm;
    aa.k_norm = d_k_norm;
    aa.rope_cos = d_rope_cos;
    aa.rope_sin = d_rope_sin;
    aa.pos_ptr = d_pos;
    aa.nt = 1;
    aa.heads = heads;
    aa.kv_heads = kv_heads;
    aa.hd = hdim;
    aa.kvdim = kv_heads * hdim;
    aa.qdim = heads * hdim;
    aa.ctx = ctx;
    aa.half = hdim / 2;
    aa.eps = eps;
    aa.scale = 1.0f / sqrtf((float)hdim);
    aa.ao = d_ao;
    aa.part = sc.part;
    aa.tickets = sc.tickets;
    aa.split_len = kDecSplit;
    aa.max_splits = splits;
    aa.trace = -1;
    const dim3 grid(kv_heads, splits), block(kDecWarps * 32);
    const size_t smem = hdim == 128 ? attn_dec_smem<128>() : attn_dec_smem<64>();
    cudaError_t e = cudaErrorInvalidValue;
#define HY_NA(HD_, G_)                                                                    \
    if (hdim == HD_ && G == G_) e = cudaLaunchKernelEx_compat(attn_decode2<HD_, G_>, grid, block, smem, st, aa);
    HY_NA(128, 4) HY_NA(128, 1) HY_NA(128, 2) HY_NA(128, 8)
    HY_NA(64, 4) HY_NA(64, 1) HY_NA(64, 2) HY_NA(64, 8)
#undef HY_NA
    if (e != cudaSuccess) return noalloc_fail(err, err_cap, -3, cudaGetErrorString(e));
    if (err && err_cap > 0) err[0] = 0;
    return 0;
}

}  // extern "C"
