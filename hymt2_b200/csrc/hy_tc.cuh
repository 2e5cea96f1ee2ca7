// hy_tc.cuh — int8 tensor-core GEMM for batched prefill / multi-sequence
// decode on sm_100a: tcgen05.mma kind::i8, accumulators in TMEM.
//
// Y[t][n] = sum_b ad[t][b] * (ws1[n][b] * S1_b[t][n] - ws2[n][b] * S2_b[t][n])
// with A the Q8_K codes of the activations (per-256-block scale ad) and the
// weight held as P int8 planes per 256-block, chosen so that every S is the
// reference's per-block integer, exactly:
//   P = 1  panel (STQ1_0 / Q2_0C): W = code * 2^shift - off, the value the
//          panel GEMV multiplies (reference src/kernels.c:565-581); S1 = A.W,
//          ws1 = the panel scale.
//   P = 2  Q6_K: W' = sc_j * (q6 - 32) split as 64 * hi + lo (lo in 0..63);
//          S1 = 64 * (A.hi) + A.lo = the reference's `acc`
//          (src/kernels.c:808-835), ws1 = d.
//   P = 3  Q4_K: W' = sc_j * q4 split the same way gives `sumi`; the third
//          plane holds the sub-block min m_j at each of its 32 elements, so
//          S2 = A.m = sum_j m_j * bsum_j is `summ` (src/kernels.c:861-877);
//          ws1 = d, ws2 = dmin.
// The blocks are combined in fp32.
//
// Operands live in global memory pre-tiled in the UMMA canonical K-major
// layout without swizzle: a tile of R rows x K is (K/16) x (R/8) core
// matrices of 8 rows x 16 bytes; core (row group g, 16-byte k chunk c) sits
// at (c * R/8 + g) * 128 bytes, so each half block (K = 128) of a tile is
// contiguous.  Activations: [m tile][block][128 x 256]; weights: [n tile]
// [block][half][P*N x 128] with the planes stacked as rows, so one bulk copy
// moves the A half or the B half of a stage and one MMA (N' = P*NM <= 256)
// multiplies the activations with every plane, reading them once.  Launches
// that multiply 64-row slices of 256 / 128-row tiles (short passes) read a
// second copy of the weight ordered slice first, [n tile][block][half]
// [slice][P*64 x 128], so a slice's half block is one bulk copy too.
//
// Persistent CTAs (one per SM) walk the (m, n) tiles m-fastest, so the
// CTAs running at one time share each weight tile through L2.  Per CTA:
// warp 0 streams half blocks (A, B planes) into a 3..8-stage ring and each
// block's scales into a ring of their own; warp 1 (one thread)
// issues 4 MMAs of K = 32 (N' = P*NM) per half block into one of two TMEM
// accumulator sets (N = 256 / 128 / 64 for P = 1 / 2 / 3, so one set is at
// most 256 columns); warps 2-17 (4 per TMEM lane quarter, N/4 columns each)
// read a finished block's int32 results with tcgen05.ld and fold them into
// fp32 registers while the MMAs of the next block (or tile) run.  A stage is
// released by the MMA commit alone, a scale entry and an accumulator set by
// the epilogue.  Every wait is bounded; TMEM is released on every exit.
#pragma once
#include "hy_common.cuh"
#include "hy_gemv.cuh"

namespace hyk {

constexpr int kTcM = 128;       // tokens per tile (TMEM lanes)
constexpr int kTcKB = 256;      // K per Q8_K block
constexpr int kTcKH = 128;      // K per stage: half a block
constexpr int kTcMaxStages = 8;      // half-block stages in flight (at most)
constexpr int kTcSmemBudget = 226 * 1024;  // of 227 KB per block, leaving the static barriers room
constexpr int kTcEpiWarps = 16;
constexpr int kTcThreads = (2 + kTcEpiWarps) * 32;  // warp 0 producer, 1 MMA, 2.. epilogue
constexpr int kTcABytes = kTcM * kTcKB;             // 32 KB
constexpr unsigned long long kTcWaitNs = 2000000000ull;

// Weight rows per tile for P planes.
__host__ __device__ constexpr int tc_n(int P) { return P == 1 ? 256 : (P == 2 ? 128 : 64); }
// Bytes of one (tile, block) of the tiled weight: 2 halves x P planes of N x 128.
__host__ __device__ constexpr int tc_bbytes(int P) { return P * tc_n(P) * kTcKB; }
// Bytes of one (tile, block) of the tiled scales: ws1[N] then ws2[N].
__host__ __device__ constexpr int tc_sbytes(int P) { return 2 * tc_n(P) * 4; }
// One stage: the A half (128 x 128) and the B half (P planes of NM x 128).
__host__ __device__ constexpr int tc_stage_bytes(int P, int NM) { return kTcABytes / 2 + P * NM * kTcKH; }
// One scale-ring entry: ws1[NM], ws2[NM], then the 128 activation scales.
__host__ __device__ constexpr int tc_slot_bytes(int NM) { return 2 * NM * 4 + kTcM * 4; }
// Stages: as many as the shared-memory budget holds (up to 8) next to a
// scale ring with an entry per block in flight plus two.
__host__ __device__ constexpr int tc_stages(int P, int NM) {
    int s = kTcMaxStages;
    while (s > 2 && s * tc_stage_bytes(P, NM) + (s / 2 + 2) * tc_slot_bytes(NM) + 1024 > kTcSmemBudget) s--;
    return s;
}
__host__ __device__ constexpr int tc_slots(int P, int NM) { return tc_stages(P, NM) / 2 + 2; }
__host__ __device__ inline size_t tc_smem_bytes(int P, int NM) {
    return (size_t)tc_stages(P, NM) * tc_stage_bytes(P, NM) + (size_t)tc_slots(P, NM) * tc_slot_bytes(NM) + 1024;
}
static_assert(tc_stages(1, 256) >= 4 && tc_stages(3, 64) >= 4, "tc pipeline too shallow");
// Planes of a device weight format (0: not on the tensor-core path).
__host__ __device__ constexpr int tc_planes(int fmt) {
    return (fmt == FMT_PANEL || fmt == FMT_STQN) ? 1 : (fmt == FMT_Q6K ? 2 : (fmt == FMT_Q4K ? 3 : 0));
}

// Byte offset of (row r, k) inside a canonical tile of R rows (any K).
__host__ __device__ inline size_t tc_tile_off(int r, int k, int R) {
    return ((size_t)(k >> 4) * (R / 8) + (r >> 3)) * 128 + (size_t)(r & 7) * 16 + (k & 15);
}
// Byte offset of (plane p, row r, k in 0..255) inside one (tile, block) of
// a tiled weight: half k / 128, then ONE canonical tile of P*N rows holding
// the planes stacked (row p*N + r), so a single MMA of N' = P*NM covers
// every plane and reads the activation tile once.
__host__ __device__ inline size_t tc_wtile_off(int P, int p, int r, int k) {
    const int N = tc_n(P);
    return (size_t)(k >> 7) * P * N * kTcKH + tc_tile_off(p * N + r, k & 127, P * N);
}

constexpr int kTcMaxW = 3;  // weights of one launch (same format, same activation)

struct TcArgs {
    const int8_t *a;   // tiled activations [ceil(T/128)][nb][128 x 256]
    const float *ad;   // activation block scales [ceil(T/128)][nb][128]
    int nw;            // weights in this launch; their tiles follow one another
    const int8_t *w[kTcMaxW];   // tiled weight [ceil(N/n)][nb][2][P][n x 128]
    const int8_t *w64[kTcMaxW]; // the same, 64-row slices first (launches with NM = 64 < n)
    const float *ws[kTcMaxW];   // tiled weight scales [ceil(N/n)][nb][2][n]
    float *out[kTcMaxW];        // [T][ldo]
    int ldo[kTcMaxW], N[kTcMaxW];
    int T, nb;
    int epi;           // 0: out = y, 1: out += y
    int *err;          // set on a bounded-wait timeout
    int32_t *ints;     // tc_gemm<P, NM, true> only: per-block integers [T][N][nb] (Q4_K: [T][N][nb][2])
};

// Number of (m, n) tiles of a GEMM whose MMAs cover NM weight rows.
__host__ __device__ inline int tc_tiles(int P, int NM, int T, int N) {
    return ((T + kTcM - 1) / kTcM) * ((N + tc_n(P) - 1) / tc_n(P)) * (tc_n(P) / NM);
}
__host__ __device__ inline int tc_tiles_all(int P, int NM, const TcArgs &a) {
    int n = 0;
    for (int i = 0; i < a.nw; i++) n += tc_tiles(P, NM, a.T, a.N[i]);
    return n;
}
// Tile -> (weight, m tile, NM-row slice of that weight).
__device__ __forceinline__ int tc_locate(int P, int NM, const TcArgs &a, int ntm, int tile, int &mt, int &ns) {
    int wi = 0;
    for (; wi < a.nw - 1; wi++) {
        const int tw = tc_tiles(P, NM, a.T, a.N[wi]);
        if (tile < tw) break;
        tile -= tw;
    }
    mt = tile % ntm;
    ns = tile / ntm;
    return wi;
}

__device__ __forceinline__ uint32_t tc_smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void tc_mbar_init(uint64_t *b, unsigned count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(tc_smem_u32(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void tc_mbar_arrive(uint64_t *b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(tc_smem_u32(b)) : "memory");
}
__device__ __forceinline__ void tc_mbar_expect(uint64_t *b, unsigned tx) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(tc_smem_u32(b)), "r"(tx) : "memory");
}
__device__ __forceinline__ bool tc_mbar_try(uint64_t *b, unsigned parity) {
    unsigned ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(tc_smem_u32(b)), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ bool tc_mbar_wait(uint64_t *b, unsigned parity, unsigned long long limit_ns = kTcWaitNs) {
    if (tc_mbar_try(b, parity)) return true;
    const unsigned long long t0 = gtimer();
    while (!tc_mbar_try(b, parity))
        if (gtimer() - t0 > limit_ns) return false;
    return true;
}
__device__ __forceinline__ void tc_bulk(void *dst, const void *src, unsigned bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     tc_smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(tc_smem_u32(bar))
                 : "memory");
}

// UMMA shared-memory descriptor of MMA step s (k chunks 2s, 2s+1) of a
// canonical tile of R rows: no swizzle, LBO = distance between k chunks,
// SBO = distance between 8-row groups, version 1.
__device__ __forceinline__ uint64_t tc_desc(const void *tile, int s, int R) {
    const uint32_t addr = tc_smem_u32(tile) + (uint32_t)s * 2u * (uint32_t)(R / 8) * 128u;
    const uint64_t lbo = (uint64_t)((R / 8) * 128) >> 4, sbo = 128 >> 4;
    return (uint64_t)((addr >> 4) & 0x3FFFu) | (lbo << 16) | (sbo << 32) | (1ull << 46);
}
// Instruction descriptor: D s32, A s8, B s8, both K-major, N, M.
__host__ __device__ constexpr uint32_t tc_idesc(int M, int N) {
    return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, int acc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc)
        : "memory");
}
__device__ __forceinline__ void tc_commit(uint64_t *b) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(tc_smem_u32(b))
                 : "memory");
}
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

// 32 lanes x 16 columns of 32-bit words from TMEM (this warp's lane quarter).
__device__ __forceinline__ void tc_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
}
// 32 lanes x 8 columns.
__device__ __forceinline__ void tc_ld8(uint32_t taddr, uint32_t (&r)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr)
                 : "memory");
}
template <int W>
__device__ __forceinline__ void tc_ld(uint32_t taddr, uint32_t (&r)[W]) {
    if constexpr (W == 16) tc_ld16(taddr, r);
    else tc_ld8(taddr, r);
}
// Wait for this thread's tcgen05.ld results.  The loads write their
// registers asynchronously, but the compiler sees those registers as defined
// by the tcgen05.ld statement itself and may move arithmetic on them above a
// wait that names no register.  So every destination register also passes
// through an empty statement after the wait (asm volatile statements keep
// their order), and each use depends on that statement's output.
template <int P, int W>
__device__ __forceinline__ void tc_wait_ld(uint32_t (&r)[P][W]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int p = 0; p < P; p++)
#pragma unroll
        for (int j = 0; j < W; j++) asm volatile("" : "+r"(r[p][j]));
}

// int32 -> fp32 for |v| < 2^22 without the conversion unit: the bits of
// 1.5 * 2^23 + v.  Exact, so fmaf(tc_magic(v), s, -1.5 * 2^23 * s) rounds
// v * s once, like fmaf on (float)v, whenever 1.5 * 2^23 * s is exact.
__device__ __forceinline__ float tc_magic(uint32_t v) { return __int_as_float((int)(v + 0x4B400000u)); }
constexpr float kTcMagic = 12582912.0f;  // 1.5 * 2^23

// P planes; MMAs of NM weight rows, a slice of the N = tc_n(P) rows of
// each weight tile (NM < N gives small token counts more CTAs).  INTS (test
// instantiations only) also stores every block's integers as the epilogue
// reads them from TMEM: the panel S = A.W, Q6_K acc = 64 S_hi + S_lo, Q4_K
// sumi = 64 S_hi + S_lo and summ = S_m.
template <int P, int NM, bool INTS = false>
__global__ void __launch_bounds__(kTcThreads, 1) tc_gemm(const __grid_constant__ TcArgs a) {
    constexpr int N = tc_n(P), SUB = N / NM, C = NM / 4, AH = kTcABytes / 2, SB = tc_sbytes(P);
    constexpr int STB = tc_stage_bytes(P, NM), SLB = tc_slot_bytes(NM);
    constexpr int kTcStages = tc_stages(P, NM), kTcScaleSlots = tc_slots(P, NM);
    // accumulator sets: as many as TMEM holds, up to 4 (the MMA runs that many blocks ahead of the epilogue)
    constexpr int NBUF = 512 / (P * NM) > 4 ? 4 : 512 / (P * NM);
    static_assert(N % NM == 0 && NM % 64 == 0, "MMA rows must be a slice of the weight tile");
    static_assert(SUB == 1 || NM == 64, "slices are read from the 64-row slice-first copy");
    extern __shared__ __align__(1024) uint8_t smem[];
    __shared__ __align__(8) uint64_t full[kTcStages], empty[kTcStages], sfull[kTcScaleSlots], sempty[kTcScaleSlots],
        accf[4], acce[4], fin;
    // launched as a programmatic dependent: barrier setup and the TMEM
    // allocation overlap the previous kernel; the producer waits for it
    // before its first copy (everything else follows the producer)
    pdl_trigger();
    __shared__ uint32_t s_tmem;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nb = a.nb, ntm = (a.T + kTcM - 1) / kTcM, ntiles = tc_tiles_all(P, NM, a);
    uint8_t *stage = (uint8_t *)(((uintptr_t)smem + 1023) & ~(uintptr_t)1023);
    uint8_t *slots = stage + (size_t)kTcStages * STB;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kTcStages; s++) {
            tc_mbar_init(&full[s], 1);
            tc_mbar_init(&empty[s], 1);  // the MMA commit
        }
        for (int s = 0; s < kTcScaleSlots; s++) {
            tc_mbar_init(&sfull[s], 1);
            tc_mbar_init(&sempty[s], kTcEpiWarps);
        }
        for (int b = 0; b < NBUF; b++) {
            tc_mbar_init(&accf[b], 1);
            tc_mbar_init(&acce[b], kTcEpiWarps);
        }
        tc_mbar_init(&fin, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(tc_smem_u32(&s_tmem))
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
        tc_fence_before();
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;
    bool ok = true;
    if (warp == 0) {
        // producer: per block its scales (weight slice, then activations),
        // then two half-block stages (A half, B planes of the slice)
        if (lane == 0) {
            pdl_wait();
            int g = 0, hs = 0;  // blocks and half blocks issued by this CTA
            for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
                int mt, ns;
                const int wi = tc_locate(P, NM, a, ntm, tile, mt, ns), nt = ns / SUB, si = ns % SUB;
                for (int kb = 0; kb < nb && ok; kb++, g++) {
                    const int sl = g % kTcScaleSlots, su = g / kTcScaleSlots;
                    if (su > 0 && !tc_mbar_wait(&sempty[sl], (su - 1) & 1)) {
                        ok = false;
                        break;
                    }
                    uint8_t *sd = slots + (size_t)sl * SLB;
                    const uint8_t *ws = (const uint8_t *)a.ws[wi] + ((size_t)nt * nb + kb) * SB + (size_t)si * NM * 4;
                    tc_mbar_expect(&sfull[sl], SLB);
                    tc_bulk(sd, ws, NM * 4, &sfull[sl]);
                    tc_bulk(sd + NM * 4, ws + N * 4, NM * 4, &sfull[sl]);
                    tc_bulk(sd + 2 * NM * 4, a.ad + ((size_t)mt * nb + kb) * kTcM, kTcM * 4, &sfull[sl]);
                    for (int h = 0; h < 2 && ok; h++, hs++) {
                        const int s = hs % kTcStages, use = hs / kTcStages;
                        if (use > 0 && !tc_mbar_wait(&empty[s], (use - 1) & 1)) {
                            ok = false;
                            break;
                        }
                        uint8_t *st = stage + (size_t)s * STB;
                        tc_mbar_expect(&full[s], STB);
                        tc_bulk(st, a.a + ((size_t)mt * nb + kb) * kTcABytes + (size_t)h * AH, AH, &full[s]);
                        const int8_t *wb = a.w[wi] + ((size_t)nt * nb + kb) * tc_bbytes(P) + (size_t)h * P * N * kTcKH;
                        if constexpr (SUB == 1) {
                            tc_bulk(st + AH, wb, P * N * kTcKH, &full[s]);
                        } else {
                            // the slice-first copy: the slice's P*64 x 128 canonical tile is contiguous
                            const int8_t *wsl = a.w64[wi] + ((size_t)nt * nb + kb) * tc_bbytes(P) +
                                                (size_t)h * P * N * kTcKH + (size_t)si * P * NM * kTcKH;
                            tc_bulk(st + AH, wsl, P * NM * kTcKH, &full[s]);
                        }
                    }
                }
            }
            if (!ok) atomicExch(a.err, 1);
        }
    } else if (warp == 1) {
        // MMA issuer: 4 MMAs (K = 32, N = P*NM: every plane at once) per half
        // block into accumulator set g % 2
        if (lane == 0) {
            constexpr uint32_t idesc = tc_idesc(kTcM, P * NM);
            int g = 0, hs = 0;
            for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
                for (int kb = 0; kb < nb && ok; kb++, g++) {
                    const int buf = g % NBUF, ub = g / NBUF;
                    if (ub > 0 && !tc_mbar_wait(&acce[buf], (ub - 1) & 1)) {
                        ok = false;
                        break;
                    }
                    for (int h = 0; h < 2; h++, hs++) {
                        const int s = hs % kTcStages, use = hs / kTcStages;
                        if (!tc_mbar_wait(&full[s], use & 1)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint8_t *st = stage + (size_t)s * STB;
#pragma unroll
                        for (int k = 0; k < kTcKH / 32; k++)
                            tc_mma(tmem + (uint32_t)(buf * P * NM), tc_desc(st, k, kTcM), tc_desc(st + AH, k, P * NM),
                                   idesc, (h | k) != 0);
                        tc_commit(&empty[s]);
                    }
                    if (ok) tc_commit(&accf[buf]);
                }
            }
            tc_commit(&fin);  // completes when every MMA issued above has
            if (!tc_mbar_wait(&fin, 0)) ok = false;
            if (!ok) atomicExch(a.err, 1);
        }
    } else {
        // epilogue: lane quarter q = warp % 4 (the TMEM lanes this warp may
        // read: tokens 32q..32q+31 of the tile), columns part*C ..; each run
        // of four consecutive warps covers all four quarters
        const int e = warp - 2, q = warp & 3, part = e >> 2;
        int g = 0;
        for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
            int mt, ns;
            const int wi = tc_locate(P, NM, a, ntm, tile, mt, ns);
            const int t = mt * kTcM + q * 32 + lane;
            float acc[C];
#pragma unroll
            for (int j = 0; j < C; j++) acc[j] = 0.f;
            for (int kb = 0; kb < nb; kb++, g++) {
                const int buf = g % NBUF, ub = g / NBUF, sl = g % kTcScaleSlots;
                if (!tc_mbar_wait(&accf[buf], ub & 1) || !tc_mbar_wait(&sfull[sl], (g / kTcScaleSlots) & 1)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const float *sd = (const float *)(slots + (size_t)sl * SLB);
                const float yd = sd[2 * NM + q * 32 + lane];  // 0 past T (the quantiser pads with zeros)
                const float4 *ws1 = (const float4 *)(sd + part * C), *ws2 = (const float4 *)(sd + NM + part * C);
                const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * P * NM + part * C);
                // P = 1 reads 8 columns at a time: its accumulators leave
                // fewer registers for the loaded words
                constexpr int CW = (P == 1 && C > 16) ? 8 : 16;
#pragma unroll
                for (int c = 0; c < C / CW; c++) {
                    uint32_t r[P][CW];
#pragma unroll
                    for (int p = 0; p < P; p++) tc_ld<CW>(tbase + (uint32_t)(p * NM + c * CW), r[p]);
                    tc_wait_ld(r);
                    if constexpr (INTS) {
                        const int nmax = a.N[wi];
                        for (int j = 0; j < CW; j++) {
                            const int n = ns * NM + part * C + c * CW + j;
                            if (t >= a.T || n >= nmax) continue;
                            const size_t o = (size_t)t * nmax + n;
                            if constexpr (P == 1) {
                                a.ints[o * nb + kb] = (int)r[0][j];
                            } else if constexpr (P == 2) {
                                a.ints[o * nb + kb] = (int)(r[0][j] << 6) + (int)r[1][j];
                            } else {
                                a.ints[(o * nb + kb) * 2] = (int)(r[0][j] << 6) + (int)r[1][j];
                                a.ints[(o * nb + kb) * 2 + 1] = (int)r[2][j];
                            }
                        }
                    }
#pragma unroll
                    for (int j4 = 0; j4 < CW / 4; j4++) {
                        const float4 w1 = ws1[c * CW / 4 + j4];
                        float4 w2 = make_float4(0.f, 0.f, 0.f, 0.f);
                        if constexpr (P != 2) w2 = ws2[c * CW / 4 + j4];
                        const float w1v[4] = {w1.x, w1.y, w1.z, w1.w}, w2v[4] = {w2.x, w2.y, w2.z, w2.w};
#pragma unroll
                        for (int jj = 0; jj < 4; jj++) {
                            const int j = j4 * 4 + jj, n = c * CW + j;
                            float v;
                            if constexpr (P == 1) {
                                // |S| <= 256 * 127 * 3 < 2^22; ws2 holds -1.5 * 2^23 * ws1 (exact: ws1 is an f16)
                                v = fmaf(tc_magic(r[0][j]), w1v[jj], w2v[jj]);
                            } else {
                                const int s1 = (int)(r[0][j] << 6) + (int)r[1][j];
                                v = (float)s1 * w1v[jj];
                                if constexpr (P == 3) v = fmaf(-(float)(int)r[2][j], w2v[jj], v);
                            }
                            acc[n] = fmaf(v, yd, acc[n]);
                        }
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    tc_mbar_arrive(&acce[buf]);
                    tc_mbar_arrive(&sempty[sl]);
                }
            }
            if (ok && t < a.T) {
                float *o = a.out[wi] + (size_t)t * a.ldo[wi];
                const int n0 = ns * NM + part * C, nmax = a.N[wi];
                if ((a.ldo[wi] & 3) == 0 && n0 + C <= nmax) {
#pragma unroll
                    for (int j = 0; j < C; j += 4) {
                        float4 v = make_float4(acc[j], acc[j + 1], acc[j + 2], acc[j + 3]);
                        if (a.epi) {
                            const float4 p = *(const float4 *)(o + n0 + j);
                            v.x += p.x;
                            v.y += p.y;
                            v.z += p.z;
                            v.w += p.w;
                        }
                        *(float4 *)(o + n0 + j) = v;
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < C; j++) {
                        const int n = n0 + j;
                        if (n < nmax) o[n] = a.epi ? o[n] + acc[j] : acc[j];
                    }
                }
            }
        }
        if (!ok && lane == 0) atomicExch(a.err, 1);
    }
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem) : "memory");
    }
}

// ---------------------------------------------------------------- operand preparation

// Integer plane values of element x (0..255) of block b of row r, and the
// block's scales, in each format's device layout (the element decode of
// dequant_elem).  Rows past n give zeros.
template <int P>
__device__ inline void tc_elem(const WDesc &w, int r, int b, int x, int (&v)[P]) {
    const uint8_t *row = w.w + (size_t)r * w.stride;
    const int nb = w.k / 256;
    if constexpr (P == 1) {
        const int ch = x >> 6, l = (x >> 4) & 3, i = x & 15;
        uint32_t byte;
        if (w.fmt == FMT_STQN) {
            const int u = b * 4 + piece_of_chunk(ch);
            const int slot = (row[(size_t)u * 8 + (i >> 1)] >> ((i & 1) * 4)) & 15;
            const uint32_t sg = row[(size_t)nb * 32 + u * 2] | ((uint32_t)row[(size_t)nb * 32 + u * 2 + 1] << 8);
            byte = stq_pattern((int)(((sg >> (4 * (i & 3) + (i >> 2))) & 1) << 4) | slot);
        } else {
            byte = row[(size_t)b * 64 + piece_of_chunk(ch) * 16 + i];
        }
        v[0] = (int)((byte >> (2 * l)) & 3) * (1 << w.shift) - w.off;
    } else if constexpr (P == 2) {
        const int half = x >> 7, q = (x & 127) >> 5, l = x & 31;
        const uint8_t lb = row[(size_t)b * 128 + half * 64 + l + (q & 1) * 32];
        const int lo = (q & 2) ? (lb >> 4) : (lb & 15);
        const int hi = (row[(size_t)nb * 128 + (size_t)b * 64 + half * 32 + l] >> (2 * q)) & 3;
        const int sc = (int8_t)row[(size_t)nb * 192 + (size_t)b * 16 + half * 8 + 2 * q + (l >> 4)];
        const int wv = sc * ((lo | (hi << 4)) - 32);  // -4096 .. 3937
        v[0] = wv >> 6;                               // arithmetic: floor
        v[1] = wv & 63;
    } else {
        const uint8_t *blk = row + (size_t)b * 144;
        const int g = x >> 6, hi = (x >> 5) & 1, l = x & 31, j = 2 * g + hi;
        const uint8_t *q = blk + 4;
        int sc, mn;
        if (j < 4) { sc = q[j] & 63; mn = q[j + 4] & 63; }
        else { sc = (q[j + 4] & 0x0f) | ((q[j - 4] >> 6) << 4); mn = (q[j + 4] >> 4) | ((q[j] >> 6) << 4); }
        const uint8_t qb = blk[16 + 32 * g + l];
        const int wv = sc * (hi ? (qb >> 4) : (qb & 15));  // 0 .. 945
        v[0] = wv >> 6;
        v[1] = wv & 63;
        v[2] = mn;
    }
}

template <int P>
__device__ inline void tc_block_scales(const WDesc &w, int r, int b, float &s1, float &s2) {
    const uint8_t *row = w.w + (size_t)r * w.stride;
    const int nb = w.k / 256;
    if constexpr (P == 1) {
        s1 = w.fmt == FMT_STQN ? h2f((uint16_t)(row[(size_t)nb * 40 + 2 * b] | (row[(size_t)nb * 40 + 2 * b + 1] << 8)))
                               : w.s[(size_t)r * nb + b];
        s2 = -kTcMagic * s1;  // exact: s1 is an f16 value
    } else if constexpr (P == 2) {
        s1 = h2f((uint16_t)(row[(size_t)nb * 208 + 2 * b] | (row[(size_t)nb * 208 + 2 * b + 1] << 8)));
        s2 = 0.f;
    } else {
        const uint8_t *blk = row + (size_t)b * 144;
        s1 = h2f((uint16_t)(blk[0] | (blk[1] << 8)));
        s2 = h2f((uint16_t)(blk[2] | (blk[3] << 8)));
    }
}

// Device weight -> tiled int8 planes and tiled block scales.  One thread per
// (padded row, block, 16-element group).
template <int P>
__global__ void tc_weight_to_tiled(const __grid_constant__ WDesc w, int8_t *tw, float *tws) {
    constexpr int N = tc_n(P);
    const int nb = w.k / 256, ntiles = (w.n + N - 1) / N;
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    const long long total = (long long)ntiles * N * nb * 16;
    if (i >= total) return;
    const int g16 = (int)(i % 16);
    const int b = (int)((i / 16) % nb);
    const int rr = (int)(i / (16LL * nb));  // padded row
    const int tile = rr / N, r = rr % N;
    int8_t *dst = tw + ((size_t)tile * nb + b) * tc_bbytes(P);
    for (int j = 0; j < 16; j++) {
        int v[P];
#pragma unroll
        for (int p = 0; p < P; p++) v[p] = 0;
        if (rr < w.n) tc_elem<P>(w, rr, b, g16 * 16 + j, v);
#pragma unroll
        for (int p = 0; p < P; p++) dst[tc_wtile_off(P, p, r, g16 * 16 + j)] = (int8_t)v[p];
    }
    if (g16 == 0) {
        float s1 = 0.f, s2 = 0.f;
        if (rr < w.n) tc_block_scales<P>(w, rr, b, s1, s2);
        float *sd = tws + ((size_t)tile * nb + b) * 2 * N;
        sd[r] = s1;
        sd[N + r] = s2;
    }
}

// The slice-first copy of a tiled weight (P planes, N = tc_n(P) > 64 rows per
// tile): each half block [chunk c][plane p][row r][16 bytes] becomes
// [slice r / 64][c][p][r % 64][16 bytes]; one thread per 16 bytes.
template <int P>
__global__ void tc_tiles_to_slices(const int8_t *tw, int8_t *tw64, long long units) {
    constexpr int N = tc_n(P), HU = (kTcKH / 16) * P * N;  // 16-byte units per half block
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= units) return;
    const long long hb = i / HU;
    const int u = (int)(i % HU), r = u % N, cp = u / N;  // cp = c * P + p
    const long long o = hb * HU + (long long)(r / 64) * ((kTcKH / 16) * P * 64) + (long long)cp * 64 + (r % 64);
    ((uint4 *)tw64)[o] = ((const uint4 *)tw)[i];
}

// Q8_K codes of one 256 block held by a warp (lane: elements 8 lane ..
// 8 lane + 7), written into the tiled operand (token row r of m tile mt)
// with its scale: quantize_block_warp's arithmetic (first index of the
// largest |x|, iscale = -127/max, d = 1/iscale, round-half-even, clip +-127,
// non-finite products -> 0).
__device__ __forceinline__ void tc_quant_store(const float (&v)[8], int8_t *ta, float *ad, int mt, int nb, int b,
                                               int r) {
    const int lane = threadIdx.x & 31;
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
            int rr = isfinite(f) ? __float2int_rn(f) : 0;
            q[j] = rr > 127 ? 127 : (rr < -127 ? -127 : rr);
        }
    }
    const uint32_t lo = (q[0] & 0xff) | ((q[1] & 0xff) << 8) | ((q[2] & 0xff) << 16) | ((uint32_t)(q[3] & 0xff) << 24);
    const uint32_t hi = (q[4] & 0xff) | ((q[5] & 0xff) << 8) | ((q[6] & 0xff) << 16) | ((uint32_t)(q[7] & 0xff) << 24);
    *(uint2 *)(ta + ((size_t)mt * nb + b) * kTcABytes + tc_tile_off(r, lane * 8, kTcM)) = make_uint2(lo, hi);
    if (lane == 0) ad[((size_t)mt * nb + b) * kTcM + r] = d;
}

// Host-made Q8_K blocks [T][nb] (natural-order codes qs, scale d) written as
// the tiled activation operand, with no prologue: the test hook that reads
// the GEMM's block integers feeds it exactly the codes the oracle uses.  One
// thread per (padded token, block, 16-byte chunk); tokens T .. tpad - 1 get
// zero codes.
__global__ void tc_from_q8k(const q8k_block *xq, int T, int tpad, int nb, int8_t *ta, float *ad) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)tpad * nb * 16) return;
    const int k16 = (int)(i % 16), b = (int)((i / 16) % nb), t = (int)(i / (16LL * nb));
    const int mt = t / kTcM, r = t % kTcM;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (t < T) v = *(const uint4 *)&xq[(size_t)t * nb + b].qs[k16 * 16];
    *(uint4 *)(ta + ((size_t)mt * nb + b) * kTcABytes + tc_tile_off(r, k16 * 16, kTcM)) = v;
    if (k16 == 0) ad[((size_t)mt * nb + b) * kTcM + r] = t < T ? xq[(size_t)t * nb + b].d : 0.f;
}

// Activation rows -> Q8_K, written as tiled int8 codes plus block scales
// (tiled too: [m tile][block][128]).
// One CTA (kGemvThreads) per token; the fp32 row is built by stage_fp32 (the
// GEMV prologues: as is, RMSNorm*w, SiLU*up) and each 256 block quantised by
// one warp with quantize_block_warp's arithmetic (bit-identical codes).
// Tokens past T (padding of the last tile) get zero codes.
// SV = float4 loads per thread (K <= 1024 * SV): the staged arithmetic is the
// same for any SV that covers K, a smaller one only needs fewer registers.
template <int SV>
__global__ void __launch_bounds__(kGemvThreads) tc_quantize(const __grid_constant__ GemvArgs a, int T, int8_t *ta,
                                                             float *ad) {
    extern __shared__ __align__(16) uint8_t smem[];
    pdl_trigger();
    pdl_wait();  // the codes and scales are still the previous GEMM's operand until it completes
    const int K = a.k, nb = K / 256, t = blockIdx.x;
    float *x = (float *)smem;
    float *red = x + K;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int mt = t / kTcM, r = t % kTcM;
    if (t >= T) {
        for (int b = warp; b < nb; b += kGemvThreads / 32) {
            int8_t *dst = ta + ((size_t)mt * nb + b) * kTcABytes + tc_tile_off(r, lane * 8, kTcM);
            *(uint2 *)dst = make_uint2(0, 0);
            if (lane == 0) ad[((size_t)mt * nb + b) * kTcM + r] = 0.f;
        }
        return;
    }
    stage_fp32<SV>(a, t, x, red, K);
    __syncthreads();
    for (int b = warp; b < nb; b += kGemvThreads / 32) {
        const float *p = x + b * 256 + lane * 8;
        const float4 v0 = *(const float4 *)&p[0], v1 = *(const float4 *)&p[4];
        const float v[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
        tc_quant_store(v, ta, ad, mt, nb, b, r);
    }
}

// Activations that need no row-wide reduction (as is; SiLU(x) * x2): one
// warp per (token, 256 block), the element arithmetic of stage_fp32 and the
// quantiser of tc_quantize, so the codes are the same; no CTA barrier, so
// every block of every token is in flight at once.  Tokens T .. tpad - 1 get
// zero codes.
__global__ void __launch_bounds__(256) tc_quantize_blocks(const __grid_constant__ GemvArgs a, int T, int tpad,
                                                          int8_t *ta, float *ad) {
    pdl_trigger();
    pdl_wait();  // the codes and scales are still the previous GEMM's operand until it completes
    const int nb = a.k / 256, lane = threadIdx.x & 31;
    const long long nw = (long long)tpad * nb;
    // the grid strides over the (token, block) pairs
    for (long long wid = (long long)blockIdx.x * 8 + (threadIdx.x >> 5); wid < nw; wid += (long long)gridDim.x * 8) {
    const int t = (int)(wid / nb), b = (int)(wid % nb), mt = t / kTcM, r = t % kTcM;
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; j++) v[j] = 0.f;
    if (t < T) {
        const size_t off = (size_t)t * a.ldx + (size_t)b * 256 + lane * 8;
        const float4 x0 = *(const float4 *)(a.x + off), x1 = *(const float4 *)(a.x + off + 4);
        const float xs[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
        if (a.act == ACT_SILU) {
            const float4 u0 = *(const float4 *)(a.x2 + off), u1 = *(const float4 *)(a.x2 + off + 4);
            const float us[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
#pragma unroll
            for (int j = 0; j < 8; j++) v[j] = __fmul_rn(xs[j] / (1.0f + expf(-xs[j])), us[j]);
        } else {
#pragma unroll
            for (int j = 0; j < 8; j++) v[j] = xs[j];
        }
    }
    tc_quant_store(v, ta, ad, mt, nb, b, r);
    }
}

}  // namespace hyk
