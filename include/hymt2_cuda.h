/* hymt2_cuda.h — C ABI of the B200 (sm_100a) device backend for hymt2.
 *
 * Drop-in entry points (what the hymt2 host binds):
 *   hy_cuda_create / hy_cuda_probe replace reference src/cuda.c:151-183 and
 *   src/cuda.c:18-34 (declared by the host in src/device.c:8-9).  The created
 *   device fills the host's `hy_device_ops` vtable (reference
 *   src/device.h:70-79) with the semantics listed there: upload / release /
 *   matmul / fused_prepare / fused_forward.
 *
 * Standalone entry points (hyc_*): the same implementation without the
 * host's device wrapper, plus the additive operations the host vtable cannot
 * express — on-device embedding, argmax and token feedback so a decode step
 * runs as one CUDA graph with no host synchronisation.
 *
 * Conventions follow the host's: bool/NULL (or int 0 / negative) for
 * success/failure, `info` strings on create, one host thread per handle.
 * After any CUDA error a handle is "broken" and refuses further work; the
 * host then falls back to its CPU path as it does today.
 */
#ifndef HYMT2_CUDA_H
#define HYMT2_CUDA_H

#include "hy_device_abi.h"

#ifdef __cplusplus
extern "C" {
#endif

#if defined(_WIN32)
#define HYC_API __declspec(dllexport)
#else
#define HYC_API __attribute__((visibility("default")))
#endif

/* ---- drop-in (replaces reference src/cuda.c) -------------------------- */

/* Replaces src/cuda.c:151 hy_cuda_create.  `pref` "auto" or a device
 * ordinal ("0", "1", ...).  Wraps the implementation with the host's
 * hy_device_wrap (src/device.c:25); returns NULL with a reason in `info` when
 * no sm_100 GPU is usable or when the host device layer is not linked in
 * (standalone shared-library use: call hyc_create instead). */
HYC_API hy_device *hy_cuda_create(const char *pref, char *info, size_t cap);
/* Replaces src/cuda.c:18 hy_cuda_probe: writes "1" when a CUDA driver and
 * device are present, else "0"; returns the same as int. */
HYC_API int hy_cuda_probe(char *out, int cap);

/* ---- standalone handle ------------------------------------------------ */

/* Create the backend on `device` (ordinal).  NULL + reason in `info` on failure. */
HYC_API void *hyc_create(int device, char *info, size_t cap);
/* The vtable hy_cuda_create registers with the host (reference
 * src/device.h:70-79 layout). */
HYC_API const hy_device_ops *hyc_device_ops(void);
/* Last error text of a handle ("" when none). */
HYC_API int hyc_last_error(void *impl, char *out, int cap);
/* cudaStream_t the handle launches on (for timing with external events). */
HYC_API void *hyc_stream(void *impl);
HYC_API int hyc_sync(void *impl);

/* ---- additive operations (no counterpart in the reference vtable) ----- */

/* Weight the device embedding lookup reads (the token embedding; may be the
 * same handle as the LM head when they are tied). */
HYC_API int hyc_set_embedding(void *impl, hy_dweight *embd);

/* Greedy generation entirely on the device: prefill prompt[keep..n) in
 * chunks (positions keep..n-1; positions < keep are reused from the device KV
 * cache, the longest-common-prefix contract of reference src/model.c:931-936),
 * then `max_new` argmax steps (first maximum over rows [0, vocab_out) wins,
 * src/model.c:945-948) with token feedback, stopping after a token in
 * stop_ids.  Writes the generated ids to out_ids and returns their count, or
 * a negative value on error.  Requires fused_prepare and hyc_set_embedding. */
HYC_API int hyc_generate(void *impl, const int *prompt, int n, int keep, int max_new, const int *stop_ids,
                         int n_stop, int vocab_out, int *out_ids);

/* Lower-level decode control used by hyc_generate and the benchmark:
 *  hyc_decode_begin: prefill like hyc_generate and leave the first generated
 *    token on the device (no synchronisation);
 *  hyc_decode_steps: enqueue `steps` greedy single-token steps (one
 *    persistent kernel launch when the model supports it and
 *    hyc_set_decode_mode has not selected the graph, else one graph per
 *    step; both give bit-identical results);
 *  hyc_decode_steps_host: the same, but every step's input token is copied
 *    from pinned host memory tok_io[s] and its result written back to
 *    tok_io[s+1] (tok_io must hold steps+1 ints, allocated with
 *    hyc_host_alloc);
 *  hyc_decode_read: synchronise and copy the emitted ids (returns count);
 *  hyc_decode_rewind: enqueue (asynchronously) a new next-token / next
 *    position; KV rows >= pos are overwritten by later steps.  Up to 500
 *    rewinds may be in flight before the stream is synchronised. */
HYC_API int hyc_decode_begin(void *impl, const int *prompt, int n, int keep, int max_new, const int *stop_ids,
                             int n_stop, int vocab_out);
HYC_API int hyc_decode_steps(void *impl, int steps);
HYC_API int hyc_decode_steps_host(void *impl, int steps, int *tok_io);
/* Resident host loop (the reference's gen_ids loop, src/model.c:943-954, with
 * the host reading every token and choosing the next input, without a launch
 * per token): hyc_decode_resident starts ONE persistent-kernel launch of up to
 * max_steps steps after hyc_decode_begin and returns at once.  io is 4 ints of
 * pinned host memory (hyc_host_alloc): [go, token in, done, token out].  Step
 * s runs once go >= s + 1 and takes its input token from io[1]; when it has
 * finished, io[3] holds its argmax and done = s + 1.  hyc_resident_go(io, s,
 * tok) releases step s with input tok (s < 0: stop the loop); call it for step
 * 0 before or after hyc_decode_resident.  hyc_resident_wait(io, s, &tok,
 * limit_ns) spins until step s is done and returns its token (0), -1 when the
 * loop ended with an error (done < 0) or -2 after limit_ns.  The kernel waits
 * for each go at most limit_ns (0: 2 s); a host that does not answer ends the
 * loop, hyc_sync then reports it once and the handle stays usable, with the
 * decode state after the last finished step.  Needs the persistent kernel
 * (hyc_decode_path() == 1); stop ids still end the emitted-id count as in
 * hyc_decode_read. */
HYC_API int hyc_decode_resident(void *impl, int max_steps, int *io, unsigned long long limit_ns);
HYC_API int hyc_resident_go(int *io, int step, int tok);
HYC_API int hyc_resident_wait(const int *io, int step, int *tok, unsigned long long limit_ns);
HYC_API int hyc_decode_read(void *impl, int *out_ids, int cap);
HYC_API int hyc_decode_rewind(void *impl, int pos, int tok);
HYC_API void *hyc_host_alloc(size_t bytes);
HYC_API void hyc_host_free(void *p);
/* Decode path selection (no reference counterpart; the reference's host
 * loop is src/model.c:914-958): mode 0 (the default) uses the persistent
 * kernel whenever the prepared model supports it (panel layer weights, Q6_K
 * head), mode 1 always the graph of per-layer launches.  hyc_decode_path returns 1 when
 * the next decode steps run the persistent kernel, 0 for the graph, and
 * writes the reason. */
HYC_API int hyc_set_decode_mode(void *impl, int mode);
/* Tensor-core path for multi-token chunks (no reference counterpart; it
 * serves the same forward_batch chunks, src/model.c:798-909): with on != 0
 * (the default) chunks of >= 32 tokens over STQ1_0 / Q2_0C panel, Q4_K and
 * Q6_K weights run the tcgen05 int8 GEMM with TMEM accumulators; 0 keeps
 * the dp4a GEMV kernels.  hyc_tc_test runs one such weight through that
 * GEMM on host inputs (act as hyc_gemv_test: 1 plain, 2 RMSNorm*w,
 * 3 SiLU(x)*x2; nt 1..256) and writes out[t*n + r]. */
HYC_API int hyc_set_tc(void *impl, int on);
/* STQ1_0 weight layout for later uploads (replaces the panel decision of
 * reference src/model.c:385-388, which always uploads the host-built panel):
 * native == 0 (the default) stores the panel (64 B of 2-bit codes + an fp32
 * scale per 256 weights, 68 B); native != 0 stores the file's own 42-byte
 * blocks (weight_t.data, row_bytes = 42 * k / 256), split per row into
 * qs | sign | d planes and decoded in registers by the GEMV kernels, with the
 * same per-block integers (reference stq1_0_dot_scalar, src/kernels.c:202-215).
 * The environment variable HYMT2_STQ_LAYOUT=native sets it at hyc_create.
 * The persistent decode kernel takes panels only; native layers decode
 * through the per-layer graph. */
HYC_API int hyc_set_stq_layout(void *impl, int native);
HYC_API int hyc_tc_test(void *impl, hy_dweight *w, int act, const float *x, const float *x2, const float *norm_w,
                        float eps, int nt, float *out);
HYC_API int hyc_decode_path(void *impl, char *why, int cap);
/* Failure detection without a fault: runs the bounded waits of the
 * persistent decode kernel (grid barrier) and of the tensor-core GEMM
 * (mbarrier) on targets nothing reaches, each giving up after limit_ns
 * (<= 1 s; the kernels themselves use 2 s).  out[0] = 1 if the barrier wait
 * passed (expected 0), out[1] = the error word it raised (expected 1, the
 * barrier timeout code the persistent kernel reports through
 * hyc_decode_read), out[2] = 1 if the mbarrier wait completed (expected 0).
 * The handle stays usable afterwards.  Returns 0 or -1. */
HYC_API int hyc_wait_probe(void *impl, unsigned long long limit_ns, int *out);

/* ---- ragged multi-sequence batches and the continuous-batching server --
 * (additive extension, no reference counterpart: the reference serves one
 * sequence per handle, src/model.c:914-958; these run many of them through
 * one forward pass).  After fused_prepare and hyc_set_embedding:
 * hyc_batch_prepare allocates a paged KV cache (pages of 16 positions in
 * every layer; each of the `slots` sequences holds up to slot_ctx rows,
 * slot_ctx <= the prepared ctx, plus a quarter more pages for the server's
 * prompt cache), and activations for up to max_tokens tokens per pass with
 * up to max_out head rows.  hyc_batch_forward runs one pass over host arrays: token t is
 * tokens[t] at position tok_pos[t] of slot tok_slot[t] (its K/V row is
 * written there; it attends to rows 0..tok_pos[t] of that slot, which must
 * be filled by this or earlier passes; no (slot, position) twice in one
 * pass).  For each i < nout, out_ids[i] is the argmax over the first
 * vocab_out logits (all when <= 0) of token out_rows[i], after the output
 * RMSNorm and LM head; `logits` (optional) receives them as [nout][n_vocab].
 * hyc_batch_kv_copy copies rows 0..npos-1 of every layer from one slot to
 * another; hyc_batch_kv_read reads one slot's layer like hyc_kv_read.
 * hyc_serve generates max_new greedy tokens for each of nreq requests
 * (request r = prompts[prompt_off[r] .. prompt_off[r+1])), as the
 * reference's gen_ids would one request at a time, with continuous batching
 * over the prepared slots: each pass feeds one token of every decoding
 * request plus prompt chunks of newly admitted ones, at most step_tokens in
 * all (<= max_tokens; max_out must be >= slots), or up to max_tokens while
 * fewer than half the slots are decoding; requests are admitted longest
 * prompt first.  Pages are allocated as
 * sequences grow and freed when they end; a fed prompt's full pages stay
 * cached (least recently used evicted first), and a new prompt shares the
 * longest chain of cached pages its leading tokens match, by reference,
 * then copies the matching first rows of one more cached page (the
 * reference's longest-common-prefix reuse, src/model.c:931-936, against
 * every cached prompt; the last prompt token is always recomputed).  A request
 * also ends at its first id in stop_ids (n_stop <= 16), as the reference's
 * loop breaks there.  out_ids is [nreq][max_new]: the ids before the stop
 * id, then the stop id, then -1; out_len[r] counts the ids before the stop
 * id (max_new when none came).  All return 0 or -1 (hyc_last_error). */
typedef struct hyc_serve_stats {
    long long steps, decode_tokens, prefill_tokens, prefix_hits, prefix_tokens, generated;
    long long shared_pages, copied_rows, evictions;  /* paged KV: pages shared by reference, rows copied, cached
                                                        pages evicted */
    long long active_seq_steps;                      /* sum over passes of the requests holding a slot */
} hyc_serve_stats;
HYC_API int hyc_batch_prepare(void *impl, int slots, int slot_ctx, int max_tokens, int max_out);
HYC_API int hyc_batch_forward(void *impl, const int *tokens, const int *tok_slot, const int *tok_pos, int nt,
                              const int *out_rows, int nout, int vocab_out, int *out_ids, float *logits);
HYC_API int hyc_batch_kv_copy(void *impl, int src_slot, int dst_slot, int npos);
HYC_API int hyc_batch_kv_read(void *impl, int slot, int layer, int npos, uint16_t *k, uint16_t *v);
HYC_API int hyc_serve(void *impl, const int *prompts, const int *prompt_off, int nreq, int max_new,
                      const int *stop_ids, int n_stop, int vocab_out, int step_tokens, int *out_ids, int *out_len,
                      hyc_serve_stats *stats);

/* ---- kernel-level hooks for parity tests (host buffers, synchronous) -- */

/* Device Q8_K quantiser on x[nt][k]; writes full host blocks. */
HYC_API int hyc_quantize_q8k(void *impl, const float *x, int k, int nt, q8k_block *y);
/* Exact per-block int32 accumulators of the GEMV for host blocks xq[nt][k/256]:
 * out[t][row][b] (Q4_K: pairs sumi, summ).  Returns ints per (t, row). */
HYC_API int hyc_block_ints(void *impl, hy_dweight *w, const q8k_block *xq, int nt, int32_t *out);
/* The same per-block integers from the tcgen05 GEMM that chunks of >= 32
 * tokens use (STQ1_0 / Q2_0C panels, Q4_K, Q6_K), read from TMEM for host
 * blocks xq[nt][k/256] (no activation prologue), nt up to 65536, with the
 * launch shape (whole or 64-row-slice tiles) the product path picks for nt:
 * out[t][row][b] (Q4_K: pairs sumi, summ; reference src/kernels.c:565-581,
 * 808-835, 861-877).  Returns ints per (t, row). */
HYC_API int hyc_tc_block_ints(void *impl, hy_dweight *w, const q8k_block *xq, int nt, int32_t *out);
/* One row of a device weight as fp32. */
HYC_API int hyc_dequant_row(void *impl, hy_dweight *w, int row, float *dst);
/* fp32-activation GEMV (Q8_0 / F16 / F32 weights): out[t*n + r]. */
HYC_API int hyc_matmul_f32(void *impl, hy_dweight *w, const float *x, int nt, float *out);
/* One GEMV with a fused activation prologue on host inputs: act 1 = x as is,
 * 2 = RMSNorm(x[t]) * norm_w, 3 = SiLU(x) * x2; the Q8_K formats then
 * quantise on the device.  epi_add != 0 adds into the given `out`. */
HYC_API int hyc_gemv_test(void *impl, hy_dweight *w, int act, const float *x, const float *x2, const float *norm_w,
                          float eps, int nt, int epi_add, float *out);
/* Up to three weights of equal k sharing one activation (act 1 plain, 2
 * RMSNorm*w), merged into launches as the fused layer merges q|k|v and
 * gate|up; outs[i] receives [nt][rows_i]. */
HYC_API int hyc_gemv_multi_test(void *impl, hy_dweight *const *ws, int cnt, int act, const float *x,
                                const float *norm_w, float eps, int nt, float *const *outs);
/* Attention with its fused rope -> q/k RMSNorm -> bf16 KV-store prologue on
 * host buffers (qkv [nt][q|k|v] pre-rope; kc/vc [ctx][kvdim] in/out;
 * ao [nt][qdim]).  nt == 1 runs the split-KV decode kernel. */
HYC_API int hyc_attention_test(void *impl, int heads, int kv_heads, int hdim, int ctx, int nt, int pos0, float eps,
                               const float *qkv, uint16_t *kc, uint16_t *vc, const float *q_norm,
                               const float *k_norm, const float *rope_cos, const float *rope_sin, float *ao);
/* Copy an internal activation buffer of the fused state to the host (after
 * synchronising): 0 residual h, 1 q|k|v, 2 attention output, 3 gate, 4 up;
 * `count` floats from the start of the buffer. */
HYC_API int hyc_debug_buffer(void *impl, int which, float *out, size_t count);
/* Debug timeline of the captured graphs: hyc_trace(impl, 1) rebuilds them
 * with one slot per kernel; hyc_trace_read copies [max_slots][4] %globaltimer
 * stamps (launch, past wait, past prologue, end), then [max_slots][4]
 * sub-phase stamps of CTA 0, then [max_slots][4] (clock64, globaltimer) of
 * CTA 0 at its wait and its end; returns the number of slots in use. */
HYC_API int hyc_trace(void *impl, int on);
HYC_API int hyc_trace_read(void *impl, unsigned long long *out, int max_slots);
/* Persistent decode kernel timeline of the last launch made while tracing:
 * %globaltimer of block 0 at each step start and before/after every grid
 * barrier (per step: 1 + 10 per layer + 2 stamps).  Returns stamps copied. */
HYC_API int hyc_mega_timeline(void *impl, unsigned long long *out, int cap);
/* bf16 KV rows [0, npos) of one layer of the fused cache. */
HYC_API int hyc_kv_read(void *impl, int layer, int npos, uint16_t *k, uint16_t *v);
/* RoPE tables exactly as the host loader computes them (src/model.c:537,576-586). */
HYC_API int hyc_rope_tables(float freq_base, float alpha, int hdim, int rope_dim, int ctx, float *cos_out,
                            float *sin_out);
/* Number of kernels this handle has enqueued so far (graph replays count
 * every kernel node of the graph). */
HYC_API long long hyc_launch_count(void *impl);
/* Enqueue `iters` launches of one hot operation of the decode step for
 * timing: 0 LM head + argmax, 1 q|k|v GEMV, 2 gate|up GEMV, 3 down GEMV,
 * 4 o_proj GEMV, 5 decode attention; layer weights rotate over all layers. */
HYC_API int hyc_bench_op(void *impl, int op, int iters);

/* ---- tensor parallelism (the optional split of config 4) -------------- */

/* One process per GPU; each handle holds one rank's share of the model,
 * uploaded and fused_prepare'd with the rank's shape: query heads
 * [r*heads/world, (r+1)*heads/world) with the KV heads they use (a KV head
 * is replicated when world > kv_heads), gate/up rows and down K-columns of
 * FFN slice r, o_proj with the rank's K-columns, and the LM head's
 * vocabulary rows [vocab0, vocab0 + n) (the embedding table whole).  The
 * layer loop then adds the sum over ranks of the o_proj and down partial
 * products to the residual (a one-shot push over NVLink peer memory, the
 * sum in rank order: every rank holds bit-identical activations), and the
 * greedy token is the largest (logit, first index) key over the ranks.
 * Splits the reference's layer loop src/model.c:824-882 and its head and
 * argmax :884-900, 945-948; no counterpart in its device interface.
 * hyc_tp_init: allocate and zero the exchange area, write its CUDA IPC
 * handle (64 bytes) to handle_out; returns the handle size or -1.
 * hyc_tp_connect: map every peer's area (handles of all ranks, 64 bytes
 * each, in rank order); call it on every rank only after every rank's
 * hyc_tp_init has returned.  Returns 0 or -1.  Decode (hyc_decode_begin /
 * steps / read, hyc_generate) then runs the split; the persistent kernel,
 * fused_forward and the batch engine are refused on a rank.  A wait for a
 * peer is bounded (2 s); a timeout marks the handle broken and hyc_sync /
 * hyc_decode_read report it. */
HYC_API int hyc_tp_init(void *impl, int rank, int world, int vocab0, unsigned char *handle_out);
HYC_API int hyc_tp_connect(void *impl, const unsigned char *handles);

/* ---- allocation-free decode attention -------------------------------- */

/* No counterpart in the reference (its CUDA path allocates every buffer in
 * fused_prepare).  For callers that cannot allocate device memory at the
 * point of the call — for example a host whose own arena or caching
 * allocator already holds all free device memory, or a serving loop that
 * must not let cudaMalloc/cudaFree synchronise the device — this runs the
 * split-KV decode attention of one token (rope -> q/k RMSNorm -> bf16 K/V
 * store at *d_pos -> causal GQA softmax over positions 0..*d_pos) on
 * caller-provided DEVICE buffers and allocates nothing: no cudaMalloc,
 * cudaFree or allocating library call.  Its scratch (split partials and
 * per-KV-head tickets) is a file-scope device array of 512 KiB + 256 B that
 * every GPU loading this library keeps until the process exits.
 *   d_qkv [q | k | v] (pre-rope, heads*hdim + 2*kv_heads*hdim floats);
 *   d_kc, d_vc [ctx][kv_heads*hdim] bf16 caches (row *d_pos is written);
 *   d_rope_cos/sin [ctx][hdim/2]; d_q_norm, d_k_norm [hdim]; d_ao [heads*hdim].
 * Limits: hdim 64 or 128; heads/kv_heads in {1,2,4,8};
 * kv_heads * ceil(ctx/128) * (heads/kv_heads) * (hdim+2) <= 131072 and
 * kv_heads <= 64 — larger shapes return -2.  Returns 0, -1 (bad argument),
 * -2 (beyond the scratch maximum) or -3 (CUDA error); `err` (optional)
 * receives a message.  Work is enqueued on `stream` (a cudaStream_t).
 * *d_pos is read on the device only, so keeping 0 <= *d_pos < ctx is the
 * caller's job: for a position outside that range the kernel writes nothing
 * (d_ao and both caches keep their contents) and the call still returns 0.
 * The first call on a device looks up the scratch address (once per device,
 * with that device current); make that first call before any stream
 * capture.  All calls share the one scratch array and it keeps the last
 * call's contents (the tickets are cleared on the stream before each
 * launch), so calls whose executions overlap on the GPU race with each
 * other: serialise them, e.g. on one stream. */
HYC_API int hyc_attention_decode_noalloc(void *stream, int heads, int kv_heads, int hdim, int ctx, const int *d_pos,
                                         float eps, float *d_qkv, uint16_t *d_kc, uint16_t *d_vc,
                                         const float *d_q_norm, const float *d_k_norm, const float *d_rope_cos,
                                         const float *d_rope_sin, float *d_ao, char *err, int err_cap);

#ifdef __cplusplus
}
#endif
#endif
