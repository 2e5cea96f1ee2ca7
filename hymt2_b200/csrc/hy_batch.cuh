// hy_batch.cuh — ragged multi-sequence batches and the continuous-batching
// server built on them.  Part of hy_backend.cu's translation unit (it uses
// HyCtx, the layer loop and the tensor-core linear defined there).
//
// A batch is a list of tokens, token t at position tok_pos[t] of sequence
// slot tok_slot[t].  The bf16 KV cache is paged: pages of kPageRows
// positions, laid out [L][npages][K | V][kPageRows][kvdim], and a page table
// [slots][page_max] maps (slot, pos / kPageRows) to a page.  The direct
// batch API gives slot s the pages s * page_max + j; the server allocates
// pages as its sequences grow and shares cached prompt pages between
// requests (hy_pages.h).  One forward pass embeds every token, runs all
// layers over the whole batch (tensor-core GEMMs from kTcMinTokens tokens
// up, so a step of 256 decode tokens or a 32 x 256 prefill is one GEMM per
// projection), then the LM head over the selected rows with one argmax per
// row (reference semantics: first maximum wins, src/model.c:945-948).
//
// The server (reference gen_ids, src/model.c:914-958, for many requests at
// once; a request ends at max_new ids or at its first stop id, which then
// frees its slot and its pages): every step feeds one token of each decoding
// sequence plus prompt chunks of newly admitted ones, up to a token budget.
// An admitted prompt first takes the longest chain of cached full pages
// matching its leading tokens by reference, then copies the matching first
// rows of one cached page that continues the chain (the reference's
// longest-common-prefix reuse, src/model.c:931-936, against every cached
// prompt instead of the previous one); the last prompt token is always
// recomputed for its logits.  When a prompt has been fed, its full pages are
// sealed into the cache.

struct Batch {
    int slots = 0, slot_ctx = 0, max_tokens = 0, max_out = 0;
    int page_max = 0;  // pages per slot: ceil(slot_ctx / kPageRows)
    int npages = 0;    // device pages: slots * page_max for the slots, the rest for cached prompt pages
    uint16_t *kv = nullptr;
    int *d_pages = nullptr, *h_pages = nullptr;  // page table [slots][page_max] (h: pinned copy)
    float *h = nullptr, *qkv = nullptr, *ao = nullptr, *g = nullptr, *u = nullptr;
    // tok [max_tokens] | slot [max_tokens] | pos [max_tokens] | rows [max_out] | qblk [2 max_tokens]
    int *d_in = nullptr;
    int *h_in = nullptr;   // pinned staging of d_in
    int nqb = 0;           // attention query blocks of the uploaded pass
    float *sel = nullptr;  // [max_out][H] residual rows for the head
    float *logits = nullptr;  // [max_out][vocab]
    int *d_ids = nullptr, *h_ids = nullptr;
    long long page_stride(const HyCtx *c) const { return (long long)2 * kPageRows * c->kvd; }
    size_t layer_stride(const HyCtx *c) const { return (size_t)npages * page_stride(c); }
    size_t kv_elems(const HyCtx *c) const { return (size_t)c->L * layer_stride(c); }
    // the direct batch API's table: slot s owns pages s * page_max + j
    void identity_pages() {
        for (int sl = 0; sl < slots; sl++)
            for (int j = 0; j < page_max; j++) h_pages[sl * page_max + j] = sl * page_max + j;
    }
    int *tok() const { return d_in; }
    int *slot() const { return d_in + max_tokens; }
    int *pos() const { return d_in + 2 * max_tokens; }
    int *rows() const { return d_in + 3 * max_tokens; }
    size_t qblk_off() const { return (size_t)3 * max_tokens + max_out; }
    size_t in_ints() const { return (size_t)5 * max_tokens + max_out; }
};

// ---------------------------------------------------------------- kernels

// sel[i] = h[rows[i]]
__global__ void batch_gather(const float *h, int H, const int *rows, float *sel) {
    const float4 *src = (const float4 *)(h + (size_t)rows[blockIdx.x] * H);
    float4 *dst = (float4 *)(sel + (size_t)blockIdx.x * H);
    for (int i = threadIdx.x; i < H / 4; i += blockDim.x) dst[i] = src[i];
}

// ids[r] = first index of the maximum of logits[r][0 .. n)
__global__ void __launch_bounds__(1024) rows_argmax(const float *logits, long long ld, int n, int *ids) {
    __shared__ unsigned long long red[32];
    const float *row = logits + (size_t)blockIdx.x * ld;
    unsigned long long best = 0;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const unsigned long long k = argmax_key(row[i], (uint32_t)i);
        if (k > best) best = k;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long v = __shfl_xor_sync(0xffffffffu, best, o);
        if (v > best) best = v;
    }
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    if (l == 0) red[w] = best;
    __syncthreads();
    if (w == 0) {
        best = l < (int)(blockDim.x >> 5) ? red[l] : 0ull;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const unsigned long long v = __shfl_xor_sync(0xffffffffu, best, o);
            if (v > best) best = v;
        }
        if (l == 0) ids[blockIdx.x] = best ? (int)argmax_index(best) : 0;
    }
}

// Rows [0, nrows) of page src -> page dst, K and V of every layer; grid
// (layers, 2); 16-byte words.
__global__ void kv_copy_page(uint16_t *kv, size_t layer_stride, long long page_stride, int kvd, int src, int dst,
                             int nrows) {
    const size_t base = (size_t)blockIdx.x * layer_stride + (blockIdx.y ? (size_t)kPageRows * kvd : 0);
    const uint4 *s = (const uint4 *)(kv + base + (size_t)src * page_stride);
    uint4 *d = (uint4 *)(kv + base + (size_t)dst * page_stride);
    const int words = nrows * kvd / 8;
    for (int i = threadIdx.x; i < words; i += blockDim.x) d[i] = s[i];
}

// ---------------------------------------------------------------- host side

void batch_free(HyCtx *c) {
    Batch *b = c->bat;
    if (!b) return;
    cudaFree(b->kv);
    cudaFree(b->h);
    cudaFree(b->qkv);
    cudaFree(b->ao);
    cudaFree(b->g);
    cudaFree(b->u);
    cudaFree(b->d_in);
    cudaFree(b->sel);
    cudaFree(b->logits);
    cudaFree(b->d_ids);
    cudaFree(b->d_pages);
    if (b->h_pages) cudaFreeHost(b->h_pages);
    if (b->h_in) cudaFreeHost(b->h_in);
    if (b->h_ids) cudaFreeHost(b->h_ids);
    delete b;
    c->bat = nullptr;
    c->max_tokens = kMaxChunk;
}

bool batch_prepare(HyCtx *c, int slots, int slot_ctx, int max_tokens, int max_out) {
    REQ(c, c->fused && c->embd && c->outw, "model not prepared (fused_prepare, embedding, LM head)");
    REQ(c, slots >= 1 && slot_ctx >= 1 && slot_ctx <= c->ctx && max_tokens >= 1 && max_out >= 1 &&
               max_out <= max_tokens,
        "bad batch geometry (slot_ctx must not exceed the prepared context)");
    if (c->bat && c->bat->slots == slots && c->bat->slot_ctx == slot_ctx && c->bat->max_tokens == max_tokens &&
        c->bat->max_out == max_out)
        return true;
    batch_free(c);
    Batch *b = new Batch();
    c->bat = b;
    b->slots = slots;
    b->slot_ctx = slot_ctx;
    b->max_tokens = max_tokens;
    b->max_out = max_out;
    b->page_max = (slot_ctx + kPageRows - 1) / kPageRows;
    // the slots' own pages, plus a quarter more (at least one slot's worth)
    // that keeps finished prompts' pages cached for later requests
    b->npages = slots * b->page_max + (slots * b->page_max / 4 > b->page_max ? slots * b->page_max / 4 : b->page_max);
    const size_t T = (size_t)max_tokens;
    CK(c, cudaMalloc(&b->kv, b->kv_elems(c) * 2));
    CK(c, cudaMemsetAsync(b->kv, 0, b->kv_elems(c) * 2, c->st));
    CK(c, cudaMalloc(&b->d_pages, (size_t)slots * b->page_max * 4));
    CK(c, cudaMallocHost(&b->h_pages, (size_t)slots * b->page_max * 4));
    b->identity_pages();
    CK(c, cudaMemcpyAsync(b->d_pages, b->h_pages, (size_t)slots * b->page_max * 4, cudaMemcpyHostToDevice, c->st));
    CK(c, cudaMalloc(&b->h, T * c->H * 4));
    CK(c, cudaMalloc(&b->qkv, T * (c->qd + 2 * c->kvd) * 4));
    CK(c, cudaMalloc(&b->ao, T * c->qd * 4));
    CK(c, cudaMalloc(&b->g, T * c->F * 4));
    CK(c, cudaMalloc(&b->u, T * c->F * 4));
    CK(c, cudaMalloc(&b->d_in, b->in_ints() * 4));
    CK(c, cudaMallocHost(&b->h_in, b->in_ints() * 4));
    CK(c, cudaMalloc(&b->sel, (size_t)max_out * c->H * 4));
    CK(c, cudaMalloc(&b->logits, (size_t)max_out * c->outw->n * 4));
    CK(c, cudaMalloc(&b->d_ids, (size_t)max_out * 4));
    CK(c, cudaMallocHost(&b->h_ids, (size_t)max_out * 4));
    c->max_tokens = max_tokens > kMaxChunk ? max_tokens : kMaxChunk;
    CK(c, cudaStreamSynchronize(c->st));
    return true;
}

Fwd fwd_batch(HyCtx *c) {
    const Batch &b = *c->bat;
    Fwd f;
    memset(&f, 0, sizeof f);
    f.h = b.h;
    f.qkv = b.qkv;
    f.ao = b.ao;
    f.g = b.g;
    f.u = b.u;
    f.kv = b.kv;
    f.layer_stride = b.layer_stride(c);
    f.pages = b.d_pages;
    f.page_max = b.page_max;
    f.page_stride = b.page_stride(c);
    f.kv_ctx = b.slot_ctx;
    f.v_rows = kPageRows;
    f.tok_pos = b.pos();
    f.tok_slot = b.slot();
    f.qblk = b.d_in + b.qblk_off();
    f.nqb = b.nqb;
    return f;
}

// Upload nt tokens (tok / slot / pos) and nout head rows from the pinned
// staging area (filled by the caller at the same offsets as on the device),
// with the attention query blocks: runs of <= kFaQ tokens of one slot at
// consecutive positions.
bool batch_upload(HyCtx *c, int nt, int nout) {
    Batch &b = *c->bat;
    const size_t T = (size_t)b.max_tokens;
    const int *slot = b.h_in + T, *pos = b.h_in + 2 * T;
    int *qb = b.h_in + b.qblk_off();
    int nqb = 0;
    for (int t = 0; t < nt; t++) {
        if (nqb > 0) {
            int *blk = qb + 2 * (nqb - 1);
            const int last = blk[0] + blk[1] - 1;
            if (blk[1] < kFaQ && slot[t] == slot[last] && pos[t] == pos[last] + 1) {
                blk[1]++;
                continue;
            }
        }
        qb[2 * nqb] = t;
        qb[2 * nqb + 1] = 1;
        nqb++;
    }
    b.nqb = nqb;
    for (int part = 0; part < 3; part++)
        CK(c, cudaMemcpyAsync(b.d_in + part * T, b.h_in + part * T, (size_t)nt * 4, cudaMemcpyHostToDevice, c->st));
    if (nout > 0)
        CK(c, cudaMemcpyAsync(b.rows(), b.h_in + 3 * T, (size_t)nout * 4, cudaMemcpyHostToDevice, c->st));
    CK(c, cudaMemcpyAsync(b.d_in + b.qblk_off(), qb, (size_t)nqb * 8, cudaMemcpyHostToDevice, c->st));
    return true;
}

// One forward pass over the uploaded batch; argmax ids of the nout head rows
// (over the first vocab_out logits) land in b.d_ids, the logits in b.logits.
bool batch_run(HyCtx *c, int nt, int nout, int vocab_out) {
    Batch &b = *c->bat;
    // every kernel of the pass is a programmatic dependent of the one before
    // (each waits for it before touching its data; setup overlaps its tail)
    if (!launch(c, embed_rows, dim3(nt), dim3(256), 0, true, desc(c->embd, nullptr, 0), (const int *)b.tok(), b.h, -1))
        return false;
    if (!layers_forward(c, fwd_batch(c), nt, true)) return false;
    if (nout < 1) return true;
    if (!launch(c, batch_gather, dim3(nout), dim3(128), 0, false, (const float *)b.h, c->H, (const int *)b.rows(),
                b.sel))
        return false;
    HyWeight *ws[1] = {c->outw};
    float *outs[1] = {b.logits};
    const int lds[1] = {c->outw->n};
    GemvArgs a = gemv_args(nout, c->H);
    a.act = ACT_NORM;
    a.x = b.sel;
    a.ldx = c->H;
    a.norm_w = c->d_out_norm;
    a.eps = c->eps;
    if (tc_usable(c, nout, ws, 1)) {
        if (!tc_linear(c, a, nout, ws, outs, lds, 1, 0, true)) return false;
    } else {
        a.epi = EPI_STORE;
        a.nw = 1;
        a.rows_total = c->outw->n;
        a.w[0] = desc(c->outw, b.logits, c->outw->n);
        if (!run_gemv(c, a, false, 2)) return false;
    }
    return launch(c, rows_argmax, dim3(nout), dim3(1024), 0, false, (const float *)b.logits, (long long)c->outw->n,
                  vocab_out, b.d_ids);
}

bool kv_copy_rows(HyCtx *c, int src_page, int dst_page, int nrows) {
    Batch &b = *c->bat;
    if (nrows < 1) return true;
    return launch(c, kv_copy_page, dim3(c->L, 2), dim3(256), 0, false, b.kv, b.layer_stride(c), b.page_stride(c),
                  c->kvd, src_page, dst_page, nrows);
}

// Rows 0 .. npos - 1 of slot src -> slot dst through the current page table.
bool kv_copy(HyCtx *c, int src, int dst, int npos) {
    Batch &b = *c->bat;
    for (int j = 0; j * kPageRows < npos; j++) {
        const int n = npos - j * kPageRows < kPageRows ? npos - j * kPageRows : kPageRows;
        if (!kv_copy_rows(c, b.h_pages[src * b.page_max + j], b.h_pages[dst * b.page_max + j], n)) return false;
    }
    return true;
}

// ---------------------------------------------------------------- server

struct ServeSeq {
    int req, slot, n, fed, gen, last;
    bool stopped;            // emitted a stop id
    bool sealed;             // its prompt pages went into the cache
    std::vector<int> pages;  // its page table row
};

bool serve_run(HyCtx *c, const int *prompts, const int *off, int nreq, int max_new, const int *stop_ids, int n_stop,
               int vocab_out, int step_tokens, int *out, int *out_len, hyc_serve_stats *st) {
    Batch &b = *c->bat;
    const int S = b.slots, T = b.max_tokens, PM = b.page_max;
    REQ(c, step_tokens >= 1 && step_tokens <= T, "step token budget exceeds the batch capacity");
    REQ(c, max_new >= 1 && b.max_out >= S, "batch head rows must cover every slot");
    for (int r = 0; r < nreq; r++) {
        const int n = off[r + 1] - off[r];
        REQ(c, n >= 1 && n + max_new - 1 <= b.slot_ctx, "request does not fit a slot's context");
    }
    PagePool pool;
    pool.reset(b.npages);
    for (int i = 0; i < S * PM; i++) b.h_pages[i] = 0;  // rows of idle slots are never read
    bool table_dirty = true;
    // the page holding position pos of q, allocated (with any before it) on first use
    auto need_page = [&](ServeSeq &q, int pos) -> bool {
        while ((int)q.pages.size() <= (pos >> kPageShift)) {
            const int pg = pool.alloc();
            REQ(c, pg >= 0, "KV page pool exhausted");
            b.h_pages[q.slot * PM + (int)q.pages.size()] = pg;
            q.pages.push_back(pg);
            table_dirty = true;
        }
        return true;
    };
    std::vector<int> free_slots;
    for (int s = S - 1; s >= 0; s--) free_slots.push_back(s);
    std::vector<ServeSeq> act;
    // admission order: longest prompts first (ties in request order), so the
    // last wave is not held up by a long prompt admitted late
    std::vector<int> order((size_t)nreq);
    for (int r = 0; r < nreq; r++) order[(size_t)r] = r;
    std::stable_sort(order.begin(), order.end(),
                     [&](int x, int y) { return off[x + 1] - off[x] > off[y + 1] - off[y]; });
    int next = 0, done = 0;
    std::vector<int> row_seq;
    memset(st, 0, sizeof *st);
    for (size_t i = 0; i < (size_t)nreq * max_new; i++) out[i] = -1;
    int *h_tok = b.h_in, *h_slot = b.h_in + T, *h_pos = b.h_in + 2 * T, *h_rows = b.h_in + 3 * T;
    while (done < nreq) {
        // admit while there are free slots
        while (!free_slots.empty() && next < nreq) {
            ServeSeq q;
            q.req = order[(size_t)next++];
            q.slot = free_slots.back();
            free_slots.pop_back();
            q.n = off[q.req + 1] - off[q.req];
            q.fed = 0;
            q.gen = 0;
            q.last = -1;
            q.stopped = false;
            q.sealed = false;
            const int *p = prompts + off[q.req];
            // cached prefix: whole pages by reference, then a copy of the first rows of one more
            PagePool::Match m = pool.match(p, q.n - 1);
            for (size_t j = 0; j < m.full.size(); j++) {
                b.h_pages[q.slot * PM + (int)j] = m.full[j];
                q.pages.push_back(m.full[j]);
            }
            table_dirty = table_dirty || !m.full.empty();
            if (m.src >= 0 && m.src_rows > 0) {
                pool.ref(m.src);  // not evictable while this request takes its own page
                const bool ok = need_page(q, m.rows - 1) && kv_copy_rows(c, m.src, q.pages.back(), m.src_rows);
                pool.unref(m.src);
                if (!ok) return false;
                st->copied_rows += m.src_rows;
            }
            q.fed = m.rows;
            if (m.rows > 0) {
                st->prefix_hits++;
                st->prefix_tokens += m.rows;
                st->shared_pages += (long long)m.full.size();
            }
            act.push_back(q);
        }
        // one step: a token of every decoding sequence, then prompt chunks; while
        // fewer than half the slots decode (waves of admissions, the drain), the
        // prompt chunks may fill the whole pass capacity
        int ndec = 0;
        for (const ServeSeq &q : act) ndec += q.fed >= q.n;
        const int budget = ndec < S / 2 ? T : step_tokens;
        st->active_seq_steps += (long long)act.size();
        int nt = 0, nout = 0;
        row_seq.clear();
        for (size_t i = 0; i < act.size(); i++) {
            ServeSeq &q = act[i];
            if (q.fed < q.n || nt >= budget) continue;
            if (!need_page(q, q.n + q.gen - 1)) return false;
            h_tok[nt] = q.last;
            h_slot[nt] = q.slot;
            h_pos[nt] = q.n + q.gen - 1;
            h_rows[nout++] = nt++;
            row_seq.push_back((int)i);
            st->decode_tokens++;
        }
        for (size_t i = 0; i < act.size() && nt < budget; i++) {
            ServeSeq &q = act[i];
            if (q.fed >= q.n) continue;
            const int *p = prompts + off[q.req];
            const int take = (q.n - q.fed) < (budget - nt) ? (q.n - q.fed) : (budget - nt);
            if (!need_page(q, q.fed + take - 1)) return false;
            for (int j = 0; j < take; j++) {
                h_tok[nt] = p[q.fed + j];
                h_slot[nt] = q.slot;
                h_pos[nt] = q.fed + j;
                nt++;
            }
            q.fed += take;
            st->prefill_tokens += take;
            if (q.fed == q.n) {
                h_rows[nout++] = nt - 1;
                row_seq.push_back((int)i);
            }
        }
        REQ(c, nt > 0, "server made no progress");
        if (table_dirty) {
            CK(c, cudaMemcpyAsync(b.d_pages, b.h_pages, (size_t)S * PM * 4, cudaMemcpyHostToDevice, c->st));
            table_dirty = false;
        }
        if (!batch_upload(c, nt, nout) || !batch_run(c, nt, nout, vocab_out)) return false;
        CK(c, cudaMemcpyAsync(b.h_ids, b.d_ids, (size_t)nout * 4, cudaMemcpyDeviceToHost, c->st));
        CK(c, cudaStreamSynchronize(c->st));
        st->steps++;
        // prompts fed in full: their full pages become shareable (each one's
        // parent must be cached, so the chain stops at a page another
        // request cached first)
        for (size_t i = 0; i < act.size(); i++) {
            ServeSeq &q = act[i];
            if (q.sealed || q.fed < q.n) continue;
            q.sealed = true;
            const int *p = prompts + off[q.req];
            for (int j = 0; (j + 1) * kPageRows <= q.n; j++)
                if (!pool.cached(q.pages[j]) && !pool.seal(q.pages[j], j ? q.pages[j - 1] : -1, p + j * kPageRows))
                    break;
        }
        for (int i = 0; i < nout; i++) {
            ServeSeq &q = act[row_seq[i]];
            const int id = b.h_ids[i];
            out[(size_t)q.req * max_new + q.gen] = id;
            q.gen++;
            q.last = id;
            for (int k = 0; k < n_stop; k++)
                if (id == stop_ids[k]) q.stopped = true;
        }
        // retire finished sequences: their slots and page references
        size_t w = 0;
        for (size_t i = 0; i < act.size(); i++) {
            ServeSeq &q = act[i];
            if (q.stopped || (q.fed == q.n && q.gen >= max_new)) {
                free_slots.push_back(q.slot);
                for (int pg : q.pages) pool.unref(pg);
                done++;
                st->generated += q.gen;
                out_len[q.req] = q.stopped ? q.gen - 1 : q.gen;  // the stop id is not output
            } else {
                if (w != i) act[w] = std::move(act[i]);
                w++;
            }
        }
        act.resize(w);
    }
    st->evictions = pool.evictions();
    // the direct batch API's table again
    b.identity_pages();
    CK(c, cudaMemcpyAsync(b.d_pages, b.h_pages, (size_t)S * PM * 4, cudaMemcpyHostToDevice, c->st));
    CK(c, cudaStreamSynchronize(c->st));
    return tc_status(c);
}
