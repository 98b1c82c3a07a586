// Forward passes, greedy generation and speculative decoding.
//
//  * predict / hidden / next_token follow engine/src/model.rs:143-240 with
//    one host sync per call (the reference's gpu_finish, gpu.m:114-128).
//  * generate (model.rs:268-285) and generate_speculative (speculative.rs:
//    43-143) run on the device: the whole loop is one CUDA graph whose WHILE
//    node repeats a round and whose IF nodes skip draft passes past the
//    budget or an end-of-sequence.  Acceptance, KV rollback (a length
//    update) and the draft catch-up are small kernels between the passes,
//    so a generation costs one host synchronisation.
//  * JL_SPEC_HOST keeps the reference's host-side control flow for
//    comparison.
#include <algorithm>
#include <chrono>
#include <cstdio>
#include <cstring>

#include "jl_internal.h"
#include "kernels.cuh"
#include "loop.cuh"
#include "ptx.cuh"
#include "timeline.cuh"

namespace jl {

jl_status add_conditional(cudaGraph_t graph, cudaGraphNode_t* deps, size_t ndeps,
                          cudaGraphConditionalHandle h, cudaGraphConditionalNodeType type,
                          cudaGraphNode_t* node, cudaGraph_t* body) {
    cudaGraphNodeParams p = {};
    p.type = cudaGraphNodeTypeConditional;
    p.conditional.handle = h;
    p.conditional.type = type;
    p.conditional.size = 1;
    JL_CUDA(cudaGraphAddNode(node, graph, deps, ndeps, &p));
    *body = p.conditional.phGraph_out[0];
    return JL_OK;
}

int att_splits_for(const jl_model* m, size_t max_ctx) {
    const size_t pages = (max_ctx + PAGE - 1) / PAGE;
    const int nwin = (int)std::max<size_t>(1, (pages + ATT_WIN - 1) / ATT_WIN);
    const int wpc = (nwin + ATT_ZMAX - 1) / ATT_ZMAX;  // as the attention kernel splits a row
    const int need = (nwin + wpc - 1) / wpc;
    int s = 1;
    while (s < need) s <<= 1;
    return std::min(s, std::max(1, m->att_smax));
}

jl_status stage_begin(jl_model* m, StageSlot** out) {
    StageSlot& sl = m->stage[m->stage_next];
    m->stage_next = (m->stage_next + 1) % STAGE_SLOTS;
    if (sl.pending) {
        JL_CUDA(cudaEventSynchronize(sl.done));
        sl.pending = false;
    }
    *out = &sl;
    return JL_OK;
}

jl_status stage_end(jl_model* m, StageSlot* s, cudaStream_t st) {
    (void)m;
    JL_CUDA(cudaEventRecord(s->done, st));
    s->pending = true;
    return JL_OK;
}

double elapsed_ms(cudaEvent_t a, cudaEvent_t b) {
    float ms = 0.f;
    cudaEventElapsedTime(&ms, a, b);
    return ms;
}

// Kernels record impossible states (a page id outside the pool, a position
// outside the RoPE table) and bounded waits that gave up in a device flag
// instead of touching memory out of range or spinning forever; surface it
// once the stream is idle.  Bits: 1 page id, 2 position, 4 a projection's
// copy or split-K wait, 8 a fused draft step's wait.
jl_status check_device_flag(jl_model* m) {
    int flag = 0;
    JL_CUDA(cudaMemcpy(&flag, m->counters, sizeof(int), cudaMemcpyDeviceToHost));
    if (flag) {
        JL_CUDA(cudaMemsetAsync(m->counters, 0, sizeof(int), m->stream));
        JL_CUDA(cudaStreamSynchronize(m->stream));
        if (flag & 3) {
            set_error("kernel guard tripped (flags 0x%x): %s", flag,
                      (flag & 1) ? "KV page id outside the pool" : "position outside the context");
            return JL_ERR_CUDA;
        }
        set_error("a bounded device wait gave up (flags 0x%x): a weight, activation or KV page copy, or a "
                  "split-K reduction, did not complete in time", flag);
        return JL_ERR_TIMEOUT;
    }
    return JL_OK;
}

namespace {
// One wait that nothing completes: an mbarrier expecting one arrival that
// never comes, polled `polls` times by the same loop the pass kernels use,
// then the same error bit they set.  No fault, no unbounded loop.
__global__ void k_wait_probe(int* err, uint32_t polls) {
    __shared__ uint64_t bar;
    if (threadIdx.x == 0) {
        ptx::mbar_init(&bar, 1);
        ptx::fence_barrier_init();
    }
    __syncthreads();
    if (threadIdx.x == 0 && !ptx::mbar_wait(&bar, 0, polls)) atomicOr(err, 4);
}
}  // namespace

jl_status wait_probe(jl_model* m, uint32_t polls) {
    if (polls == 0 || polls > (1u << 20)) {
        set_error("wait probe: polls must be 1..%u", 1u << 20);
        return JL_ERR_INVALID_ARG;
    }
    JL_CUDA(cudaSetDevice(m->device));
    k_wait_probe<<<1, 32, 0, m->stream>>>(m->counters, polls);
    JL_CUDA(cudaGetLastError());
    JL_CUDA(cudaStreamSynchronize(m->stream));
    return check_device_flag(m);
}

jl_status check_ids(const jl_model* m, const uint32_t* ids, size_t n) {
    for (size_t i = 0; i < n; ++i)
        if (ids[i] >= (uint32_t)m->embed.rows) {
            set_error("token id %u out of range (vocabulary %d)", ids[i], m->embed.rows);
            return JL_ERR_INVALID_ARG;
        }
    return JL_OK;
}

namespace {

constexpr int HEAD_CAP = 512;  // predicted rows per pass (longer all=true calls are chunked)

__device__ inline void set_row(PassBuf pb, int i, uint32_t token, int32_t pos) {
    int n = i;
    put_row(pb.row, n, token, pos, 0);
}

// Conditional handles of one round: IF nodes of draft steps 1..G-1.  Their
// values persist across WHILE iterations, so every round clears them first.
struct StepHandles {
    cudaGraphConditionalHandle h[MAX_GAMMA];
    int n;
};

// speculative.rs:79-93, first iteration: propose draft_next, then decide
// whether the draft runs again.
__global__ void k_round_begin(SpecState* st, PassBuf draft, cudaGraphConditionalHandle loop,
                              StepHandles steps, cudaGraphConditionalHandle catchup) {
    SpecState& s = *st;
    cudaGraphSetConditional(catchup, 0);
    for (int i = 1; i < steps.n; ++i) cudaGraphSetConditional(steps.h[i], 0);
    s.iterations += 1;
    if (s.iterations > s.limit + 1) s.fault = 1;  // cannot happen: each round adds a token
    int n = 0;
    if (!seq_round_begin(s, draft.row, n, 0)) {
        cudaGraphSetConditional(loop, 0);
        return;
    }
    if (n) {
        draft.hdr->rows = 1;
        draft.hdr->head_rows = 1;
        draft.head_row[0] = 0;
    }
    if (steps.n > 1) cudaGraphSetConditional(steps.h[1], n ? 1 : 0);
}

// After draft pass i of a round (speculative.rs:84-92).
__global__ void k_draft_step(SpecState* st, PassBuf draft, Oracle o, int i,
                             cudaGraphConditionalHandle next) {
    int n = 0;
    seq_draft_step(*st, o, i, draft.out_ids[0], draft.row, n, 0);
    if (next) cudaGraphSetConditional(next, n ? 1 : 0);
}

// speculative.rs:95-97: [pending correction] + proposals, predict after every row.
__global__ void k_verify_setup(SpecState* st, PassBuf target) {
    int rows = 0;
    seq_verify_rows(*st, target.row, rows, 0);
    target.hdr->rows = rows;
    target.hdr->head_rows = rows;
    for (int j = 0; j < rows; ++j) target.head_row[j] = j;
}

// speculative.rs:99-140: greedy acceptance, schedule feedback, rollback by
// length, correction / bonus token and the draft catch-up rows.
__global__ void k_accept(SpecState* st, PassBuf target, PassBuf draft, uint32_t* tokens,
                         jl_round_stats* rounds, int32_t rounds_cap,
                         cudaGraphConditionalHandle loop, cudaGraphConditionalHandle catchup) {
    int n = 0;
    if (!seq_accept(*st, target.out_ids, tokens, rounds, rounds_cap, draft.row, n, 0)) {
        cudaGraphSetConditional(loop, 0);
        cudaGraphSetConditional(catchup, 0);
        return;
    }
    draft.hdr->rows = n;
    draft.hdr->head_rows = 1;
    draft.head_row[0] = n - 1;
    cudaGraphSetConditional(catchup, 1);
}

__global__ void k_catchup_done(SpecState* st, PassBuf draft, Oracle o) {
    seq_catchup_done(*st, o, draft.out_ids[0]);
}

// Greedy loop (model.rs:277-283): after each single-row pass, append the
// prediction and stop at eos or the count.
__global__ void k_greedy_step(SpecState* st, PassBuf pb, uint32_t* tokens,
                              cudaGraphConditionalHandle loop) {
    SpecState& s = *st;
    s.target_len += 1;
    s.iterations += 1;
    const uint32_t nxt = pb.out_ids[0];
    if (s.n_tokens < s.limit) tokens[s.n_tokens++] = nxt;
    if ((int32_t)nxt == s.eos || s.n_tokens >= s.limit || s.iterations > s.limit) {
        s.done = 1;
        cudaGraphSetConditional(loop, 0);
        return;
    }
    set_row(pb, 0, nxt, s.target_len);
}

// Stages one pass's rows from the host and runs it on m->stream.
jl_status host_pass(jl_model* m, jl_cache* c, const uint32_t* ids, size_t n, int head_rows,
                    bool all, int layers, bool draft_step = false) {
    StageSlot* sl = nullptr;
    JL_TRY(stage_begin(m, &sl));
    PassHdr* h = sl->hdr;
    h->rows = (int32_t)n;
    h->head_rows = head_rows;
    h->pad0 = h->pad1 = 0;
    for (size_t i = 0; i < n; ++i) {
        sl->row[i].token = ids[i];
        sl->row[i].seq = 0;
        sl->row[i].pos = (int32_t)(c->len + i);
        sl->row[i].pad = 0;
    }
    for (int j = 0; j < head_rows; ++j) sl->head_row[j] = all ? j : (int32_t)n - 1;
    sl->page_table[0] = c->d_pages;
    cudaStream_t st = m->stream;
    JL_CUDA(cudaMemcpyAsync(m->pass.hdr, h, sizeof(PassHdr), cudaMemcpyHostToDevice, st));
    JL_CUDA(cudaMemcpyAsync(m->pass.row, sl->row, n * sizeof(RowDesc), cudaMemcpyHostToDevice, st));
    if (head_rows)
        JL_CUDA(cudaMemcpyAsync(m->pass.head_row, sl->head_row, head_rows * sizeof(int32_t),
                                cudaMemcpyHostToDevice, st));
    JL_CUDA(cudaMemcpyAsync(m->pass.page_table, sl->page_table, sizeof(int32_t*),
                            cudaMemcpyHostToDevice, st));
    JL_TRY(stage_end(m, sl, st));
    const bool full = layers == m->layers && head_rows > 0;
    // window CTAs the attention needs for this pass's longest context; a
    // captured pass is captured again when it was built for fewer
    const int splits = att_splits_for(m, c->len + n);
    if (full && draft_step && m->dec_ok && n <= 2) {
        // a speculative loop's draft step, captured on its own
        cudaGraphExec_t& exec = m->draft_graph[n - 1];
        if (exec && m->draft_graph_splits[n - 1] < splits) {
            cudaGraphExecDestroy(exec);
            exec = nullptr;
        }
        if (!exec) {
            cudaGraph_t g;
            JL_CUDA(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
            PassCtx ctx{m, st, (int)n, (int)n, true, splits};
            jl_status rs = record_pass_ctx(ctx, m->layers, true);
            cudaError_t ce = cudaStreamEndCapture(st, &g);
            if (rs != JL_OK) return rs;
            JL_CUDA(ce);
            JL_CUDA(cudaGraphInstantiate(&exec, g, 0));
            cudaGraphDestroy(g);
            m->draft_graph_splits[n - 1] = splits;
        }
        JL_CUDA(cudaGraphLaunch(exec, st));
        return JL_OK;
    }
    if (full && n <= (size_t)SMALL_M) {
        // one captured pass per row count, as the speculative loop's verify
        // pass is: the projections' MMA columns and shared-memory rings are
        // sized for the pass's rows
        const int b = (int)n - 1;
        cudaGraphExec_t& exec = m->small_graph[b];
        if (exec && m->small_graph_splits[b] < splits) {
            cudaGraphExecDestroy(exec);
            exec = nullptr;
        }
        if (!exec) {
            cudaGraph_t g;
            JL_CUDA(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
            PassCtx ctx{m, st, (int)n, (int)n, false, splits};
            jl_status rs = record_pass_ctx(ctx, m->layers, true);
            cudaError_t ce = cudaStreamEndCapture(st, &g);
            if (rs != JL_OK) return rs;
            JL_CUDA(ce);
            JL_CUDA(cudaGraphInstantiate(&exec, g, 0));
            cudaGraphDestroy(g);
            m->small_graph_splits[b] = splits;
        }
        JL_CUDA(cudaGraphLaunch(exec, st));
        return JL_OK;
    }
    PassCtx ctx{m, st, (int)n, std::max(head_rows, 1), false, splits};
    return record_pass_ctx(ctx, layers, head_rows > 0);
}

// Whether `m` runs passes over more than 16 rows as multi-chunk passes.
bool multi_chunk_model(const jl_model* m) { return m->mx.fused && m->bf_head.a && m->mx.chunks > 1; }

// A pass of 17..16*chunks rows from the host as one multi-chunk pass
// (recorded directly on m->stream).  Predicted rows: every row (`all`), or
// the last one; their ids land in out_ids at 16 * chunk + index.
jl_status host_pass_multi(jl_model* m, jl_cache* c, const uint32_t* ids, size_t n, bool all, bool head) {
    const int C = (int)((n + SMALL_M - 1) / SMALL_M);
    StageSlot* sl = nullptr;
    JL_TRY(stage_begin(m, &sl));
    const int last = (int)((n - 1) / SMALL_M);
    for (int k = 0; k < C; ++k) {
        const int rows = (int)std::min<size_t>(SMALL_M, n - (size_t)k * SMALL_M);
        PassHdr& h = sl->hdr[k];
        h.rows = rows;
        h.head_rows = !head ? 0 : all ? rows : (k == last ? 1 : 0);
        h.pad0 = h.pad1 = 0;
        for (int j = 0; j < SMALL_M; ++j) sl->head_row[k * SMALL_M + j] = all ? j : rows - 1;
    }
    for (size_t i = 0; i < n; ++i) {
        sl->row[i].token = ids[i];
        sl->row[i].seq = 0;
        sl->row[i].pos = (int32_t)(c->len + i);
        sl->row[i].pad = 0;
    }
    sl->page_table[0] = c->d_pages;
    cudaStream_t st = m->stream;
    JL_CUDA(cudaMemcpyAsync(m->pass.hdr, sl->hdr, C * sizeof(PassHdr), cudaMemcpyHostToDevice, st));
    JL_CUDA(cudaMemcpyAsync(m->pass.row, sl->row, n * sizeof(RowDesc), cudaMemcpyHostToDevice, st));
    JL_CUDA(cudaMemcpyAsync(m->pass.head_row, sl->head_row, (size_t)C * SMALL_M * sizeof(int32_t),
                            cudaMemcpyHostToDevice, st));
    JL_CUDA(cudaMemcpyAsync(m->pass.page_table, sl->page_table, sizeof(int32_t*), cudaMemcpyHostToDevice, st));
    JL_TRY(stage_end(m, sl, st));
    PassCtx ctx{m, st, C * SMALL_M, C * SMALL_M, false, att_splits_for(m, c->len + n)};
    ctx.chunks = C;
    ctx.prefill = true;
    return record_pass_ctx(ctx, m->layers, head);
}

}  // namespace

// The decode pass with every MXFP4 projection fused with its neighbours:
// five kernels per layer.  Each projection's epilogue writes the next one's
// input pieces (and, after a residual add, the sums of squares the next
// RMSNorm needs), so no normalisation or quantisation kernel runs between
// them; the q|k|v epilogue also does QK-norm, RoPE and the cache append.
jl_status record_fused_pass(const PassCtx& c, int layers) {
    const jl_model* m = c.m;
    const MxBuffers& B = m->mx;
    const int h = m->hidden, tiles = h / 128;
    const bool multi = c.chunks > 1;  // chunk strides of the piece images
    const size_t sx = multi ? B.sx : 0, sattn = multi ? B.sattn : 0, sact = multi ? B.sact : 0;
    JL_TRY(launch_embed(c));
    if (layers > 0) JL_TRY(mx_norm_pieces(c, m->s.x, h, m->lw[0].in_ln, h, B.bx, B.part));
    for (int l = 0; l < layers; ++l) {
        const LayerW& L = m->lw[l];
        MxFuse qkv;  // model.rs:174-177, lib.rs:353-396
        qkv.b = B.bx;
        qkv.part_in = B.part;
        qkv.part_tiles = tiles;
        qkv.norm_width = h;
        qkv.layer = l;
        qkv.qn = L.q_norm;
        qkv.kn = L.k_norm;
        qkv.cs_b = sx;
        JL_TRY(mx_project_fused(c, L.mx_qkv, MXE_QKV, qkv, m->s.qkv, qkv_ld(m)));
        JL_TRY(launch_attention(c, l, true));  // lib.rs:401-441
        MxFuse o;  // lib.rs:444-449 + residual, then post_attention_layernorm
        o.b = B.battn;
        o.bout = B.bx;
        o.part_out = B.part;
        o.next_w = L.post_ln;
        o.cs_b = sattn;
        o.cs_bout = sx;
        JL_TRY(mx_project_fused(c, L.mx_o, MXE_ADD, o, m->s.x, h));
        MxFuse gu;  // lib.rs:459-463
        gu.b = B.bx;
        gu.part_in = B.part;
        gu.part_tiles = tiles;
        gu.norm_width = h;
        gu.bout = B.bact;
        gu.cs_b = sx;
        gu.cs_bout = sact;
        JL_TRY(mx_project_fused(c, L.mx_gateup, MXE_SWIGLU, gu, nullptr, m->inter));
        MxFuse dn;  // lib.rs:464-467 + residual, then the next input_layernorm
        dn.b = B.bact;
        dn.cs_b = sact;
        dn.cs_bout = sx;
        if (l + 1 < layers) {
            dn.bout = B.bx;
            dn.part_out = B.part;
            dn.next_w = m->lw[l + 1].in_ln;
        }
        JL_TRY(mx_project_fused(c, L.mx_down, MXE_ADD, dn, m->s.x, h));
    }
    return JL_OK;
}

jl_status record_pass_ctx(const PassCtx& c, int layers, bool with_head) {
    tl_begin_pass();
    const jl_model* m = c.m;
    const bool dec = c.draft && m->dec_ok && c.rows_cap <= 2 && c.chunks == 1;
    if (c.chunks > 1 && !(m->mx.fused && m->bf_head.a)) {
        set_error("multi-chunk passes need the fused tensor-core pass and output table");
        return JL_ERR_INVALID_ARG;
    }
    if (dec || (m->mx.fused && (c.rows_cap <= mx_max_tokens() || c.chunks > 1))) {
        if (dec) JL_TRY(record_dec_pass(c, layers));
        else JL_TRY(record_fused_pass(c, layers));
        if (with_head && m->bf_head.a && (c.head_cap <= mx_max_tokens() || c.chunks > 1))  // model.rs:220-239
            return mx_head_fused(c, m->bf_head, m->final_norm, m->s.logits, m->vocab);
        if (with_head) {
            JL_TRY(launch_rmsnorm(c, m->s.x, m->final_norm, m->s.xh, true));  // model.rs:228
            JL_TRY(launch_head(c));                                           // model.rs:229-234
            JL_TRY(launch_argmax(c));                                         // model.rs:235-239
        }
        return JL_OK;
    }
    JL_TRY(launch_embed(c));
    for (int l = 0; l < layers; ++l) {
        const LayerW& L = m->lw[l];
        JL_TRY(launch_rmsnorm(c, m->s.x, L.in_ln, m->s.xn, false));  // model.rs:174-177
        JL_TRY(launch_qkv(c, L));                                    // lib.rs:353-355
        JL_TRY(launch_qk_rope_kv(c, l, L));                          // lib.rs:363-396
        JL_TRY(launch_attention(c, l));                              // lib.rs:401-441
        JL_TRY(launch_o(c, L));                                      // lib.rs:444-449 + residual
        JL_TRY(launch_rmsnorm(c, m->s.x, L.post_ln, m->s.xn, false));
        JL_TRY(launch_gateup(c, L));                                 // lib.rs:459-463
        JL_TRY(launch_down(c, L));                                   // lib.rs:464-467 + residual
    }
    if (with_head) {
        JL_TRY(launch_rmsnorm(c, m->s.x, m->final_norm, m->s.xh, true));  // model.rs:228
        JL_TRY(launch_head(c));                                           // model.rs:229-234
        JL_TRY(launch_argmax(c));                                         // model.rs:235-239
    }
    return JL_OK;
}


// predict(), except that the last pass's predicted ids (and logits) are left
// in flight on m->stream: predict_finish() waits for them.  Two models'
// prompts started this way run on their own streams at the same time.
struct PendingIds {
    uint32_t* dst = nullptr;
    size_t count = 0;
};

jl_status predict_start(jl_model* m, jl_cache* c, const uint32_t* ids, size_t n, bool all,
                        uint32_t* out_ids, float* out_logits, bool draft_step, PendingIds* pend) {
    *pend = PendingIds{};
    if (n == 0 || c->len + n > (size_t)m->max_positions) {  // model.rs:212
        set_error("predict needs 1..%zu tokens, got %zu", (size_t)m->max_positions - c->len, n);
        return JL_ERR_INVALID_ARG;
    }
    JL_TRY(check_ids(m, ids, n));
    JL_CUDA(cudaSetDevice(m->device));
    JL_TRY(cache_reserve(c, c->len + n, m->stream));
    // The captured decode pass takes 16 rows at a time (the kernels are
    // row-count invariant, so chunking changes no result).  On a model whose
    // pass is fused onto the tensor cores it is faster than the tiled
    // long-prompt kernels at every prompt length (B200, Qwen3-8B MXFP4: 2048
    // tokens 0.86 s against 1.13 s), so every prompt takes it; otherwise
    // prompts over 256 tokens use the long-prompt kernels.
    // A model with multi-chunk passes takes up to 16 * chunks rows at a time:
    // every kernel then runs all chunks in one launch, so the weights stream
    // from HBM about once per pass instead of once per 16 rows.
    const bool multi = multi_chunk_model(m);
    const size_t chunk = multi ? (size_t)SMALL_M * m->mx.chunks
                         : n <= 256 || m->mx.fused
                             ? (size_t)SMALL_M
                             : (all ? std::min<size_t>(m->max_rows, HEAD_CAP) : (size_t)m->max_rows);
    size_t done = 0;
    while (done < n) {
        const size_t take = std::min(chunk, n - done);
        const bool last = done + take == n;
        const int head_rows = all ? (int)take : (last ? 1 : 0);
        // where the predicted rows' ids and logits land
        size_t out_at = 0;
        if (multi && take > (size_t)SMALL_M) {
            JL_TRY(host_pass_multi(m, c, ids + done, take, all, head_rows > 0));
            if (!all) out_at = (take - 1) / SMALL_M * SMALL_M;
        } else {
            JL_TRY(host_pass(m, c, ids + done, take, head_rows, all, m->layers, draft_step));
        }
        if (head_rows) {
            const size_t first = all ? done : 0;
            JL_CUDA(cudaMemcpyAsync(m->host_out, m->pass.out_ids + out_at, head_rows * sizeof(uint32_t),
                                    cudaMemcpyDeviceToHost, m->stream));
            if (out_logits)
                JL_CUDA(cudaMemcpyAsync(out_logits + first * m->vocab, m->s.logits + out_at * m->vocab,
                                        (size_t)head_rows * m->vocab * sizeof(float),
                                        cudaMemcpyDeviceToHost, m->stream));
            if (last) {
                pend->dst = out_ids + first;
                pend->count = (size_t)head_rows;
            } else {
                JL_CUDA(cudaStreamSynchronize(m->stream));
                memcpy(out_ids + first, m->host_out, head_rows * sizeof(uint32_t));
            }
        }
        c->len += take;
        done += take;
    }
    return JL_OK;
}

jl_status predict_finish(jl_model* m, const PendingIds& p) {
    JL_CUDA(cudaSetDevice(m->device));
    JL_CUDA(cudaStreamSynchronize(m->stream));
    if (p.count) memcpy(p.dst, m->host_out, p.count * sizeof(uint32_t));
    return check_device_flag(m);
}

jl_status predict(jl_model* m, jl_cache* c, const uint32_t* ids, size_t n, bool all,
                  uint32_t* out_ids, float* out_logits, bool draft_step) {
    PendingIds p;
    JL_TRY(predict_start(m, c, ids, n, all, out_ids, out_logits, draft_step, &p));
    return predict_finish(m, p);
}

jl_status time_pass(jl_model* m, const uint32_t* prompt, size_t n, size_t rows, size_t reps,
                    double* wall_ms, double* gpu_ms, bool draft_step) {
    // model.rs:245-266
    if (rows == 0 || reps == 0 || n + rows > (size_t)m->max_positions) {
        set_error("time_pass needs rows > 0, reps > 0 and prompt + rows within the context");
        return JL_ERR_INVALID_ARG;
    }
    jl_cache* c = nullptr;
    JL_TRY(cache_create(m, &c));
    std::unique_ptr<jl_cache, void (*)(jl_cache*)> guard(c, cache_free);
    uint32_t first = 0;
    JL_TRY(predict(m, c, prompt, n, false, &first, nullptr));
    JL_TRY(tl_clear(m->stream));  // timeline build: only the timed passes' stamps remain
    std::vector<uint32_t> tokens(rows), out(rows);
    for (size_t i = 0; i < rows; ++i) tokens[i] = prompt[i % n];
    std::vector<double> wall, busy;
    for (size_t r = 0; r < reps + 2; ++r) {
        const auto t0 = std::chrono::steady_clock::now();
        JL_CUDA(cudaEventRecord(m->ev0, m->stream));
        JL_TRY(predict(m, c, tokens.data(), rows, rows > 1, out.data(), nullptr, draft_step));
        JL_CUDA(cudaEventRecord(m->ev1, m->stream));
        JL_CUDA(cudaEventSynchronize(m->ev1));
        wall.push_back(std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count());
        busy.push_back(elapsed_ms(m->ev0, m->ev1));
        c->len = n;  // cache.truncate(prompt.len())
    }
    auto median = [](std::vector<double>& v) {
        v.erase(v.begin(), v.begin() + 2);
        std::sort(v.begin(), v.end());
        return v[v.size() / 2];
    };
    *wall_ms = median(wall);
    *gpu_ms = median(busy);
    return JL_OK;
}

jl_status project(jl_model* m, int layer, int which, const float* x, size_t rows, float* y) {
    if (rows < 1 || rows > (size_t)SMALL_M || which < 0 || which > 4 ||
        (which != 4 && (layer < 0 || layer >= m->layers))) {
        set_error("project: rows must be 1..%d and layer/projection valid", SMALL_M);
        return JL_ERR_INVALID_ARG;
    }
    JL_CUDA(cudaSetDevice(m->device));
    cudaStream_t st = m->stream;
    const int QW = m->q_heads * HEAD, KVW = m->kv_heads * HEAD;
    const LayerW* L = which == 4 ? nullptr : &m->lw[layer];
    // (input buffer, width in, output buffer, width out)
    float* in = nullptr;
    float* out = nullptr;
    int win = m->hidden, wout = m->hidden;
    switch (which) {
        case 0: in = m->s.xn; out = m->s.qkv; wout = QW + 2 * KVW; break;
        case 1: in = m->s.attn; win = QW; out = m->s.x; break;
        case 2: in = m->s.xn; out = m->s.act; wout = m->inter; break;
        case 3: in = m->s.act; win = m->inter; out = m->s.x; break;
        default: in = m->s.xh; out = m->s.logits; wout = m->vocab; break;
    }
    PassHdr h{(int32_t)rows, (int32_t)rows, 0, 0};
    StageSlot* sl = nullptr;
    JL_TRY(stage_begin(m, &sl));
    *sl->hdr = h;
    JL_CUDA(cudaMemcpyAsync(m->pass.hdr, sl->hdr, sizeof(PassHdr), cudaMemcpyHostToDevice, st));
    JL_TRY(stage_end(m, sl, st));
    JL_CUDA(cudaMemcpyAsync(in, x, rows * win * sizeof(float), cudaMemcpyHostToDevice, st));
    if (which == 1 || which == 3)  // these add into the residual stream: start it at zero
        JL_CUDA(cudaMemsetAsync(out, 0, rows * wout * sizeof(float), st));
    PassCtx c{m, st, (int)rows, (int)rows};
    switch (which) {
        case 0: JL_TRY(launch_qkv(c, *L)); break;
        case 1: JL_TRY(launch_o(c, *L)); break;
        case 2: JL_TRY(launch_gateup(c, *L)); break;
        case 3: JL_TRY(launch_down(c, *L)); break;
        default: JL_TRY(launch_head(c)); break;
    }
    JL_CUDA(cudaMemcpyAsync(y, out, rows * wout * sizeof(float), cudaMemcpyDeviceToHost, st));
    JL_CUDA(cudaStreamSynchronize(st));
    return check_device_flag(m);
}

jl_status time_projection(jl_model* m, int layer, int which, int rows, int iters, double* ms,
                          size_t* bytes) {
    if (layer < 0 || layer >= m->layers || which < 0 || which > 4 || rows < 1 ||
        rows > m->max_rows || iters < 1) {
        set_error("time_projection: bad layer, projection, rows or iters");
        return JL_ERR_INVALID_ARG;
    }
    JL_CUDA(cudaSetDevice(m->device));
    const LayerW& L = m->lw[layer];
    PassHdr h{rows, which == 4 ? rows : 0, 0, 0};
    StageSlot* sl = nullptr;
    JL_TRY(stage_begin(m, &sl));
    *sl->hdr = h;
    JL_CUDA(cudaMemcpyAsync(m->pass.hdr, sl->hdr, sizeof(PassHdr), cudaMemcpyHostToDevice, m->stream));
    JL_TRY(stage_end(m, sl, m->stream));
    PassCtx c{m, m->stream, rows, rows};
    const bool fused = m->mx.fused && rows <= mx_max_tokens();
    const int hid = m->hidden, tiles = hid / 128;
    auto launch = [&]() -> jl_status {
        if (fused && which == 1) {  // o: residual add, pieces and sums of squares out
            MxFuse f;
            f.b = m->mx.battn;
            f.bout = m->mx.bx;
            f.part_out = m->mx.part;
            f.next_w = L.post_ln;
            return mx_project_fused(c, L.mx_o, MXE_ADD, f, m->s.x, hid);
        }
        if (fused && which == 2) {  // gate/up: input RMSNorm, SwiGLU, pieces out
            MxFuse f;
            f.b = m->mx.bx;
            f.part_in = m->mx.part;
            f.part_tiles = tiles;
            f.norm_width = hid;
            f.bout = m->mx.bact;
            return mx_project_fused(c, L.mx_gateup, MXE_SWIGLU, f, nullptr, m->inter);
        }
        if (which == 4 && m->bf_head.a && rows <= mx_max_tokens())  // final norm + bf16 table + argmax
            return mx_head_fused(c, m->bf_head, m->final_norm, m->s.logits, m->vocab);
        if (fused && which == 3) {  // down: residual add, pieces and sums of squares out
            MxFuse f;
            f.b = m->mx.bact;
            f.bout = m->mx.bx;
            f.part_out = m->mx.part;
            f.next_w = L.in_ln;
            return mx_project_fused(c, L.mx_down, MXE_ADD, f, m->s.x, hid);
        }
        switch (which) {
            case 0: return launch_qkv(c, L);
            case 1: return launch_o(c, L);
            case 2: return launch_gateup(c, L);
            case 3: return launch_down(c, L);
            default: return launch_head(c);
        }
    };
    JL_TRY(launch());  // warm up
    JL_CUDA(cudaEventRecord(m->ev0, m->stream));
    for (int i = 0; i < iters; ++i) JL_TRY(launch());
    JL_CUDA(cudaEventRecord(m->ev1, m->stream));
    JL_CUDA(cudaEventSynchronize(m->ev1));
    *ms = elapsed_ms(m->ev0, m->ev1) / iters;
    switch (which) {
        case 0: *bytes = L.q.bytes() + L.k.bytes() + L.v.bytes(); break;
        case 1: *bytes = L.o.bytes(); break;
        case 2: *bytes = L.gate.bytes() + L.up.bytes(); break;
        case 3: *bytes = L.down.bytes(); break;
        default: *bytes = m->head.bytes();
    }
    return JL_OK;
}

size_t pass_kernels(const jl_model* m, size_t rows, bool draft_step) {
    const size_t L = (size_t)m->layers;
    const size_t head = m->bf_head.a ? 3 : (m->mx_head.a ? 4 : 3);  // head pieces + table + argmax
    if (draft_step && m->dec_ok && rows <= 2)  // embed, 5 per layer, head
        return 1 + 5 * L + head;
    if (m->mx.fused && rows <= (size_t)mx_max_tokens())  // embed + norm pieces, 5 per layer, head
        return 2 + 5 * L + (m->bf_head.a ? 3 : (m->mx_head.a ? 4 : 3));
    // embed, 8 per layer (norm, q|k|v, rope, attention, o, norm, gate/up, down) with
    // an extra pieces kernel before each tensor-core projection, head
    const bool mx = !m->lw.empty() && m->lw[0].mx_qkv.a && rows <= (size_t)mx_max_tokens();
    return 1 + (mx ? 12 : 8) * L + (m->mx_head.a && rows <= (size_t)mx_max_tokens() ? 4 : 3);
}

jl_status hidden(jl_model* m, const uint32_t* ids, size_t n, size_t layers, float* out) {
    if (n == 0 || n > (size_t)m->max_positions || layers > (size_t)m->layers) {
        set_error("hidden needs 1..%d tokens and at most %d layers", m->max_positions, m->layers);
        return JL_ERR_INVALID_ARG;
    }
    JL_TRY(check_ids(m, ids, n));
    JL_CUDA(cudaSetDevice(m->device));
    jl_cache* c = nullptr;
    JL_TRY(cache_create(m, &c));
    std::unique_ptr<jl_cache, void (*)(jl_cache*)> guard(c, cache_free);
    JL_TRY(cache_reserve(c, n, m->stream));
    size_t done = 0;
    while (done < n) {
        const size_t take = std::min((size_t)m->max_rows, n - done);
        JL_TRY(host_pass(m, c, ids + done, take, 0, false, (int)layers));
        JL_CUDA(cudaMemcpyAsync(out + done * m->hidden, m->s.x, take * m->hidden * sizeof(float),
                                cudaMemcpyDeviceToHost, m->stream));
        JL_CUDA(cudaStreamSynchronize(m->stream));
        c->len += take;
        done += take;
    }
    return JL_OK;
}

// ---------------------------------------------------------------------------
// device-resident loops

struct SpecGraph {
    jl_model* target = nullptr;
    jl_model* draft = nullptr;  // null for the greedy loop
    int G = 0;
    int splits = 1;             // attention window CTAs per row the graph was built with
    cudaGraphExec_t exec = nullptr;
    SpecState* st = nullptr;
    uint32_t* tokens = nullptr;
    jl_round_stats* rounds = nullptr;
    int32_t cap = 0;
    uint32_t* oracle = nullptr;
    int32_t oracle_cap = 0;
    Oracle oracle_args{};
    SpecState* host_st = nullptr;
};

void spec_graph_free(SpecGraph* g) {
    if (!g) return;
    if (g->exec) cudaGraphExecDestroy(g->exec);
    cudaFree(g->st);
    cudaFree(g->tokens);
    cudaFree(g->rounds);
    cudaFree(g->oracle);
    cudaFreeHost(g->host_st);
    delete g;
}

namespace {

jl_status build_spec_graph(SpecGraph* g) {
    jl_model* T = g->target;
    jl_model* D = g->draft;
    cudaStream_t st = T->stream;
    cudaGraph_t top;
    JL_CUDA(cudaGraphCreate(&top, 0));
    std::unique_ptr<CUgraph_st, cudaError_t (*)(cudaGraph_t)> top_guard(top, cudaGraphDestroy);
    cudaGraphConditionalHandle h_loop;
    JL_CUDA(cudaGraphConditionalHandleCreate(&h_loop, top, 1, cudaGraphCondAssignDefault));
    cudaGraphNode_t loop_node;
    cudaGraph_t body;
    JL_TRY(add_conditional(top, nullptr, 0, h_loop, cudaGraphCondTypeWhile, &loop_node, &body));

    const int G = g->G;
    std::vector<cudaGraphConditionalHandle> h_step(G + 1, 0);
    for (int i = 1; i < G; ++i)
        JL_CUDA(cudaGraphConditionalHandleCreate(&h_step[i], body, 0, 0));
    cudaGraphConditionalHandle h_catch;
    JL_CUDA(cudaGraphConditionalHandleCreate(&h_catch, body, 0, 0));

    StepHandles steps{};
    steps.n = G;
    for (int i = 1; i < G; ++i) steps.h[i] = h_step[i];
    std::vector<cudaGraphNode_t> tail;
    // round begin
    JL_TRY(capture_into(body, st, nullptr, [&]() -> jl_status {
        k_round_begin<<<1, 1, 0, st>>>(g->st, D->pass, h_loop, steps, h_catch);
        JL_CUDA(cudaGetLastError());
        return JL_OK;
    }, &tail));
    cudaGraphNode_t prev = tail.at(0);
    // draft steps 1..G-1, each behind an IF node
    for (int i = 1; i < G; ++i) {
        cudaGraphNode_t ifn;
        cudaGraph_t ifb;
        JL_TRY(add_conditional(body, &prev, 1, h_step[i], cudaGraphCondTypeIf, &ifn, &ifb));
        const cudaGraphConditionalHandle nxt = i + 1 < G ? h_step[i + 1] : 0;
        JL_TRY(capture_into(ifb, st, nullptr, [&]() -> jl_status {
            PassCtx c{D, st, 1, 1, true, g->splits};
            JL_TRY(record_pass_ctx(c, D->layers, true));
            k_draft_step<<<1, 1, 0, st>>>(g->st, D->pass, g->oracle_args, i, nxt);
            JL_CUDA(cudaGetLastError());
            return JL_OK;
        }, nullptr));
        prev = ifn;
    }
    // verify + accept
    JL_TRY(capture_into(body, st, &prev, [&]() -> jl_status {
        k_verify_setup<<<1, 1, 0, st>>>(g->st, T->pass);
        JL_CUDA(cudaGetLastError());
        PassCtx c{T, st, G + 1, G + 1, false, g->splits};
        JL_TRY(record_pass_ctx(c, T->layers, true));
        k_accept<<<1, 1, 0, st>>>(g->st, T->pass, D->pass, g->tokens, g->rounds, g->cap, h_loop, h_catch);
        JL_CUDA(cudaGetLastError());
        return JL_OK;
    }, &tail));
    prev = tail.at(0);
    // draft catch-up behind an IF node
    {
        cudaGraphNode_t ifn;
        cudaGraph_t ifb;
        JL_TRY(add_conditional(body, &prev, 1, h_catch, cudaGraphCondTypeIf, &ifn, &ifb));
        JL_TRY(capture_into(ifb, st, nullptr, [&]() -> jl_status {
            PassCtx c{D, st, 2, 1, true, g->splits};
            JL_TRY(record_pass_ctx(c, D->layers, true));
            k_catchup_done<<<1, 1, 0, st>>>(g->st, D->pass, g->oracle_args);
            JL_CUDA(cudaGetLastError());
            return JL_OK;
        }, nullptr));
    }
    JL_CUDA(cudaGraphInstantiate(&g->exec, top, 0));
    return JL_OK;
}

jl_status build_greedy_graph(SpecGraph* g) {
    jl_model* T = g->target;
    cudaStream_t st = T->stream;
    cudaGraph_t top;
    JL_CUDA(cudaGraphCreate(&top, 0));
    std::unique_ptr<CUgraph_st, cudaError_t (*)(cudaGraph_t)> top_guard(top, cudaGraphDestroy);
    cudaGraphConditionalHandle h_loop;
    JL_CUDA(cudaGraphConditionalHandleCreate(&h_loop, top, 1, cudaGraphCondAssignDefault));
    cudaGraphNode_t loop_node;
    cudaGraph_t body;
    JL_TRY(add_conditional(top, nullptr, 0, h_loop, cudaGraphCondTypeWhile, &loop_node, &body));
    JL_TRY(capture_into(body, st, nullptr, [&]() -> jl_status {
        PassCtx c{T, st, 1, 1, false, g->splits};
        JL_TRY(record_pass_ctx(c, T->layers, true));
        k_greedy_step<<<1, 1, 0, st>>>(g->st, T->pass, g->tokens, h_loop);
        JL_CUDA(cudaGetLastError());
        return JL_OK;
    }, nullptr));
    JL_CUDA(cudaGraphInstantiate(&g->exec, top, 0));
    return JL_OK;
}

// The loop graph of (target, draft, G), built with at least `splits`
// attention window CTAs per row (captured again when it had fewer).
jl_status get_graph(jl_model* target, jl_model* draft, int G, int splits, SpecGraph** out) {
    for (auto* g : target->spec_graphs)
        if (g->draft == draft && g->G == G) {
            if (g->splits < splits) {
                if (g->exec) cudaGraphExecDestroy(g->exec);
                g->exec = nullptr;
                g->splits = splits;
                JL_TRY(draft ? build_spec_graph(g) : build_greedy_graph(g));
            }
            *out = g;
            return JL_OK;
        }
    std::unique_ptr<SpecGraph> g(new SpecGraph());
    g->target = target;
    g->draft = draft;
    g->G = G;
    g->splits = splits;
    g->cap = target->max_positions + 2 * MAX_GAMMA + 8;
    JL_CUDA(cudaMalloc(&g->st, sizeof(SpecState)));
    JL_CUDA(cudaMalloc(&g->tokens, (size_t)g->cap * sizeof(uint32_t)));
    JL_CUDA(cudaMalloc(&g->rounds, (size_t)g->cap * sizeof(jl_round_stats)));
    JL_CUDA(cudaMallocHost(&g->host_st, sizeof(SpecState)));
    if (draft) {
        g->oracle_cap = g->cap;
        JL_CUDA(cudaMalloc(&g->oracle, (size_t)g->oracle_cap * sizeof(uint32_t)));
        g->oracle_args = Oracle{nullptr, 0, 0.0, 0, target->vocab};
        // The kernels read oracle settings from a device copy refreshed per call.
    }
    jl_status s = draft ? build_spec_graph(g.get()) : build_greedy_graph(g.get());
    if (s != JL_OK) {
        spec_graph_free(g.release());
        return s;
    }
    *out = g.get();
    target->spec_graphs.push_back(g.release());
    return JL_OK;
}

}  // namespace

jl_status generate(jl_model* m, const uint32_t* prompt, size_t n, size_t count, uint32_t* out,
                   size_t cap, size_t* out_len) {
    // model.rs:268-285
    if (n == 0) {
        set_error("prompt is empty");
        return JL_ERR_INVALID_ARG;
    }
    const size_t limit_room = n < (size_t)m->max_positions ? (size_t)m->max_positions - n : 0;
    count = std::min(count, limit_room);
    if (cap < n + count) {
        set_error("output capacity %zu is below prompt + count = %zu", cap, n + count);
        return JL_ERR_INVALID_ARG;
    }
    JL_TRY(check_ids(m, prompt, n));
    memcpy(out, prompt, n * sizeof(uint32_t));
    *out_len = n;
    if (count == 0) return JL_OK;
    JL_CUDA(cudaSetDevice(m->device));
    jl_cache* c = nullptr;
    JL_TRY(cache_create(m, &c));
    std::unique_ptr<jl_cache, void (*)(jl_cache*)> guard(c, cache_free);
    uint32_t next = 0;
    JL_TRY(predict(m, c, prompt, n, false, &next, nullptr));
    out[n] = next;
    *out_len = n + 1;
    if ((int32_t)next == m->eos || count == 1) return JL_OK;
    // the rest of the loop runs on the device
    SpecGraph* g = nullptr;
    JL_TRY(get_graph(m, nullptr, 0, att_splits_for(m, n + count), &g));
    JL_TRY(cache_reserve(c, n + count, m->stream));
    SpecState* s = g->host_st;
    memset(s, 0, sizeof(SpecState));
    s->n_tokens = (int32_t)(n + 1);
    s->limit = (int32_t)(n + count);
    s->eos = m->eos;
    s->target_len = (int32_t)c->len;
    cudaStream_t st = m->stream;
    JL_CUDA(cudaMemcpyAsync(g->st, s, sizeof(SpecState), cudaMemcpyHostToDevice, st));
    JL_CUDA(cudaMemcpyAsync(g->tokens, out, (n + 1) * sizeof(uint32_t), cudaMemcpyHostToDevice, st));
    StageSlot* sl = nullptr;
    JL_TRY(stage_begin(m, &sl));
    PassHdr* h = sl->hdr;
    h->rows = 1;
    h->head_rows = 1;
    h->pad0 = h->pad1 = 0;
    sl->row[0] = RowDesc{next, 0, (int32_t)c->len, 0};
    sl->head_row[0] = 0;
    sl->page_table[0] = c->d_pages;
    JL_CUDA(cudaMemcpyAsync(m->pass.hdr, h, sizeof(PassHdr), cudaMemcpyHostToDevice, st));
    JL_CUDA(cudaMemcpyAsync(m->pass.row, sl->row, sizeof(RowDesc), cudaMemcpyHostToDevice, st));
    JL_CUDA(cudaMemcpyAsync(m->pass.head_row, sl->head_row, sizeof(int32_t), cudaMemcpyHostToDevice, st));
    JL_CUDA(cudaMemcpyAsync(m->pass.page_table, sl->page_table, sizeof(int32_t*),
                            cudaMemcpyHostToDevice, st));
    JL_TRY(stage_end(m, sl, st));
    JL_CUDA(cudaGraphLaunch(g->exec, st));
    JL_CUDA(cudaMemcpyAsync(s, g->st, sizeof(SpecState), cudaMemcpyDeviceToHost, st));
    JL_CUDA(cudaStreamSynchronize(st));
    JL_TRY(check_device_flag(m));
    if (s->n_tokens < (int32_t)n + 1 || s->n_tokens > (int32_t)(n + count)) {
        set_error("greedy loop ended in an inconsistent state (%d tokens)", s->n_tokens);
        return JL_ERR_CUDA;
    }
    JL_CUDA(cudaMemcpy(out, g->tokens, (size_t)s->n_tokens * sizeof(uint32_t), cudaMemcpyDeviceToHost));
    c->len = (size_t)s->target_len;
    *out_len = (size_t)s->n_tokens;
    return JL_OK;
}

namespace {

double now_ms() {
    return std::chrono::duration<double, std::milli>(
               std::chrono::steady_clock::now().time_since_epoch()).count();
}

// speculative.rs:43-143 with one host synchronisation per pass.
jl_status spec_host(jl_model* T, jl_model* D, const uint32_t* prompt, size_t n, size_t limit,
                    const jl_schedule& sched, const Oracle& o, jl_spec_result* r) {
    jl_cache *tc = nullptr, *dc = nullptr;
    JL_TRY(cache_create(T, &tc));
    std::unique_ptr<jl_cache, void (*)(jl_cache*)> g1(tc, cache_free);
    JL_TRY(cache_create(D, &dc));
    std::unique_ptr<jl_cache, void (*)(jl_cache*)> g2(dc, cache_free);
    std::vector<uint32_t> tokens(prompt, prompt + n);
    uint32_t gamma = sched.gamma;
    double t0 = now_ms();
    uint32_t first = 0, dnext = 0;
    JL_TRY(predict(T, tc, prompt, n, false, &first, nullptr));
    JL_TRY(predict(D, dc, prompt, n, false, &dnext, nullptr));
    dnext = oracle_token(o, (int32_t)dc->len, dnext);
    int64_t first_pred = first;
    r->prefill_passes = 2;
    r->prefill_ms = now_ms() - t0;
    const double decode0 = now_ms();
    int64_t pending = -1;
    std::vector<uint32_t> proposed, verification, checked(MAX_GAMMA + 2);
    while (tokens.size() < limit) {
        const size_t start = tokens.size();
        const size_t budget = std::min<size_t>(gamma, limit - start);
        proposed.clear();
        double t = now_ms();
        for (size_t i = 0; i < budget; ++i) {
            proposed.push_back(dnext);
            if (i + 1 == budget || (int32_t)dnext == T->eos) break;
            uint32_t nx = 0;
            JL_TRY(predict(D, dc, &dnext, 1, false, &nx, nullptr));
            dnext = oracle_token(o, (int32_t)dc->len, nx);
            r->draft_passes++;
        }
        r->draft_ms += now_ms() - t;
        verification.clear();
        if (pending >= 0) verification.push_back((uint32_t)pending);
        verification.insert(verification.end(), proposed.begin(), proposed.end());
        pending = -1;
        t = now_ms();
        checked.resize(verification.size());
        JL_TRY(predict(T, tc, verification.data(), verification.size(), true, checked.data(), nullptr));
        r->verify_passes++;
        r->verify_ms += now_ms() - t;
        std::vector<uint32_t> preds;
        if (first_pred >= 0) preds.push_back((uint32_t)first_pred);
        preds.insert(preds.end(), checked.begin(), checked.end());
        first_pred = -1;
        size_t accepted = 0;
        uint32_t next = preds[0];
        while (accepted < proposed.size() && proposed[accepted] == next) next = preds[++accepted];
        const uint32_t g_before = gamma;
        if (sched.adaptive && proposed.size() == gamma) {
            if (accepted == proposed.size()) gamma = std::min(gamma + 1, sched.max_gamma);
            else if (accepted < (proposed.size() + 1) / 2) gamma = std::max<uint32_t>(gamma / 2, 1);
        }
        if (r->rounds_out && r->rounds < r->rounds_cap)
            r->rounds_out[r->rounds] = jl_round_stats{g_before, (uint32_t)proposed.size(),
                                                      (uint32_t)accepted, gamma};
        r->rounds++;
        r->drafted += proposed.size();
        r->accepted += accepted;
        tokens.insert(tokens.end(), proposed.begin(), proposed.begin() + accepted);
        if ((accepted > 0 && (int32_t)tokens.back() == T->eos) || tokens.size() == limit) break;
        tc->len = start + accepted;                     // speculative.rs:127
        dc->len = std::min(start + accepted, dc->len);  // speculative.rs:128
        tokens.push_back(next);
        if ((int32_t)next == T->eos || tokens.size() == limit) break;
        pending = next;
        const size_t tail = tokens.size() - dc->len;
        t = now_ms();
        uint32_t nx = 0;
        JL_TRY(predict(D, dc, tokens.data() + dc->len, tail, false, &nx, nullptr));
        dnext = oracle_token(o, (int32_t)dc->len, nx);
        r->draft_passes++;
        r->draft_ms += now_ms() - t;
    }
    r->decode_ms = now_ms() - decode0;
    r->n_tokens = tokens.size();
    memcpy(r->tokens, tokens.data(), tokens.size() * sizeof(uint32_t));
    return JL_OK;
}

}  // namespace

jl_status generate_speculative(jl_model* T, jl_model* D, const uint32_t* prompt, size_t n,
                               size_t count, const jl_schedule& sched,
                               const jl_spec_options& opts, jl_spec_result* r) {
    if (n == 0) {
        set_error("prompt is empty");
        return JL_ERR_INVALID_ARG;
    }
    if (sched.gamma == 0 || sched.max_gamma < sched.gamma) {
        set_error("gamma must be positive and no greater than max gamma");
        return JL_ERR_INVALID_ARG;
    }
    if (T->vocab != D->vocab || T->eos != D->eos) {
        // speculative.rs:42: both models must share token ids
        set_error("target and draft must share the vocabulary");
        return JL_ERR_INVALID_ARG;
    }
    if (T->device != D->device) {
        set_error("target and draft must live on the same GPU");
        return JL_ERR_INVALID_ARG;
    }
    if (T == D) {
        set_error("use two model handles for target and draft (each owns its pass buffers)");
        return JL_ERR_INVALID_ARG;
    }
    // speculative.rs:60-67
    const size_t limit = std::min({n + count, (size_t)T->max_positions, (size_t)D->max_positions});
    if (r->tokens_cap < std::max(limit, n)) {
        set_error("tokens capacity %zu is below %zu", r->tokens_cap, std::max(limit, n));
        return JL_ERR_INVALID_ARG;
    }
    JL_TRY(check_ids(T, prompt, n));
    if (opts.oracle_stream && opts.oracle_p > 0) {
        if (opts.oracle_p > 1.0) {
            set_error("oracle_p must lie in [0, 1]");
            return JL_ERR_INVALID_ARG;
        }
    }
    if (opts.oracle_stream) JL_TRY(check_ids(T, opts.oracle_stream, opts.oracle_len));
    const size_t keep_tokens_cap = r->tokens_cap, keep_rounds_cap = r->rounds_cap;
    uint32_t* keep_tokens = r->tokens;
    jl_round_stats* keep_rounds = r->rounds_out;
    memset(r, 0, sizeof(*r));
    r->tokens = keep_tokens;
    r->tokens_cap = keep_tokens_cap;
    r->rounds_out = keep_rounds;
    r->rounds_cap = keep_rounds_cap;
    memcpy(r->tokens, prompt, n * sizeof(uint32_t));
    r->n_tokens = n;
    if (n >= limit) return JL_OK;
    JL_CUDA(cudaSetDevice(T->device));
    Oracle host_oracle{opts.oracle_stream, (int32_t)std::min(opts.oracle_len, (size_t)INT32_MAX),
                       opts.oracle_p, opts.oracle_seed, T->vocab};
    if (opts.mode == JL_SPEC_HOST)
        return spec_host(T, D, prompt, n, limit, sched, host_oracle, r);

    const int G = (int)sched.max_gamma;
    if (G > MAX_GAMMA) {
        set_error("max gamma %d exceeds %d for the device loop", G, MAX_GAMMA);
        return JL_ERR_INVALID_ARG;
    }
    jl_cache *tc = nullptr, *dc = nullptr;
    JL_TRY(cache_create(T, &tc));
    std::unique_ptr<jl_cache, void (*)(jl_cache*)> g1(tc, cache_free);
    JL_TRY(cache_create(D, &dc));
    std::unique_ptr<jl_cache, void (*)(jl_cache*)> g2(dc, cache_free);
    cudaStream_t st = T->stream;
    // prefill both models (speculative.rs:69-75), each on its own stream, at
    // the same time; the target's stream then waits for the draft's
    JL_CUDA(cudaEventRecord(T->ev0, st));
    uint32_t first = 0, dnext = 0;
    PendingIds pt, pd;
    JL_TRY(predict_start(T, tc, prompt, n, false, &first, nullptr, false, &pt));
    JL_TRY(predict_start(D, dc, prompt, n, false, &dnext, nullptr, false, &pd));
    JL_CUDA(cudaEventRecord(D->ev0, D->stream));
    JL_CUDA(cudaStreamWaitEvent(st, D->ev0, 0));
    JL_CUDA(cudaEventRecord(T->ev1, st));
    JL_TRY(predict_finish(T, pt));
    JL_TRY(predict_finish(D, pd));
    JL_CUDA(cudaEventSynchronize(T->ev1));
    r->prefill_ms = elapsed_ms(T->ev0, T->ev1);
    r->prefill_passes = 2;
    dnext = oracle_token(host_oracle, (int32_t)dc->len, dnext);

    SpecGraph* g = nullptr;
    JL_TRY(get_graph(T, D, G, std::max(att_splits_for(T, limit + G + 1), att_splits_for(D, limit + G + 1)), &g));
    // pages for every position the loop can reach
    JL_TRY(cache_reserve(tc, limit + G + 1, st));
    JL_TRY(cache_reserve(dc, limit + G + 1, st));
    // oracle stream to the device
    Oracle dev_oracle{nullptr, 0, opts.oracle_p, opts.oracle_seed, T->vocab};
    if (opts.oracle_stream) {
        const size_t len = std::min(opts.oracle_len, (size_t)g->oracle_cap);
        JL_CUDA(cudaMemcpyAsync(g->oracle, opts.oracle_stream, len * sizeof(uint32_t),
                                cudaMemcpyHostToDevice, st));
        dev_oracle.stream = g->oracle;
        dev_oracle.len = (int32_t)len;
    }
    if (memcmp(&dev_oracle, &g->oracle_args, sizeof(Oracle)) != 0) {
        // oracle settings are kernel arguments: rebuild the graph when they change
        g->oracle_args = dev_oracle;
        if (g->exec) cudaGraphExecDestroy(g->exec);
        g->exec = nullptr;
        JL_TRY(build_spec_graph(g));
    }
    SpecState* s = g->host_st;
    memset(s, 0, sizeof(SpecState));
    s->n_tokens = (int32_t)n;
    s->limit = (int32_t)limit;
    s->eos = T->eos;
    s->gamma = (int32_t)sched.gamma;
    s->max_gamma = (int32_t)sched.max_gamma;
    s->adaptive = sched.adaptive ? 1 : 0;
    s->pending = -1;
    s->first_pred = (int32_t)first;
    s->draft_next = (int32_t)dnext;
    s->target_len = (int32_t)tc->len;
    s->draft_len = (int32_t)dc->len;
    JL_CUDA(cudaMemcpyAsync(g->st, s, sizeof(SpecState), cudaMemcpyHostToDevice, st));
    JL_CUDA(cudaMemcpyAsync(g->tokens, prompt, n * sizeof(uint32_t), cudaMemcpyHostToDevice, st));
    // both models read sequence 0 from their own cache's page table
    StageSlot *ts = nullptr, *ds = nullptr;
    JL_TRY(stage_begin(T, &ts));
    JL_TRY(stage_begin(D, &ds));
    ts->page_table[0] = tc->d_pages;
    ds->page_table[0] = dc->d_pages;
    JL_CUDA(cudaMemcpyAsync(T->pass.page_table, ts->page_table, sizeof(int32_t*),
                            cudaMemcpyHostToDevice, st));
    JL_CUDA(cudaMemcpyAsync(D->pass.page_table, ds->page_table, sizeof(int32_t*),
                            cudaMemcpyHostToDevice, st));
    JL_TRY(stage_end(T, ts, st));
    JL_TRY(stage_end(D, ds, st));
    // the draft's stream must not still be using its pass buffers
    JL_CUDA(cudaStreamSynchronize(D->stream));
    JL_CUDA(cudaEventRecord(T->ev0, st));
    JL_CUDA(cudaGraphLaunch(g->exec, st));
    JL_CUDA(cudaEventRecord(T->ev1, st));
    JL_CUDA(cudaMemcpyAsync(s, g->st, sizeof(SpecState), cudaMemcpyDeviceToHost, st));
    JL_CUDA(cudaStreamSynchronize(st));
    r->decode_ms = elapsed_ms(T->ev0, T->ev1);
    JL_TRY(check_device_flag(T));
    JL_TRY(check_device_flag(D));
    if (s->fault || s->n_tokens < (int32_t)n || s->n_tokens > (int32_t)limit) {
        set_error("device loop ended in an inconsistent state (%d tokens)", s->n_tokens);
        return JL_ERR_CUDA;
    }
    JL_CUDA(cudaMemcpy(r->tokens, g->tokens, (size_t)s->n_tokens * sizeof(uint32_t),
                       cudaMemcpyDeviceToHost));
    if (r->rounds_out && r->rounds_cap)
        JL_CUDA(cudaMemcpy(r->rounds_out, g->rounds,
                           std::min((size_t)s->rounds, r->rounds_cap) * sizeof(jl_round_stats),
                           cudaMemcpyDeviceToHost));
    r->n_tokens = (size_t)s->n_tokens;
    r->drafted = (size_t)s->drafted;
    r->accepted = (size_t)s->accepted;
    r->rounds = (size_t)s->rounds;
    r->draft_passes = (size_t)s->draft_passes;
    r->verify_passes = (size_t)s->verify_passes;
    tc->len = (size_t)s->target_len;
    dc->len = (size_t)s->draft_len;
    return JL_OK;
}


// ---- kernel phase timeline (diagnostic build, timeline.cuh) ----------------

namespace {
struct Timeline {
    unsigned long long* table = nullptr;
    int device = -1;  // the table's device: launches elsewhere get no slot
    int next = 0;
    std::vector<std::string> names;
};
Timeline g_timeline;
}  // namespace

bool tl_enabled() {
#ifdef JL_TIMELINE
    return true;
#else
    return false;
#endif
}

jl_status tl_prepare() {
#ifdef JL_TIMELINE
    if (!g_timeline.table) {
        const size_t bytes = sizeof(unsigned long long) * TL_LAUNCHES * TL_CTAS * TL_POINTS;
        JL_CUDA(cudaGetDevice(&g_timeline.device));
        JL_CUDA(cudaMalloc(&g_timeline.table, bytes));
        JL_CUDA(cudaMemset(g_timeline.table, 0, bytes));
        JL_CUDA(cudaDeviceSynchronize());
    }
#endif
    return JL_OK;
}

jl_status tl_clear(cudaStream_t stream) {
    int dev = -1;
    if (!tl_enabled() || !g_timeline.table || cudaGetDevice(&dev) != cudaSuccess || dev != g_timeline.device)
        return JL_OK;
    JL_CUDA(cudaMemsetAsync(g_timeline.table, 0, sizeof(unsigned long long) * TL_LAUNCHES * TL_CTAS * TL_POINTS,
                            stream));
    return JL_OK;
}

void tl_begin_pass() {
    g_timeline.next = 0;
    g_timeline.names.clear();
}

TlSlot tl_launch(const char* kernel) {
    int dev = -1;
    if (!tl_enabled() || !g_timeline.table || g_timeline.next >= TL_LAUNCHES || cudaGetDevice(&dev) != cudaSuccess ||
        dev != g_timeline.device)
        return TlSlot{nullptr, -1};
    g_timeline.names.emplace_back(kernel);
    return TlSlot{g_timeline.table, g_timeline.next++};
}

jl_status tl_read(unsigned long long* out, size_t cap, size_t* launches) {
    if (!tl_enabled()) {
        set_error("this library was built without the kernel timeline (make timeline)");
        return JL_ERR_INVALID_ARG;
    }
    const size_t n = (size_t)g_timeline.next;
    if (launches) *launches = n;
    if (!out) return JL_OK;
    const size_t need = n * TL_CTAS * TL_POINTS;
    if (cap < need) {
        set_error("timeline: %zu stamps needed, room for %zu", need, cap);
        return JL_ERR_INVALID_ARG;
    }
    JL_CUDA(cudaSetDevice(g_timeline.device));
    JL_CUDA(cudaDeviceSynchronize());
    if (n) JL_CUDA(cudaMemcpy(out, g_timeline.table, need * sizeof(unsigned long long), cudaMemcpyDeviceToHost));
    return JL_OK;
}

const char* tl_kernel(size_t launch) {
    return launch < g_timeline.names.size() ? g_timeline.names[launch].c_str() : nullptr;
}

}  // namespace jl
