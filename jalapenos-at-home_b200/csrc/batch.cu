// Independent sequences decoded in lockstep rounds on one GPU: greedy
// (model.rs:268-285) and speculative (speculative.rs:43-143) generation of a
// batch of sequences, each exactly as the single-sequence loop decodes it.
//
// No reference counterpart exists for the batch itself (the reference
// engine decodes one sequence per call); the per-sequence rules are the
// shared steps of loop.cuh.  A round drafts for every sequence still
// running, verifies all of them in one target pass and accepts per sequence.
// A pass over more than 16 rows runs as 16-row chunk passes (the decode
// kernels take 16 rows), each behind a graph IF node its producer sets, so
// chunks without rows cost nothing.  Every row of a batched pass is predicted
// (head rows = rows); the kernels compute each row the same way whatever else
// shares its pass, so a sequence's tokens do not depend on its neighbours.
#include <algorithm>
#include <cstring>
#include <memory>

#include "jl_internal.h"
#include "kernels.cuh"
#include "loop.cuh"

namespace jl {

constexpr int BATCH_CHUNKS = 32;  // chunks of one batched pass: 512 rows

// Chunked pass buffers of one model in a batched loop.
struct BatchPass {
    PassHdr* hdr = nullptr;                // [chunks]
    RowDesc* row = nullptr;                // [chunks * SMALL_M]
    int32_t* ident = nullptr;              // [chunks * SMALL_M]: each chunk's rows 0, 1, ..., 15
    const int32_t** page_table = nullptr;  // [MAX_SEQS]: sequence b's cache
    uint32_t* out_ids = nullptr;           // [chunks * SMALL_M]
    int chunks = 0;
};

__host__ __device__ inline PassBuf chunk_view(const BatchPass& p, int c) {
    PassBuf v;
    v.hdr = p.hdr + c;
    v.row = p.row + c * SMALL_M;
    v.head_row = p.ident;
    v.page_table = p.page_table;
    v.out_ids = p.out_ids + c * SMALL_M;
    return v;
}

struct ChunkHandles {
    cudaGraphConditionalHandle h[BATCH_CHUNKS];
    int n;
};

struct BatchCtl {
    int32_t B, iterations, fault, max_limit;
    int32_t target_passes, draft_passes;  // chunk passes run
    int32_t rounds, pad;
};

struct BatchArgs {
    BatchCtl* ctl;
    SpecState* seqs;         // [B]
    const Oracle* oracles;   // [B]
    uint32_t* tokens;        // [B][tcap]
    jl_round_stats* rounds;  // [B][tcap]
    int32_t tcap;
    BatchPass tp, dp;        // target and draft pass buffers
};

// Splits `rows` rows over the chunk headers and opens the IF node of every
// chunk that has rows; returns how many do.
__device__ int set_chunks(const BatchPass& p, const ChunkHandles& ch, int rows) {
    int used = 0;
    for (int c = 0; c < p.chunks; ++c) {
        const int r = max(0, min(SMALL_M, rows - c * SMALL_M));
        p.hdr[c].rows = r;
        p.hdr[c].head_rows = r;
        if (c < ch.n) cudaGraphSetConditional(ch.h[c], r > 0 ? 1 : 0);
        used += r > 0;
    }
    return used;
}

// speculative.rs:79-93 for every running sequence; `first` are the chunk
// handles of draft step 1.
__global__ void k_batch_round_begin(BatchArgs a, cudaGraphConditionalHandle loop, ChunkHandles first) {
    BatchCtl& ctl = *a.ctl;
    ctl.iterations += 1;
    if (ctl.iterations > ctl.max_limit + 1) ctl.fault = 1;  // cannot happen: each round adds a token
    int n = 0, running = 0;
    for (int b = 0; b < ctl.B; ++b) {
        SpecState& s = a.seqs[b];
        if (ctl.fault) s.done = 1;
        running += seq_round_begin(s, a.dp.row, n, b) ? 1 : 0;
    }
    if (!running) cudaGraphSetConditional(loop, 0);
    else ctl.rounds += 1;
    ctl.draft_passes += set_chunks(a.dp, first, n);
}

// After draft pass i (speculative.rs:84-92): one row per drafting sequence,
// compacted in place for step i + 1 (a row moves only to a lower index).
__global__ void k_batch_draft_step(BatchArgs a, int i, ChunkHandles next) {
    int total = 0;
    for (int c = 0; c < a.dp.chunks; ++c) total += a.dp.hdr[c].rows;
    int n = 0;
    for (int r = 0; r < total; ++r) {
        const int b = a.dp.row[r].seq;
        seq_draft_step(a.seqs[b], a.oracles[b], i, a.dp.out_ids[r], a.dp.row, n, b);
    }
    a.ctl->draft_passes += set_chunks(a.dp, next, n);
}

// speculative.rs:95-97 for every sequence in the round.
__global__ void k_batch_verify_setup(BatchArgs a, ChunkHandles chunks) {
    int n = 0;
    for (int b = 0; b < a.ctl->B; ++b) {
        SpecState& s = a.seqs[b];
        if (s.done) {
            s.nrows = 0;
            continue;
        }
        seq_verify_rows(s, a.tp.row, n, b);
    }
    a.ctl->target_passes += set_chunks(a.tp, chunks, n);
}

// speculative.rs:99-140 per sequence, then the draft catch-up rows of every
// sequence that continues.
__global__ void k_batch_accept(BatchArgs a, cudaGraphConditionalHandle loop, ChunkHandles chunks) {
    int n = 0, running = 0;
    for (int b = 0; b < a.ctl->B; ++b) {
        SpecState& s = a.seqs[b];
        if (s.done) continue;
        running += seq_accept(s, a.tp.out_ids + s.row0, a.tokens + (size_t)b * a.tcap,
                              a.rounds + (size_t)b * a.tcap, a.tcap, a.dp.row, n, b)
                       ? 1
                       : 0;
        if (s.fault) a.ctl->fault = 1;
    }
    if (!running) cudaGraphSetConditional(loop, 0);
    a.ctl->draft_passes += set_chunks(a.dp, chunks, n);
}

__global__ void k_batch_catchup_done(BatchArgs a) {
    for (int b = 0; b < a.ctl->B; ++b) {
        SpecState& s = a.seqs[b];
        if (s.done || s.catch_rows == 0) continue;
        seq_catchup_done(s, a.oracles[b], a.dp.out_ids[s.crow]);
    }
}

// Greedy rounds (model.rs:277-283): one row per running sequence, its last
// token at the cache length.
__global__ void k_batch_greedy_begin(BatchArgs a, cudaGraphConditionalHandle loop, ChunkHandles chunks) {
    BatchCtl& ctl = *a.ctl;
    ctl.iterations += 1;
    if (ctl.iterations > ctl.max_limit + 1) ctl.fault = 1;
    int n = 0;
    for (int b = 0; b < ctl.B; ++b) {
        SpecState& s = a.seqs[b];
        if (ctl.fault || s.n_tokens >= s.limit) s.done = 1;
        if (s.done) continue;
        put_row(a.tp.row, n, a.tokens[(size_t)b * a.tcap + s.n_tokens - 1], s.target_len, b);
    }
    if (!n) cudaGraphSetConditional(loop, 0);
    else ctl.rounds += 1;
    ctl.target_passes += set_chunks(a.tp, chunks, n);
}

__global__ void k_batch_greedy_step(BatchArgs a) {
    int total = 0;
    for (int c = 0; c < a.tp.chunks; ++c) total += a.tp.hdr[c].rows;
    for (int r = 0; r < total; ++r) {
        const int b = a.tp.row[r].seq;
        SpecState& s = a.seqs[b];
        s.target_len += 1;
        s.verify_passes += 1;
        const uint32_t nxt = a.tp.out_ids[r];
        if (s.n_tokens < s.limit) a.tokens[(size_t)b * a.tcap + s.n_tokens++] = nxt;
        if ((int32_t)nxt == s.eos || s.n_tokens >= s.limit) s.done = 1;
    }
}

// ---------------------------------------------------------------------------

struct BatchGraph {
    jl_model* target = nullptr;
    jl_model* draft = nullptr;  // null for the greedy loop
    int G = 0, B = 0, splits = 1;
    int32_t tcap = 0;
    cudaGraphExec_t exec = nullptr;
    BatchArgs args{};
    std::vector<void*> dev;   // device allocations
    std::vector<void*> host;  // pinned allocations
    SpecState* host_seqs = nullptr;
    BatchCtl* host_ctl = nullptr;
    Oracle* host_oracles = nullptr;
    uint32_t* oracle_buf = nullptr;     // device: sequence b's oracle stream at b * tcap
    const int32_t** host_pt = nullptr;  // [2][MAX_SEQS]
};

void batch_graph_free(BatchGraph* g) {
    if (!g) return;
    if (g->exec) cudaGraphExecDestroy(g->exec);
    for (void* p : g->dev) cudaFree(p);
    for (void* p : g->host) cudaFreeHost(p);
    delete g;
}

namespace {

template <class T>
jl_status dev_alloc(BatchGraph* g, T** out, size_t count) {
    void* p = nullptr;
    JL_CUDA(cudaMalloc(&p, std::max<size_t>(count, 1) * sizeof(T)));
    g->dev.push_back(p);
    JL_CUDA(cudaMemset(p, 0, std::max<size_t>(count, 1) * sizeof(T)));
    // the memset runs on the legacy stream, which the model's stream does not wait for
    JL_CUDA(cudaDeviceSynchronize());
    *out = (T*)p;
    return JL_OK;
}

template <class T>
jl_status host_alloc(BatchGraph* g, T** out, size_t count) {
    void* p = nullptr;
    JL_CUDA(cudaMallocHost(&p, std::max<size_t>(count, 1) * sizeof(T)));
    g->host.push_back(p);
    memset(p, 0, std::max<size_t>(count, 1) * sizeof(T));
    *out = (T*)p;
    return JL_OK;
}

jl_status alloc_pass(BatchGraph* g, BatchPass* p, int rows) {
    p->chunks = (rows + SMALL_M - 1) / SMALL_M;
    JL_TRY(dev_alloc(g, &p->hdr, p->chunks));
    JL_TRY(dev_alloc(g, &p->row, (size_t)p->chunks * SMALL_M));
    JL_TRY(dev_alloc(g, &p->out_ids, (size_t)p->chunks * SMALL_M));
    int32_t* ident = nullptr;
    const size_t n = (size_t)p->chunks * SMALL_M;
    JL_TRY(dev_alloc(g, &ident, n));
    std::vector<int32_t> h(n);
    for (size_t j = 0; j < n; ++j) h[j] = (int32_t)(j % SMALL_M);
    JL_CUDA(cudaMemcpy(ident, h.data(), n * sizeof(int32_t), cudaMemcpyHostToDevice));
    p->ident = ident;
    const int32_t** pt = nullptr;
    JL_TRY(dev_alloc(g, &pt, MAX_SEQS));
    p->page_table = pt;
    return JL_OK;
}

// Rows of chunk c of a pass over at most `rows` rows.
int chunk_cap(int rows, int c) { return std::min(SMALL_M, rows - c * SMALL_M); }

// Whether `m` runs a pass over `rows` rows as one multi-chunk pass.
bool multi_chunk(const jl_model* m, int rows) {
    const int chunks = (rows + SMALL_M - 1) / SMALL_M;
    return chunks > 1 && m->mx.fused && m->bf_head.a && chunks <= m->mx.chunks;
}

// The passes of `m` over at most `rows` rows inside `graph` after `dep`:
// one multi-chunk pass behind the IF node of h[0] (open when chunk 0 has
// rows), or one pass per 16-row chunk, each behind the IF node of its
// handle.  Returns the last node.
jl_status add_chunk_passes(cudaGraph_t graph, cudaStream_t st, cudaGraphNode_t* dep, jl_model* m,
                           const BatchPass& p, int rows, bool draft, int splits,
                           const std::vector<cudaGraphConditionalHandle>& h, cudaGraphNode_t* last) {
    cudaGraphNode_t prev = dep ? *dep : nullptr;
    const int chunks = (rows + SMALL_M - 1) / SMALL_M;
    if (multi_chunk(m, rows)) {
        cudaGraphNode_t ifn;
        cudaGraph_t ifb;
        JL_TRY(add_conditional(graph, prev ? &prev : nullptr, prev ? 1 : 0, h[0], cudaGraphCondTypeIf, &ifn, &ifb));
        JL_TRY(capture_into(ifb, st, nullptr, [&]() -> jl_status {
            PassCtx ctx{m, st, chunks * SMALL_M, chunks * SMALL_M, draft, splits};
            ctx.chunks = chunks;
            ctx.view = chunk_view(p, 0);
            return record_pass_ctx(ctx, m->layers, true);
        }, nullptr));
        *last = ifn;
        return JL_OK;
    }
    for (int c = 0; c < chunks; ++c) {
        cudaGraphNode_t ifn;
        cudaGraph_t ifb;
        JL_TRY(add_conditional(graph, prev ? &prev : nullptr, prev ? 1 : 0, h[c], cudaGraphCondTypeIf, &ifn, &ifb));
        const int cap = chunk_cap(rows, c);
        JL_TRY(capture_into(ifb, st, nullptr, [&]() -> jl_status {
            PassCtx ctx{m, st, cap, cap, draft, splits};
            ctx.view = chunk_view(p, c);
            return record_pass_ctx(ctx, m->layers, true);
        }, nullptr));
        prev = ifn;
    }
    *last = prev;
    return JL_OK;
}

ChunkHandles to_struct(const std::vector<cudaGraphConditionalHandle>& v) {
    ChunkHandles h{};
    h.n = (int)v.size();
    for (size_t i = 0; i < v.size() && i < (size_t)BATCH_CHUNKS; ++i) h.h[i] = v[i];
    return h;
}

// IF handles of a pass site over `rows` rows of `m`: one per chunk pass.
int site_handles(const jl_model* m, int rows) {
    return multi_chunk(m, rows) ? 1 : (rows + SMALL_M - 1) / SMALL_M;
}

jl_status make_handles(cudaGraph_t graph, int n, std::vector<cudaGraphConditionalHandle>* out) {
    out->assign(n, 0);
    for (int i = 0; i < n; ++i) JL_CUDA(cudaGraphConditionalHandleCreate(&(*out)[i], graph, 0, 0));
    return JL_OK;
}

// Appends kernel `fn` to `graph` after `dep`; returns its node.
template <class F>
jl_status add_kernel(cudaGraph_t graph, cudaStream_t st, cudaGraphNode_t* dep, F fn, cudaGraphNode_t* node) {
    std::vector<cudaGraphNode_t> tail;
    JL_TRY(capture_into(graph, st, dep, [&]() -> jl_status {
        fn();
        JL_CUDA(cudaGetLastError());
        return JL_OK;
    }, &tail));
    *node = tail.at(0);
    return JL_OK;
}

// One round in the loop body: round begin, draft steps 1..G-1, verify,
// accept and the draft catch-up, each pass as chunk passes behind IF nodes
// that the kernel before them opens.  Every conditional node sits in the
// body and every handle is set each round before its node is reached.
jl_status build_batch_spec(BatchGraph* g) {
    jl_model* T = g->target;
    jl_model* D = g->draft;
    cudaStream_t st = T->stream;
    const int G = g->G, B = g->B;
    const BatchArgs a = g->args;
    cudaGraph_t top;
    JL_CUDA(cudaGraphCreate(&top, 0));
    std::unique_ptr<CUgraph_st, cudaError_t (*)(cudaGraph_t)> top_guard(top, cudaGraphDestroy);
    cudaGraphConditionalHandle h_loop;
    JL_CUDA(cudaGraphConditionalHandleCreate(&h_loop, top, 1, cudaGraphCondAssignDefault));
    cudaGraphNode_t loop_node;
    cudaGraph_t body;
    JL_TRY(add_conditional(top, nullptr, 0, h_loop, cudaGraphCondTypeWhile, &loop_node, &body));

    const int vrows = B * (G + 1), crows = 2 * B;
    std::vector<std::vector<cudaGraphConditionalHandle>> h_dc(G + 1);
    for (int i = 1; i < G; ++i) JL_TRY(make_handles(body, site_handles(D, B), &h_dc[i]));
    std::vector<cudaGraphConditionalHandle> h_vc, h_cc;
    JL_TRY(make_handles(body, site_handles(T, vrows), &h_vc));
    JL_TRY(make_handles(body, site_handles(D, crows), &h_cc));

    const ChunkHandles first = G > 1 ? to_struct(h_dc[1]) : ChunkHandles{};
    cudaGraphNode_t prev;
    JL_TRY(add_kernel(body, st, nullptr, [&] { k_batch_round_begin<<<1, 1, 0, st>>>(a, h_loop, first); }, &prev));
    for (int i = 1; i < G; ++i) {
        JL_TRY(add_chunk_passes(body, st, &prev, D, a.dp, B, true, g->splits, h_dc[i], &prev));
        const ChunkHandles next = i + 1 < G ? to_struct(h_dc[i + 1]) : ChunkHandles{};
        JL_TRY(add_kernel(body, st, &prev, [&] { k_batch_draft_step<<<1, 1, 0, st>>>(a, i, next); }, &prev));
    }
    const ChunkHandles vc = to_struct(h_vc), cc = to_struct(h_cc);
    JL_TRY(add_kernel(body, st, &prev, [&] { k_batch_verify_setup<<<1, 1, 0, st>>>(a, vc); }, &prev));
    JL_TRY(add_chunk_passes(body, st, &prev, T, a.tp, vrows, false, g->splits, h_vc, &prev));
    JL_TRY(add_kernel(body, st, &prev, [&] { k_batch_accept<<<1, 1, 0, st>>>(a, h_loop, cc); }, &prev));
    JL_TRY(add_chunk_passes(body, st, &prev, D, a.dp, crows, true, g->splits, h_cc, &prev));
    JL_TRY(add_kernel(body, st, &prev, [&] { k_batch_catchup_done<<<1, 1, 0, st>>>(a); }, &prev));
    JL_CUDA(cudaGraphInstantiate(&g->exec, top, 0));
    return JL_OK;
}

jl_status build_batch_greedy(BatchGraph* g) {
    jl_model* T = g->target;
    cudaStream_t st = T->stream;
    const BatchArgs a = g->args;
    cudaGraph_t top;
    JL_CUDA(cudaGraphCreate(&top, 0));
    std::unique_ptr<CUgraph_st, cudaError_t (*)(cudaGraph_t)> top_guard(top, cudaGraphDestroy);
    cudaGraphConditionalHandle h_loop;
    JL_CUDA(cudaGraphConditionalHandleCreate(&h_loop, top, 1, cudaGraphCondAssignDefault));
    cudaGraphNode_t loop_node;
    cudaGraph_t body;
    JL_TRY(add_conditional(top, nullptr, 0, h_loop, cudaGraphCondTypeWhile, &loop_node, &body));
    std::vector<cudaGraphConditionalHandle> h_c;
    JL_TRY(make_handles(body, site_handles(T, g->B), &h_c));
    const ChunkHandles ch = to_struct(h_c);
    cudaGraphNode_t prev;
    JL_TRY(add_kernel(body, st, nullptr, [&] { k_batch_greedy_begin<<<1, 1, 0, st>>>(a, h_loop, ch); }, &prev));
    JL_TRY(add_chunk_passes(body, st, &prev, T, a.tp, g->B, false, g->splits, h_c, &prev));
    JL_TRY(add_kernel(body, st, &prev, [&] { k_batch_greedy_step<<<1, 1, 0, st>>>(a); }, &prev));
    JL_CUDA(cudaGraphInstantiate(&g->exec, top, 0));
    return JL_OK;
}

// The batched loop graph of (target, draft, G, B), built with at least
// `splits` attention window CTAs per row.
jl_status get_batch_graph(jl_model* T, jl_model* D, int G, int B, int splits, BatchGraph** out) {
    for (auto* g : T->batch_graphs)
        if (g->draft == D && g->G == G && g->B == B) {
            if (g->splits < splits) {
                if (g->exec) cudaGraphExecDestroy(g->exec);
                g->exec = nullptr;
                g->splits = splits;
                JL_TRY(D ? build_batch_spec(g) : build_batch_greedy(g));
            }
            *out = g;
            return JL_OK;
        }
    std::unique_ptr<BatchGraph, void (*)(BatchGraph*)> g(new BatchGraph(), batch_graph_free);
    g->target = T;
    g->draft = D;
    g->G = G;
    g->B = B;
    g->splits = splits;
    g->tcap = T->max_positions + 2 * MAX_GAMMA + 8;
    BatchArgs& a = g->args;
    JL_TRY(dev_alloc(g.get(), &a.ctl, 1));
    JL_TRY(dev_alloc(g.get(), &a.seqs, B));
    Oracle* orc = nullptr;
    JL_TRY(dev_alloc(g.get(), &orc, B));
    a.oracles = orc;
    JL_TRY(dev_alloc(g.get(), &a.tokens, (size_t)B * g->tcap));
    a.tcap = g->tcap;
    JL_TRY(alloc_pass(g.get(), &a.tp, D ? B * (G + 1) : B));
    if (D) {
        JL_TRY(dev_alloc(g.get(), &a.rounds, (size_t)B * g->tcap));
        JL_TRY(alloc_pass(g.get(), &a.dp, 2 * B));
        JL_TRY(dev_alloc(g.get(), &g->oracle_buf, (size_t)B * g->tcap));
        JL_TRY(host_alloc(g.get(), &g->host_oracles, B));
    }
    JL_TRY(host_alloc(g.get(), &g->host_seqs, B));
    JL_TRY(host_alloc(g.get(), &g->host_ctl, 1));
    JL_TRY(host_alloc(g.get(), &g->host_pt, 2 * MAX_SEQS));
    JL_TRY(D ? build_batch_spec(g.get()) : build_batch_greedy(g.get()));
    *out = g.get();
    T->batch_graphs.push_back(g.release());
    return JL_OK;
}

struct Batch {
    jl_model* T;
    jl_model* D;
    size_t B;
    std::vector<jl_cache*> tc, dc;
    ~Batch() {
        for (auto* c : tc) cache_free(c);
        for (auto* c : dc) cache_free(c);
    }
};

jl_status check_batch(const jl_model* m, size_t batch, const uint32_t* const* prompts, const size_t* lens,
                      jl_spec_result* results) {
    if (batch == 0 || batch > (size_t)MAX_SEQS) {
        set_error("batch must hold 1..%d sequences, got %zu", MAX_SEQS, batch);
        return JL_ERR_INVALID_ARG;
    }
    if (!prompts || !lens || !results) {
        set_error("prompts, prompt lengths and results are required");
        return JL_ERR_INVALID_ARG;
    }
    for (size_t b = 0; b < batch; ++b) {
        if (lens[b] == 0 || !prompts[b]) {
            set_error("prompt %zu is empty", b);
            return JL_ERR_INVALID_ARG;
        }
        if (!results[b].tokens) {
            set_error("results[%zu].tokens is NULL", b);
            return JL_ERR_INVALID_ARG;
        }
        JL_TRY(check_ids(m, prompts[b], lens[b]));
    }
    return JL_OK;
}

void reset_result(jl_spec_result* r) {
    const size_t tcap = r->tokens_cap, rcap = r->rounds_cap;
    uint32_t* t = r->tokens;
    jl_round_stats* rs = r->rounds_out;
    memset(r, 0, sizeof(*r));
    r->tokens = t;
    r->tokens_cap = tcap;
    r->rounds_out = rs;
    r->rounds_cap = rcap;
}

// Runs the instantiated loop once and copies every sequence's tokens back.
jl_status run_batch(BatchGraph* g, const std::vector<size_t>& lens, jl_spec_result* results, jl_batch_stats* stats,
                    double prefill_ms) {
    jl_model* T = g->target;
    cudaStream_t st = T->stream;
    const int B = g->B;
    JL_CUDA(cudaMemcpyAsync(g->args.seqs, g->host_seqs, B * sizeof(SpecState), cudaMemcpyHostToDevice, st));
    JL_CUDA(cudaMemcpyAsync(g->args.ctl, g->host_ctl, sizeof(BatchCtl), cudaMemcpyHostToDevice, st));
    JL_CUDA(cudaMemcpyAsync(g->args.tp.page_table, g->host_pt, MAX_SEQS * sizeof(int32_t*), cudaMemcpyHostToDevice,
                            st));
    if (g->draft) {
        JL_CUDA(cudaMemcpyAsync(g->args.dp.page_table, g->host_pt + MAX_SEQS, MAX_SEQS * sizeof(int32_t*),
                                cudaMemcpyHostToDevice, st));
        JL_CUDA(cudaMemcpyAsync((void*)g->args.oracles, g->host_oracles, B * sizeof(Oracle), cudaMemcpyHostToDevice,
                                st));
        JL_CUDA(cudaStreamSynchronize(g->draft->stream));
    }
    JL_CUDA(cudaEventRecord(T->ev0, st));
    JL_CUDA(cudaGraphLaunch(g->exec, st));
    JL_CUDA(cudaEventRecord(T->ev1, st));
    JL_CUDA(cudaMemcpyAsync(g->host_seqs, g->args.seqs, B * sizeof(SpecState), cudaMemcpyDeviceToHost, st));
    JL_CUDA(cudaMemcpyAsync(g->host_ctl, g->args.ctl, sizeof(BatchCtl), cudaMemcpyDeviceToHost, st));
    JL_CUDA(cudaStreamSynchronize(st));
    const double decode_ms = elapsed_ms(T->ev0, T->ev1);
    JL_TRY(check_device_flag(T));
    if (g->draft) JL_TRY(check_device_flag(g->draft));
    if (g->host_ctl->fault) {
        set_error("batched loop stopped by a guard after %d rounds", g->host_ctl->rounds);
        return JL_ERR_CUDA;
    }
    for (int b = 0; b < B; ++b) {
        const SpecState& s = g->host_seqs[b];
        jl_spec_result* r = &results[b];
        if (s.fault || s.n_tokens < (int32_t)lens[b] || s.n_tokens > std::max(s.limit, (int32_t)lens[b])) {
            set_error("sequence %d ended in an inconsistent state (%d tokens)", b, s.n_tokens);
            return JL_ERR_CUDA;
        }
        JL_CUDA(cudaMemcpy(r->tokens, g->args.tokens + (size_t)b * g->tcap, (size_t)s.n_tokens * sizeof(uint32_t),
                           cudaMemcpyDeviceToHost));
        if (g->draft && r->rounds_out && r->rounds_cap)
            JL_CUDA(cudaMemcpy(r->rounds_out, g->args.rounds + (size_t)b * g->tcap,
                               std::min((size_t)s.rounds, r->rounds_cap) * sizeof(jl_round_stats),
                               cudaMemcpyDeviceToHost));
        r->n_tokens = (size_t)s.n_tokens;
        r->drafted = (size_t)s.drafted;
        r->accepted = (size_t)s.accepted;
        r->rounds = (size_t)s.rounds;
        r->draft_passes = (size_t)s.draft_passes;
        r->verify_passes = (size_t)s.verify_passes;
        r->prefill_passes = s.limit > (int32_t)lens[b] ? (g->draft ? 2 : 1) : 0;  // prefilled sequences
        r->prefill_ms = prefill_ms;
        r->decode_ms = decode_ms;
    }
    if (stats) {
        stats->prefill_ms = prefill_ms;
        stats->decode_ms = decode_ms;
        stats->rounds = (size_t)g->host_ctl->rounds;
        stats->target_passes = (size_t)g->host_ctl->target_passes;
        stats->draft_passes = (size_t)g->host_ctl->draft_passes;
    }
    return JL_OK;
}

}  // namespace

jl_status generate_batch(jl_model* m, size_t batch, const uint32_t* const* prompts, const size_t* lens,
                         size_t count, jl_spec_result* results, jl_batch_stats* stats) {
    JL_TRY(check_batch(m, batch, prompts, lens, results));
    if (stats) memset(stats, 0, sizeof(*stats));
    std::vector<size_t> limit(batch), plen(lens, lens + batch);
    size_t max_limit = 0;
    for (size_t b = 0; b < batch; ++b) {
        // model.rs:268-285: at most max_positions tokens in all
        const size_t room = lens[b] < (size_t)m->max_positions ? (size_t)m->max_positions - lens[b] : 0;
        limit[b] = lens[b] + std::min(count, room);
        if (results[b].tokens_cap < limit[b]) {
            set_error("results[%zu].tokens_cap %zu is below %zu", b, results[b].tokens_cap, limit[b]);
            return JL_ERR_INVALID_ARG;
        }
        max_limit = std::max(max_limit, limit[b]);
    }
    for (size_t b = 0; b < batch; ++b) {
        reset_result(&results[b]);
        memcpy(results[b].tokens, prompts[b], lens[b] * sizeof(uint32_t));
        results[b].n_tokens = lens[b];
    }
    JL_CUDA(cudaSetDevice(m->device));
    Batch bt{m, nullptr, batch, {}, {}};
    bt.tc.assign(batch, nullptr);
    for (size_t b = 0; b < batch; ++b) JL_TRY(cache_create(m, &bt.tc[b]));
    cudaStream_t st = m->stream;
    JL_CUDA(cudaEventRecord(m->ev0, st));
    std::vector<uint32_t> first(batch);
    for (size_t b = 0; b < batch; ++b)
        if (limit[b] > lens[b]) JL_TRY(predict(m, bt.tc[b], prompts[b], lens[b], false, &first[b], nullptr));
    JL_CUDA(cudaEventRecord(m->ev1, st));
    JL_CUDA(cudaEventSynchronize(m->ev1));
    const double prefill_ms = elapsed_ms(m->ev0, m->ev1);
    BatchGraph* g = nullptr;
    JL_TRY(get_batch_graph(m, nullptr, 0, (int)batch, att_splits_for(m, max_limit), &g));
    memset(g->host_seqs, 0, batch * sizeof(SpecState));
    memset(g->host_ctl, 0, sizeof(BatchCtl));
    g->host_ctl->B = (int32_t)batch;
    g->host_ctl->max_limit = (int32_t)max_limit;
    for (size_t b = 0; b < batch; ++b) {
        SpecState& s = g->host_seqs[b];
        s.limit = (int32_t)limit[b];
        s.eos = m->eos;
        s.n_tokens = (int32_t)lens[b];
        s.target_len = (int32_t)bt.tc[b]->len;
        JL_CUDA(cudaMemcpyAsync(g->args.tokens + b * g->tcap, prompts[b], lens[b] * sizeof(uint32_t),
                                cudaMemcpyHostToDevice, st));
        if (limit[b] > lens[b]) {
            // the prefill's prediction is the first new token (model.rs:277-283)
            results[b].tokens[lens[b]] = first[b];
            JL_CUDA(cudaMemcpyAsync(g->args.tokens + b * g->tcap + lens[b], &results[b].tokens[lens[b]],
                                    sizeof(uint32_t), cudaMemcpyHostToDevice, st));
            s.n_tokens += 1;
            if ((int32_t)first[b] == m->eos) s.done = 1;
            JL_TRY(cache_reserve(bt.tc[b], limit[b], st));
        } else {
            s.done = 1;
        }
        g->host_pt[b] = bt.tc[b]->d_pages;
    }
    JL_TRY(run_batch(g, plen, results, stats, prefill_ms));
    return JL_OK;
}

jl_status generate_speculative_batch(jl_model* T, jl_model* D, size_t batch, const uint32_t* const* prompts,
                                     const size_t* lens, size_t count, const jl_schedule* scheds,
                                     const jl_spec_options* opts, jl_spec_result* results, jl_batch_stats* stats) {
    JL_TRY(check_batch(T, batch, prompts, lens, results));
    if (stats) memset(stats, 0, sizeof(*stats));
    if (!scheds) {
        set_error("schedules are required");
        return JL_ERR_INVALID_ARG;
    }
    if (T->vocab != D->vocab || T->eos != D->eos) {
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
    int G = 0;
    for (size_t b = 0; b < batch; ++b) {
        const jl_schedule& s = scheds[b];
        if (s.gamma == 0 || s.max_gamma < s.gamma) {
            set_error("gamma must be positive and no greater than max gamma");
            return JL_ERR_INVALID_ARG;
        }
        G = std::max(G, (int)s.max_gamma);
        if (opts && opts[b].oracle_stream) {
            if (opts[b].oracle_p < 0 || opts[b].oracle_p > 1.0) {
                set_error("oracle_p must lie in [0, 1]");
                return JL_ERR_INVALID_ARG;
            }
            JL_TRY(check_ids(T, opts[b].oracle_stream, opts[b].oracle_len));
        }
    }
    if (G > MAX_GAMMA || (size_t)(G + 1) * batch > (size_t)BATCH_CHUNKS * SMALL_M) {
        set_error("batch %zu with max gamma %d exceeds the loop's %d verify rows (max gamma at most %d)", batch, G,
                  BATCH_CHUNKS * SMALL_M, MAX_GAMMA);
        return JL_ERR_INVALID_ARG;
    }
    std::vector<size_t> limit(batch), plen(lens, lens + batch);
    size_t max_limit = 0;
    for (size_t b = 0; b < batch; ++b) {
        // speculative.rs:60-67
        limit[b] = std::min({lens[b] + count, (size_t)T->max_positions, (size_t)D->max_positions});
        if (results[b].tokens_cap < std::max(limit[b], lens[b])) {
            set_error("results[%zu].tokens_cap %zu is below %zu", b, results[b].tokens_cap,
                      std::max(limit[b], lens[b]));
            return JL_ERR_INVALID_ARG;
        }
        max_limit = std::max(max_limit, limit[b]);
    }
    for (size_t b = 0; b < batch; ++b) {
        reset_result(&results[b]);
        memcpy(results[b].tokens, prompts[b], lens[b] * sizeof(uint32_t));
        results[b].n_tokens = lens[b];
    }
    JL_CUDA(cudaSetDevice(T->device));
    Batch bt{T, D, batch, {}, {}};
    bt.tc.assign(batch, nullptr);
    bt.dc.assign(batch, nullptr);
    for (size_t b = 0; b < batch; ++b) {
        JL_TRY(cache_create(T, &bt.tc[b]));
        JL_TRY(cache_create(D, &bt.dc[b]));
    }
    cudaStream_t st = T->stream;
    // prefill both models (speculative.rs:69-75)
    JL_CUDA(cudaEventRecord(T->ev0, st));
    std::vector<uint32_t> first(batch), dnext(batch);
    for (size_t b = 0; b < batch; ++b) {
        if (lens[b] >= limit[b]) continue;
        JL_TRY(predict(T, bt.tc[b], prompts[b], lens[b], false, &first[b], nullptr));
        JL_TRY(predict(D, bt.dc[b], prompts[b], lens[b], false, &dnext[b], nullptr));
    }
    JL_CUDA(cudaEventRecord(T->ev1, st));
    JL_CUDA(cudaEventSynchronize(T->ev1));
    const double prefill_ms = elapsed_ms(T->ev0, T->ev1);
    BatchGraph* g = nullptr;
    const size_t reach = max_limit + G + 1;
    JL_TRY(get_batch_graph(T, D, G, (int)batch, std::max(att_splits_for(T, reach), att_splits_for(D, reach)), &g));
    memset(g->host_seqs, 0, batch * sizeof(SpecState));
    memset(g->host_ctl, 0, sizeof(BatchCtl));
    g->host_ctl->B = (int32_t)batch;
    g->host_ctl->max_limit = (int32_t)max_limit;
    for (size_t b = 0; b < batch; ++b) {
        SpecState& s = g->host_seqs[b];
        const jl_schedule& sc = scheds[b];
        s.n_tokens = (int32_t)lens[b];
        s.limit = (int32_t)limit[b];
        s.eos = T->eos;
        s.gamma = (int32_t)sc.gamma;
        s.max_gamma = (int32_t)sc.max_gamma;
        s.adaptive = sc.adaptive ? 1 : 0;
        s.pending = -1;
        s.first_pred = (int32_t)first[b];
        s.target_len = (int32_t)bt.tc[b]->len;
        s.draft_len = (int32_t)bt.dc[b]->len;
        s.done = lens[b] >= limit[b] ? 1 : 0;
        // sequence b's oracle: a device copy of its stream
        Oracle& o = g->host_oracles[b];
        o = Oracle{nullptr, 0, 0.0, 0, T->vocab};
        if (opts && opts[b].oracle_stream) {
            const size_t len = std::min(opts[b].oracle_len, (size_t)g->tcap);
            uint32_t* dst = g->oracle_buf + b * g->tcap;
            JL_CUDA(cudaMemcpyAsync(dst, opts[b].oracle_stream, len * sizeof(uint32_t), cudaMemcpyHostToDevice, st));
            o = Oracle{dst, (int32_t)len, opts[b].oracle_p, opts[b].oracle_seed, T->vocab};
            const Oracle on_host{opts[b].oracle_stream, o.len, o.p, o.seed, T->vocab};
            s.draft_next = (int32_t)oracle_token(on_host, (int32_t)bt.dc[b]->len, dnext[b]);
        } else {
            s.draft_next = (int32_t)dnext[b];
        }
        JL_CUDA(cudaMemcpyAsync(g->args.tokens + b * g->tcap, prompts[b], lens[b] * sizeof(uint32_t),
                                cudaMemcpyHostToDevice, st));
        if (!s.done) {
            // pages for every position the loop can reach
            JL_TRY(cache_reserve(bt.tc[b], limit[b] + G + 1, st));
            JL_TRY(cache_reserve(bt.dc[b], limit[b] + G + 1, st));
        }
        g->host_pt[b] = bt.tc[b]->d_pages;
        g->host_pt[MAX_SEQS + b] = bt.dc[b]->d_pages;
    }
    return run_batch(g, plen, results, stats, prefill_ms);
}

}  // namespace jl
