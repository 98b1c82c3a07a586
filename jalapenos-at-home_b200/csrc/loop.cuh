// Pieces shared by the device-resident generation loops (engine.cu: one
// sequence; batch.cu: independent sequences in lockstep rounds).
//
// The per-sequence steps below restate one round of
// engine/src/speculative.rs:79-140 on a SpecState.  A step that feeds rows
// to the next forward pass appends them to `rows` at *n, tagged with the
// sequence's page-table index, so the single-sequence loop and the batched
// loop build their passes with the same code.
#pragma once

#include "jl_internal.h"

namespace jl {

__host__ __device__ inline void philox10_hd(uint32_t c[4], uint32_t k0, uint32_t k1) {
    for (int r = 0; r < 10; ++r) {
        if (r) { k0 += 0x9E3779B9u; k1 += 0xBB67AE85u; }
        const uint64_t p0 = (uint64_t)0xD2511F53u * c[0];
        const uint64_t p1 = (uint64_t)0xCD9E8D57u * c[2];
        const uint32_t n0 = (uint32_t)(p1 >> 32) ^ c[1] ^ k0, n2 = (uint32_t)(p0 >> 32) ^ c[3] ^ k1;
        c[0] = n0; c[1] = (uint32_t)p1; c[2] = n2; c[3] = (uint32_t)p0;
    }
}

// Oracle-draft proposal for `position`: the scripted stream's token, or with
// probability p a uniform id, both drawn from one Philox block keyed by the
// seed and the position.  `own` is the draft model's prediction.
struct Oracle {
    const uint32_t* stream;  // device or host, matching the caller
    int32_t len;
    double p;
    uint64_t seed;
    int32_t vocab;
};

__host__ __device__ inline uint32_t oracle_token(const Oracle& o, int32_t position, uint32_t own) {
    if (!o.stream || position >= o.len) return own;
    uint32_t c[4] = {(uint32_t)position, 0u, 0u, 0x6f726163u};
    philox10_hd(c, (uint32_t)o.seed, 0x64726166u);
    if ((double)c[0] + 0.5 < o.p * 4294967296.0) return c[1] % (uint32_t)o.vocab;
    return o.stream[position];
}

// Device-side state of one sequence's generation loop.
struct SpecState {
    int32_t n_tokens, limit, eos, start;
    int32_t gamma, max_gamma, adaptive, budget;
    int32_t n_proposed, pending, first_pred, draft_next;
    int32_t target_len, draft_len, done, catch_rows;
    int32_t drafted, accepted, rounds, draft_passes, verify_passes;
    int32_t iterations;  // loop bodies entered; every round adds >= 1 token, so <= limit
    int32_t fault;       // set when a guard stopped the loop
    int32_t row0, nrows; // this round's verify rows: first index and count
    int32_t crow;        // this round's last draft catch-up row
    int32_t proposed[MAX_GAMMA];
};

__device__ inline void put_row(RowDesc* rows, int& n, uint32_t token, int32_t pos, int32_t seq) {
    RowDesc r;
    r.token = token;
    r.seq = seq;
    r.pos = pos;
    r.pad = 0;
    rows[n++] = r;
}

// speculative.rs:79-93, first iteration: propose draft_next; when the draft
// runs again, append its row.  False once the sequence is finished.
__device__ inline bool seq_round_begin(SpecState& s, RowDesc* rows, int& n, int seq) {
    if (s.done || s.fault || s.n_tokens >= s.limit) {
        s.done = 1;
        return false;
    }
    s.start = s.n_tokens;
    s.budget = min(s.gamma, s.limit - s.start);
    s.proposed[0] = s.draft_next;
    s.n_proposed = 1;
    s.catch_rows = 0;
    if (!(s.budget == 1 || s.draft_next == s.eos)) put_row(rows, n, (uint32_t)s.draft_next, s.draft_len, seq);
    return true;
}

// After draft pass i of a round (speculative.rs:84-92); `out` is the draft's
// prediction for the sequence's row.
__device__ inline void seq_draft_step(SpecState& s, const Oracle& o, int i, uint32_t out, RowDesc* rows,
                                      int& n, int seq) {
    s.draft_len += 1;
    s.draft_passes += 1;
    const uint32_t tok = oracle_token(o, s.draft_len, out);
    s.draft_next = (int32_t)tok;
    s.proposed[i] = (int32_t)tok;
    s.n_proposed = i + 1;
    if (!(i + 1 == s.budget || (int32_t)tok == s.eos)) put_row(rows, n, tok, s.draft_len, seq);
}

// speculative.rs:95-97: [pending correction] + proposals, predict after every row.
__device__ inline void seq_verify_rows(SpecState& s, RowDesc* rows, int& n, int seq) {
    s.row0 = n;
    if (s.pending >= 0) put_row(rows, n, (uint32_t)s.pending, s.target_len, seq);
    for (int j = 0; j < s.n_proposed; ++j)
        put_row(rows, n, (uint32_t)s.proposed[j], s.target_len + (n - s.row0), seq);
    s.nrows = n - s.row0;
}

// speculative.rs:99-140: greedy acceptance, schedule feedback, rollback by
// length, correction / bonus token; `out` holds the target's predictions for
// this sequence's verify rows.  Appends the draft catch-up rows and returns
// true while the sequence continues.
__device__ inline bool seq_accept(SpecState& s, const uint32_t* out, uint32_t* tokens, jl_round_stats* rounds,
                                  int32_t rounds_cap, RowDesc* rows, int& n, int seq) {
    const int nr = s.nrows;
    s.target_len += nr;
    s.verify_passes += 1;
    int32_t preds[MAX_GAMMA + 2];
    int np = 0;
    if (s.first_pred >= 0) preds[np++] = s.first_pred;
    for (int j = 0; j < nr; ++j) preds[np++] = (int32_t)out[j];
    s.first_pred = -1;
    s.pending = -1;
    int accepted = 0;
    int32_t next = preds[0];
    while (accepted < s.n_proposed && s.proposed[accepted] == next) {
        ++accepted;
        next = preds[accepted];
    }
    // DraftSchedule::observe (scheduler.rs:33-44)
    const int gamma = s.gamma, drafted = s.n_proposed;
    if (s.adaptive && drafted == s.gamma) {
        if (accepted == drafted) s.gamma = min(s.gamma + 1, s.max_gamma);
        else if (accepted < (drafted + 1) / 2) s.gamma = max(s.gamma / 2, 1);
    }
    if (s.rounds < rounds_cap) {
        jl_round_stats r;
        r.gamma = (uint32_t)gamma;
        r.drafted = (uint32_t)drafted;
        r.accepted = (uint32_t)accepted;
        r.next_gamma = (uint32_t)s.gamma;
        rounds[s.rounds] = r;
    }
    s.rounds += 1;
    s.drafted += drafted;
    s.accepted += accepted;
    // budget <= limit - start keeps n_tokens <= limit; the guards only bound writes
    for (int j = 0; j < accepted && s.n_tokens < s.limit; ++j) tokens[s.n_tokens++] = (uint32_t)s.proposed[j];
    bool stop = (accepted > 0 && (int32_t)tokens[s.n_tokens - 1] == s.eos) || s.n_tokens >= s.limit;
    if (!stop) {
        s.target_len = s.start + accepted;
        s.draft_len = min(s.start + accepted, s.draft_len);
        tokens[s.n_tokens++] = (uint32_t)next;
        stop = next == s.eos || s.n_tokens >= s.limit;
    }
    if (stop) {
        s.done = 1;
        return false;
    }
    s.pending = next;
    // The last accepted proposal may not be in the draft cache yet: feed it
    // together with the bonus token (speculative.rs:134-138).
    const int tail = s.n_tokens - s.draft_len;
    if (tail < 1 || tail > 2) {  // cannot happen; stop rather than run a malformed pass
        s.fault = 1;
        s.done = 1;
        return false;
    }
    s.catch_rows = tail;
    for (int j = 0; j < tail; ++j) put_row(rows, n, tokens[s.draft_len + j], s.draft_len + j, seq);
    s.crow = n - 1;
    return true;
}

// After the draft catch-up pass; `out` is the prediction after its last row.
__device__ inline void seq_catchup_done(SpecState& s, const Oracle& o, uint32_t out) {
    s.draft_len += s.catch_rows;
    s.draft_passes += 1;
    s.draft_next = (int32_t)oracle_token(o, s.draft_len, out);
}

// ---- host helpers (engine.cu) ------------------------------------------------

double elapsed_ms(cudaEvent_t a, cudaEvent_t b);
// Surfaces the device guard flag kernels set instead of touching memory out
// of range (and clears it).
jl_status check_device_flag(jl_model* m);
jl_status check_ids(const jl_model* m, const uint32_t* ids, size_t n);

jl_status add_conditional(cudaGraph_t graph, cudaGraphNode_t* deps, size_t ndeps,
                          cudaGraphConditionalHandle h, cudaGraphConditionalNodeType type,
                          cudaGraphNode_t* node, cudaGraph_t* body);

// Captures the kernels that `fn` launches on `stream` into `graph`, after
// `dep` (or as roots when dep is null); returns the capture's last nodes.
template <class F>
jl_status capture_into(cudaGraph_t graph, cudaStream_t stream, cudaGraphNode_t* dep, F fn,
                       std::vector<cudaGraphNode_t>* tail) {
    JL_CUDA(cudaStreamBeginCaptureToGraph(stream, graph, dep, nullptr, dep ? 1 : 0,
                                          cudaStreamCaptureModeThreadLocal));
    jl_status rs = fn();
    if (rs == JL_OK && tail) {
        cudaStreamCaptureStatus cs;
        const cudaGraphNode_t* deps = nullptr;
        size_t nd = 0;
        cudaError_t e = cudaStreamGetCaptureInfo(stream, &cs, nullptr, nullptr, &deps, &nd);
        if (e == cudaSuccess) tail->assign(deps, deps + nd);
    }
    cudaGraph_t out;
    cudaError_t ce = cudaStreamEndCapture(stream, &out);
    if (rs != JL_OK) return rs;
    JL_CUDA(ce);
    return JL_OK;
}

}  // namespace jl
