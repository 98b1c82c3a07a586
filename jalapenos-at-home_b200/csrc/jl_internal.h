// Internal declarations of the B200 Qwen3 decode engine.
//
// Data layout in HBM (one CUDA context per GPU, one model per handle):
//  * Weights live in one arena.  A projection is row-major [out, in]:
//    bf16 as u16[out*in]; MXFP4 exactly as the reference checkpoint stores it
//    (python/quantize_mxfp4.py:37-38): packed u8[out, in/2] with the even
//    element in the low nibble, and E8M0 scales u8[out, in/32].
//  * The KV cache is a pool of pages of PAGE tokens shared by every cache of a
//    model: [layer][K|V][page][kv_head][PAGE][128], bf16 or f32.  A cache is a
//    page table plus a length; truncation (KvCache::truncate,
//    engine/src/model.rs:45-51) only moves the length.
//  * A forward pass reads its rows (token, sequence, position) from a
//    device-resident PassBuf, so one captured CUDA graph serves any row count
//    up to the bucket it was captured for.
#pragma once

#include <cuda.h>  // CUtensorMap (a type only: the driver entry point is looked up at run time)
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstddef>
#include <cstdint>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "../../include/jalapeno.h"

namespace jl {

constexpr int HEAD = 128;        // head_dim of every Qwen3 model (engine/src/lib.rs:24)
constexpr int HALF = 64;         // RoPE rotates (i, i + 64) pairs (engine/src/lib.rs:297)
constexpr int PAGE = 64;         // tokens per KV page
constexpr int SMALL_M = 16;      // passes up to this many rows use the decode kernels (tensor-core MXFP4)
constexpr int ATT_WIN = 2;       // KV pages per decode-attention window (one CTA per window over long contexts)
constexpr int ATT_PART = 4 + HEAD;  // floats of one window's partial: max, sum, 2 pad, 128 outputs
constexpr int ATT_ZMAX = 64;     // window CTAs per row at most: past 64 windows each CTA takes several
// Window CTAs per row at most in the decode attention of passes whose q|k|v
// arrive normalised (greedy, verify, batched; the model's raw draft steps
// keep ATT_ZMAX): a verify pass's rows then fill the GPU with fewer,
// longer CTAs.  Every such pass of a model uses the same cap, so a row's
// result does not depend on the pass.
constexpr int ATT_ZMAX_DECODE = 8;
constexpr int MAX_SEQS = 64;     // sequences one pass may touch
constexpr int MAX_CHUNKS = 32;   // 16-row chunks of one multi-chunk pass (fused decode kernels)
constexpr int MAX_GAMMA = 16;    // largest draft length of the device-resident loop

// ---- errors --------------------------------------------------------------

void set_error(const char* fmt, ...) __attribute__((format(printf, 1, 2)));
const char* last_error();

struct Status {
    jl_status code = JL_OK;
    bool ok() const { return code == JL_OK; }
};

#define JL_TRY(expr)                                   \
    do {                                               \
        jl_status _s = (expr);                         \
        if (_s != JL_OK) return _s;                    \
    } while (0)

jl_status cuda_fail(cudaError_t e, const char* what, const char* file, int line);
#define JL_CUDA(call)                                                          \
    do {                                                                       \
        cudaError_t _e = (call);                                               \
        if (_e != cudaSuccess) return ::jl::cuda_fail(_e, #call, __FILE__, __LINE__); \
    } while (0)

// ---- host weights (engine::load) -------------------------------------------

struct HostTensor {
    std::string name;
    jl_dtype dtype = JL_BF16;
    std::vector<size_t> shape;       // logical shape
    std::vector<uint16_t> bf16;      // JL_BF16
    std::vector<uint8_t> packed;     // JL_MXFP4
    std::vector<uint8_t> scales;     // JL_MXFP4
};

struct HostConfig {
    int layers = 0, max_positions = 0, eos = 0;
};

// Where a tensor's bytes lie in a checkpoint file.
struct FileRange {
    std::string path;
    uint64_t offset = 0, bytes = 0;
};

// A checkpoint's tensors after every header check, with the payloads left in
// the files: BF16 values (little-endian u16) or MXFP4 packed codes at `data`.
// MXFP4 scales are read while scanning (a NaN scale is a format error), and
// are 1/16 of the packed bytes.
struct IndexTensor {
    std::string name;
    jl_dtype dtype = JL_BF16;
    std::vector<size_t> shape;     // logical shape
    FileRange data;
    std::vector<uint8_t> scales;   // JL_MXFP4
};

struct WeightIndex {
    std::map<std::string, IndexTensor> tensors;
};

}  // namespace jl

struct jl_weights {
    std::map<std::string, jl::HostTensor> tensors;
};

namespace jl {

jl_status load_weights(const std::string& dir, jl_weights* out);
jl_status scan_weights(const std::string& dir, WeightIndex* out);
jl_status read_range(const FileRange& r, void* dst, size_t offset, size_t bytes);
jl_status load_config(const std::string& dir, HostConfig* out);

// ---- device structures -------------------------------------------------------

enum MatKind : int { MAT_BF16 = 0, MAT_MXFP4 = 1 };

struct Mat {
    int kind = MAT_BF16;
    int rows = 0, cols = 0;
    const void* data = nullptr;      // bf16 [rows][cols] or packed [rows][cols/2]
    const uint8_t* scales = nullptr; // [rows][cols/32] for MXFP4
    size_t bytes() const {
        return kind == MAT_MXFP4 ? (size_t)rows * cols / 2 + (size_t)rows * cols / 32
                                 : (size_t)rows * cols * 2;
    }
};

// An MXFP4 projection re-laid out for the tensor-core kernel (mx_mma.cu):
// T tiles of 128 weight rows (gate/up: 64 gate + 64 up rows), S stages of 256
// K-elements, K split into `ksplit` slices across CTAs.
struct MxProj {
    const uint8_t* a = nullptr;     // [T][S] swizzled 16 KB weight stages, each then (MXFP4) its scales
    int T = 0, S = 0, K = 0, ksplit = 1, out_rows = 0;
    bool swiglu = false;
};

struct MxBuffers {
    uint8_t* bimg = nullptr;   // activation pieces, [S][N*128 + 1024]
    float* ws = nullptr;       // split-K partials
    int* tickets = nullptr;    // split-K arrival counters (kept at zero between launches)
    void* arena = nullptr;     // tiled weights
    void* scratch = nullptr;   // bimg, ws, tickets and the fused-pass buffers below
    // Fused decode pass (every layer MXFP4, widths multiples of 256): piece
    // images of the normalised residual stream (x), the attention output and
    // the SwiGLU activations, and per-tile sums of squares of x.
    bool fused = false;
    uint8_t* bx = nullptr;
    uint8_t* battn = nullptr;
    uint8_t* bact = nullptr;
    float* part = nullptr;     // [hidden / 128][MX_PART_STRIDE]
    // bf16 output table on the tensor cores: its input pieces and each
    // tile's first maximum per row
    uint8_t* bhead = nullptr;  // [hidden / 64][64 * 128]
    float* amax_v = nullptr;   // [T][MX_PART_STRIDE]
    int* amax_i = nullptr;
    // Multi-chunk passes: `chunks` copies of every buffer above from bx on,
    // chunk c's at c * (its stride): bytes for the piece images, elements for
    // part, amax_v and amax_i.
    int chunks = 1;
    size_t sx = 0, sattn = 0, sact = 0, spart = 0, shead = 0, samax = 0;
};

struct LayerW {
    MxProj mx_qkv, mx_o, mx_gateup, mx_down;
    Mat q, k, v, o, gate, up, down;
    const uint16_t* in_ln = nullptr;
    const uint16_t* post_ln = nullptr;
    const uint16_t* q_norm = nullptr;
    const uint16_t* k_norm = nullptr;
};

struct RowDesc {
    uint32_t token;
    int32_t seq;   // index into PassBuf::page_table
    int32_t pos;   // absolute position of this token in its sequence
    int32_t pad;
};

struct PassHdr {
    int32_t rows;       // active rows of this pass
    int32_t head_rows;  // rows whose next token is predicted
    int32_t pad0, pad1;
};

// Device pointers describing one pass; written by the host (jl_predict) or by
// the speculative-loop kernels, read by every pass kernel.
struct PassBuf {
    PassHdr* hdr = nullptr;
    RowDesc* row = nullptr;            // [max_rows]
    int32_t* head_row = nullptr;       // [max_rows] row index of each predicted row
    const int32_t** page_table = nullptr;  // [MAX_SEQS]
    uint32_t* out_ids = nullptr;       // [max_rows]
};

// One slot of a model's pinned descriptor staging ring.
constexpr int STAGE_SLOTS = 4;
struct StageSlot {
    PassHdr* hdr = nullptr;
    RowDesc* row = nullptr;                // [max_rows]
    int32_t* head_row = nullptr;           // [max_rows]
    const int32_t** page_table = nullptr;  // [MAX_SEQS]
    cudaEvent_t done = nullptr;            // recorded after the copies that read the slot
    bool pending = false;
};

struct Scratch {
    float* x = nullptr;       // [rows, hidden] residual stream
    float* xn = nullptr;      // [rows, max(hidden, q_width)] normalised input
    float* qkv = nullptr;     // [rows, q_width + 2*kv_width]
    float* attn = nullptr;    // [rows, q_width]
    float* act = nullptr;     // [rows, inter] silu(gate) * up
    float* xh = nullptr;      // [rows, hidden] final-norm rows to predict
    float* logits = nullptr;  // [rows, vocab]
};

struct KvPool {
    jl_kv_dtype dtype = JL_KV_BF16;
    int elem = 2;
    size_t pages = 0;
    void* base = nullptr;                 // [layers][2][pages][kv_heads][PAGE][HEAD]
    std::vector<int32_t> free_list;
    size_t page_elems = 0;                // kv_heads * PAGE * HEAD
};

struct SpecGraph;   // device-resident speculative loop (engine.cu)
struct BatchGraph;  // device-resident loop over a batch of sequences (batch.cu)

}  // namespace jl

struct jl_model {
    int device = 0;
    int sms = 148;                        // streaming multiprocessors of the device
    int layers = 0, hidden = 0, q_heads = 0, kv_heads = 0, inter = 0, vocab = 0;
    int max_positions = 0, eos = 0;
    bool tied = false;
    jl::Mat embed, head;
    jl::MxProj mx_head;                   // tensor-core copy of an MXFP4 output table
    jl::MxProj bf_head;                   // tensor-core copy of a bf16 output table (fused pass)
    bool dec_ok = false;                  // draft steps may run on the CUDA-core kernels
    jl::MxBuffers mx;
    const uint16_t* final_norm = nullptr;
    std::vector<jl::LayerW> lw;
    void* arena = nullptr;
    size_t arena_bytes = 0;
    float2* rope = nullptr;               // [max_positions][HALF] (cos, sin)
    jl::KvPool kv;
    // TMA tensor maps of each layer's K and V pages ([layer][K|V]) for the
    // tensor-core prompt attention; empty for f32 pools and pools too large
    // for 32-bit coordinates (the CUDA-core kernel serves those)
    std::vector<CUtensorMap> kv_tmaps;
    bool prompt_attn_cuda_cores = false;  // jl_model_prompt_attention(m, 0, ...)
    int max_rows = 0;
    jl::PassBuf pass;                     // device
    // Pinned staging of pass descriptors: a ring of slots (jl::stage_begin /
    // jl::stage_end).  An upload's copies run only when the stream reaches
    // them, after the work queued before; a slot is written again only once
    // they have run, so a pass never reads a later pass's descriptors.
    jl::StageSlot stage[jl::STAGE_SLOTS];
    int stage_next = 0;
    // decode attention over long contexts: one CTA per window of pages (up
    // to att_smax per row), a partial-sum workspace of att_rows rows
    // [kv_heads][rows][att_smax][group][4 + 128] f32 and per (kv head, row)
    // arrival counters (zero between launches)
    int att_smax = 1;
    int att_rows = 16;
    float* att_ws = nullptr;
    int* att_cnt = nullptr;
    int small_graph_splits[jl::SMALL_M] = {};  // att_splits each small_graph was captured with
    int draft_graph_splits[2] = {};
    uint32_t* host_out = nullptr;
    float* host_logits = nullptr;
    jl::Scratch s;
    void* scratch_arena = nullptr;
    cudaStream_t stream = nullptr;
    cudaEvent_t ev0 = nullptr, ev1 = nullptr;
    cudaGraphExec_t small_graph[jl::SMALL_M] = {};  // full pass of 1..16 rows, one per row count
    cudaGraphExec_t draft_graph[2] = {};  // draft-step pass of 1 or 2 rows (profiling)
    std::vector<jl::SpecGraph*> spec_graphs;  // owned; freed by model_free
    std::vector<jl::BatchGraph*> batch_graphs;  // owned; freed by model_free
    std::vector<jl_cache*> caches;              // live caches; detached by model_free
    int* counters = nullptr;              // zeroed split-K / reduction counters
    std::map<std::string, std::pair<const void*, size_t>> tensor_index;  // name -> device bytes
};
namespace jl {
// The next slot of m's staging ring, once the copies that last read it have
// run; stage_end records that the copies just queued on `st` read it.
jl_status stage_begin(jl_model* m, StageSlot** out);
jl_status stage_end(jl_model* m, StageSlot* s, cudaStream_t st);
}  // namespace jl


struct jl_cache {
    jl_model* m = nullptr;
    std::vector<int32_t> pages;
    int32_t* d_pages = nullptr;           // device page table [max_pages]
    int32_t* h_pages = nullptr;           // pinned mirror
    size_t max_pages = 0;
    size_t len = 0;
};

namespace jl {

// ---- model construction (model.cu) --------------------------------------------
jl_status model_from_checkpoint(const WeightIndex& w, const HostConfig& cfg, const jl_model_options& o,
                                jl_model** out);
jl_status model_synthesize(const jl_synth_config& c, const jl_model_options& o, jl_model** out);
void model_free(jl_model* m);
jl_status cache_create(jl_model* m, jl_cache** out);
void cache_free(jl_cache* c);
jl_status cache_reserve(jl_cache* c, size_t tokens, cudaStream_t stream);

// ---- passes and generation (engine.cu) ---------------------------------------
// Records the kernels of one forward pass on `stream`.  rows_cap bounds the
// rows the pass may have; `layers` < m->layers stops early (Model::hidden);
// with_head adds final norm, lm_head and argmax.
struct PassCtx;
jl_status record_pass_ctx(const PassCtx& c, int layers, bool with_head);
// Sets kernel attributes once per device, before any stream capture.
jl_status configure_kernels();
// Tensor-core prompt attention (attn_prefill_tc.cu).
jl_status kv_tensor_maps(jl_model* m);
jl_status configure_prefill_tc();
bool prefill_tc_supported(const jl_model* m);
jl_status launch_attention_prefill_tc(const PassCtx& c, int layer, uint8_t* bout, int bN);
jl_status predict(jl_model* m, jl_cache* c, const uint32_t* ids, size_t n, bool all,
                  uint32_t* out_ids, float* out_logits, bool draft_step = false);
jl_status hidden(jl_model* m, const uint32_t* ids, size_t n, size_t layers, float* out);
// One bounded device wait that nothing completes (tests the timeout path).
jl_status wait_probe(jl_model* m, uint32_t polls);
jl_status time_pass(jl_model* m, const uint32_t* prompt, size_t n, size_t rows, size_t reps,
                    double* wall_ms, double* gpu_ms, bool draft_step = false);
jl_status time_projection(jl_model* m, int layer, int which, int rows, int iters, double* ms,
                          size_t* bytes);
jl_status project(jl_model* m, int layer, int which, const float* x, size_t rows, float* y);
size_t pass_kernels(const jl_model* m, size_t rows, bool draft_step);
jl_status generate(jl_model* m, const uint32_t* prompt, size_t n, size_t count, uint32_t* out,
                   size_t cap, size_t* out_len);
jl_status generate_speculative(jl_model* target, jl_model* draft, const uint32_t* prompt,
                               size_t n, size_t count, const jl_schedule& sched,
                               const jl_spec_options& opts, jl_spec_result* res);
void spec_graph_free(SpecGraph* g);
// A batch of independent sequences decoded in lockstep rounds (batch.cu).
jl_status generate_batch(jl_model* m, size_t batch, const uint32_t* const* prompts, const size_t* lens,
                         size_t count, jl_spec_result* results, jl_batch_stats* stats);
jl_status generate_speculative_batch(jl_model* target, jl_model* draft, size_t batch,
                                     const uint32_t* const* prompts, const size_t* lens, size_t count,
                                     const jl_schedule* schedules, const jl_spec_options* opts,
                                     jl_spec_result* results, jl_batch_stats* stats);
void batch_graph_free(BatchGraph* g);

// ---- kernel launchers (kernels.cu) ---------------------------------------------
struct PassCtx {
    const jl_model* m;
    cudaStream_t stream;
    int rows_cap;   // rows the pass may hold
    int head_cap;   // predicted rows the pass may hold
    bool draft = false;  // a speculative loop's draft step (may take the CUDA-core path)
    int att_splits = 1;  // decode attention: window CTAs per row in the launch grid (att_splits_for)
    // A multi-chunk pass (fused decode kernels only): `chunks` > 1 chunks of
    // 16 rows, rows_cap = head_cap = 16 * chunks.  Chunk c has its own header
    // (hdr[c]); its rows are row[16c ..], its predicted rows are listed in
    // head_row[16c ..] as indices within the chunk and predicted into
    // out_ids[16c ..].  Each kernel runs every chunk in one launch.
    int chunks = 1;
    // A multi-chunk pass over one sequence's prompt at consecutive positions
    // (predict): attention shares each K/V page among 8 rows.
    bool prefill = false;
    // The rows this pass reads: by default the model's own pass buffer; a
    // batched loop points each pass at its own buffers.
    PassBuf view{};
    const PassBuf& pass() const { return view.hdr ? view : m->pass; }
};
// Window CTAs per row a decode attention launch needs to cover contexts of
// up to max_ctx positions: a power of two (so graphs rebuild rarely), at most
// the model's att_smax.
int att_splits_for(const jl_model* m, size_t max_ctx);
jl_status launch_embed(const PassCtx& c);
jl_status launch_rmsnorm(const PassCtx& c, const float* x, const uint16_t* w, float* out,
                         bool head_rows);
jl_status launch_qkv(const PassCtx& c, const LayerW& L);
jl_status launch_qk_rope_kv(const PassCtx& c, int layer, const LayerW& L);
jl_status launch_attention(const PassCtx& c, int layer, bool pieces = false);
// Decode attention on raw q|k|v rows: it applies QK-RMSNorm and RoPE itself
// and appends this pass's K/V to the cache (the draft-step pass).
jl_status launch_attention_raw(const PassCtx& c, int layer, const uint16_t* qn, const uint16_t* kn);
jl_status launch_o(const PassCtx& c, const LayerW& L);
jl_status launch_gateup(const PassCtx& c, const LayerW& L);
jl_status launch_down(const PassCtx& c, const LayerW& L);
jl_status launch_head(const PassCtx& c);
jl_status launch_argmax(const PassCtx& c);

jl_status launch_synth_bf16(uint64_t seed, uint32_t tensor_index, size_t n, uint16_t* out,
                            cudaStream_t stream);

// ---- tensor-core MXFP4 projections (mx_mma.cu) ---------------------------------
enum MxEpi : int { MXE_STORE = 0, MXE_ADD = 1, MXE_SWIGLU = 2, MXE_QKV = 3 };
constexpr int MX_PART_STRIDE = 16;  // rows per tile in the sum-of-squares partials
// Fused decode-pass projection (mx_project_fused): its input pieces are
// already in b, written by the kernel before it.
struct MxFuse {
    const uint8_t* b = nullptr;        // input pieces
    const float* part_in = nullptr;    // input RMSNorm: per-tile sums of squares of x
    int part_tiles = 0, norm_width = 0;
    uint8_t* bout = nullptr;           // pieces of (output * next_w) for the next projection
    float* part_out = nullptr;         // per-tile sums of squares of the output (residual add)
    const uint16_t* next_w = nullptr;
    int layer = 0;                     // q|k|v: cache layer and QK-norm weights
    const uint16_t* qn = nullptr;
    const uint16_t* kn = nullptr;
    size_t cs_b = 0, cs_bout = 0;      // multi-chunk passes: chunk strides of b and bout (bytes)
};
jl_status mx_configure();
int mx_max_tokens();
size_t mx_tile_bytes(int out_rows, int K, bool swiglu);
jl_status mx_build(const Mat* const* mats, int nmats, bool swiglu, uint8_t* dst, int sms,
                   MxProj* out, cudaStream_t stream);
jl_status mx_project(const PassCtx& c, const MxProj& p, int epi, int use_head, const float* x,
                     int ldx, const uint16_t* norm, float* y, int ldy);
// Scratch one launch of `p` over `mcap` rows needs when the caller supplies
// it: split-K tickets (zero at launch), the piece image and split-K
// partials, in that order, each 256-byte aligned.
struct MxScratchPlan {
    size_t tickets = 0, bimg = 0, ws = 0, total = 0;
};
MxScratchPlan mx_scratch_plan(const MxProj& p, int mcap);
jl_status mx_project_fused(const PassCtx& c, const MxProj& p, int epi, const MxFuse& f, float* y,
                           int ldy);
// Pieces of x * w and per-tile sums of squares of x for the first projection
// of a fused pass (after the embedding).
jl_status mx_norm_pieces(const PassCtx& c, const float* x, int ldx, const uint16_t* w, int width,
                         uint8_t* bout, float* part);
// bf16 output table on the tensor cores (kind::f16): load-time tiles, and the
// fused final norm + logits + argmax of a decode pass.
size_t bf16_tile_bytes(int rows, int K);
jl_status mx_build_bf16(const Mat& w, uint8_t* dst, MxProj* out, cudaStream_t stream);
jl_status mx_head_fused(const PassCtx& c, const MxProj& p, const uint16_t* norm, float* logits, int ldy);
// Draft-step passes of 1..2 rows on CUDA cores (dec.cu).
bool dec_supported(const jl_model* m);
jl_status dec_configure();
jl_status record_dec_pass(const PassCtx& c, int layers);
// mx_project over caller-owned memory: `hdr` (rows read on the device),
// `scratch` laid out as mx_scratch_plan says, `err` the device error flag.
jl_status mx_project_with(const MxProj& p, int epi, const PassHdr* hdr, int mcap, const float* x,
                          int ldx, float* y, int ldy, uint8_t* scratch, int* err, int sms,
                          cudaStream_t stream);
jl_status project_noalloc(jl_model* m, int layer, int which, const float* x, size_t rows, float* y,
                          cudaStream_t stream);
// Loads project_noalloc's module, array and kernels on the current device
// and pins its host flag word, so that no call of it loads or allocates.
jl_status noalloc_prepare(int device);
// Builds the tensor-core copies of every MXFP4 projection of `m` (model.cu).
jl_status build_mx(jl_model* m);
jl_status launch_fill_u16(uint16_t* out, size_t n, uint16_t value, cudaStream_t stream);
jl_status launch_quantize_mxfp4(const uint16_t* bf16, int rows, int cols, uint8_t* packed,
                                uint8_t* scales, cudaStream_t stream);

// ---- kernel phase timeline (the device side is timeline.cuh) ----

constexpr int TL_LAUNCHES = 512, TL_CTAS = 512, TL_POINTS = 8;

// A launch's rows of the table (a kernel argument); table null: no stamps.
struct TlSlot {
    unsigned long long* table;
    int id;
};

// Host side (engine.cu).  tl_begin_pass restarts the launch ids; tl_launch
// returns the slot of the next launch of the pass being recorded and keeps
// its kernel name for the reader.  Both do nothing in the normal build.
void tl_begin_pass();
TlSlot tl_launch(const char* kernel);
bool tl_enabled();
// allocates the table (timeline build, once per process, on the current
// device) when a model is created, never while a pass is being captured
jl_status tl_prepare();
// zeroes the table on `stream` (outside a capture), so rows that the passes
// timed next do not write read as zeros rather than as older stamps
jl_status tl_clear(cudaStream_t stream);
// launches recorded in the last pass; copies their rows (launches x TL_CTAS
// x TL_POINTS stamps) when `out` is non-null and `cap` holds them all
jl_status tl_read(unsigned long long* out, size_t cap, size_t* launches);
const char* tl_kernel(size_t launch);

}  // namespace jl
