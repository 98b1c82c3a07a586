/*
 * jalapeno.h -- C ABI of the B200 speculative-decoding engine for Qwen3.
 *
 * This ABI replaces the reference engine crate's public Rust API
 * (fawwaz46/jalapenos-at-home, engine/src/lib.rs:16-21) and its native GPU
 * bridge (engine/src/gpu.rs:19-42 -> engine/src/gpu.m:21-128).  Each entry
 * point names the reference item it stands in for.
 *
 * Conventions
 *  - Every call returns jl_status; JL_OK is 0.  On failure,
 *    jl_last_error() returns a thread-local message (never NULL).
 *  - Token ids are uint32_t (the reference uses usize; Qwen3's vocabulary
 *    fits in 32 bits).
 *  - The caller owns every host buffer it passes; the library owns device
 *    memory.  Handles are not thread safe: use one handle from one thread at
 *    a time.  Different handles are independent (one model per GPU replica).
 *  - There is no CPU fallback: calls that compute fail with
 *    JL_ERR_NO_DEVICE when no CUDA device is present.
 */
#ifndef JALAPENO_H
#define JALAPENO_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum jl_status {
    JL_OK = 0,
    JL_ERR_INVALID_ARG = 1, /* reference: assert!/panic on bad arguments */
    JL_ERR_FORMAT = 2,      /* reference: Err(...) from try_load / Mxfp4::validate */
    JL_ERR_OOM = 3,         /* reference: "could not allocate GPU memory" panic */
    JL_ERR_CUDA = 4,        /* reference: gpu_finish() returning -1 (gpu.m:114-128) */
    JL_ERR_TIMEOUT = 5,     /* a bounded device wait gave up */
    JL_ERR_IO = 6,          /* reference: io::Error from try_load */
    JL_ERR_NO_DEVICE = 7    /* no CUDA device: this engine has no CPU path */
} jl_status;

/* Thread-local description of the last failure on this thread. */
const char* jl_last_error(void);
/* Library version string, e.g. "0.1.0 sm_100a". */
const char* jl_version(void);
/* Number of visible CUDA devices (0 when none); never fails. */
int jl_device_count(void);

/* ------------------------------------------------------------------------
 * Weights on the host: engine::load / try_load (engine/src/lib.rs:85-202),
 * Tensor / Mxfp4 / Weights (lib.rs:27-71, mxfp4.rs:5-26).  Needs no GPU.
 * ---------------------------------------------------------------------- */

typedef struct jl_weights jl_weights;

typedef enum jl_dtype { JL_BF16 = 0, JL_MXFP4 = 1 } jl_dtype;

typedef struct jl_tensor_view {
    const char* name;        /* HF name without the .mxfp4_* suffix */
    jl_dtype dtype;
    int ndim;                /* 1 or 2 */
    size_t shape[2];         /* logical shape: [rows, cols] (cols in elements) */
    const uint16_t* bf16;    /* JL_BF16: shape product bf16 values, else NULL */
    const uint8_t* packed;   /* JL_MXFP4: rows*cols/2 bytes, low nibble = even index */
    const uint8_t* scales;   /* JL_MXFP4: rows*cols/32 E8M0 bytes (bias 127) */
} jl_tensor_view;

/* Reads every *.safetensors file of `dir` (sorted by name), with the
 * reference loader's validation: header <= 1e8 bytes, offsets in range,
 * BF16 tensors (U16 allowed in "jalapenos-mxfp4-v1" files), .mxfp4_packed /
 * .mxfp4_scales pairs, no duplicates, no orphaned scales, no NaN scale. */
jl_status jl_weights_load(const char* dir, jl_weights** out);
void jl_weights_free(jl_weights* w);
size_t jl_weights_count(const jl_weights* w);
/* i-th tensor in name order. */
jl_status jl_weights_at(const jl_weights* w, size_t i, jl_tensor_view* view);
jl_status jl_weights_get(const jl_weights* w, const char* name, jl_tensor_view* view);

/* ------------------------------------------------------------------------
 * Models on the GPU: Model::load / load_with_prefill (engine/src/model.rs:
 * 54-108) with Backend::Gpu, GpuModel::new (engine/src/gpu.rs:336-428).
 * ---------------------------------------------------------------------- */

typedef struct jl_model jl_model;
typedef struct jl_cache jl_cache;

typedef enum jl_kv_dtype { JL_KV_BF16 = 0, JL_KV_F32 = 1 } jl_kv_dtype;

typedef struct jl_model_options {
    int device;              /* CUDA device ordinal (default 0) */
    jl_kv_dtype kv_dtype;    /* KV cache element type (default bf16) */
    size_t kv_pool_tokens;   /* KV page pool capacity in tokens; 0 = context limit + 1024 */
    size_t max_pass_rows;    /* largest rows per forward pass; 0 = 4096 */
} jl_model_options;

/* Fills `o` with the defaults above. */
void jl_model_options_default(jl_model_options* o);

/* Loads config.json (num_hidden_layers, max_position_embeddings,
 * eos_token_id) and every .safetensors file of `dir`, uploads to the GPU.  bf16 and MXFP4
 * tensors may be mixed; a tied lm_head (absent or equal to the embedding
 * table) is stored once.  Every header is checked before any payload is
 * read (the checks and messages of jl_weights_load); payloads then go from
 * the files to the device through two 16 MB pinned buffers, so host memory
 * never holds the checkpoint.  opts may be NULL.
 * Replaces Model::load (engine/src/model.rs:55-57). */
jl_status jl_model_load(const char* dir, const jl_model_options* opts, jl_model** out);

/* Architecture of a seeded synthetic model (no file I/O): the same tensors a
 * checkpoint written from the seeded stream would hold.  Used by benchmarks
 * and tests; weights are generated on the GPU. */
typedef struct jl_synth_config {
    int layers, hidden, q_heads, kv_heads, inter, vocab;
    int tied;                /* 1: lm_head is the embedding table */
    int max_positions;       /* config.json max_position_embeddings */
    int eos;                 /* config.json eos_token_id */
    uint64_t seed;
    int mxfp4;               /* 1: q/k/v/o/gate/up/down quantized to MXFP4 */
    int mxfp4_embed;         /* 1: embedding and lm_head quantized too */
} jl_synth_config;
jl_status jl_model_synthesize(const jl_synth_config* cfg, const jl_model_options* opts,
                              jl_model** out);
void jl_model_free(jl_model* m);

typedef struct jl_model_info {
    int layers, hidden, q_heads, kv_heads, inter, vocab, max_positions, eos;
    int tied;
    int mxfp4_projections;   /* 1 when the layer projections are MXFP4 */
    int mxfp4_head;          /* 1 when the output table is MXFP4 */
    size_t weight_bytes;     /* bytes of weights resident on the GPU */
    size_t pass_bytes;       /* weight bytes one single-row forward pass reads */
    size_t kv_bytes_per_token;
} jl_model_info;
jl_status jl_model_info_get(const jl_model* m, jl_model_info* info);

/* Copies one weight tensor back to the host in its device format (for
 * tests).  bf16: rows*cols*2 bytes; MXFP4: packed then scales. */
jl_status jl_model_read_tensor(const jl_model* m, const char* name, void* dst, size_t cap,
                               size_t* written);

/* ------------------------------------------------------------------------
 * KV cache: Model::cache / KvCache::truncate (engine/src/model.rs:37-52,
 * 124-133), GpuCache (engine/src/gpu.rs:272-300).  Pages of the model's
 * pool are taken as the sequence grows; truncation only moves the length.
 * ---------------------------------------------------------------------- */

jl_status jl_cache_create(jl_model* m, jl_cache** out);
void jl_cache_free(jl_cache* c);
size_t jl_cache_len(const jl_cache* c);
/* len must not exceed the current length (KvCache::truncate asserts). */
jl_status jl_cache_truncate(jl_cache* c, size_t len);

/* ------------------------------------------------------------------------
 * Forward passes: Model::predict / next_token / hidden (model.rs:143-240),
 * GpuModel::run (gpu.rs:544-634).  One host sync per call.
 * ---------------------------------------------------------------------- */

/* Appends `n` tokens to `c` and predicts after the last row (all == 0, one
 * id) or after every row (all != 0, n ids).  out_logits (nullable) receives
 * [rows_predicted, vocab] f32 logits. */
jl_status jl_predict(jl_model* m, jl_cache* c, const uint32_t* ids, size_t n, int all,
                     uint32_t* out_ids, float* out_logits);
/* jl_predict for a speculative loop's draft step: n = 1 or 2 tokens,
 * predicting after the last, through the kernels the loop's draft passes
 * run (on a model whose layer projections are all MXFP4, CUDA-core
 * projections with rounding of their own; otherwise the same pass as
 * jl_predict).  Stands in for the draft's proposal passes of
 * generate_scheduled (engine/src/speculative.rs:84-92, 136-138, which call
 * Model::predict); it lets callers check those kernels' logits. */
jl_status jl_predict_draft(jl_model* m, jl_cache* c, const uint32_t* ids, size_t n,
                           uint32_t* out_id, float* out_logits);
/* Model::next_token (model.rs:203-205): predict after a fresh prompt. */
jl_status jl_next_token(jl_model* m, const uint32_t* ids, size_t n, uint32_t* out_id);
/* Model::hidden (model.rs:143-154): residual stream after `layers` layers
 * for `n` tokens on a fresh cache, [n, hidden] f32. */
jl_status jl_hidden(jl_model* m, const uint32_t* ids, size_t n, size_t layers, float* out);

/* ------------------------------------------------------------------------
 * Generation: Model::generate (model.rs:268-285), generate_speculative /
 * generate_scheduled (speculative.rs:32-143), DraftSchedule (scheduler.rs).
 * ---------------------------------------------------------------------- */

/* Greedy decode.  out receives prompt + generated ids (capacity `cap`,
 * which must be >= n + count); *out_len is set to their number. */
jl_status jl_generate(jl_model* m, const uint32_t* prompt, size_t n, size_t count,
                      uint32_t* out, size_t cap, size_t* out_len);

typedef struct jl_schedule {
    uint32_t gamma;          /* initial draft length */
    uint32_t max_gamma;      /* adaptive upper bound (== gamma when fixed) */
    int adaptive;
} jl_schedule;
/* DraftSchedule::fixed (scheduler.rs:9-16): gamma must be positive. */
jl_status jl_schedule_fixed(uint32_t gamma, jl_schedule* out);
/* DraftSchedule::adaptive (scheduler.rs:18-27): 0 < initial <= maximum. */
jl_status jl_schedule_adaptive(uint32_t initial, uint32_t maximum, jl_schedule* out);

typedef struct jl_round_stats {
    uint32_t gamma, drafted, accepted, next_gamma; /* RoundStats (speculative.rs:13-19) */
} jl_round_stats;

typedef enum jl_spec_mode {
    JL_SPEC_DEVICE = 0,      /* whole loop on the GPU in one CUDA graph, one host sync */
    JL_SPEC_HOST = 1         /* reference control flow on the host, one sync per pass */
} jl_spec_mode;

typedef struct jl_spec_options {
    jl_spec_mode mode;
    /* Oracle-draft mode (benchmarks): when oracle_stream is non-NULL, the
     * draft model still runs every pass but its prediction for position P is
     * replaced by oracle_stream[P] (P < oracle_len), or with probability
     * oracle_p by a uniform id drawn from (oracle_seed, P). */
    const uint32_t* oracle_stream;
    size_t oracle_len;
    double oracle_p;
    uint64_t oracle_seed;
} jl_spec_options;
void jl_spec_options_default(jl_spec_options* o);

typedef struct jl_spec_result {
    /* caller-provided outputs */
    uint32_t* tokens;        /* prompt + generated ids, capacity tokens_cap */
    size_t tokens_cap;
    jl_round_stats* rounds_out; /* per-round stats, capacity rounds_cap (nullable) */
    size_t rounds_cap;
    /* filled by the call (SpeculativeResult, speculative.rs:21-30) */
    size_t n_tokens;
    size_t drafted, accepted, rounds;
    size_t prefill_passes, draft_passes, verify_passes;
    double prefill_ms;       /* both prefills, GPU time */
    double decode_ms;        /* everything after prefill, GPU time */
    double draft_ms, verify_ms; /* per phase (JL_SPEC_HOST only; 0 otherwise) */
} jl_spec_result;

/* The projections of one layer as the forward pass runs them: the
 * reference's public matmul (engine/src/lib.rs:240-266, y = x . W^T) applied
 * to `rows` f32 input rows, in the fused forms this engine uses.
 *   JL_PROJ_QKV     y = [x.Wq^T | x.Wk^T | x.Wv^T]   (q_width + 2*kv_width)
 *   JL_PROJ_O       y = x . Wo^T                      (hidden)
 *   JL_PROJ_GATE_UP y = silu(x.Wgate^T) * (x.Wup^T)   (intermediate, lib.rs:459-463)
 *   JL_PROJ_DOWN    y = x . Wdown^T                   (hidden)
 *   JL_PROJ_HEAD    y = x . Whead^T                   (vocab; layer ignored)
 * Inputs are NOT normalised first.  rows must be at most 16. */
typedef enum jl_projection {
    JL_PROJ_QKV = 0, JL_PROJ_O = 1, JL_PROJ_GATE_UP = 2, JL_PROJ_DOWN = 3, JL_PROJ_HEAD = 4
} jl_projection;
jl_status jl_project(jl_model* m, int layer, jl_projection which, const float* x, size_t rows,
                     float* y);

/* jl_project for callers that cannot allocate device memory when they call
 * it (a host running under a fixed device-memory reservation, or code that
 * cannot take cudaMalloc's implicit synchronisation).  No counterpart in the
 * reference: it exists for this engine's C ABI only.
 *   x: device pointer, rows x input width f32; y: device pointer, rows x
 *   output width f32 (widths as for jl_project); stream: a cudaStream_t of
 *   m's device, or NULL for the model's own stream.
 * MXFP4 projections on the tensor-core path only; rows 1..8.  All scratch
 * comes from one fixed 4 MiB device array per device (no allocation of any
 * kind); a projection whose scratch would exceed it is rejected with
 * JL_ERR_INVALID_ARG.  Calls share that array, so calls that overlap on
 * the GPU race.  Creating or loading a model on a device sets the array up
 * (module load, address lookup, a pinned flag word), so no call loads or
 * allocates anything.
 * Returns after the projection has finished (the stream is synchronised). */
jl_status jl_project_noalloc(jl_model* m, int layer, jl_projection which, const float* x,
                             size_t rows, float* y, void* stream);

/* ------------------------------------------------------------------------
 * Profiling.
 * ---------------------------------------------------------------------- */

/* Model::time_pass (engine/src/model.rs:242-266, the CLI's --time-rows):
 * prefills `prompt`, then times `reps` + 2 passes of `rows` tokens that
 * predict after every row (rolling the cache back after each), drops the
 * first two and returns the median wall and GPU milliseconds. */
jl_status jl_time_pass(jl_model* m, const uint32_t* prompt, size_t n, size_t rows, size_t reps,
                       double* wall_ms, double* gpu_ms);

/* Launches one projection kernel of `layer` for `rows` input rows `iters`
 * times back to back on the model's stream and returns the mean device time
 * per launch (CUDA events) and the weight bytes each launch reads.  On a
 * model whose decode pass is fused (every projection MXFP4), O, GATE_UP and
 * DOWN time the fused kernel that pass runs, on the input pieces a previous
 * pass left behind, and HEAD with a bf16 table the final norm + tensor-core
 * table + argmax kernels; otherwise the standalone projection.  No reference
 * counterpart: it feeds the per-kernel roofline report. */
jl_status jl_time_projection(jl_model* m, int layer, jl_projection which, int rows, int iters,
                             double* ms_per_launch, size_t* weight_bytes);

/* jl_time_pass for one row taking the path a speculative loop's draft step
 * takes (on a model whose draft steps have a path of their own; otherwise
 * the same as jl_time_pass with rows = 1).  No reference counterpart: it
 * feeds the profile of a speculative round. */
jl_status jl_time_pass_draft(jl_model* m, const uint32_t* prompt, size_t n, size_t reps,
                             double* wall_ms, double* gpu_ms);

/* Kernels one forward pass of `rows` rows (with its next-token prediction)
 * launches: `draft_step` nonzero for a speculative loop's draft step.  No
 * reference counterpart: it feeds the launch count of the benchmark. */
jl_status jl_pass_kernels(const jl_model* m, size_t rows, int draft_step, size_t* kernels);

/* Runs one device wait that nothing completes, bounded by `polls` polls
 * (1..2^20) of the poll loop every pass kernel's waits use, which then sets
 * the same error bit: returns JL_ERR_TIMEOUT with the bounded-wait message
 * and leaves the model usable.  No reference counterpart: it tests the
 * timeout path without faulting or hanging the GPU. */
jl_status jl_wait_probe(jl_model* m, uint32_t polls);

/* Chooses the kernel of prompt attention for the prompt passes recorded
 * after the call: tensor_cores = 1 (the default) runs it on tcgen05 MMAs
 * wherever the model allows (fused MXFP4 model, bf16 KV pool, GQA group of
 * 1, 2, 4 or 8), 0 keeps the CUDA-core kernel.  *active (may be NULL)
 * receives 1 when prompts now run on tensor cores.  No reference
 * counterpart: it lets tests compare the two kernels on identical inputs. */
jl_status jl_model_prompt_attention(jl_model* m, int tensor_cores, int* active);

/* Kernel phase timeline, from the diagnostic build of this library
 * (`make -C jalapenos-at-home_b200 timeline` -> lib/libjalapeno_timeline.so):
 * the decode-pass kernels stamp the GPU's nanosecond clock at fixed points
 * of their critical path.  jl_timeline_read copies the stamps of the last
 * recorded pass (jl_time_pass / jl_time_pass_draft record one pass and
 * replay it), launches x JL_TIMELINE_CTAS x JL_TIMELINE_POINTS values, 0
 * where a CTA or point did not stamp; `stamps` NULL returns the launch
 * count only.  JL_ERR_INVALID_ARG from the normal build.  No reference
 * counterpart: it backs the per-kernel phase profiles. */
#define JL_TIMELINE_CTAS 512
#define JL_TIMELINE_POINTS 8
jl_status jl_timeline_read(uint64_t* stamps, size_t cap, size_t* launches);
/* Kernel of launch i of that pass (NULL past the last). */
const char* jl_timeline_kernel(size_t launch);

/* generate_scheduled: both models share token ids; the target has the
 * final say, so the output equals jl_generate(target, ...) whenever the
 * forward pass is row-count invariant (it is here). opts may be NULL. */
jl_status jl_generate_speculative(jl_model* target, jl_model* draft, const uint32_t* prompt,
                                  size_t n, size_t count, const jl_schedule* schedule,
                                  const jl_spec_options* opts, jl_spec_result* result);

/* ------------------------------------------------------------------------
 * A batch of independent sequences on one GPU, decoded in lockstep rounds
 * (the benchmark configuration with a per-GPU batch of sequences).  The
 * reference engine has no batch call: it decodes one sequence per call
 * (model.rs:268-285, speculative.rs:43-143), and each sequence here gets
 * exactly the tokens and counters that call gives it alone.  Weights are
 * read once per round for the whole batch.
 * ---------------------------------------------------------------------- */
#define JL_MAX_BATCH 64

typedef struct jl_batch_stats {
    double prefill_ms;       /* every sequence's prefill, GPU time */
    double decode_ms;        /* the batched loop, GPU time */
    size_t rounds;           /* lockstep rounds */
    size_t target_passes;    /* target passes of up to 16 rows */
    size_t draft_passes;     /* draft passes of up to 16 rows */
} jl_batch_stats;

/* Greedy decode of `batch` sequences (1..JL_MAX_BATCH): prompts[i] holds
 * prompt_lens[i] ids.  results[i].tokens (capacity tokens_cap, at least
 * prompt_lens[i] + count or the context limit) receives prompt + generated
 * ids and n_tokens its length; the other result fields are zero except
 * verify_passes (passes the sequence took part in), prefill_ms and
 * decode_ms (the whole batch's).  stats may be NULL. */
jl_status jl_generate_batch(jl_model* m, size_t batch, const uint32_t* const* prompts,
                            const size_t* prompt_lens, size_t count, jl_spec_result* results,
                            jl_batch_stats* stats);

/* jl_generate_speculative for each of `batch` sequences: schedules[i] and
 * opts[i] (opts may be NULL; its mode is ignored, the loop runs on the
 * device) belong to sequence i, and results[i] is filled as that call
 * fills it, with prefill_ms and decode_ms the whole batch's.  batch x
 * (largest max_gamma + 1) must not exceed 512.  stats may be NULL. */
jl_status jl_generate_speculative_batch(jl_model* target, jl_model* draft, size_t batch,
                                        const uint32_t* const* prompts, const size_t* prompt_lens,
                                        size_t count, const jl_schedule* schedules,
                                        const jl_spec_options* opts, jl_spec_result* results,
                                        jl_batch_stats* stats);

#ifdef __cplusplus
}
#endif
#endif /* JALAPENO_H */
