/*
 * jl_oracle.h -- CPU restatement of the reference engine's algorithm.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product (the CUDA library under
 * jalapenos-at-home_b200/) links, loads or calls this code.  Only tests/,
 * __graft_entry__.smoke() and bench.py's cpu_baseline leg use it, as the
 * checker the GPU path is compared against.
 *
 * Every function states the reference file:line it restates (paths are
 * relative to the reference project root, fawwaz46/jalapenos-at-home).
 * Floating-point code is compiled with -ffp-contract=off so that products and
 * sums round exactly as the Rust code's separate f32 operations do.
 */
#ifndef JL_ORACLE_H
#define JL_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- scalar formats -------------------------------------------------- */

/* bf16 is the top half of an f32 (engine/src/lib.rs:73-76). */
float jlo_bf16_to_f32(uint16_t bits);
/* Round-to-nearest-even f32 -> bf16 (torch's .to(bfloat16) rounding). */
uint16_t jlo_f32_to_bf16(float value);

/* ---- MXFP4 codec ----------------------------------------------------- */

/* Mxfp4::validate (engine/src/mxfp4.rs:11-25).  Returns 0 when valid, or a
 * negative code: -1 bad shape, -2 length mismatch, -3 NaN scale (255). */
int jlo_mxfp4_validate(size_t rows, size_t cols, size_t packed_len, size_t scales_len,
                       const uint8_t* scales);
/* Mxfp4::value (engine/src/mxfp4.rs:28-33): element `index` of a row-major
 * [rows, cols] MXFP4 tensor.  Low nibble holds the even index. */
float jlo_mxfp4_value(const uint8_t* packed, const uint8_t* scales, size_t index);
/* Mxfp4::values over [start, end) (engine/src/mxfp4.rs:35-49). */
void jlo_mxfp4_values(const uint8_t* packed, const uint8_t* scales, size_t start, size_t end,
                      float* out);
/* quantize_mxfp4.quantize (python/quantize_mxfp4.py:18-39).  `values` is
 * row-major [rows, width] f32.  Returns 0, -1 (width % 32 != 0) or -2
 * (non-finite input); outputs are untouched on error. */
int jlo_mxfp4_quantize(const float* values, size_t rows, size_t width, uint8_t* packed,
                       uint8_t* scales);

/* ---- seeded synthetic weights --------------------------------------- */

/* Philox4x32-10 block (Salmon et al., SC'11), key (k0, k1). */
void jlo_philox4x32_10(const uint32_t ctr[4], uint32_t k0, uint32_t k1, uint32_t out[4]);
/* Element i of synthetic tensor `tensor_index` of a model seeded `seed`:
 * N(0, 0.02) by Box-Muller in double precision from Philox words, rounded
 * to f32 then to bf16 (RNE).  Writes n bf16 values starting at `first`. */
void jlo_synth_bf16(uint64_t seed, uint32_t tensor_index, uint64_t first, size_t n, uint16_t* out);

/* ---- model ----------------------------------------------------------- */

typedef struct jlo_model jlo_model;
typedef struct jlo_cache jlo_cache;

enum { JLO_BF16 = 0, JLO_MXFP4 = 1 };
enum {
    JLO_Q = 0, JLO_K, JLO_V, JLO_O, JLO_GATE, JLO_UP, JLO_DOWN, /* projections */
    JLO_INPUT_LN = 16, JLO_POST_LN, JLO_Q_NORM, JLO_K_NORM,      /* per-layer norms */
    JLO_EMBED = 32, JLO_HEAD, JLO_FINAL_NORM                      /* model-level */
};

/* Creates an empty model.  Dimensions follow engine/src/gpu.rs:398-406:
 * q/kv heads are counted in 128-wide heads.  Tensor storage is borrowed: the
 * caller keeps every array passed to jlo_model_set_* alive. */
jlo_model* jlo_model_new(int layers, int hidden, int q_heads, int kv_heads, int inter, int vocab,
                         int max_positions, int eos);
void jlo_model_free(jlo_model* m);
/* Matrix `which` of layer `layer` (ignored for model-level tensors).
 * kind JLO_BF16 uses `bf16`; JLO_MXFP4 uses `packed` + `scales`.  A NULL head
 * falls back to the embedding table (engine/src/model.rs:229-233). */
int jlo_model_set_matrix(jlo_model* m, int which, int layer, int kind, int rows, int cols,
                         const uint16_t* bf16, const uint8_t* packed, const uint8_t* scales);
int jlo_model_set_norm(jlo_model* m, int which, int layer, const uint16_t* bf16);

/* KvCache (engine/src/model.rs:37-52, lib.rs:323-335): f32 keys and values per
 * layer.  round_bf16 != 0 stores keys and values rounded to bf16 (RNE): that
 * is NOT the reference's behaviour; it mirrors a bf16 KV cache so that a bf16
 * cache can be compared token for token. */
jlo_cache* jlo_cache_new(const jlo_model* m, int round_bf16);
void jlo_cache_free(jlo_cache* c);
size_t jlo_cache_len(const jlo_cache* c);
int jlo_cache_truncate(jlo_cache* c, size_t len); /* KvCache::truncate, asserts len <= current */

/* Model::append_hidden (engine/src/model.rs:156-201): embeds `n` tokens, runs
 * `layers` decoder layers appending to `cache`, writes the residual stream
 * [n, hidden] to `out`.  Returns 0 or a negative error. */
int jlo_append_hidden(const jlo_model* m, jlo_cache* c, const uint32_t* tokens, size_t n,
                      int layers, float* out);
/* Model::predict (engine/src/model.rs:209-240): all != 0 predicts after every
 * row, else after the last row only.  out_ids gets one id per predicted row;
 * out_logits (nullable) gets [rows_predicted, vocab]. */
int jlo_predict(const jlo_model* m, jlo_cache* c, const uint32_t* tokens, size_t n, int all,
                uint32_t* out_ids, float* out_logits);

/* Building blocks, exported for unit tests. */
/* matmul (engine/src/lib.rs:240-266): y[rows, out] = x[rows, in] . W^T. */
int jlo_matmul(const jlo_model* m, int which, int layer, const float* x, size_t rows, float* y);
/* matmul on a free-standing matrix (kind JLO_BF16 or JLO_MXFP4, [rows, cols]). */
int jlo_matmul_raw(int kind, int rows, int cols, const uint16_t* bf16, const uint8_t* packed,
                   const uint8_t* scales, const float* x, size_t n, float* y);
/* rms_norm (engine/src/lib.rs:268-290) with bf16 gains w[width]. */
void jlo_rms_norm(const float* x, size_t rows, size_t width, const uint16_t* w, float* out);
/* rope (engine/src/lib.rs:291-321) in place over [rows, heads*128]. */
void jlo_rope(float* x, size_t rows, size_t heads, size_t offset);
/* argmax, first maximum wins (engine/src/model.rs:288-296). */
uint32_t jlo_argmax(const float* values, size_t n);

/* Number of OpenMP threads the oracle uses (for reporting). */
int jlo_threads(void);
/* Sets the OpenMP thread count of later calls (n > 0). */
void jlo_set_threads(int n);

#ifdef __cplusplus
}
#endif
#endif
