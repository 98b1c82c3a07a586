// extern "C" entry points declared in include/jalapeno.h.  Each validates
// its arguments, converts them to the internal engine calls and reports
// failures through the thread-local jl_last_error().
#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>

#include "jl_internal.h"

namespace jl {

namespace {
thread_local char g_error[1024] = "";
}

void set_error(const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_error, sizeof g_error, fmt, ap);
    va_end(ap);
}

const char* last_error() { return g_error; }

jl_status cuda_fail(cudaError_t e, const char* what, const char* file, int line) {
    set_error("CUDA error %s (%s) in %s at %s:%d", cudaGetErrorName(e), cudaGetErrorString(e), what,
              file, line);
    if (e == cudaErrorMemoryAllocation) return JL_ERR_OOM;
    if (e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver) return JL_ERR_NO_DEVICE;
    return JL_ERR_CUDA;
}

}  // namespace jl

using namespace jl;

#define JL_NEED(cond, msg)                        \
    do {                                          \
        if (!(cond)) {                            \
            set_error("%s", msg);                 \
            return JL_ERR_INVALID_ARG;            \
        }                                         \
    } while (0)

#define JL_GUARD(...)                                             \
    try {                                                         \
        __VA_ARGS__                                               \
    } catch (const std::bad_alloc&) {                             \
        set_error("host allocation failed");                      \
        return JL_ERR_OOM;                                        \
    } catch (const std::exception& e) {                           \
        set_error("internal error: %s", e.what());                \
        return JL_ERR_INVALID_ARG;                                \
    }

extern "C" {

const char* jl_last_error(void) { return last_error(); }

const char* jl_version(void) { return "0.1.0 sm_100a"; }

int jl_device_count(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return n;
}

// ---- weights -------------------------------------------------------------

jl_status jl_weights_load(const char* dir, jl_weights** out) {
    JL_NEED(dir && out, "dir and out must be non-null");
    *out = nullptr;
    JL_GUARD({
        std::unique_ptr<jl_weights> w(new jl_weights());
        JL_TRY(load_weights(dir, w.get()));
        *out = w.release();
        return JL_OK;
    })
}

void jl_weights_free(jl_weights* w) { delete w; }

size_t jl_weights_count(const jl_weights* w) { return w ? w->tensors.size() : 0; }

static void fill_view(const HostTensor& t, jl_tensor_view* v) {
    memset(v, 0, sizeof *v);
    v->name = t.name.c_str();
    v->dtype = t.dtype;
    v->ndim = (int)t.shape.size();
    for (int i = 0; i < v->ndim && i < 2; ++i) v->shape[i] = t.shape[i];
    if (t.dtype == JL_MXFP4) {
        v->packed = t.packed.data();
        v->scales = t.scales.data();
    } else {
        v->bf16 = t.bf16.data();
    }
}

jl_status jl_weights_at(const jl_weights* w, size_t i, jl_tensor_view* view) {
    JL_NEED(w && view, "weights and view must be non-null");
    JL_NEED(i < w->tensors.size(), "tensor index out of range");
    auto it = w->tensors.begin();
    std::advance(it, i);
    fill_view(it->second, view);
    return JL_OK;
}

jl_status jl_weights_get(const jl_weights* w, const char* name, jl_tensor_view* view) {
    JL_NEED(w && name && view, "weights, name and view must be non-null");
    auto it = w->tensors.find(name);
    if (it == w->tensors.end()) {
        set_error("missing tensor %s", name);
        return JL_ERR_INVALID_ARG;
    }
    fill_view(it->second, view);
    return JL_OK;
}

// ---- models ----------------------------------------------------------------

void jl_model_options_default(jl_model_options* o) {
    if (!o) return;
    memset(o, 0, sizeof *o);
    o->device = 0;
    o->kv_dtype = JL_KV_BF16;
    o->kv_pool_tokens = 0;
    o->max_pass_rows = 0;
}

static jl_status check_options(const jl_model_options* opts, jl_model_options* o) {
    jl_model_options_default(o);
    if (opts) *o = *opts;
    JL_NEED(o->kv_dtype == JL_KV_BF16 || o->kv_dtype == JL_KV_F32, "kv_dtype must be bf16 or f32");
    JL_NEED(o->max_pass_rows == 0 || (o->max_pass_rows >= (size_t)SMALL_M && o->max_pass_rows <= 65536),
            "max_pass_rows must lie in [32, 65536]");
    return JL_OK;
}

jl_status jl_model_load(const char* dir, const jl_model_options* opts, jl_model** out) {
    JL_NEED(dir && out, "dir and out must be non-null");
    *out = nullptr;
    jl_model_options o;
    JL_TRY(check_options(opts, &o));
    JL_GUARD({
        HostConfig cfg;
        JL_TRY(load_config(dir, &cfg));
        WeightIndex w;
        JL_TRY(scan_weights(dir, &w));
        return model_from_checkpoint(w, cfg, o, out);
    })
}

jl_status jl_model_synthesize(const jl_synth_config* cfg, const jl_model_options* opts,
                              jl_model** out) {
    JL_NEED(cfg && out, "cfg and out must be non-null");
    *out = nullptr;
    jl_model_options o;
    JL_TRY(check_options(opts, &o));
    JL_GUARD({ return model_synthesize(*cfg, o, out); })
}

void jl_model_free(jl_model* m) { model_free(m); }

jl_status jl_model_info_get(const jl_model* m, jl_model_info* info) {
    JL_NEED(m && info, "model and info must be non-null");
    memset(info, 0, sizeof *info);
    info->layers = m->layers;
    info->hidden = m->hidden;
    info->q_heads = m->q_heads;
    info->kv_heads = m->kv_heads;
    info->inter = m->inter;
    info->vocab = m->vocab;
    info->max_positions = m->max_positions;
    info->eos = m->eos;
    info->tied = m->tied ? 1 : 0;
    info->mxfp4_projections = m->lw.empty() ? 0 : (m->lw[0].q.kind == MAT_MXFP4);
    info->mxfp4_head = m->head.kind == MAT_MXFP4;
    info->weight_bytes = m->arena_bytes;
    size_t pass = m->head.bytes();
    for (const auto& L : m->lw)
        pass += L.q.bytes() + L.k.bytes() + L.v.bytes() + L.o.bytes() + L.gate.bytes() +
                L.up.bytes() + L.down.bytes();
    info->pass_bytes = pass;
    info->kv_bytes_per_token = (size_t)m->layers * 2 * m->kv_heads * HEAD * m->kv.elem;
    return JL_OK;
}

jl_status jl_model_read_tensor(const jl_model* m, const char* name, void* dst, size_t cap,
                               size_t* written) {
    JL_NEED(m && name && dst, "model, name and dst must be non-null");
    auto it = m->tensor_index.find(name);
    if (it == m->tensor_index.end()) {
        set_error("missing tensor %s", name);
        return JL_ERR_INVALID_ARG;
    }
    const void* src = it->second.first;
    size_t bytes = it->second.second;
    // MXFP4: packed and scales are adjacent allocations; copy both
    for (const auto& L : m->lw) {
        const Mat* mats[7] = {&L.q, &L.k, &L.v, &L.o, &L.gate, &L.up, &L.down};
        for (const Mat* mt : mats)
            if (mt->data == src && mt->kind == MAT_MXFP4) bytes = mt->bytes();
    }
    JL_NEED(cap >= bytes, "destination too small");
    JL_CUDA(cudaSetDevice(m->device));
    const Mat* mat = nullptr;
    for (const auto& L : m->lw) {
        const Mat* mats[7] = {&L.q, &L.k, &L.v, &L.o, &L.gate, &L.up, &L.down};
        for (const Mat* mt : mats)
            if (mt->data == src) mat = mt;
    }
    if (m->embed.data == src) mat = &m->embed;
    if (m->head.data == src) mat = &m->head;
    if (mat && mat->kind == MAT_MXFP4) {
        const size_t pb = (size_t)mat->rows * mat->cols / 2, sb = (size_t)mat->rows * mat->cols / 32;
        JL_CUDA(cudaMemcpy(dst, mat->data, pb, cudaMemcpyDeviceToHost));
        JL_CUDA(cudaMemcpy((char*)dst + pb, mat->scales, sb, cudaMemcpyDeviceToHost));
        bytes = pb + sb;
    } else {
        JL_CUDA(cudaMemcpy(dst, src, bytes, cudaMemcpyDeviceToHost));
    }
    if (written) *written = bytes;
    return JL_OK;
}

// ---- caches ----------------------------------------------------------------

jl_status jl_cache_create(jl_model* m, jl_cache** out) {
    JL_NEED(m && out, "model and out must be non-null");
    *out = nullptr;
    JL_GUARD({ return cache_create(m, out); })
}

void jl_cache_free(jl_cache* c) { cache_free(c); }

size_t jl_cache_len(const jl_cache* c) { return c ? c->len : 0; }

jl_status jl_cache_truncate(jl_cache* c, size_t len) {
    JL_NEED(c, "cache must be non-null");
    // KvCache::truncate asserts len <= self.len (engine/src/model.rs:46)
    JL_NEED(len <= c->len, "truncate length exceeds the cache length");
    c->len = len;
    return JL_OK;
}

// ---- passes ------------------------------------------------------------------

jl_status jl_predict(jl_model* m, jl_cache* c, const uint32_t* ids, size_t n, int all,
                     uint32_t* out_ids, float* out_logits) {
    JL_NEED(m && c && ids && out_ids, "model, cache, ids and out_ids must be non-null");
    JL_NEED(c->m == m, "this cache belongs to another model");
    JL_GUARD({ return predict(m, c, ids, n, all != 0, out_ids, out_logits); })
}

jl_status jl_predict_draft(jl_model* m, jl_cache* c, const uint32_t* ids, size_t n, uint32_t* out_id,
                           float* out_logits) {
    JL_NEED(m && c && ids && out_id, "model, cache, ids and out_id must be non-null");
    JL_NEED(c->m == m, "this cache belongs to another model");
    JL_NEED(n == 1 || n == 2, "a draft step takes 1 or 2 tokens");
    JL_GUARD({ return predict(m, c, ids, n, false, out_id, out_logits, true); })
}

jl_status jl_next_token(jl_model* m, const uint32_t* ids, size_t n, uint32_t* out_id) {
    JL_NEED(m && ids && out_id, "model, ids and out_id must be non-null");
    JL_GUARD({
        jl_cache* c = nullptr;
        JL_TRY(cache_create(m, &c));
        std::unique_ptr<jl_cache, void (*)(jl_cache*)> guard(c, cache_free);
        return predict(m, c, ids, n, false, out_id, nullptr);
    })
}

jl_status jl_hidden(jl_model* m, const uint32_t* ids, size_t n, size_t layers, float* out) {
    JL_NEED(m && ids && out, "model, ids and out must be non-null");
    JL_GUARD({ return hidden(m, ids, n, layers, out); })
}

// ---- generation ----------------------------------------------------------------

jl_status jl_generate(jl_model* m, const uint32_t* prompt, size_t n, size_t count, uint32_t* out,
                      size_t cap, size_t* out_len) {
    JL_NEED(m && prompt && out && out_len, "model, prompt, out and out_len must be non-null");
    JL_GUARD({ return generate(m, prompt, n, count, out, cap, out_len); })
}

jl_status jl_time_pass(jl_model* m, const uint32_t* prompt, size_t n, size_t rows, size_t reps,
                       double* wall_ms, double* gpu_ms) {
    JL_NEED(m && prompt && wall_ms && gpu_ms, "model, prompt and outputs must be non-null");
    JL_GUARD({ return time_pass(m, prompt, n, rows, reps, wall_ms, gpu_ms); })
}

jl_status jl_project(jl_model* m, int layer, jl_projection which, const float* x, size_t rows,
                     float* y) {
    JL_NEED(m && x && y, "model, x and y must be non-null");
    JL_GUARD({ return project(m, layer, (int)which, x, rows, y); })
}

jl_status jl_time_pass_draft(jl_model* m, const uint32_t* prompt, size_t n, size_t reps,
                             double* wall_ms, double* gpu_ms) {
    JL_NEED(m && prompt && wall_ms && gpu_ms, "model, prompt and outputs must be non-null");
    JL_GUARD({ return time_pass(m, prompt, n, 1, reps, wall_ms, gpu_ms, true); })
}

jl_status jl_pass_kernels(const jl_model* m, size_t rows, int draft_step, size_t* kernels) {
    JL_NEED(m && kernels, "model and output must be non-null");
    JL_NEED(rows >= 1, "a pass has at least one row");
    *kernels = pass_kernels(m, rows, draft_step != 0);
    return JL_OK;
}

jl_status jl_wait_probe(jl_model* m, uint32_t polls) {
    JL_NEED(m, "model must be non-null");
    JL_GUARD({ return wait_probe(m, polls); })
}

jl_status jl_model_prompt_attention(jl_model* m, int tensor_cores, int* active) {
    JL_NEED(m, "model must be non-null");
    JL_NEED(tensor_cores == 0 || tensor_cores == 1, "tensor_cores must be 0 or 1");
    m->prompt_attn_cuda_cores = tensor_cores == 0;
    if (active) *active = prefill_tc_supported(m) ? 1 : 0;
    return JL_OK;
}

jl_status jl_timeline_read(uint64_t* stamps, size_t cap, size_t* launches) {
    static_assert(JL_TIMELINE_CTAS == jl::TL_CTAS && JL_TIMELINE_POINTS == jl::TL_POINTS, "timeline table shape");
    JL_NEED(launches, "launches must be non-null");
    JL_GUARD({ return tl_read(reinterpret_cast<unsigned long long*>(stamps), cap, launches); })
}

const char* jl_timeline_kernel(size_t launch) { return jl::tl_kernel(launch); }

jl_status jl_project_noalloc(jl_model* m, int layer, jl_projection which, const float* x,
                             size_t rows, float* y, void* stream) {
    JL_NEED(m && x && y, "model, x and y must be non-null");
    JL_GUARD({ return project_noalloc(m, layer, (int)which, x, rows, y, (cudaStream_t)stream); })
}

jl_status jl_time_projection(jl_model* m, int layer, jl_projection which, int rows, int iters,
                             double* ms_per_launch, size_t* weight_bytes) {
    JL_NEED(m && ms_per_launch && weight_bytes, "model and outputs must be non-null");
    JL_GUARD({ return time_projection(m, layer, (int)which, rows, iters, ms_per_launch, weight_bytes); })
}

jl_status jl_schedule_fixed(uint32_t gamma, jl_schedule* out) {
    JL_NEED(out, "out must be non-null");
    JL_NEED(gamma > 0, "gamma must be positive");  // scheduler.rs:10
    out->gamma = gamma;
    out->max_gamma = gamma;
    out->adaptive = 0;
    return JL_OK;
}

jl_status jl_schedule_adaptive(uint32_t initial, uint32_t maximum, jl_schedule* out) {
    JL_NEED(out, "out must be non-null");
    // scheduler.rs:19-21
    JL_NEED(initial > 0 && initial <= maximum,
            "adaptive gamma must be positive and no greater than max gamma");
    out->gamma = initial;
    out->max_gamma = maximum;
    out->adaptive = 1;
    return JL_OK;
}

void jl_spec_options_default(jl_spec_options* o) {
    if (!o) return;
    memset(o, 0, sizeof *o);
    o->mode = JL_SPEC_DEVICE;
}

jl_status jl_generate_speculative(jl_model* target, jl_model* draft, const uint32_t* prompt,
                                  size_t n, size_t count, const jl_schedule* schedule,
                                  const jl_spec_options* opts, jl_spec_result* result) {
    JL_NEED(target && draft && prompt && schedule && result && result->tokens,
            "target, draft, prompt, schedule, result and result->tokens must be non-null");
    jl_spec_options o;
    jl_spec_options_default(&o);
    if (opts) o = *opts;
    JL_NEED(o.mode == JL_SPEC_DEVICE || o.mode == JL_SPEC_HOST, "unknown speculative mode");
    JL_NEED(o.oracle_p >= 0.0 && o.oracle_p <= 1.0, "oracle_p must lie in [0, 1]");
    JL_GUARD({ return generate_speculative(target, draft, prompt, n, count, *schedule, o, result); })
}

jl_status jl_generate_batch(jl_model* m, size_t batch, const uint32_t* const* prompts,
                            const size_t* prompt_lens, size_t count, jl_spec_result* results,
                            jl_batch_stats* stats) {
    JL_NEED(m && prompts && prompt_lens && results, "model, prompts, prompt_lens and results must be non-null");
    JL_GUARD({ return generate_batch(m, batch, prompts, prompt_lens, count, results, stats); })
}

jl_status jl_generate_speculative_batch(jl_model* target, jl_model* draft, size_t batch,
                                        const uint32_t* const* prompts, const size_t* prompt_lens,
                                        size_t count, const jl_schedule* schedules,
                                        const jl_spec_options* opts, jl_spec_result* results,
                                        jl_batch_stats* stats) {
    JL_NEED(target && draft && prompts && prompt_lens && schedules && results,
            "target, draft, prompts, prompt_lens, schedules and results must be non-null");
    JL_GUARD({
        return generate_speculative_batch(target, draft, batch, prompts, prompt_lens, count, schedules, opts,
                                          results, stats);
    })
}

}  // extern "C"
