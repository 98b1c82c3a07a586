// Device model construction (GpuModel::new, engine/src/gpu.rs:336-428),
// the paged KV pool and caches (GpuCache, engine/src/gpu.rs:272-300).
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>

#include "jl_internal.h"

namespace jl {

namespace {

constexpr size_t ALIGN = 256;

size_t align_up(size_t n) { return (n + ALIGN - 1) / ALIGN * ALIGN; }

// Tensor layout within the arena, planned before allocation.
struct Plan {
    size_t bytes = 0;
    size_t take(size_t n) {
        size_t at = bytes;
        bytes += align_up(n);
        return at;
    }
};

const char* PROJ_NAMES[7] = {"self_attn.q_proj.weight", "self_attn.k_proj.weight",
                             "self_attn.v_proj.weight", "self_attn.o_proj.weight",
                             "mlp.gate_proj.weight",    "mlp.up_proj.weight",
                             "mlp.down_proj.weight"};
const char* NORM_NAMES[4] = {"input_layernorm.weight", "post_attention_layernorm.weight",
                             "self_attn.q_norm.weight", "self_attn.k_norm.weight"};

Mat* proj_slot(LayerW& L, int i) {
    Mat* m[7] = {&L.q, &L.k, &L.v, &L.o, &L.gate, &L.up, &L.down};
    return m[i];
}
const uint16_t** norm_slot(LayerW& L, int i) {
    const uint16_t** n[4] = {&L.in_ln, &L.post_ln, &L.q_norm, &L.k_norm};
    return n[i];
}

// RoPE angles exactly as engine/src/lib.rs:307-311 computes them in f32:
// freq = 1 / theta^(i / 64), angle = position * freq, then cos and sin.
void rope_table(int positions, std::vector<float2>& out) {
    out.resize((size_t)positions * HALF);
    float freq[HALF];
    for (int i = 0; i < HALF; ++i) freq[i] = 1.0f / powf(1000000.0f, (float)i / (float)HALF);
    for (int p = 0; p < positions; ++p) {
        const float position = (float)p;
        for (int i = 0; i < HALF; ++i) {
            const float angle = position * freq[i];
            out[(size_t)p * HALF + i] = make_float2(cosf(angle), sinf(angle));
        }
    }
}

jl_status check_dims(int layers, int hidden, int q_heads, int kv_heads, int inter, int vocab) {
    if (layers < 1 || hidden <= 0 || q_heads <= 0 || kv_heads <= 0 || inter <= 0 || vocab <= 0) {
        set_error("the GPU engine needs at least one layer and positive dimensions");
        return JL_ERR_INVALID_ARG;
    }
    if (q_heads % kv_heads) {
        set_error("unexpected attention shapes: %d query heads over %d kv heads", q_heads, kv_heads);
        return JL_ERR_FORMAT;
    }
    if (hidden % 32 || inter % 32) {
        set_error("hidden (%d) and intermediate (%d) sizes must be multiples of 32", hidden, inter);
        return JL_ERR_FORMAT;
    }
    return JL_OK;
}

// Allocates everything but the weights: KV pool, scratch, pass buffers, RoPE.
jl_status finish_model(jl_model* m, const jl_model_options& o) {
    JL_CUDA(cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking));
    JL_CUDA(cudaEventCreate(&m->ev0));
    JL_CUDA(cudaEventCreate(&m->ev1));
    // RoPE table for every position the model accepts
    std::vector<float2> rope;
    rope_table(m->max_positions, rope);
    JL_CUDA(cudaMalloc(&m->rope, rope.size() * sizeof(float2)));
    JL_CUDA(cudaMemcpy(m->rope, rope.data(), rope.size() * sizeof(float2), cudaMemcpyHostToDevice));
    // KV pool
    m->kv.dtype = o.kv_dtype;
    m->kv.elem = o.kv_dtype == JL_KV_F32 ? 4 : 2;
    size_t tokens = o.kv_pool_tokens ? o.kv_pool_tokens : (size_t)m->max_positions + 1024;
    m->kv.pages = (tokens + PAGE - 1) / PAGE;
    m->kv.page_elems = (size_t)m->kv_heads * PAGE * HEAD;
    const size_t kv_bytes = (size_t)m->layers * 2 * m->kv.pages * m->kv.page_elems * m->kv.elem;
    if (cudaMalloc(&m->kv.base, kv_bytes) != cudaSuccess) {
        cudaGetLastError();
        set_error("cannot allocate a KV pool of %zu bytes (%zu tokens)", kv_bytes, tokens);
        return JL_ERR_OOM;
    }
    JL_TRY(kv_tensor_maps(m));  // the tensor-core prompt attention's TMA view of the pool
    m->kv.free_list.resize(m->kv.pages);
    for (size_t i = 0; i < m->kv.pages; ++i) m->kv.free_list[i] = (int32_t)(m->kv.pages - 1 - i);
    // decode attention over long contexts: the partial sums of up to
    // ATT_ZMAX window CTAs for every row of the largest multi-chunk pass
    m->att_smax = ATT_ZMAX;
    m->att_rows = std::max(SMALL_M, std::min(o.max_pass_rows ? (int)o.max_pass_rows : 4096, SMALL_M * MAX_CHUNKS));
    {
        const size_t group = (size_t)m->q_heads / m->kv_heads;
        const size_t floats = (size_t)m->kv_heads * m->att_rows * m->att_smax * group * ATT_PART;
        if (cudaMalloc(&m->att_ws, floats * sizeof(float)) != cudaSuccess ||
            cudaMalloc(&m->att_cnt, (size_t)m->kv_heads * SMALL_M * MAX_CHUNKS * sizeof(int)) != cudaSuccess) {
            cudaGetLastError();
            set_error("cannot allocate the attention split workspace");
            return JL_ERR_OOM;
        }
        JL_CUDA(cudaMemset(m->att_cnt, 0, (size_t)m->kv_heads * SMALL_M * MAX_CHUNKS * sizeof(int)));
    }
    // scratch
    const int R = m->max_rows = o.max_pass_rows ? (int)o.max_pass_rows : 4096;
    const size_t H = m->hidden, QW = (size_t)m->q_heads * HEAD, KVW = (size_t)m->kv_heads * HEAD;
    Plan sp;
    const size_t off_x = sp.take((size_t)R * H * 4);
    const size_t off_xn = sp.take((size_t)R * std::max(H, QW) * 4);
    const size_t off_qkv = sp.take((size_t)R * (QW + 2 * KVW) * 4);
    const size_t off_attn = sp.take((size_t)R * QW * 4);
    const size_t off_act = sp.take((size_t)R * m->inter * 4);
    const size_t off_xh = sp.take((size_t)R * H * 4);
    const size_t off_logits = sp.take((size_t)R * m->vocab * 4);
    const size_t off_hdr = sp.take(MAX_CHUNKS * sizeof(PassHdr));
    const size_t off_row = sp.take((size_t)R * sizeof(RowDesc));
    const size_t off_head = sp.take((size_t)R * sizeof(int32_t));
    const size_t off_pt = sp.take((size_t)MAX_SEQS * sizeof(int32_t*));
    const size_t off_out = sp.take((size_t)R * sizeof(uint32_t));
    const size_t off_cnt = sp.take(4096 * sizeof(int));
    if (cudaMalloc(&m->scratch_arena, sp.bytes) != cudaSuccess) {
        cudaGetLastError();
        set_error("cannot allocate %zu bytes of pass scratch for %d rows", sp.bytes, R);
        return JL_ERR_OOM;
    }
    JL_CUDA(cudaMemset(m->scratch_arena, 0, sp.bytes));
    char* b = (char*)m->scratch_arena;
    m->s.x = (float*)(b + off_x);
    m->s.xn = (float*)(b + off_xn);
    m->s.qkv = (float*)(b + off_qkv);
    m->s.attn = (float*)(b + off_attn);
    m->s.act = (float*)(b + off_act);
    m->s.xh = (float*)(b + off_xh);
    m->s.logits = (float*)(b + off_logits);
    m->pass.hdr = (PassHdr*)(b + off_hdr);
    m->pass.row = (RowDesc*)(b + off_row);
    m->pass.head_row = (int32_t*)(b + off_head);
    m->pass.page_table = (const int32_t**)(b + off_pt);
    m->pass.out_ids = (uint32_t*)(b + off_out);
    m->counters = (int*)(b + off_cnt);
    // pinned staging for host-driven passes
    for (StageSlot& sl : m->stage) {
        JL_CUDA(cudaMallocHost(&sl.hdr, MAX_CHUNKS * sizeof(PassHdr)));
        JL_CUDA(cudaMallocHost(&sl.row, (size_t)R * sizeof(RowDesc)));
        JL_CUDA(cudaMallocHost(&sl.head_row, (size_t)R * sizeof(int32_t)));
        JL_CUDA(cudaMallocHost(&sl.page_table, (size_t)MAX_SEQS * sizeof(int32_t*)));
        JL_CUDA(cudaEventCreateWithFlags(&sl.done, cudaEventDisableTiming));
    }
    JL_CUDA(cudaMallocHost(&m->host_out, (size_t)R * sizeof(uint32_t)));
    return JL_OK;
}

// Set-up work (weight synthesis and tiling, memsets of the scratch and
// counters) runs on the legacy default stream, which the model's
// non-blocking stream does not wait for: without this, a first pass can
// start while a memset is still clearing its pass descriptors.
jl_status creation_done(jl_model* m) {
    JL_CUDA(cudaSetDevice(m->device));
    JL_CUDA(cudaDeviceSynchronize());
    return JL_OK;
}

jl_status begin_model(const jl_model_options& o, jl_model** out) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
        cudaGetLastError();
        set_error("no CUDA device: this engine has no CPU path");
        return JL_ERR_NO_DEVICE;
    }
    if (o.device < 0 || o.device >= n) {
        set_error("device %d out of range (%d devices)", o.device, n);
        return JL_ERR_INVALID_ARG;
    }
    JL_CUDA(cudaSetDevice(o.device));
    JL_TRY(configure_kernels());
    *out = new jl_model();
    (*out)->device = o.device;
    JL_CUDA(cudaDeviceGetAttribute(&(*out)->sms, cudaDevAttrMultiProcessorCount, o.device));
    return JL_OK;
}

}  // namespace

// Tensor-core copies of the MXFP4 projections: q|k|v stacked, gate/up
// interleaved per 64 rows (the SwiGLU epilogue needs both halves of an
// output in one tile), o, down and an MXFP4 output table.  The row-major
// checkpoint copy stays for the long-prompt kernel.
jl_status build_mx(jl_model* m) {
    auto is_mx = [](const Mat& a) { return a.kind == MAT_MXFP4; };
    bool all = !m->lw.empty();
    for (const auto& L : m->lw)
        all = all && is_mx(L.q) && is_mx(L.k) && is_mx(L.v) && is_mx(L.o) && is_mx(L.gate) &&
              is_mx(L.up) && is_mx(L.down);
    const bool head = is_mx(m->head);
    if (!all && !head) return JL_OK;
    int dev = 0, sms = 148;
    JL_CUDA(cudaGetDevice(&dev));
    JL_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    const int QW = m->q_heads * HEAD, KVW = m->kv_heads * HEAD;
    // fused decode pass: piece images need whole 256-element stages; a bf16
    // output table then also runs on the tensor cores
    const bool fused = all && m->hidden % 256 == 0 && QW % 256 == 0 && m->inter % 256 == 0;
    const bool head_bf = fused && m->head.kind == MAT_BF16;
    Plan plan;
    std::vector<size_t> offs;
    if (all)
        for (size_t l = 0; l < m->lw.size(); ++l) {
            offs.push_back(plan.take(mx_tile_bytes(QW + 2 * KVW, m->hidden, false)));
            offs.push_back(plan.take(mx_tile_bytes(m->hidden, QW, false)));
            offs.push_back(plan.take(mx_tile_bytes(m->inter, m->hidden, true)));
            offs.push_back(plan.take(mx_tile_bytes(m->hidden, m->inter, false)));
        }
    const size_t head_off = head ? plan.take(mx_tile_bytes(m->vocab, m->hidden, false)) : 0;
    const size_t bfh_off = head_bf ? plan.take(bf16_tile_bytes(m->vocab, m->hidden)) : 0;
    if (cudaMalloc(&m->mx.arena, plan.bytes) != cudaSuccess) {
        cudaGetLastError();
        set_error("cannot allocate %zu bytes for tensor-core weight tiles", plan.bytes);
        return JL_ERR_OOM;
    }
    uint8_t* base = (uint8_t*)m->mx.arena;
    int maxS = 1, maxT = 1;
    size_t ws_floats = 1;
    auto track = [&](const MxProj& p) {
        maxS = std::max(maxS, p.S);
        maxT = std::max(maxT, p.T);
        ws_floats = std::max(ws_floats, (size_t)p.T * p.ksplit * mx_max_tokens() * 128);
    };
    if (all)
        for (size_t l = 0; l < m->lw.size(); ++l) {
            LayerW& L = m->lw[l];
            const Mat* qkv[3] = {&L.q, &L.k, &L.v};
            const Mat* o[1] = {&L.o};
            const Mat* gu[2] = {&L.gate, &L.up};
            const Mat* dn[1] = {&L.down};
            JL_TRY(mx_build(qkv, 3, false, base + offs[4 * l], sms, &L.mx_qkv, 0));
            JL_TRY(mx_build(o, 1, false, base + offs[4 * l + 1], sms, &L.mx_o, 0));
            JL_TRY(mx_build(gu, 2, true, base + offs[4 * l + 2], sms, &L.mx_gateup, 0));
            JL_TRY(mx_build(dn, 1, false, base + offs[4 * l + 3], sms, &L.mx_down, 0));
            track(L.mx_qkv);
            track(L.mx_o);
            track(L.mx_gateup);
            track(L.mx_down);
        }
    if (head) {
        const Mat* h[1] = {&m->head};
        JL_TRY(mx_build(h, 1, false, base + head_off, sms, &m->mx_head, 0));
        track(m->mx_head);
    }
    if (head_bf) JL_TRY(mx_build_bf16(m->head, base + bfh_off, &m->bf_head, 0));
    m->dec_ok = dec_supported(m);
    Plan sp;
    // piece images: per 256-element stage, up to 16 rows x 8 pieces x 128
    // bytes of codes, then 1 KB of scale atoms
    const size_t img_stage = (size_t)mx_max_tokens() * 8 * 128 + 1024;
    const size_t off_b = sp.take((size_t)maxS * img_stage);
    const size_t off_ws = sp.take(ws_floats * sizeof(float));
    const size_t off_t = sp.take((size_t)maxT * sizeof(int));
    // fused-pass buffers: one copy per chunk a multi-chunk pass may hold
    const int C = fused ? std::max(1, std::min(MAX_CHUNKS, m->max_rows / SMALL_M)) : 1;
    MxBuffers& X = m->mx;
    X.chunks = C;
    X.sx = (size_t)(m->hidden / 256) * img_stage;
    X.sattn = (size_t)(QW / 256) * img_stage;
    X.sact = (size_t)(m->inter / 256) * img_stage;
    X.spart = (size_t)(m->hidden / 128) * MX_PART_STRIDE;
    X.shead = (size_t)(m->hidden / 64) * (4 * mx_max_tokens()) * 128;
    X.samax = head_bf ? (size_t)m->bf_head.T * MX_PART_STRIDE : 0;
    size_t off_fx = 0, off_fa = 0, off_ff = 0, off_fp = 0;
    if (fused) {
        off_fx = sp.take(C * X.sx);
        off_fa = sp.take(C * X.sattn);
        off_ff = sp.take(C * X.sact);
        off_fp = sp.take(C * X.spart * sizeof(float));
    }
    size_t off_bh = 0, off_av = 0, off_ai = 0;
    if (head_bf) {
        off_bh = sp.take(C * X.shead);
        off_av = sp.take(C * X.samax * sizeof(float));
        off_ai = sp.take(C * X.samax * sizeof(int));
    }
    if (cudaMalloc(&m->mx.scratch, sp.bytes) != cudaSuccess) {
        cudaGetLastError();
        set_error("cannot allocate tensor-core scratch");
        return JL_ERR_OOM;
    }
    JL_CUDA(cudaMemset(m->mx.scratch, 0, sp.bytes));
    uint8_t* s = (uint8_t*)m->mx.scratch;
    m->mx.bimg = s + off_b;
    m->mx.ws = (float*)(s + off_ws);
    m->mx.tickets = (int*)(s + off_t);
    if (fused) {
        m->mx.fused = true;
        m->mx.bx = s + off_fx;
        m->mx.battn = s + off_fa;
        m->mx.bact = s + off_ff;
        m->mx.part = (float*)(s + off_fp);
    }
    if (head_bf) {
        m->mx.bhead = s + off_bh;
        m->mx.amax_v = (float*)(s + off_av);
        m->mx.amax_i = (int*)(s + off_ai);
    }
    JL_CUDA(cudaDeviceSynchronize());
    return JL_OK;
}

namespace {

static_assert(__BYTE_ORDER__ == __ORDER_LITTLE_ENDIAN__,
              "safetensors BF16 payloads (little-endian u16) are copied to the device as they are");

// Streams checkpoint payloads from their files to device memory through two
// pinned buffers: the read of one chunk overlaps the copy of the other, and
// the host never holds more than two chunks of the checkpoint.
class Stager {
  public:
    static constexpr size_t CHUNK = 16u << 20;

    ~Stager() {
        if (stream_) cudaStreamSynchronize(stream_);
        for (int i = 0; i < 2; ++i) {
            if (ev_[i]) cudaEventDestroy(ev_[i]);
            if (buf_[i]) cudaFreeHost(buf_[i]);
        }
        if (stream_) cudaStreamDestroy(stream_);
    }

    jl_status init() {
        JL_CUDA(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking));
        for (int i = 0; i < 2; ++i) {
            if (cudaHostAlloc(&buf_[i], CHUNK, cudaHostAllocDefault) != cudaSuccess) {
                cudaGetLastError();
                buf_[i] = nullptr;
                set_error("could not allocate %zu bytes of pinned host memory for loading", CHUNK);
                return JL_ERR_OOM;
            }
            JL_CUDA(cudaEventCreateWithFlags(&ev_[i], cudaEventDisableTiming));
        }
        return JL_OK;
    }

    // The bytes of `r` to dst (device memory).
    jl_status file(const FileRange& r, char* dst) {
        for (uint64_t off = 0; off < r.bytes; off += CHUNK) {
            const size_t n = (size_t)std::min<uint64_t>(CHUNK, r.bytes - off);
            const int i = next_;
            next_ ^= 1;
            JL_CUDA(cudaEventSynchronize(ev_[i]));  // the copy out of this buffer is done
            JL_TRY(read_range(r, buf_[i], (size_t)off, n));
            JL_CUDA(cudaMemcpyAsync(dst + off, buf_[i], n, cudaMemcpyHostToDevice, stream_));
            JL_CUDA(cudaEventRecord(ev_[i], stream_));
        }
        return JL_OK;
    }

    // `n` bytes already in host memory (MXFP4 scales) to dst.
    jl_status host(const void* src, size_t n, char* dst) {
        JL_CUDA(cudaMemcpyAsync(dst, src, n, cudaMemcpyHostToDevice, stream_));
        return JL_OK;
    }

    jl_status finish() {
        JL_CUDA(cudaStreamSynchronize(stream_));
        return JL_OK;
    }

  private:
    cudaStream_t stream_ = nullptr;
    void* buf_[2] = {nullptr, nullptr};
    cudaEvent_t ev_[2] = {nullptr, nullptr};
    int next_ = 0;
};

// Whether two tensors hold the same bytes: compared chunk by chunk from the
// files, stopping at the first difference.
jl_status same_payload(const IndexTensor& a, const IndexTensor& b, bool* same) {
    *same = false;
    if (a.dtype != b.dtype || a.shape != b.shape || a.data.bytes != b.data.bytes || a.scales != b.scales)
        return JL_OK;
    constexpr size_t CH = 4u << 20;
    std::vector<uint8_t> x(CH), y(CH);
    for (uint64_t off = 0; off < a.data.bytes; off += CH) {
        const size_t n = (size_t)std::min<uint64_t>(CH, a.data.bytes - off);
        JL_TRY(read_range(a.data, x.data(), (size_t)off, n));
        JL_TRY(read_range(b.data, y.data(), (size_t)off, n));
        if (memcmp(x.data(), y.data(), n) != 0) return JL_OK;
    }
    *same = true;
    return JL_OK;
}

}  // namespace

jl_status model_from_checkpoint(const WeightIndex& w, const HostConfig& cfg, const jl_model_options& o,
                                jl_model** out) {
    auto& T = w.tensors;
    auto find = [&](const std::string& name) -> const IndexTensor* {
        auto it = T.find(name);
        return it == T.end() ? nullptr : &it->second;
    };
    // Shapes (engine/src/gpu.rs:398-406)
    const IndexTensor* embed = find("model.embed_tokens.weight");
    const IndexTensor* q0 = find("model.layers.0.self_attn.q_proj.weight");
    const IndexTensor* k0 = find("model.layers.0.self_attn.k_proj.weight");
    const IndexTensor* g0 = find("model.layers.0.mlp.gate_proj.weight");
    if (!embed || embed->shape.size() != 2) {
        set_error("missing tensor model.embed_tokens.weight");
        return JL_ERR_FORMAT;
    }
    if (cfg.layers < 1 || !q0 || !k0 || !g0) {
        set_error("model has no layers");
        return JL_ERR_FORMAT;
    }
    const int hidden = (int)embed->shape[1];
    const int q_heads = (int)(q0->shape[0] / HEAD), kv_heads = (int)(k0->shape[0] / HEAD);
    const int inter = (int)g0->shape[0];
    const IndexTensor* head = find("lm_head.weight");
    // A head identical to the embedding table is stored once (gpu.rs:340-357).
    bool tied = !head;
    if (head) JL_TRY(same_payload(*head, *embed, &tied));
    const int vocab = (int)(tied ? embed->shape[0] : head->shape[0]);
    if (q0->shape[1] != (size_t)hidden || q0->shape[0] % HEAD || k0->shape[0] % HEAD) {
        set_error("unexpected attention shapes");
        return JL_ERR_FORMAT;
    }
    JL_TRY(check_dims(cfg.layers, hidden, q_heads, kv_heads, inter, vocab));
    if (!tied && head->shape[1] != (size_t)hidden) {
        set_error("lm_head width %zu does not match hidden %d", head->shape[1], hidden);
        return JL_ERR_FORMAT;
    }
    // Collect and check every tensor the pass reads.
    struct Want {
        std::string name;
        size_t rows, cols;  // cols == 0: 1-D norm of `rows` values
        Mat* mat;
        const uint16_t** norm;
    };
    jl_model* m = nullptr;
    JL_TRY(begin_model(o, &m));
    std::unique_ptr<jl_model, void (*)(jl_model*)> guard(m, model_free);
    m->layers = cfg.layers;
    m->hidden = hidden;
    m->q_heads = q_heads;
    m->kv_heads = kv_heads;
    m->inter = inter;
    m->vocab = vocab;
    m->max_positions = cfg.max_positions;
    m->eos = cfg.eos;
    m->tied = tied;
    m->lw.resize(cfg.layers);
    std::vector<Want> wants;
    const size_t QW = (size_t)q_heads * HEAD, KVW = (size_t)kv_heads * HEAD;
    wants.push_back({"model.embed_tokens.weight", (size_t)vocab, (size_t)hidden, &m->embed, nullptr});
    if (!tied) wants.push_back({"lm_head.weight", (size_t)vocab, (size_t)hidden, &m->head, nullptr});
    wants.push_back({"model.norm.weight", (size_t)hidden, 0, nullptr, &m->final_norm});
    for (int l = 0; l < cfg.layers; ++l) {
        const std::string p = "model.layers." + std::to_string(l) + ".";
        const size_t shapes[7][2] = {{QW, (size_t)hidden}, {KVW, (size_t)hidden}, {KVW, (size_t)hidden},
                                     {(size_t)hidden, QW}, {(size_t)inter, (size_t)hidden},
                                     {(size_t)inter, (size_t)hidden}, {(size_t)hidden, (size_t)inter}};
        for (int i = 0; i < 7; ++i)
            wants.push_back({p + PROJ_NAMES[i], shapes[i][0], shapes[i][1], proj_slot(m->lw[l], i), nullptr});
        const size_t nlen[4] = {(size_t)hidden, (size_t)hidden, (size_t)HEAD, (size_t)HEAD};
        for (int i = 0; i < 4; ++i)
            wants.push_back({p + NORM_NAMES[i], nlen[i], 0, nullptr, norm_slot(m->lw[l], i)});
    }
    Plan plan;
    std::vector<size_t> offs(wants.size()), offs2(wants.size());
    for (size_t i = 0; i < wants.size(); ++i) {
        auto& wt = wants[i];
        const IndexTensor* t = find(wt.name);
        if (!t) {
            set_error("missing tensor %s", wt.name.c_str());
            return JL_ERR_FORMAT;
        }
        if (wt.cols == 0) {
            if (t->dtype != JL_BF16 || t->shape.size() != 1 || t->shape[0] != wt.rows) {
                set_error("expected a bf16 norm weight: %s", wt.name.c_str());
                return JL_ERR_FORMAT;
            }
            offs[i] = plan.take(wt.rows * 2);
            continue;
        }
        if (t->shape.size() != 2 || t->shape[0] != wt.rows || t->shape[1] != wt.cols) {
            set_error("unexpected shape for %s", wt.name.c_str());
            return JL_ERR_FORMAT;
        }
        if (t->dtype == JL_MXFP4) {
            offs[i] = plan.take(wt.rows * wt.cols / 2);
            offs2[i] = plan.take(wt.rows * wt.cols / 32);
        } else {
            offs[i] = plan.take(wt.rows * wt.cols * 2);
        }
    }
    if (cudaMalloc(&m->arena, plan.bytes) != cudaSuccess) {
        cudaGetLastError();
        set_error("could not allocate %zu bytes of GPU memory for weights", plan.bytes);
        return JL_ERR_OOM;
    }
    m->arena_bytes = plan.bytes;
    char* base = (char*)m->arena;
    // Payloads go from the files straight to the arena (engine/src/gpu.rs:359-375
    // uploads each tensor once from host memory).
    Stager st;
    JL_TRY(st.init());
    for (size_t i = 0; i < wants.size(); ++i) {
        auto& wt = wants[i];
        const IndexTensor* t = find(wt.name);
        JL_TRY(st.file(t->data, base + offs[i]));
        if (wt.cols == 0) {
            *wt.norm = (const uint16_t*)(base + offs[i]);
            m->tensor_index[wt.name] = {base + offs[i], wt.rows * 2};
            continue;
        }
        Mat& mat = *wt.mat;
        mat.rows = (int)wt.rows;
        mat.cols = (int)wt.cols;
        mat.data = base + offs[i];
        if (t->dtype == JL_MXFP4) {
            mat.kind = MAT_MXFP4;
            JL_TRY(st.host(t->scales.data(), t->scales.size(), base + offs2[i]));
            mat.scales = (const uint8_t*)(base + offs2[i]);
        } else {
            mat.kind = MAT_BF16;
        }
        m->tensor_index[wt.name] = {mat.data, mat.bytes()};
    }
    JL_TRY(st.finish());
    if (tied) m->head = m->embed;
    JL_TRY(finish_model(m, o));
    JL_TRY(build_mx(m));
    JL_TRY(creation_done(m));
    *out = guard.release();
    return JL_OK;
}

jl_status model_synthesize(const jl_synth_config& c, const jl_model_options& o, jl_model** out) {
    JL_TRY(check_dims(c.layers, c.hidden, c.q_heads, c.kv_heads, c.inter, c.vocab));
    if (c.max_positions <= 0) {
        set_error("max_positions must be positive");
        return JL_ERR_INVALID_ARG;
    }
    jl_model* m = nullptr;
    JL_TRY(begin_model(o, &m));
    std::unique_ptr<jl_model, void (*)(jl_model*)> guard(m, model_free);
    m->layers = c.layers;
    m->hidden = c.hidden;
    m->q_heads = c.q_heads;
    m->kv_heads = c.kv_heads;
    m->inter = c.inter;
    m->vocab = c.vocab;
    m->max_positions = c.max_positions;
    m->eos = c.eos;
    m->tied = c.tied != 0;
    m->lw.resize(c.layers);
    const size_t H = c.hidden, QW = (size_t)c.q_heads * HEAD, KVW = (size_t)c.kv_heads * HEAD;
    // Tensor order of the seeded stream: embed, per layer (q, k, v, o, q_norm,
    // k_norm, gate, up, down, input_ln, post_ln), final norm, lm_head.
    struct Item {
        std::string name;
        uint32_t index;
        size_t rows, cols;
        bool quant;
        Mat* mat;
        const uint16_t** norm;
        size_t off = 0, off2 = 0;
    };
    std::vector<Item> items;
    items.push_back({"model.embed_tokens.weight", 0, (size_t)c.vocab, H, c.mxfp4_embed != 0, &m->embed, nullptr});
    const char* order[11] = {"q", "k", "v", "o", "q_norm", "k_norm", "gate", "up", "down", "in", "post"};
    for (int l = 0; l < c.layers; ++l) {
        const std::string p = "model.layers." + std::to_string(l) + ".";
        LayerW& L = m->lw[l];
        for (int j = 0; j < 11; ++j) {
            const uint32_t idx = 1 + 11 * (uint32_t)l + (uint32_t)j;
            const std::string key = order[j];
            if (key == "q") items.push_back({p + PROJ_NAMES[0], idx, QW, H, c.mxfp4 != 0, &L.q, nullptr});
            if (key == "k") items.push_back({p + PROJ_NAMES[1], idx, KVW, H, c.mxfp4 != 0, &L.k, nullptr});
            if (key == "v") items.push_back({p + PROJ_NAMES[2], idx, KVW, H, c.mxfp4 != 0, &L.v, nullptr});
            if (key == "o") items.push_back({p + PROJ_NAMES[3], idx, H, QW, c.mxfp4 != 0, &L.o, nullptr});
            if (key == "q_norm") items.push_back({p + NORM_NAMES[2], idx, (size_t)HEAD, 0, false, nullptr, &L.q_norm});
            if (key == "k_norm") items.push_back({p + NORM_NAMES[3], idx, (size_t)HEAD, 0, false, nullptr, &L.k_norm});
            if (key == "gate") items.push_back({p + PROJ_NAMES[4], idx, (size_t)c.inter, H, c.mxfp4 != 0, &L.gate, nullptr});
            if (key == "up") items.push_back({p + PROJ_NAMES[5], idx, (size_t)c.inter, H, c.mxfp4 != 0, &L.up, nullptr});
            if (key == "down") items.push_back({p + PROJ_NAMES[6], idx, H, (size_t)c.inter, c.mxfp4 != 0, &L.down, nullptr});
            if (key == "in") items.push_back({p + NORM_NAMES[0], idx, H, 0, false, nullptr, &L.in_ln});
            if (key == "post") items.push_back({p + NORM_NAMES[1], idx, H, 0, false, nullptr, &L.post_ln});
        }
    }
    items.push_back({"model.norm.weight", 1 + 11 * (uint32_t)c.layers, H, 0, false, nullptr, &m->final_norm});
    if (!c.tied)
        items.push_back({"lm_head.weight", 2 + 11 * (uint32_t)c.layers, (size_t)c.vocab, H,
                         c.mxfp4_embed != 0, &m->head, nullptr});
    Plan plan;
    size_t tmp_elems = 0;
    for (auto& it : items) {
        if (it.cols == 0) {
            it.off = plan.take(it.rows * 2);
        } else if (it.quant) {
            if (it.cols % 32) {
                set_error("MXFP4 requires a width divisible by 32: %s", it.name.c_str());
                return JL_ERR_INVALID_ARG;
            }
            it.off = plan.take(it.rows * it.cols / 2);
            it.off2 = plan.take(it.rows * it.cols / 32);
            tmp_elems = std::max(tmp_elems, it.rows * it.cols);
        } else {
            it.off = plan.take(it.rows * it.cols * 2);
        }
    }
    if (cudaMalloc(&m->arena, plan.bytes) != cudaSuccess) {
        cudaGetLastError();
        set_error("could not allocate %zu bytes of GPU memory for weights", plan.bytes);
        return JL_ERR_OOM;
    }
    m->arena_bytes = plan.bytes;
    uint16_t* tmp = nullptr;
    if (tmp_elems && cudaMalloc(&tmp, tmp_elems * 2) != cudaSuccess) {
        cudaGetLastError();
        set_error("could not allocate quantization staging");
        return JL_ERR_OOM;
    }
    char* base = (char*)m->arena;
    jl_status st = JL_OK;
    for (auto& it : items) {
        if (it.cols == 0) {
            // norm gains are exactly 1.0
            st = launch_fill_u16((uint16_t*)(base + it.off), it.rows, 0x3F80, 0);
            *it.norm = (const uint16_t*)(base + it.off);
            m->tensor_index[it.name] = {base + it.off, it.rows * 2};
        } else if (it.quant) {
            st = launch_synth_bf16(c.seed, it.index, it.rows * it.cols, tmp, 0);
            if (st == JL_OK)
                st = launch_quantize_mxfp4(tmp, (int)it.rows, (int)it.cols, (uint8_t*)(base + it.off),
                                           (uint8_t*)(base + it.off2), 0);
            it.mat->kind = MAT_MXFP4;
            it.mat->rows = (int)it.rows;
            it.mat->cols = (int)it.cols;
            it.mat->data = base + it.off;
            it.mat->scales = (const uint8_t*)(base + it.off2);
            m->tensor_index[it.name] = {it.mat->data, it.mat->bytes()};
        } else {
            st = launch_synth_bf16(c.seed, it.index, it.rows * it.cols, (uint16_t*)(base + it.off), 0);
            it.mat->kind = MAT_BF16;
            it.mat->rows = (int)it.rows;
            it.mat->cols = (int)it.cols;
            it.mat->data = base + it.off;
            m->tensor_index[it.name] = {it.mat->data, it.mat->bytes()};
        }
        if (st != JL_OK) break;
    }
    cudaError_t e = cudaDeviceSynchronize();
    if (tmp) cudaFree(tmp);
    if (st != JL_OK) return st;
    if (e != cudaSuccess) return cuda_fail(e, "weight synthesis", __FILE__, __LINE__);
    if (c.tied) m->head = m->embed;
    JL_TRY(finish_model(m, o));
    JL_TRY(build_mx(m));
    JL_TRY(creation_done(m));
    *out = guard.release();
    return JL_OK;
}

void model_free(jl_model* m) {
    if (!m) return;
    cudaSetDevice(m->device);
    if (m->stream) cudaStreamSynchronize(m->stream);
    for (auto* g : m->spec_graphs) spec_graph_free(g);
    m->spec_graphs.clear();
    for (auto* g : m->batch_graphs) batch_graph_free(g);
    m->batch_graphs.clear();
    // caches may outlive their model (a garbage collector frees both in any
    // order): they keep their own page tables and forget the model
    for (jl_cache* c : m->caches) c->m = nullptr;
    m->caches.clear();
    for (auto& g : m->small_graph)
        if (g) cudaGraphExecDestroy(g);
    for (auto& g : m->draft_graph)
        if (g) cudaGraphExecDestroy(g);
    cudaFree(m->arena);
    cudaFree(m->rope);
    cudaFree(m->kv.base);
    cudaFree(m->scratch_arena);
    cudaFree(m->mx.arena);
    cudaFree(m->mx.scratch);
    cudaFree(m->att_ws);
    cudaFree(m->att_cnt);
    for (StageSlot& sl : m->stage) {
        if (sl.done) cudaEventDestroy(sl.done);
        cudaFreeHost(sl.hdr);
        cudaFreeHost(sl.row);
        cudaFreeHost(sl.head_row);
        cudaFreeHost((void*)sl.page_table);
    }
    cudaFreeHost(m->host_out);
    cudaFreeHost(m->host_logits);
    if (m->ev0) cudaEventDestroy(m->ev0);
    if (m->ev1) cudaEventDestroy(m->ev1);
    if (m->stream) cudaStreamDestroy(m->stream);
    cudaGetLastError();
    delete m;
}

jl_status cache_create(jl_model* m, jl_cache** out) {
    JL_CUDA(cudaSetDevice(m->device));
    jl_cache* c = new jl_cache();
    c->m = m;
    c->max_pages = ((size_t)m->max_positions + 2 * MAX_GAMMA + PAGE - 1) / PAGE;
    cudaError_t e1 = cudaMalloc(&c->d_pages, c->max_pages * sizeof(int32_t));
    cudaError_t e2 = cudaMallocHost(&c->h_pages, c->max_pages * sizeof(int32_t));
    if (e1 != cudaSuccess || e2 != cudaSuccess) {
        cudaGetLastError();
        cache_free(c);
        set_error("cannot allocate a page table");
        return JL_ERR_OOM;
    }
    m->caches.push_back(c);
    *out = c;
    return JL_OK;
}

void cache_free(jl_cache* c) {
    if (!c) return;
    if (c->m) {
        jl_model* m = c->m;
        cudaSetDevice(m->device);
        if (m->stream) cudaStreamSynchronize(m->stream);
        for (int32_t p : c->pages) m->kv.free_list.push_back(p);
        m->caches.erase(std::remove(m->caches.begin(), m->caches.end(), c), m->caches.end());
    }
    cudaFree(c->d_pages);
    cudaFreeHost(c->h_pages);
    cudaGetLastError();
    delete c;
}

// Makes sure pages exist for positions [0, tokens).  New page-table entries
// are copied to the device on `stream`, ahead of the pass that uses them.
jl_status cache_reserve(jl_cache* c, size_t tokens, cudaStream_t stream) {
    const size_t need = (tokens + PAGE - 1) / PAGE;
    if (need <= c->pages.size()) return JL_OK;
    if (need > c->max_pages) {
        set_error("sequence of %zu tokens exceeds the context limit", tokens);
        return JL_ERR_INVALID_ARG;
    }
    auto& fl = c->m->kv.free_list;
    if (need - c->pages.size() > fl.size()) {
        set_error("KV pool exhausted: need %zu more pages, %zu free (raise kv_pool_tokens)",
                  need - c->pages.size(), fl.size());
        return JL_ERR_OOM;
    }
    const size_t first = c->pages.size();
    while (c->pages.size() < need) {
        c->h_pages[c->pages.size()] = fl.back();
        c->pages.push_back(fl.back());
        fl.pop_back();
    }
    JL_CUDA(cudaMemcpyAsync(c->d_pages + first, c->h_pages + first, (need - first) * sizeof(int32_t),
                            cudaMemcpyHostToDevice, stream));
    return JL_OK;
}

}  // namespace jl
