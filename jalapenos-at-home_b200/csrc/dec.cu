// Draft-step projections on CUDA cores: passes of one or two rows.
//
// A draft model's proposal step is one token through every layer.  With so
// little arithmetic, what a projection costs is latency: the tensor-core
// path (activation pieces, TMEM, split-K reduction, the next projection's
// pieces) takes several round trips after its inputs are ready.  These
// kernels take almost none: each CTA owns a tile of weight rows and copies
// them (MXFP4 codes and scales, exactly as the checkpoint stores them) into
// shared memory with bulk copies BEFORE it waits for the previous kernel
// (weights never depend on it).  After the wait it loads the f32 input rows,
// normalises them (the same arithmetic as k_rmsnorm), and each warp computes
// its rows' dot products: lanes take 32-element blocks, decode E2M1 pairs in
// hardware (cvt.rn.f16x2.e2m1x2), apply the block's E8M0 scale, and the warp
// sums.  Epilogues: q|k|v (QK-RMSNorm, RoPE, K/V appended to the cache),
// residual add, SwiGLU (lib.rs:337-468).
//
// The rounding differs from the tensor-core path, so a model runs these
// kernels only as the draft of a speculative loop: the draft's proposals are
// checked by the target, whose passes all take one path.
#include <cuda_runtime.h>

#include <algorithm>

#include "jl_internal.h"
#include "kernels.cuh"
#include "launch.cuh"
#include "mx_pieces.cuh"
#include "ptx.cuh"

namespace jl {

namespace {

constexpr int DEC_MAXROWS = 2;
constexpr uint32_t DEC_WAIT = 1u << 22;  // polls before the weight copy reports failure

// One weight tile: `rows` rows of an MXFP4 matrix of width K starting at row r0.
struct DecTile {
    const uint8_t* packed;   // matrix codes, row-major [rows][K/2]
    const uint8_t* scales;   // matrix scales, [rows][K/32]
};

// x chunk c (4 floats) of row m lives at xs4[m * K4 + swz(c)]: lanes reading
// chunk i of 32-element blocks b, b+1, ... hit distinct banks.
__device__ __forceinline__ int dec_swz(int c) { return c ^ ((c >> 3) & 7); }

// Copies rows [r0, r0 + n) of a tile's codes and scales to shared memory.
__device__ __forceinline__ void dec_copy_rows(const DecTile& t, int r0, int n, int K, uint8_t* wdst,
                                              uint8_t* sdst, uint64_t* bar) {
    const uint32_t wb = (uint32_t)n * (K / 2), sb = (uint32_t)n * (K / 32);
    ptx::bulk_g2s(wdst, t.packed + (size_t)r0 * (K / 2), wb, bar);
    ptx::bulk_g2s(sdst, t.scales + (size_t)r0 * (K / 32), sb, bar);
}

// Loads M input rows (f32, width K) into shared memory in the swizzled chunk
// layout; with `w` set, as the RMSNorm x / sqrt(mean(x^2) + 1e-6) * w
// (lib.rs:268-290, the arithmetic of k_rmsnorm).  Whole CTA.
__device__ __forceinline__ void dec_load_x(const float* __restrict__ x, int ldx, int M, int K,
                                           const uint16_t* __restrict__ w, float4* xs4, float* red) {
    const int K4 = K / 4;
    for (int m = 0; m < M; ++m) {
        const float* xr = x + (size_t)m * ldx;
        float size = 1.f;
        if (w) {
            float ss = 0.f;
            for (int j = threadIdx.x; j < K; j += blockDim.x) ss = fmaf(xr[j], xr[j], ss);
            ss = block_sum(ss, red);
            size = sqrtf(__fadd_rn(__fdiv_rn(ss, (float)K), 1e-6f));
        }
        for (int c = threadIdx.x; c < K4; c += blockDim.x) {
            float4 v = reinterpret_cast<const float4*>(xr)[c];
            if (w) {
                const uint2 wv = *reinterpret_cast<const uint2*>(w + 4 * c);
                v.x = __fmul_rn(__fdiv_rn(v.x, size), bf16f(wv.x & 0xffffu));
                v.y = __fmul_rn(__fdiv_rn(v.y, size), bf16f(wv.x >> 16));
                v.z = __fmul_rn(__fdiv_rn(v.z, size), bf16f(wv.y & 0xffffu));
                v.w = __fmul_rn(__fdiv_rn(v.w, size), bf16f(wv.y >> 16));
            }
            xs4[m * K4 + dec_swz(c)] = v;
        }
    }
}

// Dot products of one weight row (codes `wr`, scales `sr`, width K) with the
// M staged input rows; every lane gets the totals.  Whole warp.
template <int M>
__device__ __forceinline__ void dec_dot(const uint8_t* wr, const uint8_t* sr, int K, const float4* xs4,
                                        int lane, float (&out)[M]) {
    const int nb = K / 32, K4 = K / 4;
    float acc[M];
#pragma unroll
    for (int m = 0; m < M; ++m) acc[m] = 0.f;
    for (int b = lane; b < nb; b += 32) {
        const uint4 w = *reinterpret_cast<const uint4*>(wr + (size_t)b * 16);
        const float sc = e8m0(sr[b]);
        const uint32_t words[4] = {w.x, w.y, w.z, w.w};
        float part[M];
#pragma unroll
        for (int m = 0; m < M; ++m) part[m] = 0.f;
#pragma unroll
        for (int q = 0; q < 4; ++q) {  // 8 codes = 8 elements per word
            const float2 l01 = mx::e2m1x2_levels(words[q] & 0xffu);
            const float2 l23 = mx::e2m1x2_levels((words[q] >> 8) & 0xffu);
            const float2 l45 = mx::e2m1x2_levels((words[q] >> 16) & 0xffu);
            const float2 l67 = mx::e2m1x2_levels(words[q] >> 24);
#pragma unroll
            for (int m = 0; m < M; ++m) {
                const float4 xa = xs4[m * K4 + dec_swz(b * 8 + 2 * q)];
                const float4 xb = xs4[m * K4 + dec_swz(b * 8 + 2 * q + 1)];
                float p = part[m];
                p = fmaf(l01.x, xa.x, p);
                p = fmaf(l01.y, xa.y, p);
                p = fmaf(l23.x, xa.z, p);
                p = fmaf(l23.y, xa.w, p);
                p = fmaf(l45.x, xb.x, p);
                p = fmaf(l45.y, xb.y, p);
                p = fmaf(l67.x, xb.z, p);
                p = fmaf(l67.y, xb.w, p);
                part[m] = p;
            }
        }
#pragma unroll
        for (int m = 0; m < M; ++m) acc[m] = fmaf(part[m], sc, acc[m]);
    }
#pragma unroll
    for (int m = 0; m < M; ++m) out[m] = warp_sum(acc[m]);
}

// ---------------------------------------------------------------------------
// q|k|v: CTA = one head (128 rows of q, k or v), 16 warps x 8 rows.

struct DecQkvArgs {
    DecTile q, k, v;
    int K, q_heads, kv_heads;
    const float* x;          // residual stream [rows][K]
    const uint16_t* norm;    // input_layernorm
    const uint16_t* qn;      // q_norm / k_norm
    const uint16_t* kn;
    const float2* rope;
    PassBuf pb;
    KvView kv;
    float* q_out;            // [rows][ld]
    int ld;
    int mcap;
};

template <int M>
__global__ void __launch_bounds__(512) k_dec_qkv(DecQkvArgs a) {
    extern __shared__ __align__(128) uint8_t dsm[];
    __shared__ uint64_t bar;
    __shared__ float red[32];
    __shared__ float res[DEC_MAXROWS][HEAD];
    const int h = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int K = a.K;
    const bool is_q = h < a.q_heads, is_k = !is_q && h < a.q_heads + a.kv_heads;
    const int kvh = is_k ? h - a.q_heads : h - a.q_heads - a.kv_heads;
    const DecTile& t = is_q ? a.q : (is_k ? a.k : a.v);
    const int r0 = is_q ? h * HEAD : kvh * HEAD;
    uint8_t* wsm = dsm;
    uint8_t* ssm = dsm + HEAD * (K / 2);
    float4* xs4 = reinterpret_cast<float4*>(ssm + HEAD * (K / 32));
    if (threadIdx.x == 0) {
        ptx::mbar_init(&bar, 1);
        ptx::fence_barrier_init();
        ptx::mbar_arrive_expect_tx(&bar, (uint32_t)(HEAD * (K / 2) + HEAD * (K / 32)));
        dec_copy_rows(t, r0, HEAD, K, wsm, ssm, &bar);
    }
    __syncthreads();  // the barrier is initialised before anyone waits on it
    ptx::grid_dependency_wait();
    ptx::launch_dependents();
    const int rows = min(a.pb.hdr->rows, a.mcap);
    // warp m finishes row m: its position, RoPE factors and cache page are
    // fetched now, while the input loads and the dot products run
    RowDesc rd = {};
    float2 c0 = make_float2(1.f, 0.f), c1 = make_float2(1.f, 0.f);
    int page = -1;
    bool row_ok = false;
    if (warp < M && warp < rows) {
        rd = a.pb.row[warp];
        row_ok = rd.pos >= 0 && rd.pos < a.kv.max_pos && (unsigned)rd.seq < (unsigned)MAX_SEQS;
        if (row_ok) {
            c0 = a.rope[(size_t)rd.pos * HALF + lane];
            c1 = a.rope[(size_t)rd.pos * HALF + lane + 32];
            if (!is_q) page = a.pb.page_table[rd.seq][rd.pos / PAGE];
        }
    }
    dec_load_x(a.x, K, M, K, a.norm, xs4, red);
    const bool ok = ptx::mbar_wait(&bar, 0, DEC_WAIT);
    __syncthreads();
    if (!ok) {
        if (threadIdx.x == 0) atomicOr(a.kv.err, 4);
        return;
    }
    for (int i = 0; i < HEAD / 16; ++i) {
        const int r = warp * (HEAD / 16) + i;
        float o[M];
        dec_dot<M>(wsm + (size_t)r * (K / 2), ssm + (size_t)r * (K / 32), K, xs4, lane, o);
        if (lane == 0)
#pragma unroll
            for (int m = 0; m < M; ++m) res[m][r] = o[m];
    }
    __syncthreads();
    // warp m finishes row m, as k_qk_rope_kv does: lane owns dims l, l+32, l+64, l+96
    if (warp >= M || warp >= rows) return;
    const int m = warp;
    float a0 = res[m][lane], a1 = res[m][lane + 32], a2 = res[m][lane + 64], a3 = res[m][lane + 96];
    if (!row_ok) {
        if (lane == 0) atomicOr(a.kv.err, 2);
        return;
    }
    if (is_q || is_k) {
        const uint16_t* gw = is_q ? a.qn : a.kn;
        float ss = fmaf(a0, a0, fmaf(a1, a1, fmaf(a2, a2, a3 * a3)));
        ss = warp_sum(ss);
        const float size = sqrtf(__fadd_rn(__fdiv_rn(ss, 128.0f), 1e-6f));
        a0 = __fmul_rn(__fdiv_rn(a0, size), bf16f(gw[lane]));
        a1 = __fmul_rn(__fdiv_rn(a1, size), bf16f(gw[lane + 32]));
        a2 = __fmul_rn(__fdiv_rn(a2, size), bf16f(gw[lane + 64]));
        a3 = __fmul_rn(__fdiv_rn(a3, size), bf16f(gw[lane + 96]));
        // lib.rs:306-313: out[i] = a cos - b sin; out[i+64] = b cos + a sin
        const float b0 = __fsub_rn(__fmul_rn(a0, c0.x), __fmul_rn(a2, c0.y));
        const float b2 = __fadd_rn(__fmul_rn(a2, c0.x), __fmul_rn(a0, c0.y));
        const float b1 = __fsub_rn(__fmul_rn(a1, c1.x), __fmul_rn(a3, c1.y));
        const float b3 = __fadd_rn(__fmul_rn(a3, c1.x), __fmul_rn(a1, c1.y));
        a0 = b0; a1 = b1; a2 = b2; a3 = b3;
    }
    if (is_q) {
        float* d = a.q_out + (size_t)m * a.ld + h * HEAD;
        d[lane] = a0; d[lane + 32] = a1; d[lane + 64] = a2; d[lane + 96] = a3;
        return;
    }
    if (!page_ok(a.kv, page)) return;
    const size_t idx = kv_index(page, kvh, rd.pos % PAGE, a.kv.kv_heads);
    if (a.kv.f32) {
        float* d = (float*)(is_k ? a.kv.k : a.kv.v) + idx;
        d[lane] = a0; d[lane + 32] = a1; d[lane + 64] = a2; d[lane + 96] = a3;
    } else {
        uint16_t* d = (uint16_t*)(is_k ? a.kv.k : a.kv.v) + idx;
        d[lane] = f2bf16(a0); d[lane + 32] = f2bf16(a1);
        d[lane + 64] = f2bf16(a2); d[lane + 96] = f2bf16(a3);
    }
}

// ---------------------------------------------------------------------------
// residual add (o, down) and SwiGLU (gate/up): CTA = DEC_TR output rows
// (SwiGLU: DEC_TR gate rows and the matching up rows), 8 warps.

constexpr int DEC_TR = 32;

struct DecArgs {
    DecTile w0, w1;          // the matrix (SwiGLU: gate, up)
    int K, out_rows;
    const float* x;          // input rows [rows][K]
    const uint16_t* norm;    // RMSNorm weight applied to x first, or null
    float* y;                // output rows [rows][ldy]
    int ldy;
    const PassHdr* hdr;
    int mcap;
    int* err;
};

template <int M, bool SWIGLU>
__global__ void __launch_bounds__(256) k_dec_proj(DecArgs a) {
    extern __shared__ __align__(128) uint8_t dsm[];
    __shared__ uint64_t bar;
    __shared__ float red[32];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int K = a.K;
    const int r0 = blockIdx.x * DEC_TR;
    const int n = min(DEC_TR, a.out_rows - r0);
    const int nm = SWIGLU ? 2 : 1;
    uint8_t* wsm = dsm;                                   // [nm][DEC_TR][K/2]
    uint8_t* ssm = dsm + nm * DEC_TR * (K / 2);           // [nm][DEC_TR][K/32]
    float4* xs4 = reinterpret_cast<float4*>(ssm + nm * DEC_TR * (K / 32));
    if (threadIdx.x == 0) {
        ptx::mbar_init(&bar, 1);
        ptx::fence_barrier_init();
        ptx::mbar_arrive_expect_tx(&bar, (uint32_t)(nm * n * (K / 2 + K / 32)));
        dec_copy_rows(a.w0, r0, n, K, wsm, ssm, &bar);
        if (SWIGLU)
            dec_copy_rows(a.w1, r0, n, K, wsm + DEC_TR * (K / 2), ssm + DEC_TR * (K / 32), &bar);
    }
    __syncthreads();  // the barrier is initialised before anyone waits on it
    ptx::grid_dependency_wait();
    ptx::launch_dependents();
    const int rows = min(a.hdr->rows, a.mcap);
    dec_load_x(a.x, K, M, K, a.norm, xs4, red);
    const bool ok = ptx::mbar_wait(&bar, 0, DEC_WAIT);
    __syncthreads();
    if (!ok) {
        if (threadIdx.x == 0) atomicOr(a.err, 4);
        return;
    }
    for (int r = warp; r < n; r += 8) {
        float o[M];
        dec_dot<M>(wsm + (size_t)r * (K / 2), ssm + (size_t)r * (K / 32), K, xs4, lane, o);
        if (SWIGLU) {
            float u[M];
            dec_dot<M>(wsm + (size_t)(DEC_TR + r) * (K / 2), ssm + (size_t)(DEC_TR + r) * (K / 32), K, xs4,
                       lane, u);
            if (lane == 0)
#pragma unroll
                for (int m = 0; m < M; ++m)  // lib.rs:459-463
                    if (m < rows)
                        a.y[(size_t)m * a.ldy + r0 + r] =
                            __fmul_rn(__fdiv_rn(o[m], __fadd_rn(1.0f, expf(-o[m]))), u[m]);
        } else if (lane == 0) {
#pragma unroll
            for (int m = 0; m < M; ++m)
                if (m < rows) {
                    float* d = a.y + (size_t)m * a.ldy + r0 + r;
                    *d = __fadd_rn(*d, o[m]);  // residual (model.rs:178-186)
                }
        }
    }
}

template <int M, bool SWIGLU>
jl_status configure_dec_proj(int smem) {
    JL_CUDA(cudaFuncSetAttribute(k_dec_proj<M, SWIGLU>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    return JL_OK;
}

size_t dec_proj_smem(int K, bool swiglu) {
    const int nm = swiglu ? 2 : 1;
    return (size_t)nm * DEC_TR * (K / 2 + K / 32) + (size_t)DEC_MAXROWS * K * 4;
}

size_t dec_qkv_smem(int K) { return (size_t)HEAD * (K / 2 + K / 32) + (size_t)DEC_MAXROWS * K * 4; }

DecTile tile_of(const Mat& w) { return DecTile{(const uint8_t*)w.data, w.scales}; }

}  // namespace

bool dec_supported(const jl_model* m) {
    if (m->lw.empty()) return false;
    const int QW = m->q_heads * HEAD;
    auto ok = [](int K) { return K % 512 == 0; };  // scale rows of whole 16-byte words
    for (const auto& L : m->lw)
        if (L.q.kind != MAT_MXFP4 || L.k.kind != MAT_MXFP4 || L.v.kind != MAT_MXFP4 || L.o.kind != MAT_MXFP4 ||
            L.gate.kind != MAT_MXFP4 || L.up.kind != MAT_MXFP4 || L.down.kind != MAT_MXFP4)
            return false;
    return ok(m->hidden) && ok(QW) && ok(m->inter) && dec_qkv_smem(m->hidden) <= 200 * 1024 &&
           dec_proj_smem(std::max(m->hidden, std::max(QW, m->inter)), true) <= 200 * 1024 &&
           m->q_heads / m->kv_heads <= 8;
}

constexpr int DEC_SMEM_MAX = 200 * 1024;  // dec_supported keeps every launch under this

jl_status dec_configure() {
    const int proj = DEC_SMEM_MAX;
    JL_TRY((configure_dec_proj<1, false>(proj)));
    JL_TRY((configure_dec_proj<2, false>(proj)));
    JL_TRY((configure_dec_proj<1, true>(proj)));
    JL_TRY((configure_dec_proj<2, true>(proj)));
    const int qkv = DEC_SMEM_MAX;
    JL_CUDA(cudaFuncSetAttribute(k_dec_qkv<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, qkv));
    JL_CUDA(cudaFuncSetAttribute(k_dec_qkv<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, qkv));
    return JL_OK;
}

// The draft-step pass: embedding, then per layer q|k|v, attention, o, gate/up
// and down on CUDA cores (attention as in the decode pass).
jl_status record_dec_pass(const PassCtx& c, int layers) {
    const jl_model* m = c.m;
    const int M = c.rows_cap;
    if (M < 1 || M > DEC_MAXROWS) {
        set_error("draft-step pass takes 1..%d rows", DEC_MAXROWS);
        return JL_ERR_INVALID_ARG;
    }
    const int h = m->hidden, QW = m->q_heads * HEAD;
    JL_TRY(launch_embed(c));
    for (int l = 0; l < layers; ++l) {
        const LayerW& L = m->lw[l];
        DecQkvArgs q{};
        q.q = tile_of(L.q);
        q.k = tile_of(L.k);
        q.v = tile_of(L.v);
        q.K = h;
        q.q_heads = m->q_heads;
        q.kv_heads = m->kv_heads;
        q.x = m->s.x;
        q.norm = L.in_ln;
        q.qn = L.q_norm;
        q.kn = L.k_norm;
        q.rope = (const float2*)m->rope;
        q.pb = m->pass;
        q.kv = kv_view(m, l);
        q.q_out = m->s.qkv;
        q.ld = qkv_ld(m);
        q.mcap = M;
        const dim3 qg(m->q_heads + 2 * m->kv_heads);
        const size_t qs = dec_qkv_smem(h);
        if (M == 1) JL_TRY(launch_pdl(k_dec_qkv<1>, qg, dim3(512), qs, c.stream, q));
        else JL_TRY(launch_pdl(k_dec_qkv<2>, qg, dim3(512), qs, c.stream, q));
        JL_TRY(launch_attention(c, l, false));  // lib.rs:401-441
        auto proj = [&](const Mat& w0, const Mat* w1, int K, const float* x, const uint16_t* norm, float* y,
                        int ldy, int out_rows) -> jl_status {
            DecArgs d{};
            d.w0 = tile_of(w0);
            if (w1) d.w1 = tile_of(*w1);
            d.K = K;
            d.out_rows = out_rows;
            d.x = x;
            d.norm = norm;
            d.y = y;
            d.ldy = ldy;
            d.hdr = m->pass.hdr;
            d.mcap = M;
            d.err = m->counters;
            const dim3 g((out_rows + DEC_TR - 1) / DEC_TR);
            const size_t sm = dec_proj_smem(K, w1 != nullptr);
            if (w1) {
                if (M == 1) return launch_pdl(k_dec_proj<1, true>, g, dim3(256), sm, c.stream, d);
                return launch_pdl(k_dec_proj<2, true>, g, dim3(256), sm, c.stream, d);
            }
            if (M == 1) return launch_pdl(k_dec_proj<1, false>, g, dim3(256), sm, c.stream, d);
            return launch_pdl(k_dec_proj<2, false>, g, dim3(256), sm, c.stream, d);
        };
        JL_TRY(proj(L.o, nullptr, QW, m->s.attn, nullptr, m->s.x, h, h));                // lib.rs:444-449
        JL_TRY(proj(L.gate, &L.up, h, m->s.x, L.post_ln, m->s.act, m->inter, m->inter));  // lib.rs:459-463
        JL_TRY(proj(L.down, nullptr, m->inter, m->s.act, nullptr, m->s.x, h, h));         // lib.rs:464-467
    }
    return JL_OK;
}

}  // namespace jl
