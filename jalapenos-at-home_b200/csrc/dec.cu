// Draft-step projections on CUDA cores: passes of one or two rows.
//
// A draft model's proposal step is one token through every layer.  With so
// little arithmetic, what a projection costs is latency: the tensor-core
// path (activation pieces, TMEM, split-K reduction, the next projection's
// pieces) takes several round trips after its inputs are ready.  These
// kernels take almost none: each CTA owns a tile of weight rows and copies
// them (MXFP4 codes and scales, exactly as the checkpoint stores them) into
// shared memory with bulk copies BEFORE it waits for the previous kernel
// (weights never depend on it).  After the wait it loads the f32 input rows
// (times the RMSNorm weight), and each warp computes its rows' dot products:
// lanes take 32-element blocks, decode E2M1 pairs in hardware
// (cvt.rn.f16x2.e2m1x2), apply the block's E8M0 scale, and the warp sums; the
// RMSNorm division (lib.rs:268-290) is applied to those sums, so no
// block-wide reduction stands between the input load and the dot products.  Epilogues: q|k|v (QK-RMSNorm, RoPE, K/V appended to the cache),
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
#include "timeline.cuh"

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
// layout; with `w` set, as x * w, and warp j's share of row m's sum of
// squares goes to ssq[m * 8 + j].  The RMSNorm division (lib.rs:268-290) is
// applied to the dot products instead (dec_rms): W (x * w) / rms, so the
// dot products need not wait for a block-wide sum.  Whole CTA (8 warps).
// Each thread holds at most DEC_XCHUNKS float4 chunks of a row in registers,
// so x is read from global memory once.  The thread's norm weights (wv, from
// dec_norm_weights) are fetched before the dependency wait: they never depend
// on the previous kernel.
constexpr int DEC_XCHUNKS = 4;

__device__ __forceinline__ void dec_norm_weights(const uint16_t* __restrict__ w, int K,
                                                 uint2 (&wv)[DEC_XCHUNKS]) {
#pragma unroll
    for (int i = 0; i < DEC_XCHUNKS; ++i) {
        const int c = threadIdx.x + i * blockDim.x;
        wv[i] = (w && c < K / 4) ? *reinterpret_cast<const uint2*>(w + 4 * c) : make_uint2(0u, 0u);
    }
}

__device__ __forceinline__ void dec_load_x(const float* __restrict__ x, int ldx, int M, int K,
                                           const uint16_t* __restrict__ w, const uint2 (&wv)[DEC_XCHUNKS],
                                           float4* xs4, float* ssq) {
    const int K4 = K / 4;
    for (int m = 0; m < M; ++m) {
        const float* xr = x + (size_t)m * ldx;
        float4 v[DEC_XCHUNKS];
#pragma unroll
        for (int i = 0; i < DEC_XCHUNKS; ++i) {
            const int c = threadIdx.x + i * blockDim.x;
            v[i] = c < K4 ? reinterpret_cast<const float4*>(xr)[c] : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        if (w) {
            float ss = 0.f;
#pragma unroll
            for (int i = 0; i < DEC_XCHUNKS; ++i) {
                ss = fmaf(v[i].x, v[i].x, ss);
                ss = fmaf(v[i].y, v[i].y, ss);
                ss = fmaf(v[i].z, v[i].z, ss);
                ss = fmaf(v[i].w, v[i].w, ss);
            }
            ss = warp_sum(ss);
            if ((threadIdx.x & 31) == 0) ssq[m * 8 + (threadIdx.x >> 5)] = ss;
        }
#pragma unroll
        for (int i = 0; i < DEC_XCHUNKS; ++i) {
            const int c = threadIdx.x + i * blockDim.x;
            if (c >= K4) continue;
            if (w) {
                v[i].x = __fmul_rn(v[i].x, bf16f(wv[i].x & 0xffffu));
                v[i].y = __fmul_rn(v[i].y, bf16f(wv[i].x >> 16));
                v[i].z = __fmul_rn(v[i].z, bf16f(wv[i].y & 0xffffu));
                v[i].w = __fmul_rn(v[i].w, bf16f(wv[i].y >> 16));
            }
            xs4[m * K4 + dec_swz(c)] = v[i];
        }
    }
}

// sqrt(mean(x^2) + 1e-6) of row m from the warps' shares (in warp order),
// after the barrier that publishes them; 1 without a norm.
__device__ __forceinline__ float dec_rms(const float* ssq, int m, int K, bool norm) {
    if (!norm) return 1.f;
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) ss = __fadd_rn(ss, ssq[m * 8 + j]);
    return sqrtf(__fadd_rn(__fdiv_rn(ss, (float)K), 1e-6f));
}

// Dot products of R weight rows (codes wr[i], scales sr[i], width K) with
// the M staged input rows; every lane gets the totals out[i][m].  The rows'
// dependent chains are independent, so one pass over K interleaves them;
// each row's arithmetic is the same as on its own.  Whole warp.
template <int R, int M>
__device__ __forceinline__ void dec_dot(const uint8_t* const (&wr)[R], const uint8_t* const (&sr)[R], int K,
                                        const float4* xs4, int lane, float (&out)[R][M]) {
    const int nb = K / 32, K4 = K / 4;
    float acc[R][M];
#pragma unroll
    for (int i = 0; i < R; ++i)
#pragma unroll
        for (int m = 0; m < M; ++m) acc[i][m] = 0.f;
    for (int b = lane; b < nb; b += 32) {
        float4 xa[4][M], xb[4][M];
#pragma unroll
        for (int q = 0; q < 4; ++q)
#pragma unroll
            for (int m = 0; m < M; ++m) {
                xa[q][m] = xs4[m * K4 + dec_swz(b * 8 + 2 * q)];
                xb[q][m] = xs4[m * K4 + dec_swz(b * 8 + 2 * q + 1)];
            }
#pragma unroll
        for (int i = 0; i < R; ++i) {
            const uint4 w = *reinterpret_cast<const uint4*>(wr[i] + (size_t)b * 16);
            const float sc = e8m0(sr[i][b]);
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
                    float p = part[m];
                    p = fmaf(l01.x, xa[q][m].x, p);
                    p = fmaf(l01.y, xa[q][m].y, p);
                    p = fmaf(l23.x, xa[q][m].z, p);
                    p = fmaf(l23.y, xa[q][m].w, p);
                    p = fmaf(l45.x, xb[q][m].x, p);
                    p = fmaf(l45.y, xb[q][m].y, p);
                    p = fmaf(l67.x, xb[q][m].z, p);
                    p = fmaf(l67.y, xb[q][m].w, p);
                    part[m] = p;
                }
            }
#pragma unroll
            for (int m = 0; m < M; ++m) acc[i][m] = fmaf(part[m], sc, acc[i][m]);
        }
    }
#pragma unroll
    for (int i = 0; i < R; ++i)
#pragma unroll
        for (int m = 0; m < M; ++m) out[i][m] = warp_sum(acc[i][m]);
}

// ---------------------------------------------------------------------------
// CTA = TR output rows (8 or 16), 8 warps of TR / 8 rows each.  Output rows
// are numbered across up to three stacked matrices (q | k | v; a tile never
// straddles two); SwiGLU tiles take TR gate rows and the matching up rows.
// The dot products are latency, not work: o, gate/up and down take one row
// per warp; q|k|v (the widest output, 4096 rows on the 0.6B) takes two, as
// 512 CTAs all loading x cost more than a second interleaved row.

constexpr int DEC_TR = 16;  // the largest tile
enum : int { DEC_STORE = 0, DEC_ADD = 1, DEC_SWIGLU = 2 };

struct DecArgs {
    DecTile w[3];            // stacked matrices (SwiGLU: gate, up)
    int rows[3];             // their row counts (unused entries 0)
    int K, out_rows;
    const float* x;          // input rows [rows][K]
    const uint16_t* norm;    // RMSNorm weight applied to x first, or null
    float* y;                // output rows [rows][ldy]
    int ldy;
    const PassHdr* hdr;
    int mcap;
    int* err;
    TlSlot tl;  // phase stamps (timeline build)
};

template <int M, int EPI, int TR>
__global__ void __launch_bounds__(256) k_dec_proj(DecArgs a) {
    extern __shared__ __align__(128) uint8_t dsm[];
    __shared__ uint64_t bar;
    __shared__ float red[32];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) tl_stamp(a.tl, 0);
    const int K = a.K;
    const int r0 = blockIdx.x * TR;
    const int n = min(TR, a.out_rows - r0);
    constexpr int NM = EPI == DEC_SWIGLU ? 2 : 1;
    // the matrix this tile's rows come from, and the first local row
    int mat = 0, lr0 = r0;
    if (EPI != DEC_SWIGLU)
        while (mat < 2 && lr0 >= a.rows[mat]) lr0 -= a.rows[mat++];
    uint8_t* wsm = dsm;                                   // [NM][TR][K/2]
    uint8_t* ssm = dsm + NM * TR * (K / 2);           // [NM][TR][K/32]
    float4* xs4 = reinterpret_cast<float4*>(ssm + NM * TR * (K / 32));
    if (threadIdx.x == 0) {
        ptx::mbar_init(&bar, 1);
        ptx::fence_barrier_init();
        ptx::mbar_arrive_expect_tx(&bar, (uint32_t)(NM * n * (K / 2 + K / 32)));
        dec_copy_rows(a.w[mat], lr0, n, K, wsm, ssm, &bar);
        if (EPI == DEC_SWIGLU)
            dec_copy_rows(a.w[1], r0, n, K, wsm + TR * (K / 2), ssm + TR * (K / 32), &bar);
    }
    uint2 wv[DEC_XCHUNKS];
    dec_norm_weights(a.norm, K, wv);
    __syncthreads();  // the barrier is initialised before anyone waits on it
    ptx::grid_dependency_wait();
    if (threadIdx.x == 0) tl_stamp(a.tl, 1);
    ptx::launch_dependents();
    const int rows = min(a.hdr->rows, a.mcap);
    // residual add: the x values lane 0 of this warp adds to, read now so the
    // load overlaps the input load and the dot products (only this CTA
    // writes these rows of x)
    float xold[TR / 8][M];
#pragma unroll
    for (int h = 0; h < TR / 8; ++h)
#pragma unroll
        for (int m = 0; m < M; ++m)
            xold[h][m] = EPI == DEC_ADD && lane == 0 && warp + 8 * h < n && m < rows
                             ? a.y[(size_t)m * a.ldy + r0 + warp + 8 * h]
                             : 0.f;
    dec_load_x(a.x, K, M, K, a.norm, wv, xs4, red);
    const bool ok = ptx::mbar_wait(&bar, 0, DEC_WAIT);
    __syncthreads();
    if (!ok) {
        if (threadIdx.x == 0) atomicOr(a.err, 4);
        return;
    }
    if (threadIdx.x == 0) tl_stamp(a.tl, 2);
    // warp w owns tile rows w, w + 8, ... (RPW of them; rows past n are
    // computed from unloaded shared memory and dropped)
    constexpr int RPW = TR / 8;
    static_assert(TR % 8 == 0 && RPW <= 2, "one or two rows per warp of an 8-warp CTA");
    if (warp >= n) return;
    float rms[M];
#pragma unroll
    for (int m = 0; m < M; ++m) rms[m] = dec_rms(red, m, K, a.norm != nullptr);
    if (EPI == DEC_SWIGLU) {
        const uint8_t* wr[2 * RPW];
        const uint8_t* sr[2 * RPW];
#pragma unroll
        for (int h = 0; h < RPW; ++h) {
            const int r = warp + 8 * h;
            wr[h] = wsm + (size_t)r * (K / 2);
            sr[h] = ssm + (size_t)r * (K / 32);
            wr[RPW + h] = wsm + (size_t)(TR + r) * (K / 2);
            sr[RPW + h] = ssm + (size_t)(TR + r) * (K / 32);
        }
        float o[2 * RPW][M];
        dec_dot<2 * RPW, M>(wr, sr, K, xs4, lane, o);
        if (lane == 0)
#pragma unroll
            for (int h = 0; h < RPW; ++h) {
                const int r = warp + 8 * h;
                if (r >= n) continue;
#pragma unroll
                for (int m = 0; m < M; ++m)  // lib.rs:459-463
                    if (m < rows) {
                        const float g = __fdiv_rn(o[h][m], rms[m]), u = __fdiv_rn(o[RPW + h][m], rms[m]);
                        a.y[(size_t)m * a.ldy + r0 + r] = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);
                    }
            }
        if (threadIdx.x == 0) tl_stamp(a.tl, 3);
    } else {
        const uint8_t* wr[RPW];
        const uint8_t* sr[RPW];
#pragma unroll
        for (int h = 0; h < RPW; ++h) {
            wr[h] = wsm + (size_t)(warp + 8 * h) * (K / 2);
            sr[h] = ssm + (size_t)(warp + 8 * h) * (K / 32);
        }
        float o[RPW][M];
        dec_dot<RPW, M>(wr, sr, K, xs4, lane, o);
        if (lane == 0)
#pragma unroll
            for (int h = 0; h < RPW; ++h) {
                const int r = warp + 8 * h;
                if (r >= n) continue;
#pragma unroll
                for (int m = 0; m < M; ++m)
                    if (m < rows) {
                        float* d = a.y + (size_t)m * a.ldy + r0 + r;
                        const float v = __fdiv_rn(o[h][m], rms[m]);
                        *d = EPI == DEC_ADD ? __fadd_rn(xold[h][m], v) : v;  // residual (model.rs:178-186)
                    }
            }
        if (threadIdx.x == 0) tl_stamp(a.tl, 3);
    }
}

template <int M, int EPI>
jl_status configure_dec_proj(int smem) {
    constexpr int TR = EPI == DEC_STORE ? 16 : 8;
    JL_CUDA(cudaFuncSetAttribute(k_dec_proj<M, EPI, TR>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    return JL_OK;
}

size_t dec_proj_smem(int K, bool swiglu, int tr = DEC_TR) {
    const int nm = swiglu ? 2 : 1;
    return (size_t)nm * tr * (K / 2 + K / 32) + (size_t)DEC_MAXROWS * K * 4;
}

DecTile tile_of(const Mat& w) { return DecTile{(const uint8_t*)w.data, w.scales}; }

}  // namespace


bool dec_supported(const jl_model* m) {
    if (m->lw.empty()) return false;
    const int QW = m->q_heads * HEAD, KVW = m->kv_heads * HEAD;
    auto ok = [](int K) { return K % 512 == 0; };  // scale rows of whole 16-byte words
    for (const auto& L : m->lw)
        if (L.q.kind != MAT_MXFP4 || L.k.kind != MAT_MXFP4 || L.v.kind != MAT_MXFP4 || L.o.kind != MAT_MXFP4 ||
            L.gate.kind != MAT_MXFP4 || L.up.kind != MAT_MXFP4 || L.down.kind != MAT_MXFP4)
            return false;
    const int widest = std::max(m->hidden, std::max(QW, m->inter));
    if (widest / 4 > DEC_XCHUNKS * 256) return false;  // input row in registers (256-thread CTAs)
    return ok(m->hidden) && ok(QW) && ok(m->inter) && QW % DEC_TR == 0 && KVW % DEC_TR == 0 &&
           dec_proj_smem(widest, true) <= 200 * 1024 && m->q_heads / m->kv_heads <= 8;
}

constexpr int DEC_SMEM_MAX = 200 * 1024;  // dec_supported keeps every launch under this

jl_status dec_configure() {
    JL_TRY((configure_dec_proj<1, DEC_STORE>(DEC_SMEM_MAX)));
    JL_TRY((configure_dec_proj<2, DEC_STORE>(DEC_SMEM_MAX)));
    JL_TRY((configure_dec_proj<1, DEC_ADD>(DEC_SMEM_MAX)));
    JL_TRY((configure_dec_proj<2, DEC_ADD>(DEC_SMEM_MAX)));
    JL_TRY((configure_dec_proj<1, DEC_SWIGLU>(DEC_SMEM_MAX)));
    JL_TRY((configure_dec_proj<2, DEC_SWIGLU>(DEC_SMEM_MAX)));
    return JL_OK;
}

// The draft-step pass: embedding, then per layer the raw q|k|v projection,
// attention (which applies QK-RMSNorm and RoPE and appends K/V), o, gate/up
// and down, all projections on CUDA cores.
jl_status record_dec_pass(const PassCtx& c, int layers) {
    const jl_model* m = c.m;
    const int M = c.rows_cap;
    if (M < 1 || M > DEC_MAXROWS) {
        set_error("draft-step pass takes 1..%d rows", DEC_MAXROWS);
        return JL_ERR_INVALID_ARG;
    }
    const int h = m->hidden, QW = m->q_heads * HEAD, KVW = m->kv_heads * HEAD;
    JL_TRY(launch_embed(c));
    for (int l = 0; l < layers; ++l) {
        const LayerW& L = m->lw[l];
        auto proj = [&](int epi, const Mat* w0, const Mat* w1, const Mat* w2, int K, const float* x,
                        const uint16_t* norm, float* y, int ldy, int out_rows) -> jl_status {
            DecArgs d{};
            const Mat* ws[3] = {w0, w1, w2};
            for (int i = 0; i < 3; ++i)
                if (ws[i]) {
                    d.w[i] = tile_of(*ws[i]);
                    d.rows[i] = ws[i]->rows;
                }
            d.K = K;
            d.out_rows = out_rows;
            d.x = x;
            d.norm = norm;
            d.y = y;
            d.ldy = ldy;
            d.hdr = c.pass().hdr;
            d.mcap = M;
            d.err = m->counters;
            d.tl = tl_launch(epi == DEC_STORE ? "k_dec_proj<qkv>"
                             : epi == DEC_ADD ? "k_dec_proj<add>"
                                              : "k_dec_proj<swiglu>");
            const int tr = epi == DEC_STORE ? 16 : 8;
            const dim3 g((out_rows + tr - 1) / tr);
            const size_t sm = dec_proj_smem(K, epi == DEC_SWIGLU, tr);
            const dim3 b(256);
            switch (epi * 2 + (M - 1)) {
                case DEC_STORE * 2: return launch_pdl(k_dec_proj<1, DEC_STORE, 16>, g, b, sm, c.stream, d);
                case DEC_STORE * 2 + 1: return launch_pdl(k_dec_proj<2, DEC_STORE, 16>, g, b, sm, c.stream, d);
                case DEC_ADD * 2: return launch_pdl(k_dec_proj<1, DEC_ADD, 8>, g, b, sm, c.stream, d);
                case DEC_ADD * 2 + 1: return launch_pdl(k_dec_proj<2, DEC_ADD, 8>, g, b, sm, c.stream, d);
                case DEC_SWIGLU * 2: return launch_pdl(k_dec_proj<1, DEC_SWIGLU, 8>, g, b, sm, c.stream, d);
                default: return launch_pdl(k_dec_proj<2, DEC_SWIGLU, 8>, g, b, sm, c.stream, d);
            }
        };
        // lib.rs:353-355: raw q | k | v, normalised and rotated by the attention kernel
        JL_TRY(proj(DEC_STORE, &L.q, &L.k, &L.v, h, m->s.x, L.in_ln, m->s.qkv, qkv_ld(m), QW + 2 * KVW));
        JL_TRY(launch_attention_raw(c, l, L.q_norm, L.k_norm));                                  // lib.rs:363-441
        JL_TRY(proj(DEC_ADD, &L.o, nullptr, nullptr, QW, m->s.attn, nullptr, m->s.x, h, h));         // lib.rs:444-449
        JL_TRY(proj(DEC_SWIGLU, &L.gate, &L.up, nullptr, h, m->s.x, L.post_ln, m->s.act, m->inter,
                    m->inter));                                                                     // lib.rs:459-463
        JL_TRY(proj(DEC_ADD, &L.down, nullptr, nullptr, m->inter, m->s.act, nullptr, m->s.x, h, h));  // lib.rs:464-467
    }
    return JL_OK;
}

}  // namespace jl
