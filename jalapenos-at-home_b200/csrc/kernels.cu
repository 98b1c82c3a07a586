// Forward-pass kernels for sm_100a, first generation (CUDA cores).
//
// Every kernel reads its row count from the device PassHdr, so a pass
// recorded once into a CUDA graph replays for any number of rows.  Every
// output value is computed by one warp in a fixed order that does not depend
// on how many rows the pass holds: a token's logits are bit-identical whether
// it is decoded alone, verified among k+1 draft tokens, or fed in a two-row
// draft catch-up.  That is what makes speculative output equal greedy output
// exactly (engine/tests/generation.rs:69-92 asserts it on the reference).
#include <cstdio>

#include "jl_internal.h"
#include "kernels.cuh"
#include "launch.cuh"
#include "mx_pieces.cuh"
#include "ptx.cuh"
#include "timeline.cuh"

namespace jl {

namespace {

enum Epi : int { EPI_STORE = 0, EPI_ADD = 1, EPI_SWIGLU = 2 };

// Up to three matrices stacked along the output dimension (q, k, v), or the
// (gate, up) pair of EPI_SWIGLU.  All share the input width K and kind.
struct Proj {
    const void* w[3];
    const uint8_t* s[3];
    int n[3];
    int K;
    int total;  // output columns (EPI_SWIGLU: rows of one matrix)
};

__device__ __forceinline__ void pick(const Proj& p, int r, int& mat, int& local) {
    if (r < p.n[0]) { mat = 0; local = r; }
    else if (r < p.n[0] + p.n[1]) { mat = 1; local = r - p.n[0]; }
    else { mat = 2; local = r - p.n[0] - p.n[1]; }
}

// Shared-memory slot of 16-byte x chunk c.  MXFP4 lanes read the eight
// chunks of one 32-element block each; bf16 lanes read two adjacent chunks.
// The XOR swizzles keep every 8-lane phase of an LDS.128 on distinct banks.
__device__ __forceinline__ int swz_mx(int c) { return c ^ ((c >> 3) & 7); }
__device__ __forceinline__ int swz_bf(int c) { return c ^ ((c >> 3) & 1); }

__device__ __forceinline__ float silu_mul(float g, float u) {
    // lib.rs:462: (gate / (1 + exp(-gate))) * up
    return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);
}

// ---------------------------------------------------------------------------
// Skinny projection: y[m, r] (op)= sum_k x[m, k] * W[r, k] for M <= SMALL_M.
// CTA = 8 warps; a warp owns R output rows at a time, its lanes split K;
// MR input rows are staged in shared memory per sweep over the weights.

template <int KIND, int EPI, int R, int MR>
__global__ void __launch_bounds__(256) k_skinny(const PassHdr* __restrict__ hdr, int use_head,
                                                int max_m, const float* __restrict__ x, int ldx, Proj p,
                                                float* __restrict__ y, int ldy) {
    extern __shared__ float4 xs4[];
    ptx::grid_dependency_wait();  // PDL: the previous kernel's writes are visible past here
    ptx::launch_dependents();
    const int M = min(use_head ? hdr->head_rows : hdr->rows, max_m);  // never past the buffers
    const int K = p.K, K4 = K >> 2;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int groups = (p.total + R - 1) / R;
    constexpr int NV = EPI == EPI_SWIGLU ? 2 : 1;  // dot products per output
    for (int m0 = 0; m0 < M; m0 += MR) {
        const int mr = min(MR, M - m0);
        __syncthreads();
        for (int i = threadIdx.x; i < MR * K4; i += blockDim.x) {
            const int m = i / K4, c = i - m * K4;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (m < mr) v = reinterpret_cast<const float4*>(x + (size_t)(m0 + m) * ldx)[c];
            xs4[m * K4 + (KIND == MAT_MXFP4 ? swz_mx(c) : swz_bf(c))] = v;
        }
        __syncthreads();
        for (int g = blockIdx.x * 8 + warp; g < groups; g += gridDim.x * 8) {
            const uint8_t* wrow[R][NV];
            const uint8_t* srow[R][NV];
            bool valid[R];
#pragma unroll
            for (int j = 0; j < R; ++j) {
                const int r = g * R + j;
                valid[j] = r < p.total;
                const int rr = valid[j] ? r : 0;
#pragma unroll
                for (int v = 0; v < NV; ++v) {
                    int mat, local;
                    if (EPI == EPI_SWIGLU) { mat = v; local = rr; }
                    else pick(p, rr, mat, local);
                    if (KIND == MAT_MXFP4) {
                        wrow[j][v] = (const uint8_t*)p.w[mat] + (size_t)local * (K >> 1);
                        srow[j][v] = p.s[mat] + (size_t)local * (K >> 5);
                    } else {
                        wrow[j][v] = (const uint8_t*)p.w[mat] + (size_t)local * K * 2;
                        srow[j][v] = nullptr;
                    }
                }
            }
            float acc[R][NV][MR];
#pragma unroll
            for (int j = 0; j < R; ++j)
#pragma unroll
                for (int v = 0; v < NV; ++v)
#pragma unroll
                    for (int m = 0; m < MR; ++m) acc[j][v][m] = 0.f;

            if (KIND == MAT_MXFP4) {
                const int nb = K >> 5;
                for (int b = lane; b < nb; b += 32) {
                    uint4 wv[R][NV];
                    uint32_t sb[R][NV];
#pragma unroll
                    for (int j = 0; j < R; ++j)
#pragma unroll
                        for (int v = 0; v < NV; ++v) {
                            wv[j][v] = valid[j] ? ldg_stream(wrow[j][v] + (size_t)b * 16)
                                                : make_uint4(0, 0, 0, 0);
                            sb[j][v] = valid[j] ? srow[j][v][b] : 127u;
                        }
                    float part[R][NV][MR];
#pragma unroll
                    for (int j = 0; j < R; ++j)
#pragma unroll
                        for (int v = 0; v < NV; ++v)
#pragma unroll
                            for (int m = 0; m < MR; ++m) part[j][v][m] = 0.f;
#pragma unroll
                    for (int q = 0; q < 8; ++q) {
                        float4 xv[MR];
#pragma unroll
                        for (int m = 0; m < MR; ++m) xv[m] = xs4[m * K4 + b * 8 + (q ^ (b & 7))];
#pragma unroll
                        for (int j = 0; j < R; ++j)
#pragma unroll
                            for (int v = 0; v < NV; ++v) {
                                const uint32_t w4 = q < 2 ? wv[j][v].x : q < 4 ? wv[j][v].y
                                                  : q < 6 ? wv[j][v].z : wv[j][v].w;
                                const uint32_t word = w4 >> ((q & 1) * 16);
                                const float l0 = e2m1(word), l1 = e2m1(word >> 4);
                                const float l2 = e2m1(word >> 8), l3 = e2m1(word >> 12);
#pragma unroll
                                for (int m = 0; m < MR; ++m) {
                                    float a = part[j][v][m];
                                    a = fmaf(l0, xv[m].x, a);
                                    a = fmaf(l1, xv[m].y, a);
                                    a = fmaf(l2, xv[m].z, a);
                                    a = fmaf(l3, xv[m].w, a);
                                    part[j][v][m] = a;
                                }
                            }
                    }
#pragma unroll
                    for (int j = 0; j < R; ++j)
#pragma unroll
                        for (int v = 0; v < NV; ++v) {
                            const float sc = e8m0(sb[j][v]);
#pragma unroll
                            for (int m = 0; m < MR; ++m)
                                acc[j][v][m] = fmaf(part[j][v][m], sc, acc[j][v][m]);
                        }
                }
            } else {
                for (int e0 = lane * 8; e0 < K; e0 += 256) {
                    uint4 wv[R][NV];
#pragma unroll
                    for (int j = 0; j < R; ++j)
#pragma unroll
                        for (int v = 0; v < NV; ++v)
                            wv[j][v] = valid[j] ? ldg_stream(wrow[j][v] + (size_t)e0 * 2)
                                                : make_uint4(0, 0, 0, 0);
                    const int c = e0 >> 2;
                    float4 xa[MR], xb[MR];
#pragma unroll
                    for (int m = 0; m < MR; ++m) {
                        xa[m] = xs4[m * K4 + swz_bf(c)];
                        xb[m] = xs4[m * K4 + swz_bf(c + 1)];
                    }
#pragma unroll
                    for (int j = 0; j < R; ++j)
#pragma unroll
                        for (int v = 0; v < NV; ++v) {
                            const uint4 w = wv[j][v];
                            const float w0 = __uint_as_float(w.x << 16), w1 = __uint_as_float(w.x & 0xffff0000u);
                            const float w2 = __uint_as_float(w.y << 16), w3 = __uint_as_float(w.y & 0xffff0000u);
                            const float w4 = __uint_as_float(w.z << 16), w5 = __uint_as_float(w.z & 0xffff0000u);
                            const float w6 = __uint_as_float(w.w << 16), w7 = __uint_as_float(w.w & 0xffff0000u);
#pragma unroll
                            for (int m = 0; m < MR; ++m) {
                                float a = acc[j][v][m];
                                a = fmaf(w0, xa[m].x, a);
                                a = fmaf(w1, xa[m].y, a);
                                a = fmaf(w2, xa[m].z, a);
                                a = fmaf(w3, xa[m].w, a);
                                a = fmaf(w4, xb[m].x, a);
                                a = fmaf(w5, xb[m].y, a);
                                a = fmaf(w6, xb[m].z, a);
                                a = fmaf(w7, xb[m].w, a);
                                acc[j][v][m] = a;
                            }
                        }
                }
            }
            // fixed-order reduction across the 32 lanes
#pragma unroll
            for (int j = 0; j < R; ++j)
#pragma unroll
                for (int v = 0; v < NV; ++v)
#pragma unroll
                    for (int m = 0; m < MR; ++m) acc[j][v][m] = warp_sum(acc[j][v][m]);
            if (lane == 0) {
#pragma unroll
                for (int j = 0; j < R; ++j) {
                    if (!valid[j]) continue;
                    const int r = g * R + j;
#pragma unroll
                    for (int m = 0; m < MR; ++m) {
                        if (m >= mr) continue;
                        float* out = y + (size_t)(m0 + m) * ldy + r;
                        if (EPI == EPI_STORE) *out = acc[j][0][m];
                        else if (EPI == EPI_ADD) *out = __fadd_rn(*out, acc[j][0][m]);
                        else *out = silu_mul(acc[j][0][m], acc[j][NV - 1][m]);
                    }
                }
            }
        }
    }
}

// ---------------------------------------------------------------------------
// Tiled projection for long prompts (M > SMALL_M): 64 tokens x 64 outputs per
// CTA, weights decoded to exact f32 in shared memory.

template <int KIND, int EPI>
__global__ void __launch_bounds__(256) k_gemm(const PassHdr* __restrict__ hdr, int use_head,
                                              int max_m, const float* __restrict__ x, int ldx, Proj p,
                                              float* __restrict__ y, int ldy) {
    constexpr int BM = 64, BN = 64, BK = 32;
    ptx::grid_dependency_wait();  // PDL: the previous kernel's writes are visible past here
    ptx::launch_dependents();
    constexpr int NV = EPI == EPI_SWIGLU ? 2 : 1;
    __shared__ float xs[BK][BM + 4];
    __shared__ float ws[NV][BK][BN + 4];
    const int M = min(use_head ? hdr->head_rows : hdr->rows, max_m);  // never past the buffers
    const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
    if (m0 >= M || n0 >= p.total) return;
    const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
    const int K = p.K;
    float acc[NV][4][4] = {};
    for (int k0 = 0; k0 < K; k0 += BK) {
        // x tile: 64 rows x 32 k, transposed into xs[k][m]
        for (int i = tid; i < BM * BK / 4; i += 256) {
            const int m = i / (BK / 4), c = i % (BK / 4);
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (m0 + m < M) v = *reinterpret_cast<const float4*>(x + (size_t)(m0 + m) * ldx + k0 + c * 4);
            xs[c * 4 + 0][m] = v.x;
            xs[c * 4 + 1][m] = v.y;
            xs[c * 4 + 2][m] = v.z;
            xs[c * 4 + 3][m] = v.w;
        }
        // weight tile: 64 output rows x 32 k
#pragma unroll
        for (int v = 0; v < NV; ++v) {
            if (KIND == MAT_MXFP4) {
                if (tid < BN) {
                    const int r = n0 + tid;
                    float vals[32];
                    if (r < p.total) {
                        int mat, local;
                        if (EPI == EPI_SWIGLU) { mat = v; local = r; }
                        else pick(p, r, mat, local);
                        const uint8_t* wr = (const uint8_t*)p.w[mat] + (size_t)local * (K >> 1) + (k0 >> 1);
                        const uint4 wv = *reinterpret_cast<const uint4*>(wr);
                        const float sc = e8m0(p.s[mat][(size_t)local * (K >> 5) + (k0 >> 5)]);
                        const uint32_t words[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
                        for (int e = 0; e < 32; ++e)
                            vals[e] = __fmul_rn(e2m1(words[e >> 3] >> ((e & 7) * 4)), sc);
                    } else {
#pragma unroll
                        for (int e = 0; e < 32; ++e) vals[e] = 0.f;
                    }
#pragma unroll
                    for (int e = 0; e < 32; ++e) ws[v][e][tid] = vals[e];
                }
            } else {
                for (int i = tid; i < BN * BK / 8; i += 256) {
                    const int n = i / (BK / 8), c = i % (BK / 8);
                    const int r = n0 + n;
                    uint4 wv = make_uint4(0, 0, 0, 0);
                    if (r < p.total) {
                        int mat, local;
                        if (EPI == EPI_SWIGLU) { mat = v; local = r; }
                        else pick(p, r, mat, local);
                        wv = *reinterpret_cast<const uint4*>((const uint16_t*)p.w[mat] + (size_t)local * K + k0 + c * 8);
                    }
                    const uint32_t words[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
                    for (int e = 0; e < 8; ++e)
                        ws[v][c * 8 + e][n] = __uint_as_float(e & 1 ? (words[e >> 1] & 0xffff0000u)
                                                                    : (words[e >> 1] << 16));
                }
            }
        }
        __syncthreads();
#pragma unroll 8
        for (int k = 0; k < BK; ++k) {
            float a[4], b[NV][4];
#pragma unroll
            for (int i = 0; i < 4; ++i) a[i] = xs[k][ty * 4 + i];
#pragma unroll
            for (int v = 0; v < NV; ++v)
#pragma unroll
                for (int i = 0; i < 4; ++i) b[v][i] = ws[v][k][tx * 4 + i];
#pragma unroll
            for (int v = 0; v < NV; ++v)
#pragma unroll
                for (int i = 0; i < 4; ++i)
#pragma unroll
                    for (int jj = 0; jj < 4; ++jj) acc[v][i][jj] = fmaf(a[i], b[v][jj], acc[v][i][jj]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int m = m0 + ty * 4 + i;
        if (m >= M) continue;
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
            const int n = n0 + tx * 4 + jj;
            if (n >= p.total) continue;
            float* out = y + (size_t)m * ldy + n;
            if (EPI == EPI_STORE) *out = acc[0][i][jj];
            else if (EPI == EPI_ADD) *out = __fadd_rn(*out, acc[0][i][jj]);
            else *out = silu_mul(acc[0][i][jj], acc[NV - 1][i][jj]);
        }
    }
}

// ---------------------------------------------------------------------------

__global__ void k_embed(PassBuf pb, Mat e, float* __restrict__ x, int hidden, int chunked) {
    // lib.rs:213-235, model.rs:167-170
    ptx::grid_dependency_wait();  // PDL: the previous kernel's writes are visible past here
    ptx::launch_dependents();
    const int row = blockIdx.x;
    if (chunked ? row % SMALL_M >= pb.hdr[row / SMALL_M].rows : row >= pb.hdr->rows) return;
    uint32_t tok = pb.row[row].token;
    if (tok >= (uint32_t)e.rows) tok = 0;  // ids are validated on the host
    float* out = x + (size_t)row * hidden;
    for (int i = threadIdx.x; i < hidden; i += blockDim.x) {
        const size_t idx = (size_t)tok * hidden + i;
        if (e.kind == MAT_MXFP4) {
            const uint8_t byte = ((const uint8_t*)e.data)[idx >> 1];
            const float v = __fmul_rn(e2m1(byte >> ((idx & 1) * 4)), e8m0(e.scales[idx >> 5]));
            out[i] = __uint_as_float(__float_as_uint(v) & 0xffff0000u);  // truncation, lib.rs:227
        } else {
            out[i] = bf16f(((const uint16_t*)e.data)[idx]);
        }
    }
}

__global__ void k_rmsnorm(PassBuf pb, const float* __restrict__ x, int ldx,
                          const uint16_t* __restrict__ w, float* __restrict__ out, int ldo,
                          int width, int head_rows) {
    // lib.rs:268-290: x / sqrt(mean(x^2) + 1e-6) * w
    __shared__ float red[32];
    ptx::grid_dependency_wait();  // PDL: the previous kernel's writes are visible past here
    ptx::launch_dependents();
    const int i = blockIdx.x;
    const int n = head_rows ? pb.hdr->head_rows : pb.hdr->rows;
    if (i >= n) return;
    const int src = head_rows ? pb.head_row[i] : i;
    const float* xr = x + (size_t)src * ldx;
    float ss = 0.f;
    for (int j = threadIdx.x; j < width; j += blockDim.x) ss = fmaf(xr[j], xr[j], ss);
    ss = block_sum(ss, red);
    const float size = sqrtf(__fadd_rn(__fdiv_rn(ss, (float)width), 1e-6f));
    float* o = out + (size_t)i * ldo;
    for (int j = threadIdx.x; j < width; j += blockDim.x)
        o[j] = __fmul_rn(__fdiv_rn(xr[j], size), bf16f(w[j]));
}

// Per-head QK-RMSNorm and RoPE of q and k, then K and V appended to the cache
// (lib.rs:363-396): one warp per head, lane owns dims {l, l+32, l+64, l+96}
// so both RoPE pairs (i, i+64) stay in the lane.
__global__ void __launch_bounds__(256) k_qk_rope_kv(PassBuf pb, float* __restrict__ qkv, int ld,
                                                    int q_heads, const uint16_t* __restrict__ qn,
                                                    const uint16_t* __restrict__ kn,
                                                    const float2* __restrict__ rope, KvView kv) {
    ptx::grid_dependency_wait();  // PDL: the previous kernel's writes are visible past here
    ptx::launch_dependents();
    const int row = blockIdx.x;
    if (row >= pb.hdr->rows) return;
    const RowDesc rd = pb.row[row];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int kv_heads = kv.kv_heads;
    const int heads = q_heads + 2 * kv_heads;
    if (rd.pos < 0 || rd.pos >= kv.max_pos || (unsigned)rd.seq >= (unsigned)MAX_SEQS) {
        atomicOr(kv.err, 2);
        return;
    }
    const int32_t* pt = pb.page_table[rd.seq];
    const int page = pt[rd.pos / PAGE], t = rd.pos % PAGE;
    if (!page_ok(kv, page)) return;
    float* base = qkv + (size_t)row * ld;
    for (int h = warp; h < heads; h += 8) {
        float* src = base + h * HEAD;  // q heads, then k heads, then v heads
        float a0 = src[lane], a1 = src[lane + 32], a2 = src[lane + 64], a3 = src[lane + 96];
        if (h < q_heads + kv_heads) {
            const uint16_t* gw = h < q_heads ? qn : kn;
            float ss = fmaf(a0, a0, fmaf(a1, a1, fmaf(a2, a2, a3 * a3)));
            ss = warp_sum(ss);
            const float size = sqrtf(__fadd_rn(__fdiv_rn(ss, 128.0f), 1e-6f));
            a0 = __fmul_rn(__fdiv_rn(a0, size), bf16f(gw[lane]));
            a1 = __fmul_rn(__fdiv_rn(a1, size), bf16f(gw[lane + 32]));
            a2 = __fmul_rn(__fdiv_rn(a2, size), bf16f(gw[lane + 64]));
            a3 = __fmul_rn(__fdiv_rn(a3, size), bf16f(gw[lane + 96]));
            // lib.rs:306-313: out[i] = a cos - b sin; out[i+64] = b cos + a sin
            const float2 r0 = rope[(size_t)rd.pos * HALF + lane];
            const float2 r1 = rope[(size_t)rd.pos * HALF + lane + 32];
            const float b0 = __fsub_rn(__fmul_rn(a0, r0.x), __fmul_rn(a2, r0.y));
            const float b2 = __fadd_rn(__fmul_rn(a2, r0.x), __fmul_rn(a0, r0.y));
            const float b1 = __fsub_rn(__fmul_rn(a1, r1.x), __fmul_rn(a3, r1.y));
            const float b3 = __fadd_rn(__fmul_rn(a3, r1.x), __fmul_rn(a1, r1.y));
            a0 = b0; a1 = b1; a2 = b2; a3 = b3;
        }
        if (h < q_heads) {
            src[lane] = a0; src[lane + 32] = a1; src[lane + 64] = a2; src[lane + 96] = a3;
        } else {
            const bool is_k = h < q_heads + kv_heads;
            const int kvh = is_k ? h - q_heads : h - q_heads - kv_heads;
            const size_t idx = kv_index(page, kvh, t, kv_heads);
            if (kv.f32) {
                float* d = (float*)(is_k ? kv.k : kv.v) + idx;
                d[lane] = a0; d[lane + 32] = a1; d[lane + 64] = a2; d[lane + 96] = a3;
            } else {
                uint16_t* d = (uint16_t*)(is_k ? kv.k : kv.v) + idx;
                d[lane] = f2bf16(a0); d[lane + 32] = f2bf16(a1);
                d[lane + 64] = f2bf16(a2); d[lane + 96] = f2bf16(a3);
            }
        }
    }
}

template <int F32>
__device__ __forceinline__ float kv_load(const void* base, size_t idx) {
    if (F32) return ((const float*)base)[idx];
    return bf16f(((const uint16_t*)base)[idx]);
}

// Causal GQA attention for one (q head, row): softmax(q.k / sqrt(128)) . v
// over positions [0, pos] of the row's sequence (lib.rs:401-441), in chunks
// of 128 positions with a running max.
//
// With `bout` set, the output row also goes out as the o projection's input
// pieces (one 32-block per warp), and rows past the pass's row count get
// zero pieces so every MMA column of the next projection is defined.
template <int F32>
__global__ void __launch_bounds__(128) k_attention(PassBuf pb, const float* __restrict__ qkv,
                                                   int ld, int q_heads, int group, KvView kv,
                                                   float* __restrict__ out, uint8_t* __restrict__ bout,
                                                   int bN) {
    __shared__ __align__(16) float qs[HEAD];
    __shared__ float pr[128];
    __shared__ float red[32];
    ptx::grid_dependency_wait();  // PDL: the previous kernel's writes are visible past here
    ptx::launch_dependents();
    const int h = blockIdx.x, row = blockIdx.y;
    const int t = threadIdx.x;
    if (row >= pb.hdr->rows) {
        if (bout) mx::emit_pieces_smem(qs, HEAD, 4, row, 0, 1, t, 128, h * HEAD, bN, bout);
        return;
    }
    const RowDesc rd = pb.row[row];
    const int kvh = h / group;
    if (rd.pos < 0 || rd.pos >= kv.max_pos || (unsigned)rd.seq >= (unsigned)MAX_SEQS) {
        if (t == 0) atomicOr(kv.err, 2);
        out[(size_t)row * (q_heads * HEAD) + h * HEAD + t] = 0.f;
        if (bout) mx::emit_pieces_smem(qs, HEAD, 4, row, 0, 1, t, 128, h * HEAD, bN, bout);
        return;
    }
    const int visible = rd.pos + 1;
    const int32_t* pt = pb.page_table[rd.seq];
    qs[t] = qkv[(size_t)row * ld + h * HEAD + t];
    __syncthreads();
    const float scale = sqrtf(128.0f);
    float m = -INFINITY, l = 0.f, acc = 0.f;
    for (int s0 = 0; s0 < visible; s0 += 128) {
        const int s = s0 + t;
        float sc = -INFINITY;
        if (s < visible && page_ok(kv, pt[s / PAGE])) {
            const size_t idx = kv_index(pt[s / PAGE], kvh, s % PAGE, kv.kv_heads);
            float dot = 0.f;
            if (F32) {
                const float4* kr = (const float4*)((const float*)kv.k + idx);
#pragma unroll 8
                for (int i = 0; i < 32; ++i) {
                    const float4 k4 = kr[i];
                    dot = fmaf(qs[4 * i], k4.x, dot);
                    dot = fmaf(qs[4 * i + 1], k4.y, dot);
                    dot = fmaf(qs[4 * i + 2], k4.z, dot);
                    dot = fmaf(qs[4 * i + 3], k4.w, dot);
                }
            } else {
                const uint4* kr = (const uint4*)((const uint16_t*)kv.k + idx);
#pragma unroll 4
                for (int i = 0; i < 16; ++i) {
                    const uint4 k8 = kr[i];
                    const uint32_t w[4] = {k8.x, k8.y, k8.z, k8.w};
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        dot = fmaf(qs[8 * i + 2 * e], __uint_as_float(w[e] << 16), dot);
                        dot = fmaf(qs[8 * i + 2 * e + 1], __uint_as_float(w[e] & 0xffff0000u), dot);
                    }
                }
            }
            sc = __fdiv_rn(dot, scale);
        }
        const float cmax = block_max(sc, red);
        const float nm = fmaxf(m, cmax);
        const float corr = expf(m - nm);
        const float e = s < visible ? expf(sc - nm) : 0.f;
        pr[t] = e;
        const float esum = block_sum(e, red);  // also orders pr[] writes before reads
        l = fmaf(l, corr, esum);
        acc *= corr;
        const int n = min(128, visible - s0);
        for (int j = 0; j < n; ++j) {
            const int sp = s0 + j;
            const int page = pt[sp / PAGE];
            if ((unsigned)page >= (unsigned)kv.pages) continue;  // flagged in the score loop
            const size_t idx = kv_index(page, kvh, sp % PAGE, kv.kv_heads) + t;
            acc = fmaf(pr[j], kv_load<F32>(kv.v, idx), acc);
        }
        m = nm;
        __syncthreads();
    }
    const float o = __fdiv_rn(acc, l);
    out[(size_t)row * (q_heads * HEAD) + h * HEAD + t] = o;
    if (bout) {  // every thread is past its last read of qs (the loop ends on a barrier)
        qs[t] = o;
        __syncthreads();
        mx::emit_pieces_smem(qs, HEAD, 4, row, 1, 1, t, 128, h * HEAD, bN, bout);
    }
}

// Decode attention (lib.rs:401-441) for passes of at most a few rows: one CTA
// per (KV head, row), one warp per query head of the GQA group, sharing the
// head's K and V.  The cache keeps a (page, KV head) as one contiguous
// PAGE x 128 block, so one thread copies a window of ATT_WIN pages of K and V
// into shared memory with bulk copies and a single (bounded) mbarrier wait.
// Positions then go 32 at a time: lane j scores position c0 + j, reading its
// K row with the 16-byte chunks rotated by j (no bank conflicts); the warp
// updates the running max and sum, and lanes switch to owning 4 of the 128
// dimensions to accumulate the 32 V rows.  The output row also goes out as
// the o projection's input pieces; rows past the pass's row count get zero
// pieces.
constexpr uint32_t ATT_WAIT = 1u << 22;  // polls before the page copy reports failure

__host__ __device__ constexpr int att_page_bytes(int f32) { return PAGE * HEAD * (f32 ? 4 : 2); }
__host__ __device__ constexpr int att_smem(int f32) { return 2 * ATT_WIN * att_page_bytes(f32); }

// RAW (passes of at most two rows, the draft-step pass): q|k|v are the raw
// projections.  Each warp normalises (QK-RMSNorm) and rotates (RoPE) its
// query head; warp j computes row j's K (normalised, rotated) and V for this
// KV head, which stand in for the cache rows of this pass, and the row's own
// K/V are appended to the cache (lib.rs:363-396).
struct AttnRaw {
    const uint16_t* qn;   // q_norm / k_norm weights
    const uint16_t* kn;
    const float2* rope;
    int k_off, v_off;     // columns of k and v in a q|k|v row
};

// Position-split workspace of the decode attention: per (kv head, row slot,
// window, query head) the window's softmax max, sum and unnormalised output
// (ATT_PART floats), and per (kv head, row slot) an arrival counter that the
// last window CTA resets to zero.
struct AttnSplit {
    float* ws;
    int* cnt;
    // a multi-chunk pass: row r is row r % 16 of chunk r / 16, whose header
    // is hdr[r / 16] and whose attention pieces start at bout + chunk * cs_bout
    int chunked;
    size_t cs_bout;
    int zmax;   // window CTAs per row at most (ATT_ZMAX or ATT_ZMAX_DECODE)
    TlSlot tl;  // phase stamps (timeline build)
};

// `split` warps serve each query head, taking every split-th 32-position
// chunk with their own running max and sum; the head's first warp merges
// them in warp order at the end.
constexpr int ATT_MAXWARPS = 16;

// Warps per query head: up to 4, at most 16 warps in the CTA.
__host__ __device__ constexpr int att_split(int group) { return group >= 8 ? 2 : 4; }

template <int F32, int RAW>
__global__ void __launch_bounds__(512) k_attn_decode(PassBuf pb, const float* __restrict__ qkv, int ld,
                                                     int group, int split, KvView kv, float* __restrict__ out,
                                                     int out_ld, uint8_t* __restrict__ bout, int bN,
                                                     AttnRaw raw, AttnSplit sp) {
    static_assert(PAGE % 32 == 0, "chunks of 32 positions stay inside a page");
    __shared__ float nk[2][HEAD], nv[2][HEAD];  // RAW: this pass's rows of this KV head
    __shared__ int npos[2];
    constexpr int PB = att_page_bytes(F32);
    extern __shared__ __align__(128) uint8_t kvs[];  // [ATT_WIN][K|V][PAGE][HEAD]
    __shared__ __align__(16) float qsh[8][HEAD];
    __shared__ float cm[ATT_MAXWARPS], cl[ATT_MAXWARPS];  // per-warp running max and sum
    __shared__ __align__(16) float cacc[ATT_MAXWARPS][HEAD];
    __shared__ uint64_t bar;
    __shared__ int page_s[ATT_WIN];
    if (threadIdx.x == 0) tl_stamp(sp.tl, 0);
    const int g = blockIdx.x, row = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nw = blockDim.x >> 5;
    const int hw = warp % group, sub = warp / group;  // query head of the group, chunk share
    const int h = g * group + hw;
    const int kvh = g;
    float* qw = qsh[hw];
    // The pass's rows and page tables were written before this pass began,
    // and the cache rows before this row's position by earlier passes: the
    // first window of pages is copied before waiting for the q|k|v kernel,
    // which writes only this row's own K/V (fetched again after the wait).
    const int crow = sp.chunked ? row % SMALL_M : row;  // row within its chunk
    const int rows = pb.hdr[sp.chunked ? row / SMALL_M : 0].rows;
    if (bout && sp.chunked) bout += (row / SMALL_M) * sp.cs_bout;
    bool valid = crow < rows;
    RowDesc rd = {};
    if (valid) {
        rd = pb.row[row];
        valid = rd.pos >= 0 && rd.pos < kv.max_pos && (unsigned)rd.seq < (unsigned)MAX_SEQS;
    }
    const int visible = valid ? rd.pos + 1 : 0;
    const int npages = (visible + PAGE - 1) / PAGE;
    // Position splits (blockIdx.z): a row whose context spans more than one
    // window of ATT_WIN pages takes one CTA per window, up to sp.zmax CTAs
    // (past that each CTA takes consecutive windows), and the last of them
    // to finish merges their partial softmax sums in CTA order; a row
    // within one window is done by CTA z = 0 alone, as a whole.  The split
    // depends only on the row's position and sp.zmax, which every pass of a
    // kind shares; the host sizes every grid for its pass's longest row (a
    // grid too small for a row, which no launch here makes, falls back to
    // CTA z = 0 doing every window).
    const int nwin = max(1, (npages + ATT_WIN - 1) / ATT_WIN);
    const int wpc = (nwin + sp.zmax - 1) / sp.zmax;  // consecutive windows per CTA (1 up to zmax windows)
    const int need = (nwin + wpc - 1) / wpc;
    const int nsplit = need <= (int)gridDim.z ? need : 1;
    const int zs = blockIdx.z;
    if (zs >= (valid ? nsplit : 1)) return;  // uniform over the CTA
    const int w_lo = nsplit > 1 ? zs * wpc * ATT_WIN : 0;
    const int w_hi = nsplit > 1 ? min(npages, w_lo + wpc * ATT_WIN) : npages;
    const int32_t* pt = valid ? pb.page_table[rd.seq] : nullptr;
    if (valid && threadIdx.x == 0) {
        ptx::mbar_init(&bar, 1);
        ptx::fence_barrier_init();
    }
    auto issue_window = [&](int w0) {  // thread 0: copy pages w0 .. w0+ATT_WIN-1
        const int wn = min(ATT_WIN, npages - w0);
        uint32_t bytes = 0;
        int pg[ATT_WIN];
        for (int i = 0; i < wn; ++i) {
            pg[i] = pt[w0 + i];
            if (!page_ok(kv, pg[i])) pg[i] = -1;
            else bytes += 2 * PB;
            page_s[i] = pg[i];
        }
        ptx::mbar_arrive_expect_tx(&bar, bytes);
        for (int i = 0; i < wn; ++i) {
            if (pg[i] < 0) continue;
            const size_t off = kv_index(pg[i], kvh, 0, kv.kv_heads) * (F32 ? 4 : 2);
            ptx::bulk_g2s(kvs + (2 * i) * PB, (const uint8_t*)kv.k + off, PB, &bar);
            ptx::bulk_g2s(kvs + (2 * i + 1) * PB, (const uint8_t*)kv.v + off, PB, &bar);
        }
    };
    if (valid && threadIdx.x == 0) issue_window(w_lo);
    // RAW: the norm weights, rotation factors, this pass's row descriptors
    // and the row's cache page, all fixed before the pass began
    NormRope qnr = {}, knr = {};
    RowDesc rj = {};
    bool kgood = false;
    int kpage = -1;
    if (RAW && valid) {
        if (sub == 0) qnr = norm_rope_args(raw.qn, raw.rope, rd.pos, lane);
        if (warp <= row && warp < 2) {
            rj = pb.row[warp];
            kgood = rj.pos >= 0 && rj.pos < kv.max_pos && rj.seq == rd.seq;
            knr = norm_rope_args(raw.kn, raw.rope, kgood ? rj.pos : 0, lane);
            if (warp == row && kgood && zs == nsplit - 1) kpage = pt[rj.pos / PAGE];
        }
    }
    // Not RAW: this pass wrote the K/V of the sequence's rows just before
    // this one (`back` of them, at consecutive positions) and of this row;
    // the page of the position this warp re-fetches after the wait
    // (position pos - back + warp).
    int back = 0;
    if (!RAW && valid) {
        for (int base = 0; base < row; base += 32) {
            const int r = row - 1 - base - lane;
            bool same = false;
            if (r >= 0) {
                const RowDesc q = pb.row[r];
                same = q.seq == rd.seq && q.pos == rd.pos - (row - r);
            }
            const unsigned stop = __ballot_sync(0xffffffffu, !same);
            if (stop) {
                back = base + __ffs(stop) - 1;
                break;
            }
            back = base + 32;
        }
        back = min(back, row);
    }
    int own_p = -1, own_pg = -1;
    if (!RAW && valid && warp <= back && rd.pos - back + warp >= 0) {
        own_p = rd.pos - back + warp;
        own_pg = pt[own_p / PAGE];
    }
    __syncthreads();  // the barrier is initialised before anyone waits on it
    ptx::grid_dependency_wait();
    if (threadIdx.x == 0) tl_stamp(sp.tl, 1);
    ptx::launch_dependents();
    if (crow < rows && !valid && sub == 0) {  // uniform over the CTA
        if (threadIdx.x == 0) atomicOr(kv.err, 2);
        *(float4*)(out + (size_t)row * out_ld + h * HEAD + 4 * lane) = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    if (!valid) {
        if (bout && sub == 0) mx::emit_pieces_smem(qw, HEAD, 4, crow, 0, 1, lane, 32, h * HEAD, bN, bout);
        return;
    }
    if (RAW) {
        if (sub == 0) {
            const float* qr = qkv + (size_t)row * ld + h * HEAD;
            float a0 = qr[lane], a1 = qr[lane + 32], a2 = qr[lane + 64], a3 = qr[lane + 96];
            norm_rope4(a0, a1, a2, a3, qnr);
            qw[lane] = a0; qw[lane + 32] = a1; qw[lane + 64] = a2; qw[lane + 96] = a3;
        }
        if (warp <= row && warp < 2) {  // row j = warp of this pass (same sequence)
            const int j = warp;
            const bool good = kgood;
            const float* kr = qkv + (size_t)j * ld + raw.k_off + kvh * HEAD;
            const float* vr = qkv + (size_t)j * ld + raw.v_off + kvh * HEAD;
            float k0 = kr[lane], k1 = kr[lane + 32], k2 = kr[lane + 64], k3 = kr[lane + 96];
            const float v0 = vr[lane], v1 = vr[lane + 32], v2 = vr[lane + 64], v3 = vr[lane + 96];
            norm_rope4(k0, k1, k2, k3, knr);
            nk[j][lane] = k0; nk[j][lane + 32] = k1; nk[j][lane + 64] = k2; nk[j][lane + 96] = k3;
            nv[j][lane] = v0; nv[j][lane + 32] = v1; nv[j][lane + 64] = v2; nv[j][lane + 96] = v3;
            if (lane == 0) npos[j] = good ? rj.pos : -1;
            if (j == row && good && zs == nsplit - 1) {  // the row's own K/V go to the cache (once)
                const int pg = kpage;
                if (page_ok(kv, pg)) {
                    const size_t idx = kv_index(pg, kvh, rj.pos % PAGE, kv.kv_heads);
                    if (F32) {
                        float* dk = (float*)kv.k + idx;
                        float* dv = (float*)kv.v + idx;
                        dk[lane] = k0; dk[lane + 32] = k1; dk[lane + 64] = k2; dk[lane + 96] = k3;
                        dv[lane] = v0; dv[lane + 32] = v1; dv[lane + 64] = v2; dv[lane + 96] = v3;
                    } else {
                        uint16_t* dk = (uint16_t*)kv.k + idx;
                        uint16_t* dv = (uint16_t*)kv.v + idx;
                        dk[lane] = f2bf16(k0); dk[lane + 32] = f2bf16(k1);
                        dk[lane + 64] = f2bf16(k2); dk[lane + 96] = f2bf16(k3);
                        dv[lane] = f2bf16(v0); dv[lane + 32] = f2bf16(v1);
                        dv[lane + 64] = f2bf16(v2); dv[lane + 96] = f2bf16(v3);
                    }
                }
            }
        }
        __syncthreads();  // nk, nv, npos
    } else if (sub == 0) {
        *(float4*)(qw + 4 * lane) = *(const float4*)(qkv + (size_t)row * ld + h * HEAD + 4 * lane);
    }
    if (threadIdx.x == 0) tl_stamp(sp.tl, 2);
    const float scale = sqrtf(128.0f);
    float m = -INFINITY, l = 0.f;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    bool ok = true;
    for (int w0 = w_lo, it = 0; w0 < w_hi; w0 += ATT_WIN, ++it) {
        const int wn = min(ATT_WIN, npages - w0);
        if (threadIdx.x == 0 && w0 > w_lo) issue_window(w0);
        if (!ptx::mbar_wait(&bar, it & 1, ATT_WAIT)) ok = false;
        if (RAW) {
            // this pass's rows (computed above, in the cache's element type)
            // over the early copy
            for (int j = warp; j <= row && j < 2; j += nw) {
                const int p = npos[j];
                const int i = p / PAGE - w0;
                if (p < 0 || i < 0 || i >= wn) continue;
                const size_t at = (size_t)(p % PAGE) * HEAD;
                for (int d = lane; d < HEAD; d += 32) {
                    if (F32) {
                        ((float*)(kvs + (2 * i) * PB))[at + d] = nk[j][d];
                        ((float*)(kvs + (2 * i + 1) * PB))[at + d] = nv[j][d];
                    } else {
                        ((uint16_t*)(kvs + (2 * i) * PB))[at + d] = f2bf16(nk[j][d]);
                        ((uint16_t*)(kvs + (2 * i + 1) * PB))[at + d] = f2bf16(nv[j][d]);
                    }
                }
            }
        } else {
        // The q|k|v kernel of this pass wrote this row's K/V and those of the
        // pass's earlier rows of the sequence (`back` positions back): fetch
        // them again over the early copy.
            constexpr int RB = HEAD * (F32 ? 4 : 2);  // bytes of one row: 256 or 512
            const int lo = max(rd.pos - back, w0 * PAGE), hi = min(rd.pos, (w0 + wn) * PAGE - 1);
            for (int p = lo + warp; p <= hi; p += nw) {
                const int pg = p == own_p ? own_pg : pt[p / PAGE];
                if ((unsigned)pg >= (unsigned)kv.pages) continue;  // flagged when the window was copied
                const int i = p / PAGE - w0;
                const size_t src = kv_index(pg, kvh, p % PAGE, kv.kv_heads) * (F32 ? 4 : 2);
                const size_t dst = (size_t)(p % PAGE) * RB;
                for (int o = lane * 16; o < RB; o += 32 * 16) {
                    *(uint4*)(kvs + (2 * i) * PB + dst + o) = *(const uint4*)((const uint8_t*)kv.k + src + o);
                    *(uint4*)(kvs + (2 * i + 1) * PB + dst + o) = *(const uint4*)((const uint8_t*)kv.v + src + o);
                }
            }
        }
        __syncthreads();  // page_s and the fresh rows are visible
        if (ok) {
            for (int i = 0; i < wn; ++i) {
                if (page_s[i] < 0) continue;  // flagged: its positions are left out
                const uint8_t* Ks = kvs + (2 * i) * PB;
                const uint8_t* Vs = kvs + (2 * i + 1) * PB;
                for (int half = 0; half < PAGE / 32; ++half) {
                    const int c0 = (w0 + i) * PAGE + half * 32;
                    if (c0 >= visible) break;
                    if ((c0 / 32) % split != sub) continue;  // another warp's chunk
                    const int r = half * 32 + lane;  // row of this lane's position in the page
                    float sc = -INFINITY;
                    if (c0 + lane < visible) {
                        float dot = 0.f;
                        if (F32) {
                            const float4* kr = (const float4*)(Ks + (size_t)r * HEAD * 4);
#pragma unroll 8
                            for (int c = 0; c < 32; ++c) {
                                const int cc = (c + lane) & 31;
                                const float4 k4 = kr[cc];
                                const float4 q4 = *(const float4*)(qw + 4 * cc);
                                dot = fmaf(q4.x, k4.x, dot);
                                dot = fmaf(q4.y, k4.y, dot);
                                dot = fmaf(q4.z, k4.z, dot);
                                dot = fmaf(q4.w, k4.w, dot);
                            }
                        } else {
                            const uint4* kr = (const uint4*)(Ks + (size_t)r * HEAD * 2);
#pragma unroll 4
                            for (int c = 0; c < 16; ++c) {
                                const int cc = (c + lane) & 15;
                                const uint4 k8 = kr[cc];
                                const float4 qa = *(const float4*)(qw + 8 * cc);
                                const float4 qb = *(const float4*)(qw + 8 * cc + 4);
                                dot = fmaf(qa.x, __uint_as_float(k8.x << 16), dot);
                                dot = fmaf(qa.y, __uint_as_float(k8.x & 0xffff0000u), dot);
                                dot = fmaf(qa.z, __uint_as_float(k8.y << 16), dot);
                                dot = fmaf(qa.w, __uint_as_float(k8.y & 0xffff0000u), dot);
                                dot = fmaf(qb.x, __uint_as_float(k8.z << 16), dot);
                                dot = fmaf(qb.y, __uint_as_float(k8.z & 0xffff0000u), dot);
                                dot = fmaf(qb.z, __uint_as_float(k8.w << 16), dot);
                                dot = fmaf(qb.w, __uint_as_float(k8.w & 0xffff0000u), dot);
                            }
                        }
                        sc = __fdiv_rn(dot, scale);
                    }
                    const float cmax = warp_max(sc);
                    const float nm = fmaxf(m, cmax);
                    const float corr = nm == -INFINITY ? 1.f : expf(m - nm);
                    const float p = sc == -INFINITY ? 0.f : expf(sc - nm);
                    l = fmaf(l, corr, warp_sum(p));
#pragma unroll
                    for (int d = 0; d < 4; ++d) acc[d] *= corr;
                    m = nm;
                    const int n = min(32, visible - c0);
#pragma unroll 8
                    for (int jj = 0; jj < n; ++jj) {
                        const float pj = __shfl_sync(0xffffffffu, p, jj);
                        const int vr = half * 32 + jj;
                        float v[4];
                        if (F32) {
                            const float4 v4 = *(const float4*)(Vs + ((size_t)vr * HEAD + 4 * lane) * 4);
                            v[0] = v4.x; v[1] = v4.y; v[2] = v4.z; v[3] = v4.w;
                        } else {
                            const uint2 v2 = *(const uint2*)(Vs + ((size_t)vr * HEAD + 4 * lane) * 2);
                            v[0] = __uint_as_float(v2.x << 16);
                            v[1] = __uint_as_float(v2.x & 0xffff0000u);
                            v[2] = __uint_as_float(v2.y << 16);
                            v[3] = __uint_as_float(v2.y & 0xffff0000u);
                        }
#pragma unroll
                        for (int d = 0; d < 4; ++d) acc[d] = fmaf(pj, v[d], acc[d]);
                    }
                }
            }
        }
        if (w0 + ATT_WIN < w_hi) __syncthreads();  // the window is free for the next copy (uniform)
    }
    if (!ok && threadIdx.x == 0) atomicOr(kv.err, 4);  // a page copy did not arrive in time
    if (threadIdx.x == 0) tl_stamp(sp.tl, 3);
    // merge the head's warps in warp order
    if (lane == 0) {
        cm[warp] = m;
        cl[warp] = l;
    }
    *(float4*)(&cacc[warp][4 * lane]) = make_float4(acc[0], acc[1], acc[2], acc[3]);
    __syncthreads();
    // merge the head's warps in warp order (sub == 0 warps)
    float M = -INFINITY, L = 0.f, o[4] = {0.f, 0.f, 0.f, 0.f};
    if (sub == 0) {
        for (int s2 = 0; s2 < split; ++s2) M = fmaxf(M, cm[s2 * group + hw]);
        for (int s2 = 0; s2 < split; ++s2) {
            const int w2 = s2 * group + hw;
            if (cm[w2] == -INFINITY) continue;  // no position fell to that warp
            const float f = expf(cm[w2] - M);
            L = fmaf(cl[w2], f, L);
            const float4 a4 = *(const float4*)(&cacc[w2][4 * lane]);
            o[0] = fmaf(a4.x, f, o[0]);
            o[1] = fmaf(a4.y, f, o[1]);
            o[2] = fmaf(a4.z, f, o[2]);
            o[3] = fmaf(a4.w, f, o[3]);
        }
    }
    if (nsplit > 1) {
        // publish this window's (max, sum, unnormalised output) per head;
        // the last window CTA of the row to arrive merges them all
        __shared__ int last_s;
        float* part = sp.ws + (((size_t)(g * gridDim.y + row) * gridDim.z) * group) * ATT_PART;
        if (sub == 0) {
            float* P = part + ((size_t)zs * group + hw) * ATT_PART;
            if (lane == 0) {
                P[0] = M;
                P[1] = L;
            }
            *(float4*)(P + 4 + 4 * lane) = make_float4(o[0], o[1], o[2], o[3]);
        }
        __threadfence();
        __syncthreads();
        if (threadIdx.x == 0) {
            int* cnt = sp.cnt + g * gridDim.y + row;
            const int t = atomicAdd(cnt, 1);
            last_s = t == nsplit - 1;
            if (last_s) *cnt = 0;  // every window has arrived: ready for the next pass
        }
        __syncthreads();
        if (!last_s) return;
        __threadfence();  // the other windows' partials are visible
        if (sub != 0) return;
        // Lane z (and z + 32) fetches window z's max and sum, so those loads
        // go out together; the sums then run in window order through
        // shuffles, the output loads several windows at a time.
        static_assert(ATT_ZMAX <= 64, "two windows per lane");
        float mz_l[2], lz_l[2], f_l[2];
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int z = lane + 32 * i;
            const float* P = part + ((size_t)z * group + hw) * ATT_PART;
            mz_l[i] = z < nsplit ? __ldcg(P) : -INFINITY;
            lz_l[i] = z < nsplit ? __ldcg(P + 1) : 0.f;
        }
        M = warp_max(fmaxf(mz_l[0], mz_l[1]));
#pragma unroll
        for (int i = 0; i < 2; ++i) f_l[i] = mz_l[i] == -INFINITY ? 0.f : expf(mz_l[i] - M);
        L = 0.f;
        o[0] = o[1] = o[2] = o[3] = 0.f;
        constexpr int ZB = F32 && RAW ? 2 : 4;  // windows per batch of loads (registers of the f32 raw variant)
        for (int z0 = 0; z0 < nsplit; z0 += ZB) {
            float4 a4[ZB];
#pragma unroll
            for (int j = 0; j < ZB; ++j) {
                const int z = z0 + j;
                a4[j] = z < nsplit ? __ldcg((const float4*)(part + ((size_t)z * group + hw) * ATT_PART + 4 + 4 * lane))
                                   : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int j = 0; j < ZB; ++j) {
                const int z = z0 + j;
                if (z >= nsplit) break;
                const float mz = __shfl_sync(0xffffffffu, z < 32 ? mz_l[0] : mz_l[1], z & 31);
                const float f = __shfl_sync(0xffffffffu, z < 32 ? f_l[0] : f_l[1], z & 31);
                const float lz = __shfl_sync(0xffffffffu, z < 32 ? lz_l[0] : lz_l[1], z & 31);
                if (mz == -INFINITY) continue;  // a window whose pages were all flagged
                L = fmaf(lz, f, L);
                o[0] = fmaf(a4[j].x, f, o[0]);
                o[1] = fmaf(a4[j].y, f, o[1]);
                o[2] = fmaf(a4[j].z, f, o[2]);
                o[3] = fmaf(a4[j].w, f, o[3]);
            }
        }
    }
    if (sub != 0) return;
#pragma unroll
    for (int d = 0; d < 4; ++d) o[d] = __fdiv_rn(o[d], L);
    *(float4*)(out + (size_t)row * out_ld + h * HEAD + 4 * lane) = make_float4(o[0], o[1], o[2], o[3]);
    if (threadIdx.x == 0) tl_stamp(sp.tl, 4);
    if (bout) {
        __syncwarp();  // every lane has finished reading q
        *(float4*)(qw + 4 * lane) = make_float4(o[0], o[1], o[2], o[3]);
        __syncwarp();
        mx::emit_pieces_smem(qw, HEAD, 4, crow, 1, 1, lane, 32, h * HEAD, bN, bout);
        if (threadIdx.x == 0) tl_stamp(sp.tl, 5);
    }
}

// Prefill attention (lib.rs:401-441) for a multi-chunk pass whose rows are
// one sequence at consecutive positions, as predict builds them: a CTA per
// (KV head, PF_ROWS rows) streams the sequence's K/V pages once through
// shared memory (two page buffers) for all its rows x `group` query heads.
// Each (row, head) pair belongs to one warp, which keeps its running max and
// sum over the pages in order: lanes score positions lane and lane + 32 of a
// page (causal per row), then own 4 of the 128 output dimensions; a warp
// keeps NP = group / 2 pairs (group <= 8).  The output goes out as in
// k_attn_decode: f32 rows and the o projection's pieces.
constexpr int PF_ROWS = 8;
constexpr int PF_WARPS = 16;
__host__ __device__ constexpr size_t pf_smem(int f32, int group) {
    return 4 * (size_t)att_page_bytes(f32) + (size_t)PF_ROWS * group * HEAD * 4 + PF_WARPS * HEAD * 4;
}

template <int F32, int NP>
__global__ void __launch_bounds__(PF_WARPS * 32) k_attn_prefill(PassBuf pb, const float* __restrict__ qkv, int ld,
                                                               int group, KvView kv, float* __restrict__ out,
                                                               int out_ld, uint8_t* __restrict__ bout, int bN,
                                                               size_t cs_bout) {
    constexpr int PB = att_page_bytes(F32);
    extern __shared__ __align__(128) uint8_t pf[];  // [2 buffers][K|V][PB], q [pairs][HEAD], o [warps][HEAD]
    float* qs = (float*)(pf + 4 * PB);
    float* os = qs + PF_ROWS * group * HEAD;
    __shared__ uint64_t bar[2];
    __shared__ int page_s[2];
    const int g = blockIdx.x, r0 = blockIdx.y * PF_ROWS;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int chunk = r0 / SMALL_M, lr0 = r0 % SMALL_M;
    if (bout) bout += chunk * cs_bout;
    if (threadIdx.x == 0) {
        ptx::mbar_init(&bar[0], 1);
        ptx::mbar_init(&bar[1], 1);
        ptx::fence_barrier_init();
    }
    __syncthreads();
    ptx::grid_dependency_wait();  // q and this pass's K/V come from the q|k|v kernel
    ptx::launch_dependents();
    const int rows = pb.hdr[chunk].rows;
    const RowDesc first = pb.row[r0];
    const bool seq_ok = lr0 < rows && (unsigned)first.seq < (unsigned)MAX_SEQS;
    const int32_t* pt = seq_ok ? pb.page_table[first.seq] : nullptr;
    // live rows of this CTA: the same sequence at consecutive positions
    int nlive = 0, last_pos = -1;
    for (int i = 0; i < PF_ROWS && lr0 + i < rows; ++i) {
        const RowDesc rd = pb.row[r0 + i];
        if (!seq_ok || rd.seq != first.seq || rd.pos != first.pos + i || rd.pos < 0 || rd.pos >= kv.max_pos) {
            if (threadIdx.x == 0) atomicOr(kv.err, 2);
            break;
        }
        nlive = i + 1;
        last_pos = rd.pos;
    }
    const int pairs = PF_ROWS * group;
    // q of every live pair (QK-normalised and rotated by the q|k|v kernel)
    for (int i = threadIdx.x; i < pairs * (HEAD / 4); i += blockDim.x) {
        const int pr = i / (HEAD / 4), d4 = i % (HEAD / 4);
        const int r = pr / group, h = g * group + pr % group;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (r < nlive) v = *(const float4*)(qkv + (size_t)(r0 + r) * ld + h * HEAD + 4 * d4);
        *(float4*)(qs + (size_t)pr * HEAD + 4 * d4) = v;
    }
    const int npages = nlive ? last_pos / PAGE + 1 : 0;
    __syncthreads();  // every pair's q is in shared memory
    auto issue = [&](int p) {  // thread 0: K and V of page p into buffer p & 1
        const int pg = pt[p];
        const int b = p & 1;
        page_s[b] = page_ok(kv, pg) ? pg : -1;
        if (page_s[b] < 0) {
            ptx::mbar_arrive(&bar[b]);
            return;
        }
        ptx::mbar_arrive_expect_tx(&bar[b], 2 * PB);
        const size_t off = kv_index(pg, g, 0, kv.kv_heads) * (F32 ? 4 : 2);
        ptx::bulk_g2s(pf + (2 * b) * PB, (const uint8_t*)kv.k + off, PB, &bar[b]);
        ptx::bulk_g2s(pf + (2 * b + 1) * PB, (const uint8_t*)kv.v + off, PB, &bar[b]);
    };
    if (threadIdx.x == 0 && npages > 0) issue(0);
    float m[NP], l[NP], acc[NP][4];
#pragma unroll
    for (int j = 0; j < NP; ++j) {
        m[j] = -INFINITY;
        l[j] = 0.f;
        acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
    }
    const float scale = sqrtf(128.0f);
    bool ok = true;
    for (int p = 0; p < npages; ++p) {
        const int b = p & 1;
        if (threadIdx.x == 0 && p + 1 < npages) issue(p + 1);  // the other buffer was freed below
        if (!ptx::mbar_wait(&bar[b], (p >> 1) & 1, ATT_WAIT)) ok = false;
        if (page_s[b] >= 0) {
            const uint8_t* Ks = pf + (2 * b) * PB;
            const uint8_t* Vs = pf + (2 * b + 1) * PB;
#pragma unroll
            for (int j = 0; j < NP; ++j) {
                const int pr = warp + j * PF_WARPS;
                const int r = pr / group;
                if (pr >= pairs || r >= nlive) continue;  // uniform over the warp
                const int vis = first.pos + r + 1 - p * PAGE;  // positions of this page the row sees
                if (vis <= 0) continue;
                const float* qw = qs + (size_t)pr * HEAD;
                float sc[2];
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    const int t = lane + 32 * half;
                    float d[4] = {0.f, 0.f, 0.f, 0.f};  // four chains, summed at the end
                    if (F32) {
                        const float4* kr = (const float4*)(Ks + (size_t)t * HEAD * 4);
#pragma unroll 8
                        for (int c = 0; c < 32; ++c) {
                            const int cc = (c + lane) & 31;
                            const float4 k4 = kr[cc];
                            const float4 q4 = *(const float4*)(qw + 4 * cc);
                            d[0] = fmaf(q4.x, k4.x, d[0]);
                            d[1] = fmaf(q4.y, k4.y, d[1]);
                            d[2] = fmaf(q4.z, k4.z, d[2]);
                            d[3] = fmaf(q4.w, k4.w, d[3]);
                        }
                    } else {
                        const uint4* kr = (const uint4*)(Ks + (size_t)t * HEAD * 2);
#pragma unroll 4
                        for (int c = 0; c < 16; ++c) {
                            const int cc = (c + lane) & 15;
                            const uint4 k8 = kr[cc];
                            const float4 qa = *(const float4*)(qw + 8 * cc);
                            const float4 qb = *(const float4*)(qw + 8 * cc + 4);
                            d[0] = fmaf(qa.x, __uint_as_float(k8.x << 16), d[0]);
                            d[1] = fmaf(qa.y, __uint_as_float(k8.x & 0xffff0000u), d[1]);
                            d[2] = fmaf(qa.z, __uint_as_float(k8.y << 16), d[2]);
                            d[3] = fmaf(qa.w, __uint_as_float(k8.y & 0xffff0000u), d[3]);
                            d[0] = fmaf(qb.x, __uint_as_float(k8.z << 16), d[0]);
                            d[1] = fmaf(qb.y, __uint_as_float(k8.z & 0xffff0000u), d[1]);
                            d[2] = fmaf(qb.z, __uint_as_float(k8.w << 16), d[2]);
                            d[3] = fmaf(qb.w, __uint_as_float(k8.w & 0xffff0000u), d[3]);
                        }
                    }
                    const float dot = __fadd_rn(__fadd_rn(d[0], d[1]), __fadd_rn(d[2], d[3]));
                    sc[half] = t < vis ? __fdiv_rn(dot, scale) : -INFINITY;
                }
                const float nm = fmaxf(m[j], warp_max(fmaxf(sc[0], sc[1])));
                const float corr = m[j] == -INFINITY ? 0.f : expf(m[j] - nm);
                const float p0 = sc[0] == -INFINITY ? 0.f : expf(sc[0] - nm);
                const float p1 = sc[1] == -INFINITY ? 0.f : expf(sc[1] - nm);
                l[j] = fmaf(l[j], corr, warp_sum(p0 + p1));
#pragma unroll
                for (int d = 0; d < 4; ++d) acc[j][d] *= corr;
                m[j] = nm;
                const int n = min(PAGE, vis);
                // the page's weights go through this warp's row of shared
                // memory: each lane then reads them as broadcasts
                float* pw = os + (size_t)warp * HEAD;
                __syncwarp();
                pw[lane] = p0;
                pw[lane + 32] = p1;
                __syncwarp();
#pragma unroll 8
                for (int t = 0; t < n; ++t) {
                    const float pt_ = pw[t];
                    float v[4];
                    if (F32) {
                        const float4 v4 = *(const float4*)(Vs + ((size_t)t * HEAD + 4 * lane) * 4);
                        v[0] = v4.x; v[1] = v4.y; v[2] = v4.z; v[3] = v4.w;
                    } else {
                        const uint2 v2 = *(const uint2*)(Vs + ((size_t)t * HEAD + 4 * lane) * 2);
                        v[0] = __uint_as_float(v2.x << 16);
                        v[1] = __uint_as_float(v2.x & 0xffff0000u);
                        v[2] = __uint_as_float(v2.y << 16);
                        v[3] = __uint_as_float(v2.y & 0xffff0000u);
                    }
#pragma unroll
                    for (int d = 0; d < 4; ++d) acc[j][d] = fmaf(pt_, v[d], acc[j][d]);
                }
            }
        }
        __syncthreads();  // buffer b is free for page p + 2
    }
    if (!ok && threadIdx.x == 0) atomicOr(kv.err, 4);  // a page copy did not arrive in time
    // outputs: f32 rows, then the o projection's pieces (zero for dead rows)
#pragma unroll
    for (int j = 0; j < NP; ++j) {
        const int pr = warp + j * PF_WARPS;
        if (pr >= pairs) continue;
        const int r = pr / group, h = g * group + pr % group;
        if (lr0 + r >= SMALL_M) continue;
        const bool live = r < nlive && l[j] > 0.f;
        float o[4];
#pragma unroll
        for (int d = 0; d < 4; ++d) o[d] = live ? __fdiv_rn(acc[j][d], l[j]) : 0.f;
        if (lr0 + r < rows) *(float4*)(out + (size_t)(r0 + r) * out_ld + h * HEAD + 4 * lane) = make_float4(o[0], o[1], o[2], o[3]);
        if (bout) {
            float* ow = os + (size_t)warp * HEAD;
            __syncwarp();
            *(float4*)(ow + 4 * lane) = make_float4(o[0], o[1], o[2], o[3]);
            __syncwarp();
            mx::emit_pieces_smem(ow, HEAD, 4, lr0 + r, 1, 1, lane, 32, h * HEAD, bN, bout);
        }
    }
}

// First maximum of each predicted row, ties to the lower index
// (model.rs:288-296, gpu.metal:176-212).
__global__ void __launch_bounds__(1024) k_argmax(PassBuf pb, const float* __restrict__ logits,
                                                 int vocab) {
    __shared__ float bv[32];
    __shared__ uint32_t bi[32];
    ptx::grid_dependency_wait();  // PDL: the previous kernel's writes are visible past here
    ptx::launch_dependents();
    const int r = blockIdx.x;
    if (r >= pb.hdr->head_rows) return;
    const float* x = logits + (size_t)r * vocab;
    float best = -INFINITY;
    uint32_t idx = 0xffffffffu;
    for (int i = threadIdx.x; i < vocab; i += blockDim.x) {
        const float v = x[i];
        if (v > best) { best = v; idx = i; }
    }
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_down_sync(0xffffffffu, best, o);
        const uint32_t oi = __shfl_down_sync(0xffffffffu, idx, o);
        if (ov > best || (ov == best && oi < idx)) { best = ov; idx = oi; }
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) { bv[warp] = best; bi[warp] = idx; }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
            if (bv[w] > best || (bv[w] == best && bi[w] < idx)) { best = bv[w]; idx = bi[w]; }
        pb.out_ids[r] = idx == 0xffffffffu ? 0u : idx;
    }
}

// ---------------------------------------------------------------------------
// Seeded synthetic weights: Philox4x32-10 (Salmon et al., SC'11) keyed by the
// model seed, counter (group, tensor index); Box-Muller in double precision;
// 0.02 * z rounded to f32, then to bf16.

__device__ __forceinline__ void philox10(uint32_t c[4], uint32_t k0, uint32_t k1) {
#pragma unroll
    for (int r = 0; r < 10; ++r) {
        if (r) { k0 += 0x9E3779B9u; k1 += 0xBB67AE85u; }
        const uint32_t hi0 = __umulhi(0xD2511F53u, c[0]), lo0 = 0xD2511F53u * c[0];
        const uint32_t hi1 = __umulhi(0xCD9E8D57u, c[2]), lo1 = 0xCD9E8D57u * c[2];
        const uint32_t n0 = hi1 ^ c[1] ^ k0, n2 = hi0 ^ c[3] ^ k1;
        c[0] = n0; c[1] = lo1; c[2] = n2; c[3] = lo0;
    }
}

__global__ void k_synth(uint64_t seed, uint32_t tensor, size_t n, uint16_t* __restrict__ out) {
    const double two_pi = 6.283185307179586476925286766559;
    const double inv32 = 1.0 / 4294967296.0;
    const uint32_t k0 = (uint32_t)seed ^ (uint32_t)(seed >> 32);
    const size_t groups = (n + 3) / 4;
    for (size_t g = blockIdx.x * (size_t)blockDim.x + threadIdx.x; g < groups;
         g += (size_t)gridDim.x * blockDim.x) {
        uint32_t c[4] = {(uint32_t)g, (uint32_t)(g >> 32), tensor, 0x6a616c61u};
        philox10(c, k0, 0x70656e6fu);
        const double u0 = ((double)c[0] + 0.5) * inv32, u1 = ((double)c[1] + 0.5) * inv32;
        const double u2 = ((double)c[2] + 0.5) * inv32, u3 = ((double)c[3] + 0.5) * inv32;
        const double a = sqrt(-2.0 * log(u0)), b = sqrt(-2.0 * log(u2));
        const double z[4] = {a * cos(two_pi * u1), a * sin(two_pi * u1), b * cos(two_pi * u3),
                             b * sin(two_pi * u3)};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const size_t e = g * 4 + j;
            if (e < n) out[e] = f2bf16((float)(0.02 * z[j]));
        }
    }
}

__global__ void k_fill_u16(uint16_t* out, size_t n, uint16_t v) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        out[i] = v;
}

// MXFP4 quantization of bf16 weights, one 32-block per thread.  Same steps as
// python/quantize_mxfp4.py:26-38: exponent = frexp(max|v|) - 3 clipped to
// [-127, 127] (-127 for an all-zero block), codes by nearest level with ties
// to the even code, sign in bit 3, even element in the low nibble.
__global__ void k_quantize(const uint16_t* __restrict__ in, size_t blocks, uint8_t* __restrict__ packed,
                           uint8_t* __restrict__ scales) {
    const float mid[7] = {0.25f, 0.75f, 1.25f, 1.75f, 2.5f, 3.5f, 5.0f};
    for (size_t b = blockIdx.x * (size_t)blockDim.x + threadIdx.x; b < blocks;
         b += (size_t)gridDim.x * blockDim.x) {
        const uint16_t* v = in + b * 32;
        float mx = 0.f;
        for (int i = 0; i < 32; ++i) mx = fmaxf(mx, fabsf(bf16f(v[i])));
        int e;
        frexpf(mx, &e);
        int ex = e - 3;
        ex = ex < -127 ? -127 : (ex > 127 ? 127 : ex);
        if (mx == 0.f) ex = -127;
        uint8_t* p = packed + b * 16;
        for (int j = 0; j < 16; ++j) {
            uint32_t codes[2];
            for (int h = 0; h < 2; ++h) {
                const float f = bf16f(v[2 * j + h]);
                const float sc = ldexpf(fabsf(f), -ex);
                uint32_t c = 0;
                while (c < 7 && mid[c] < sc) ++c;
                if ((c & 1u) && sc == mid[c < 6 ? c : 6]) c += 1;
                if (signbit(f)) c |= 8u;
                codes[h] = c;
            }
            p[j] = (uint8_t)(codes[0] | (codes[1] << 4));
        }
        scales[b] = (uint8_t)(ex + 127);
    }
}

// ---------------------------------------------------------------------------
// launch helpers

int sm_count() {
    static int n = 0;
    if (!n) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) n = 148;
    }
    return n;
}

Proj make_proj(std::initializer_list<const Mat*> mats) {
    Proj p{};
    int i = 0;
    for (const Mat* m : mats) {
        p.w[i] = m->data;
        p.s[i] = m->scales;
        p.n[i] = m->rows;
        p.K = m->cols;
        p.total += m->rows;
        ++i;
    }
    for (; i < 3; ++i) { p.w[i] = nullptr; p.s[i] = nullptr; p.n[i] = 0; }
    return p;
}

template <int KIND, int EPI, int R, int MR>
jl_status run_skinny(const PassCtx& c, int use_head, const float* x, int ldx, const Proj& p,
                     float* y, int ldy) {
    auto kern = k_skinny<KIND, EPI, R, MR>;
    const size_t smem = (size_t)MR * p.K * sizeof(float);
    const int groups = (p.total + R - 1) / R;
    const int per_sm = smem <= 48 * 1024 ? 4 : (smem <= 100 * 1024 ? 2 : 1);
    int grid = std::min((groups + 7) / 8, sm_count() * per_sm);
    grid = std::max(grid, 1);
    return launch_pdl(kern, dim3(grid), dim3(256), smem, c.stream, (const PassHdr*)c.pass().hdr, use_head,
                      c.m->max_rows, x, ldx, p, y, ldy);
}

template <int KIND, int EPI>
jl_status run_proj_kind(const PassCtx& c, int use_head, const float* x, int ldx, const Proj& p,
                        float* y, int ldy) {
    const int cap = use_head ? c.head_cap : c.rows_cap;
    if (cap <= SMALL_M) {
        if ((size_t)4 * p.K * sizeof(float) <= 100 * 1024)
            return run_skinny<KIND, EPI, 2, 4>(c, use_head, x, ldx, p, y, ldy);
        return run_skinny<KIND, EPI, 2, 2>(c, use_head, x, ldx, p, y, ldy);
    }
    dim3 grid((p.total + 63) / 64, (cap + 63) / 64);
    return launch_pdl(k_gemm<KIND, EPI>, grid, dim3(256), 0, c.stream, (const PassHdr*)c.pass().hdr,
                      use_head, cap, x, ldx, p, y, ldy);
}

template <int EPI>
jl_status run_proj(const PassCtx& c, int kind, int use_head, const float* x, int ldx,
                   const Proj& p, float* y, int ldy) {
    if (kind == MAT_MXFP4) return run_proj_kind<MAT_MXFP4, EPI>(c, use_head, x, ldx, p, y, ldy);
    return run_proj_kind<MAT_BF16, EPI>(c, use_head, x, ldx, p, y, ldy);
}


template <int KIND, int EPI>
jl_status configure_skinny() {
    JL_CUDA(cudaFuncSetAttribute(k_skinny<KIND, EPI, 2, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 200 * 1024));
    JL_CUDA(cudaFuncSetAttribute(k_skinny<KIND, EPI, 2, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 200 * 1024));
    return JL_OK;
}

}  // namespace

jl_status configure_kernels() {
    int dev = 0;
    JL_CUDA(cudaGetDevice(&dev));
    static bool done[64] = {};
    if (dev < 64 && done[dev]) return JL_OK;
    sm_count();
    JL_TRY((configure_skinny<MAT_BF16, EPI_STORE>()));
    JL_TRY((configure_skinny<MAT_BF16, EPI_ADD>()));
    JL_TRY((configure_skinny<MAT_BF16, EPI_SWIGLU>()));
    JL_TRY((configure_skinny<MAT_MXFP4, EPI_STORE>()));
    JL_TRY((configure_skinny<MAT_MXFP4, EPI_ADD>()));
    JL_TRY((configure_skinny<MAT_MXFP4, EPI_SWIGLU>()));
    JL_CUDA(cudaFuncSetAttribute(k_attn_prefill<0, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pf_smem(0, 8)));
    JL_CUDA(cudaFuncSetAttribute(k_attn_prefill<0, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pf_smem(0, 8)));
    JL_CUDA(cudaFuncSetAttribute(k_attn_prefill<0, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pf_smem(0, 8)));
    JL_CUDA(cudaFuncSetAttribute(k_attn_prefill<1, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pf_smem(1, 8)));
    JL_CUDA(cudaFuncSetAttribute(k_attn_prefill<1, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pf_smem(1, 8)));
    JL_CUDA(cudaFuncSetAttribute(k_attn_prefill<1, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pf_smem(1, 8)));
    JL_CUDA(cudaFuncSetAttribute(k_attn_decode<0, 0>, cudaFuncAttributeMaxDynamicSharedMemorySize, att_smem(0)));
    JL_CUDA(cudaFuncSetAttribute(k_attn_decode<1, 0>, cudaFuncAttributeMaxDynamicSharedMemorySize, att_smem(1)));
    JL_CUDA(cudaFuncSetAttribute(k_attn_decode<0, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, att_smem(0)));
    JL_CUDA(cudaFuncSetAttribute(k_attn_decode<1, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, att_smem(1)));
    JL_TRY(mx_configure());
    JL_TRY(dec_configure());
    JL_TRY(configure_prefill_tc());
    JL_TRY(noalloc_prepare(dev));
    JL_TRY(tl_prepare());
    if (dev < 64) done[dev] = true;
    return JL_OK;
}

jl_status launch_embed(const PassCtx& c) {
    return launch_pdl(k_embed, dim3(c.rows_cap), dim3(256), 0, c.stream, c.pass(), c.m->embed, c.m->s.x,
                      c.m->hidden, c.chunks > 1 ? 1 : 0);
}

jl_status launch_rmsnorm(const PassCtx& c, const float* x, const uint16_t* w, float* out,
                         bool head_rows) {
    const int h = c.m->hidden;
    return launch_pdl(k_rmsnorm, dim3(head_rows ? c.head_cap : c.rows_cap), dim3(256), 0, c.stream,
                      c.pass(), x, h, w, out, h, h, head_rows ? 1 : 0);
}

jl_status launch_qkv(const PassCtx& c, const LayerW& L) {
    if (L.mx_qkv.a && c.rows_cap <= mx_max_tokens())
        return mx_project(c, L.mx_qkv, MXE_STORE, 0, c.m->s.xn, c.m->hidden, nullptr, c.m->s.qkv,
                          qkv_ld(c.m));
    Proj p = make_proj({&L.q, &L.k, &L.v});
    return run_proj<EPI_STORE>(c, L.q.kind, 0, c.m->s.xn, c.m->hidden, p, c.m->s.qkv, qkv_ld(c.m));
}

jl_status launch_qk_rope_kv(const PassCtx& c, int layer, const LayerW& L) {
    return launch_pdl(k_qk_rope_kv, dim3(c.rows_cap), dim3(256), 0, c.stream, c.pass(), c.m->s.qkv,
                      qkv_ld(c.m), c.m->q_heads, L.q_norm, L.k_norm, (const float2*)c.m->rope,
                      kv_view(c.m, layer));
}

// Window CTAs per row in a decode attention launch: what the pass context
// asks for, within the workspace the model holds.
int att_grid_splits(const PassCtx& c) { return std::max(1, std::min(c.att_splits, c.m->att_smax)); }

jl_status launch_attention(const PassCtx& c, int layer, bool pieces) {
    dim3 grid(c.m->q_heads, c.rows_cap);
    const int group = c.m->q_heads / c.m->kv_heads;
    uint8_t* bout = pieces ? c.m->mx.battn : nullptr;
    const bool chunked = c.chunks > 1;
    const int bN = 8 * (chunked ? SMALL_M : c.rows_cap);
    // one sequence's prompt on tensor cores (bf16 pools, groups of 1, 2, 4, 8)
    if (chunked && c.prefill && prefill_tc_supported(c.m)) return launch_attention_prefill_tc(c, layer, bout, bN);
    if (chunked && c.prefill && group <= 8) {  // one sequence's prompt: K/V pages shared by 8 rows
        const dim3 g3(c.m->kv_heads, c.rows_cap / PF_ROWS), blk(PF_WARPS * 32);
        const int qw = c.m->q_heads * HEAD;
        const int f32 = c.m->kv.dtype == JL_KV_F32 ? 1 : 0;
        const int np = group <= 2 ? 1 : group <= 4 ? 2 : 4;  // (row, head) pairs per warp
        auto go = [&](auto kern) {
            return launch_pdl(kern, g3, blk, pf_smem(f32, group), c.stream, c.pass(), (const float*)c.m->s.qkv,
                              qkv_ld(c.m), group, kv_view(c.m, layer), c.m->s.attn, qw, bout, bN, c.m->mx.sattn);
        };
        switch (f32 * 3 + (np == 1 ? 0 : np == 2 ? 1 : 2)) {
            case 0: return go(k_attn_prefill<0, 1>);
            case 1: return go(k_attn_prefill<0, 2>);
            case 2: return go(k_attn_prefill<0, 4>);
            case 3: return go(k_attn_prefill<1, 1>);
            case 4: return go(k_attn_prefill<1, 2>);
            default: return go(k_attn_prefill<1, 4>);
        }
    }
    if ((c.rows_cap <= SMALL_M || chunked) && group <= 8) {  // decode passes: a warp per query head
        const int split = att_split(group);
        // the split workspace holds att_rows rows x att_smax windows (a row
        // whose context needs more CTAs than a grid has is done by one CTA;
        // with at most ATT_ZMAX_DECODE CTAs per row the halving never runs).
        int z = std::min(att_grid_splits(c), ATT_ZMAX_DECODE);
        while (z > 1 && (size_t)c.rows_cap * z > (size_t)c.m->att_rows * c.m->att_smax) z >>= 1;
        const dim3 g2(c.m->kv_heads, c.rows_cap, z), blk(32 * group * split);
        const int qw = c.m->q_heads * HEAD;
        const AttnRaw none{};
        const AttnSplit sp{c.m->att_ws, c.m->att_cnt, chunked ? 1 : 0, chunked ? c.m->mx.sattn : 0,
                           ATT_ZMAX_DECODE, tl_launch("k_attn_decode")};
        if (c.m->kv.dtype == JL_KV_F32)
            return launch_pdl(k_attn_decode<1, 0>, g2, blk, att_smem(1), c.stream, c.pass(),
                              (const float*)c.m->s.qkv, qkv_ld(c.m), group, split, kv_view(c.m, layer),
                              c.m->s.attn, qw, bout, bN, none, sp);
        return launch_pdl(k_attn_decode<0, 0>, g2, blk, att_smem(0), c.stream, c.pass(),
                          (const float*)c.m->s.qkv, qkv_ld(c.m), group, split, kv_view(c.m, layer), c.m->s.attn,
                          qw, bout, bN, none, sp);
    }
    if (c.m->kv.dtype == JL_KV_F32)
        return launch_pdl(k_attention<1>, grid, dim3(128), 0, c.stream, c.pass(), (const float*)c.m->s.qkv,
                          qkv_ld(c.m), c.m->q_heads, group, kv_view(c.m, layer), c.m->s.attn, bout, bN);
    return launch_pdl(k_attention<0>, grid, dim3(128), 0, c.stream, c.pass(), (const float*)c.m->s.qkv,
                      qkv_ld(c.m), c.m->q_heads, group, kv_view(c.m, layer), c.m->s.attn, bout, bN);
}

jl_status launch_o(const PassCtx& c, const LayerW& L) {
    if (L.mx_o.a && c.rows_cap <= mx_max_tokens())
        return mx_project(c, L.mx_o, MXE_ADD, 0, c.m->s.attn, c.m->q_heads * HEAD, nullptr, c.m->s.x,
                          c.m->hidden);
    Proj p = make_proj({&L.o});
    return run_proj<EPI_ADD>(c, L.o.kind, 0, c.m->s.attn, c.m->q_heads * HEAD, p, c.m->s.x, c.m->hidden);
}

jl_status launch_gateup(const PassCtx& c, const LayerW& L) {
    if (L.mx_gateup.a && c.rows_cap <= mx_max_tokens())
        return mx_project(c, L.mx_gateup, MXE_SWIGLU, 0, c.m->s.xn, c.m->hidden, nullptr, c.m->s.act,
                          c.m->inter);
    Proj p = make_proj({&L.gate, &L.up});
    p.total = L.gate.rows;
    return run_proj<EPI_SWIGLU>(c, L.gate.kind, 0, c.m->s.xn, c.m->hidden, p, c.m->s.act, c.m->inter);
}

jl_status launch_down(const PassCtx& c, const LayerW& L) {
    if (L.mx_down.a && c.rows_cap <= mx_max_tokens())
        return mx_project(c, L.mx_down, MXE_ADD, 0, c.m->s.act, c.m->inter, nullptr, c.m->s.x,
                          c.m->hidden);
    Proj p = make_proj({&L.down});
    return run_proj<EPI_ADD>(c, L.down.kind, 0, c.m->s.act, c.m->inter, p, c.m->s.x, c.m->hidden);
}

jl_status launch_head(const PassCtx& c) {
    if (c.m->mx_head.a && c.head_cap <= mx_max_tokens())
        return mx_project(c, c.m->mx_head, MXE_STORE, 1, c.m->s.xh, c.m->hidden, nullptr, c.m->s.logits,
                          c.m->vocab);
    Proj p = make_proj({&c.m->head});
    return run_proj<EPI_STORE>(c, c.m->head.kind, 1, c.m->s.xh, c.m->hidden, p, c.m->s.logits,
                               c.m->vocab);
}

jl_status launch_attention_raw(const PassCtx& c, int layer, const uint16_t* qn, const uint16_t* kn) {
    const jl_model* m = c.m;
    const int group = m->q_heads / m->kv_heads;
    if (c.rows_cap > 2 || group > 8 || group < 2) {
        set_error("attention on raw q|k|v takes passes of at most 2 rows and GQA groups of 2..8");
        return JL_ERR_INVALID_ARG;
    }
    const int split = att_split(group);
    const dim3 g2(m->kv_heads, c.rows_cap, att_grid_splits(c)), blk(32 * group * split);
    const int qw = m->q_heads * HEAD;
    const AttnSplit sp{m->att_ws, m->att_cnt, 0, 0, ATT_ZMAX, tl_launch("k_attn_decode<raw>")};
    AttnRaw raw;
    raw.qn = qn;
    raw.kn = kn;
    raw.rope = (const float2*)m->rope;
    raw.k_off = qw;
    raw.v_off = qw + m->kv_heads * HEAD;
    if (m->kv.dtype == JL_KV_F32)
        return launch_pdl(k_attn_decode<1, 1>, g2, blk, att_smem(1), c.stream, c.pass(), (const float*)m->s.qkv,
                          qkv_ld(m), group, split, kv_view(m, layer), m->s.attn, qw, (uint8_t*)nullptr, 0,
                          raw, sp);
    return launch_pdl(k_attn_decode<0, 1>, g2, blk, att_smem(0), c.stream, c.pass(), (const float*)m->s.qkv,
                      qkv_ld(m), group, split, kv_view(m, layer), m->s.attn, qw, (uint8_t*)nullptr, 0,
                      raw, sp);
}

jl_status launch_argmax(const PassCtx& c) {
    return launch_pdl(k_argmax, dim3(c.head_cap), dim3(1024), 0, c.stream, c.pass(),
                      (const float*)c.m->s.logits, c.m->vocab);
}

jl_status launch_synth_bf16(uint64_t seed, uint32_t tensor_index, size_t n, uint16_t* out,
                            cudaStream_t stream) {
    const size_t groups = (n + 3) / 4;
    const int grid = (int)std::min<size_t>((groups + 255) / 256, (size_t)sm_count() * 16);
    k_synth<<<std::max(grid, 1), 256, 0, stream>>>(seed, tensor_index, n, out);
    JL_CUDA(cudaGetLastError());
    return JL_OK;
}

jl_status launch_fill_u16(uint16_t* out, size_t n, uint16_t value, cudaStream_t stream) {
    const int grid = (int)std::min<size_t>((n + 255) / 256, (size_t)sm_count() * 8);
    k_fill_u16<<<std::max(grid, 1), 256, 0, stream>>>(out, n, value);
    JL_CUDA(cudaGetLastError());
    return JL_OK;
}

jl_status launch_quantize_mxfp4(const uint16_t* bf16, int rows, int cols, uint8_t* packed,
                                uint8_t* scales, cudaStream_t stream) {
    const size_t blocks = (size_t)rows * cols / 32;
    const int grid = (int)std::min<size_t>((blocks + 127) / 128, (size_t)sm_count() * 16);
    k_quantize<<<std::max(grid, 1), 128, 0, stream>>>(bf16, blocks, packed, scales);
    JL_CUDA(cudaGetLastError());
    return JL_OK;
}

}  // namespace jl
