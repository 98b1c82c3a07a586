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
};

template <int M, int EPI, int TR>
__global__ void __launch_bounds__(256) k_dec_proj(DecArgs a) {
    extern __shared__ __align__(128) uint8_t dsm[];
    __shared__ uint64_t bar;
    __shared__ float red[32];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
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

// ===========================================================================
// The draft step as one persistent kernel (k_draft_fused)
// ===========================================================================
//
// One CTA per SM runs every layer of a one- or two-row draft step.  Each
// layer has five phases, each a share of rows per CTA:
//   P1 q|k|v rows (grouped by KV head), P2 attention (per KV head, its
//   positions split into 128-position windows over up to 16 CTAs), P3 o rows
//   + residual, P4 gate/up pairs + SwiGLU, P5 down rows + residual.
// A phase waits for the one before it through device counters: a CTA that
// finishes its share adds its unit count, and a CTA about to start polls
// (acquire, bounded) until the count is complete; attention of a KV head
// waits only for that head's q|k|v rows.  A loader warp streams each CTA's
// weight rows for the coming phases (codes and scales exactly as the
// checkpoint stores them) through a ring of shared-memory slots with bulk
// copies, running ahead across phases and layers: weights never depend on
// activations, so what is left per phase is the dependency and the
// activation load.  Activations written by other CTAs are read through L2
// (ld.global.cg), never from a stale L1 line.
//
// Every wait is bounded.  A wait that gives up sets bit 3 of the model's
// error flag and an abort word that every later wait sees, so all CTAs
// leave promptly, each first waiting (bounded) for its own copies in
// flight.  The last CTA to leave resets the counters for the next launch.
// The kernel never triggers its dependents early: the next kernel starts
// only when every CTA is done, and one CTA per SM keeps the whole grid
// resident while CTAs wait for one another.

constexpr int DM_COMPUTE = 256;               // 8 compute warps
constexpr int DM_THREADS = DM_COMPUTE + 32;   // + 1 loader warp
constexpr int DM_MAXSLOTS = 8;
constexpr int DM_WIN = 128;                   // attention positions per window
constexpr int DM_MAXUNITS = 16;               // attention CTAs per KV head at most
constexpr uint32_t DM_WAIT = 1u << 21;        // polls of a counter or barrier before giving up (about a second)
constexpr int DM_SMEM_MAX = 200 * 1024;       // dynamic shared memory (static: under 12 KB)

// Counters of one layer: q|k|v rows done per KV head, attention tickets per
// KV head, then KV heads whose attention is done, o rows, gate/up pairs,
// down rows.  After the layers: the exit counter and the abort word.
__host__ __device__ inline int dm_layer_counters(int kv_heads) { return 2 * kv_heads + 4; }

struct DmLayer {
    const uint8_t* codes[7];   // q, k, v, o, gate, up, down: [rows][K/2]
    const uint8_t* scales[7];  // [rows][K/32]
    const uint16_t* in_ln;
    const uint16_t* post_ln;
    const uint16_t* qn;
    const uint16_t* kn;
};

struct DmArgs {
    const DmLayer* layers;
    int L, H, QW, KVW, I, kv_heads, group;
    const uint16_t* embed;     // bf16 [vocab][H]
    const float2* rope;        // [max_pos][HALF]
    char* kv_base;             // [layer][K|V] pools
    size_t kv_layer_bytes;     // bytes of one layer's K (or V) pool
    int kv_f32, kv_pages, max_pos;
    PassBuf pb;
    float* x;                  // [M][H] residual stream (the output table reads it next)
    float* qkv;                // [M][QW + 2 KVW]
    float* attn;               // [M][QW]
    float* act;                // [M][I]
    float* part;               // attention partials [kv_heads][DM_MAXUNITS][M][group][ATT_PART]
    int* cnt;                  // [L][dm_layer_counters], exit, abort
    int* err;
    int slot_bytes, nslots;
};

__device__ __forceinline__ void dm_sync() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

// Barrier of the compute warps that also returns the AND of `v` over them,
// so a decision to stop is the same in every thread.
__device__ __forceinline__ bool dm_sync_and(bool v) {
    uint32_t r;
    asm volatile(
        "{\n .reg .pred pi, po;\n"
        " setp.ne.u32 pi, %1, 0;\n"
        " bar.red.and.pred po, 1, 256, pi;\n"
        " selp.u32 %0, 1, 0, po;\n}"
        : "=r"(r)
        : "r"((uint32_t)v)
        : "memory");
    return r != 0;
}

__device__ __forceinline__ int ld_acquire(const int* p) {
    int v;
    asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__host__ __device__ inline void dm_range(int R, int nb, int b, int& u0, int& u1) {
    u0 = (int)((long long)R * b / nb);
    u1 = (int)((long long)R * (b + 1) / nb);
}

// A P1 unit's place: its weight matrix (0 q, 1 k, 2 v), the row in it, the
// output column in a q|k|v row, and how many units from it on stay in that
// matrix.  Units run over KV heads g, each with its group's query rows,
// then its K rows, then its V rows.
struct DmQkvUnit {
    int mat, row, col, run;
};
__host__ __device__ inline DmQkvUnit dm_qkv_unit(int u, int group, int QW, int KVW) {
    const int GU = (group + 2) * HEAD;
    const int g = u / GU, i = u % GU;
    DmQkvUnit r;
    if (i < group * HEAD) {
        r.mat = 0; r.row = g * group * HEAD + i; r.col = r.row; r.run = group * HEAD - i;
    } else if (i < (group + 1) * HEAD) {
        r.mat = 1; r.row = g * HEAD + i - group * HEAD; r.col = QW + r.row; r.run = (group + 1) * HEAD - i;
    } else {
        r.mat = 2; r.row = g * HEAD + i - (group + 1) * HEAD; r.col = QW + KVW + r.row; r.run = GU - i;
    }
    return r;
}

// Weight stage q of a layer (0 q|k|v, 1 o, 2 gate/up, 3 down) for CTA b:
// K, its units [u0, u1) and the bytes its slot receives.
struct DmPhase {
    int K, u0, u1;
    uint32_t bytes;
};
__host__ __device__ inline DmPhase dm_phase(int q, int nb, int b, int H, int QW, int I, int kv_heads,
                                            int group) {
    DmPhase p;
    int R = 0;
    switch (q) {
        case 0: p.K = H; R = kv_heads * (group + 2) * HEAD; break;
        case 1: p.K = QW; R = H; break;
        case 2: p.K = H; R = I; break;
        default: p.K = I; R = H; break;
    }
    dm_range(R, nb, b, p.u0, p.u1);
    const uint32_t n = (uint32_t)(p.u1 - p.u0);
    p.bytes = (q == 2 ? 2u : 1u) * n * (uint32_t)(p.K / 2 + p.K / 32);
    return p;
}

// Bounded poll of a counter (acquire); false once it gave up or another CTA
// did (the abort word).
__device__ bool dm_wait_count(const int* c, int target, int* abort_w, int* err) {
    for (uint32_t i = 0; i < DM_WAIT; ++i) {
        if (ld_acquire(c) >= target) return true;
        if ((i & 255u) == 255u && *(volatile int*)abort_w) return false;
    }
    atomicOr(err, 8);
    atomicExch(abort_w, 1);
    return false;
}

// Rows of the pass into the swizzled layout dec_dot reads, as x * w when w
// is given, with warp j's share of row m's sum of squares in ssq[m * 8 + j]
// (the RMSNorm division is applied to the dot products).  Source: f32 rows
// read through L2 (written by other CTAs of this launch), or the bf16
// embedding rows of the pass's tokens.  Rows >= `rows` are zero.
template <int M>
__device__ void dm_load_x(const float* src, int ld, const uint16_t* embed, const int* tok, int rows, int K,
                          const uint16_t* w, float4* xs4, float* ssq) {
    const int K4 = K / 4;
    const int t = threadIdx.x, warp = t >> 5;
#pragma unroll
    for (int m = 0; m < M; ++m) {
        float4 v[DEC_XCHUNKS];
#pragma unroll
        for (int i = 0; i < DEC_XCHUNKS; ++i) {
            const int c = t + i * DM_COMPUTE;
            v[i] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (c < K4 && m < rows) {
                if (embed) {
                    const uint2 e = *reinterpret_cast<const uint2*>(embed + (size_t)tok[m] * K + 4 * c);
                    v[i] = make_float4(bf16f(e.x & 0xffffu), bf16f(e.x >> 16), bf16f(e.y & 0xffffu), bf16f(e.y >> 16));
                } else {
                    v[i] = __ldcg(reinterpret_cast<const float4*>(src + (size_t)m * ld) + c);
                }
            }
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
            if ((t & 31) == 0) ssq[m * 8 + warp] = ss;
        }
#pragma unroll
        for (int i = 0; i < DEC_XCHUNKS; ++i) {
            const int c = t + i * DM_COMPUTE;
            if (c >= K4) continue;
            if (w) {
                const uint2 wv = *reinterpret_cast<const uint2*>(w + 4 * c);
                v[i].x = __fmul_rn(v[i].x, bf16f(wv.x & 0xffffu));
                v[i].y = __fmul_rn(v[i].y, bf16f(wv.x >> 16));
                v[i].z = __fmul_rn(v[i].z, bf16f(wv.y & 0xffffu));
                v[i].w = __fmul_rn(v[i].w, bf16f(wv.y >> 16));
            }
            xs4[m * K4 + dec_swz(c)] = v[i];
        }
    }
}

// Dot products of this warp's rows j = warp, warp + 8, ... (< n) of a slot
// holding NM matrices of n rows (codes [NM][n][K/2], then scales
// [NM][n][K/32]), R rows per interleaved sweep; emit(j, vals[NM][M]) gets
// the totals on lane 0.
template <int R, int M, int NM, typename Emit>
__device__ __forceinline__ void dm_dots(const uint8_t* slot, int n, int K, const float4* xs4, int warp, int lane,
                                        Emit emit) {
    const size_t cb = (size_t)K / 2, sb = (size_t)K / 32;
    for (int j0 = warp; j0 < n; j0 += 8 * R) {
        const uint8_t* wr[R * NM];
        const uint8_t* sr[R * NM];
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const int j = min(j0 + 8 * r, n - 1);
#pragma unroll
            for (int q = 0; q < NM; ++q) {
                wr[r * NM + q] = slot + ((size_t)q * n + j) * cb;
                sr[r * NM + q] = slot + (size_t)NM * n * cb + ((size_t)q * n + j) * sb;
            }
        }
        float o[R * NM][M];
        dec_dot<R * NM, M>(wr, sr, K, xs4, lane, o);
        if (lane == 0) {
#pragma unroll
            for (int r = 0; r < R; ++r) {
                const int j = j0 + 8 * r;
                if (j >= n) continue;
                float v[NM][M];
#pragma unroll
                for (int q = 0; q < NM; ++q)
#pragma unroll
                    for (int m = 0; m < M; ++m) v[q][m] = o[r * NM + q][m];
                emit(j, v);
            }
        }
    }
}

struct DmShared {
    uint64_t full[DM_MAXSLOTS], empty[DM_MAXSLOTS];
    float ssq[2 * 8];
    int tok[2], pos[2], rows, seq, flag;
    volatile int loader_issued;  // stages whose copies the loader issued (set when it stops)
    volatile int loader_done;
    volatile int stop;           // the compute warps have left: the loader issues no more
    float wm[8], wl[8];
    float q[8][HEAD];            // normalised, rotated queries of the (row, query head) pairs
    float k[2][HEAD], v[2][HEAD];  // this pass's K (normalised, rotated) and V, in the cache's rounding
    float wacc[8][HEAD];         // per-warp unnormalised attention outputs
};

template <int M>
__global__ void __launch_bounds__(DM_THREADS, 1) k_draft_fused(DmArgs a) {
    extern __shared__ __align__(128) uint8_t dsm[];
    __shared__ DmShared sh;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
    const int nb = gridDim.x, b = blockIdx.x;
    const int NC = dm_layer_counters(a.kv_heads);
    int* exit_c = a.cnt + a.L * NC;
    int* abort_w = exit_c + 1;
    uint8_t* ring = dsm;
    float4* xs4 = reinterpret_cast<float4*>(dsm + (size_t)a.nslots * a.slot_bytes);
    const int stages = 4 * a.L;
    const int H = a.H, QW = a.QW, KVW = a.KVW, I = a.I, G = a.group;

    if (tid == 0) {
        for (int s = 0; s < a.nslots; ++s) {
            ptx::mbar_init(&sh.full[s], 1);
            ptx::mbar_init(&sh.empty[s], 1);
        }
        ptx::fence_barrier_init();
        sh.loader_issued = 0;
        sh.loader_done = 0;
        sh.stop = 0;
    }
    __syncthreads();

    if (warp == 8) {
        // ---- loader: this CTA's weight stages in the order they are consumed ----
        if (lane == 0) {
            int k = 0;
            for (; k < stages; ++k) {
                const int l = k / 4, q = k % 4, s = k % a.nslots, it = k / a.nslots;
                bool ok = false;  // the slot's previous stage has been consumed
                for (uint32_t i = 0; i < DM_WAIT; ++i) {
                    if (ptx::mbar_try_wait(&sh.empty[s], (it & 1) ^ 1)) { ok = true; break; }
                    if ((i & 255u) == 255u && (sh.stop || *(volatile int*)abort_w)) break;
                }
                if (!ok) break;
                const DmLayer& Lw = a.layers[l];
                const DmPhase ph = dm_phase(q, nb, b, H, QW, I, a.kv_heads, G);
                uint8_t* dst = ring + (size_t)s * a.slot_bytes;
                ptx::mbar_arrive_expect_tx(&sh.full[s], ph.bytes);
                const int n = ph.u1 - ph.u0;
                const size_t cb = (size_t)ph.K / 2, sbt = (size_t)ph.K / 32;
                if (n > 0 && q == 0) {
                    for (int u = ph.u0, j = 0; u < ph.u1;) {
                        const DmQkvUnit un = dm_qkv_unit(u, G, QW, KVW);
                        const int c = min(un.run, ph.u1 - u);
                        ptx::bulk_g2s(dst + (size_t)j * cb, Lw.codes[un.mat] + (size_t)un.row * cb,
                                      (uint32_t)(c * cb), &sh.full[s]);
                        ptx::bulk_g2s(dst + (size_t)n * cb + (size_t)j * sbt, Lw.scales[un.mat] + (size_t)un.row * sbt,
                                      (uint32_t)(c * sbt), &sh.full[s]);
                        u += c;
                        j += c;
                    }
                } else if (n > 0) {
                    const int nm = q == 2 ? 2 : 1;
                    for (int t = 0; t < nm; ++t) {
                        const int mat = q == 1 ? 3 : (q == 2 ? 4 + t : 6);
                        ptx::bulk_g2s(dst + (size_t)t * n * cb, Lw.codes[mat] + (size_t)ph.u0 * cb,
                                      (uint32_t)(n * cb), &sh.full[s]);
                        ptx::bulk_g2s(dst + (size_t)nm * n * cb + (size_t)t * n * sbt,
                                      Lw.scales[mat] + (size_t)ph.u0 * sbt, (uint32_t)(n * sbt), &sh.full[s]);
                    }
                }
            }
            sh.loader_issued = k;
            __threadfence_block();
            sh.loader_done = 1;
        }
        return;
    }

    // ---- compute warps ----
    ptx::grid_dependency_wait();
    if (tid == 0) {
        const int rows = min(a.pb.hdr->rows, M);
        sh.rows = rows;
        sh.seq = rows > 0 ? a.pb.row[0].seq : 0;
        for (int m = 0; m < M; ++m) {
            const RowDesc rd = a.pb.row[m < rows ? m : 0];
            sh.tok[m] = (int)rd.token;
            sh.pos[m] = rd.pos;
        }
    }
    dm_sync();
    const int rows = sh.rows;
    bool alive = rows > 0 && (unsigned)sh.seq < (unsigned)MAX_SEQS;
    for (int m = 0; m < rows; ++m)
        if (sh.pos[m] < 0 || sh.pos[m] >= a.max_pos || sh.pos[m] != sh.pos[0] + m) alive = false;
    if (!alive && tid == 0 && rows > 0) atomicOr(a.err, 2);
    const int32_t* pt = alive ? a.pb.page_table[sh.seq] : nullptr;
    const int ldq = QW + 2 * KVW;
    int consumed = 0;  // ring stages consumed

    // thread 0 polls a counter; the outcome is the same in every compute thread
    auto wait_count = [&](const int* c, int target) {
        bool ok = true;
        if (tid == 0) ok = alive && dm_wait_count(c, target, abort_w, a.err);
        if (!dm_sync_and(alive && ok)) alive = false;
    };
    // the next ring stage, once its copies have landed
    auto take_slot = [&]() -> const uint8_t* {
        const int s = consumed % a.nslots, it = consumed / a.nslots;
        const bool ok = ptx::mbar_wait(&sh.full[s], it & 1, DM_WAIT);
        if (!dm_sync_and(ok)) {
            if (tid == 0) {
                atomicOr(a.err, 8);
                atomicExch(abort_w, 1);
            }
            alive = false;
        }
        return ring + (size_t)s * a.slot_bytes;
    };
    // after the warps' stores: release the slot, then publish `count` units
    auto finish = [&](int* c, int count) {
        __threadfence();
        dm_sync();
        if (tid == 0) {
            ptx::mbar_arrive(&sh.empty[consumed % a.nslots]);
            if (count) atomicAdd(c, count);
        }
        ++consumed;
    };

    for (int l = 0; l < a.L && alive; ++l) {
        const DmLayer& Lw = a.layers[l];
        int* C = a.cnt + l * NC;
        int* c_qkv = C;                       // [kv_heads]
        int* c_tk = C + a.kv_heads;           // [kv_heads]
        int* c_att = C + 2 * a.kv_heads;
        int* c_o = c_att + 1;
        int* c_gu = c_att + 2;
        int* c_dn = c_att + 3;
        const uint16_t* emb = l == 0 ? a.embed : nullptr;

        // ---- P1: q|k|v rows (lib.rs:353-355), the input RMSNorm applied to the sums ----
        {
            const DmPhase ph = dm_phase(0, nb, b, H, QW, I, a.kv_heads, G);
            const int n = ph.u1 - ph.u0;
            if (l > 0) wait_count(a.cnt + (l - 1) * NC + 2 * a.kv_heads + 3, H);
            if (!alive) break;
            if (n > 0) dm_load_x<M>(a.x, H, emb, sh.tok, rows, H, Lw.in_ln, xs4, sh.ssq);
            dm_sync();
            const uint8_t* slot = take_slot();
            if (!alive) break;
            if (n > 0) {
                float rms[M];
#pragma unroll
                for (int m = 0; m < M; ++m) rms[m] = dec_rms(sh.ssq, m, H, true);
                dm_dots<4, M, 1>(slot, n, H, xs4, warp, lane, [&](int j, float (&v)[1][M]) {
                    const DmQkvUnit un = dm_qkv_unit(ph.u0 + j, G, QW, KVW);
#pragma unroll
                    for (int m = 0; m < M; ++m)
                        if (m < rows) a.qkv[(size_t)m * ldq + un.col] = __fdiv_rn(v[0][m], rms[m]);
                });
            }
            __threadfence();
            dm_sync();
            if (tid == 0) {
                ptx::mbar_arrive(&sh.empty[consumed % a.nslots]);
                const int GU = (G + 2) * HEAD;  // this CTA's rows, per KV head
                for (int u = ph.u0; u < ph.u1;) {
                    const int g = u / GU, e = min(ph.u1, (g + 1) * GU);
                    atomicAdd(c_qkv + g, e - u);
                    u = e;
                }
            }
            ++consumed;
        }

        // ---- P2: attention of one KV head over a range of windows (lib.rs:363-441) ----
        const int vis = sh.pos[rows - 1] + 1;
        const int nwin = (vis + DM_WIN - 1) / DM_WIN;
        const int per = nb / a.kv_heads;
        const int U = min(min(nwin, DM_MAXUNITS), per);
        const int g = b / per, j = b % per;
        if (g < a.kv_heads && j < U) {
            const int p_lo = (j * nwin / U) * DM_WIN, p_hi = min(((j + 1) * nwin / U) * DM_WIN, vis);
            wait_count(c_qkv + g, (G + 2) * HEAD);
            if (!alive) break;
            const char* kb = a.kv_base + (size_t)l * 2 * a.kv_layer_bytes;
            const char* vb = kb + a.kv_layer_bytes;
            const int P = rows * G;  // (row, query head) pairs, at most 8
            // queries, and this pass's K and V of the head: one warp per job
            for (int job = warp; job < P + rows; job += 8) {
                const bool isq = job < P;
                const int m = isq ? job / G : job - P;
                const int col = isq ? (g * G + job % G) * HEAD : QW + g * HEAD;
                const float* src = a.qkv + (size_t)m * ldq + col;
                float a0 = __ldcg(src + lane), a1 = __ldcg(src + lane + 32);
                float a2 = __ldcg(src + lane + 64), a3 = __ldcg(src + lane + 96);
                const NormRope nr = norm_rope_args(isq ? Lw.qn : Lw.kn, a.rope, sh.pos[m], lane);
                norm_rope4(a0, a1, a2, a3, nr);  // lib.rs:363-388
                if (isq) {
                    sh.q[job][lane] = a0; sh.q[job][lane + 32] = a1;
                    sh.q[job][lane + 64] = a2; sh.q[job][lane + 96] = a3;
                    continue;
                }
                const float* vs = src + KVW;
                float v0 = __ldcg(vs + lane), v1 = __ldcg(vs + lane + 32);
                float v2 = __ldcg(vs + lane + 64), v3 = __ldcg(vs + lane + 96);
                if (!a.kv_f32) {  // attend to this pass's rows as the cache will hold them
                    a0 = bf16f(f2bf16(a0)); a1 = bf16f(f2bf16(a1)); a2 = bf16f(f2bf16(a2)); a3 = bf16f(f2bf16(a3));
                    v0 = bf16f(f2bf16(v0)); v1 = bf16f(f2bf16(v1)); v2 = bf16f(f2bf16(v2)); v3 = bf16f(f2bf16(v3));
                }
                sh.k[m][lane] = a0; sh.k[m][lane + 32] = a1; sh.k[m][lane + 64] = a2; sh.k[m][lane + 96] = a3;
                sh.v[m][lane] = v0; sh.v[m][lane + 32] = v1; sh.v[m][lane + 64] = v2; sh.v[m][lane + 96] = v3;
                if (j == U - 1) {  // the pass's K/V go to the cache (lib.rs:393-396), once
                    const int pos = sh.pos[m];
                    const int pg = pt[pos / PAGE];
                    if ((unsigned)pg < (unsigned)a.kv_pages) {
                        const size_t idx = kv_index(pg, g, pos % PAGE, a.kv_heads);
                        if (a.kv_f32) {
                            float* dk = (float*)kb + idx;
                            float* dv = (float*)vb + idx;
                            dk[lane] = a0; dk[lane + 32] = a1; dk[lane + 64] = a2; dk[lane + 96] = a3;
                            dv[lane] = v0; dv[lane + 32] = v1; dv[lane + 64] = v2; dv[lane + 96] = v3;
                        } else {
                            uint16_t* dk = (uint16_t*)kb + idx;
                            uint16_t* dv = (uint16_t*)vb + idx;
                            dk[lane] = f2bf16(a0); dk[lane + 32] = f2bf16(a1);
                            dk[lane + 64] = f2bf16(a2); dk[lane + 96] = f2bf16(a3);
                            dv[lane] = f2bf16(v0); dv[lane + 32] = f2bf16(v1);
                            dv[lane + 64] = f2bf16(v2); dv[lane + 96] = f2bf16(v3);
                        }
                    } else if (lane == 0) {
                        atomicOr(a.err, 1);
                    }
                }
            }
            dm_sync();
            // scores and online softmax: pair warp % P, every nsub-th chunk of 32 positions
            const float scale = sqrtf(128.0f);
            const int nsub = 8 / P, pi = warp % P, sub = warp / P;
            if (sub < nsub) {
                const int m = pi / G;
                const int pvis = sh.pos[m] + 1;
                float mx = -INFINITY, sum = 0.f;
                float acc[4] = {0.f, 0.f, 0.f, 0.f};
                const float* qv = sh.q[pi];
                for (int c0 = p_lo + sub * 32; c0 < min(p_hi, pvis); c0 += 32 * nsub) {
                    const int p = c0 + lane;
                    float sc = -INFINITY;
                    if (p < pvis) {
                        int fresh = -1;  // this pass's rows come from shared memory
                        for (int mm = 0; mm < rows; ++mm)
                            if (sh.pos[mm] == p) fresh = mm;
                        float dot = 0.f;
                        bool good = true;
                        if (fresh >= 0) {
#pragma unroll 8
                            for (int d = 0; d < HEAD; ++d) dot = fmaf(qv[d], sh.k[fresh][d], dot);
                        } else {
                            const int pg = pt[p / PAGE];
                            good = (unsigned)pg < (unsigned)a.kv_pages;
                            if (good) {
                                const size_t idx = kv_index(pg, g, p % PAGE, a.kv_heads);
                                if (a.kv_f32) {
                                    const float4* kr = (const float4*)((const float*)kb + idx);
#pragma unroll 8
                                    for (int c = 0; c < 32; ++c) {
                                        const float4 k4 = __ldcg(kr + c);
                                        dot = fmaf(qv[4 * c], k4.x, dot);
                                        dot = fmaf(qv[4 * c + 1], k4.y, dot);
                                        dot = fmaf(qv[4 * c + 2], k4.z, dot);
                                        dot = fmaf(qv[4 * c + 3], k4.w, dot);
                                    }
                                } else {
                                    const uint4* kr = (const uint4*)((const uint16_t*)kb + idx);
#pragma unroll 4
                                    for (int c = 0; c < 16; ++c) {
                                        const uint4 k8 = __ldcg(kr + c);
                                        const float* qq = qv + 8 * c;
                                        dot = fmaf(qq[0], __uint_as_float(k8.x << 16), dot);
                                        dot = fmaf(qq[1], __uint_as_float(k8.x & 0xffff0000u), dot);
                                        dot = fmaf(qq[2], __uint_as_float(k8.y << 16), dot);
                                        dot = fmaf(qq[3], __uint_as_float(k8.y & 0xffff0000u), dot);
                                        dot = fmaf(qq[4], __uint_as_float(k8.z << 16), dot);
                                        dot = fmaf(qq[5], __uint_as_float(k8.z & 0xffff0000u), dot);
                                        dot = fmaf(qq[6], __uint_as_float(k8.w << 16), dot);
                                        dot = fmaf(qq[7], __uint_as_float(k8.w & 0xffff0000u), dot);
                                    }
                                }
                            } else {
                                atomicOr(a.err, 1);
                            }
                        }
                        if (good) sc = __fdiv_rn(dot, scale);
                    }
                    const float nm = fmaxf(mx, warp_max(sc));
                    if (nm == -INFINITY) continue;
                    const float corr = mx == -INFINITY ? 0.f : expf(mx - nm);
                    const float pw = sc == -INFINITY ? 0.f : expf(sc - nm);
                    sum = fmaf(sum, corr, warp_sum(pw));
#pragma unroll
                    for (int d = 0; d < 4; ++d) acc[d] *= corr;
                    mx = nm;
                    for (int t = 0; t < 32; ++t) {  // V: lane holds dims 4 lane .. 4 lane + 3
                        const float w = __shfl_sync(0xffffffffu, pw, t);
                        if (w == 0.f) continue;
                        const int pp = c0 + t;
                        int fresh = -1;
                        for (int mm = 0; mm < rows; ++mm)
                            if (sh.pos[mm] == pp) fresh = mm;
                        float4 v4;
                        if (fresh >= 0) {
                            v4 = *reinterpret_cast<const float4*>(&sh.v[fresh][4 * lane]);
                        } else {
                            const size_t idx = kv_index(pt[pp / PAGE], g, pp % PAGE, a.kv_heads);
                            if (a.kv_f32) {
                                v4 = __ldcg((const float4*)((const float*)vb + idx) + lane);
                            } else {
                                const uint2 u = __ldcg((const uint2*)((const uint16_t*)vb + idx) + lane);
                                v4 = make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xffff0000u),
                                                 __uint_as_float(u.y << 16), __uint_as_float(u.y & 0xffff0000u));
                            }
                        }
                        acc[0] = fmaf(w, v4.x, acc[0]);
                        acc[1] = fmaf(w, v4.y, acc[1]);
                        acc[2] = fmaf(w, v4.z, acc[2]);
                        acc[3] = fmaf(w, v4.w, acc[3]);
                    }
                }
                if (lane == 0) {
                    sh.wm[warp] = mx;
                    sh.wl[warp] = sum;
                }
                *reinterpret_cast<float4*>(&sh.wacc[warp][4 * lane]) = make_float4(acc[0], acc[1], acc[2], acc[3]);
            }
            dm_sync();
            // merge each pair's warps in warp order: the output, or this unit's partial
            if (warp < P) {
                const int m = warp / G, hq = warp % G;
                float M_ = -INFINITY;
                for (int s2 = 0; s2 < nsub; ++s2) M_ = fmaxf(M_, sh.wm[warp + s2 * P]);
                float Ls = 0.f;
                float o4[4] = {0.f, 0.f, 0.f, 0.f};
                for (int s2 = 0; s2 < nsub; ++s2) {
                    const int w2 = warp + s2 * P;
                    const float f = sh.wm[w2] == -INFINITY ? 0.f : expf(sh.wm[w2] - M_);
                    Ls = fmaf(sh.wl[w2], f, Ls);
                    const float4 v4 = *reinterpret_cast<const float4*>(&sh.wacc[w2][4 * lane]);
                    o4[0] = fmaf(v4.x, f, o4[0]);
                    o4[1] = fmaf(v4.y, f, o4[1]);
                    o4[2] = fmaf(v4.z, f, o4[2]);
                    o4[3] = fmaf(v4.w, f, o4[3]);
                }
                if (U == 1) {
                    float* o = a.attn + (size_t)m * QW + (g * G + hq) * HEAD + 4 * lane;
                    *reinterpret_cast<float4*>(o) = make_float4(__fdiv_rn(o4[0], Ls), __fdiv_rn(o4[1], Ls),
                                                                __fdiv_rn(o4[2], Ls), __fdiv_rn(o4[3], Ls));
                } else {
                    float* pp = a.part + ((((size_t)g * DM_MAXUNITS + j) * M + m) * G + hq) * ATT_PART;
                    if (lane == 0) {
                        pp[0] = M_;
                        pp[1] = Ls;
                    }
                    *reinterpret_cast<float4*>(pp + 4 + 4 * lane) = make_float4(o4[0], o4[1], o4[2], o4[3]);
                }
            }
            __threadfence();
            dm_sync();
            bool last = U == 1;
            if (U > 1) {
                if (tid == 0) sh.flag = atomicAdd(c_tk + g, 1) == U - 1 ? 1 : 0;
                dm_sync();
                last = sh.flag != 0;
                if (last) {
                    __threadfence();
                    if (warp < P) {  // the units' partials, in unit order
                        const int m = warp / G, hq = warp % G;
                        auto part_of = [&](int u) {
                            return a.part + ((((size_t)g * DM_MAXUNITS + u) * M + m) * G + hq) * ATT_PART;
                        };
                        float M_ = -INFINITY;
                        for (int u = 0; u < U; ++u) M_ = fmaxf(M_, __ldcg(part_of(u)));
                        float Ls = 0.f;
                        float o4[4] = {0.f, 0.f, 0.f, 0.f};
                        for (int u = 0; u < U; ++u) {
                            const float* pp = part_of(u);
                            const float mu = __ldcg(pp);
                            const float f = mu == -INFINITY ? 0.f : expf(mu - M_);
                            Ls = fmaf(__ldcg(pp + 1), f, Ls);
                            const float4 v4 = __ldcg(reinterpret_cast<const float4*>(pp + 4) + lane);
                            o4[0] = fmaf(v4.x, f, o4[0]);
                            o4[1] = fmaf(v4.y, f, o4[1]);
                            o4[2] = fmaf(v4.z, f, o4[2]);
                            o4[3] = fmaf(v4.w, f, o4[3]);
                        }
                        float* o = a.attn + (size_t)m * QW + (g * G + hq) * HEAD + 4 * lane;
                        *reinterpret_cast<float4*>(o) = make_float4(__fdiv_rn(o4[0], Ls), __fdiv_rn(o4[1], Ls),
                                                                    __fdiv_rn(o4[2], Ls), __fdiv_rn(o4[3], Ls));
                    }
                    __threadfence();
                }
                dm_sync();  // sh.flag is free again
            }
            if (last && tid == 0) atomicAdd(c_att, 1);
        }

        // ---- P3: o rows + residual (lib.rs:444-449, model.rs:178-186) ----
        {
            const DmPhase ph = dm_phase(1, nb, b, H, QW, I, a.kv_heads, G);
            const int n = ph.u1 - ph.u0;
            wait_count(c_att, a.kv_heads);
            if (!alive) break;
            if (n > 0) dm_load_x<M>(a.attn, QW, nullptr, sh.tok, rows, QW, nullptr, xs4, sh.ssq);
            dm_sync();
            const uint8_t* slot = take_slot();
            if (!alive) break;
            if (n > 0)
                dm_dots<1, M, 1>(slot, n, QW, xs4, warp, lane, [&](int jj, float (&v)[1][M]) {
                    const int r = ph.u0 + jj;
#pragma unroll
                    for (int m = 0; m < M; ++m)
                        if (m < rows) {
                            const float old = emb ? bf16f(emb[(size_t)sh.tok[m] * H + r]) : __ldcg(a.x + (size_t)m * H + r);
                            a.x[(size_t)m * H + r] = __fadd_rn(old, v[0][m]);
                        }
                });
            finish(c_o, n);
        }

        // ---- P4: gate/up pairs + SwiGLU (lib.rs:459-463) ----
        {
            const DmPhase ph = dm_phase(2, nb, b, H, QW, I, a.kv_heads, G);
            const int n = ph.u1 - ph.u0;
            wait_count(c_o, H);
            if (!alive) break;
            if (n > 0) dm_load_x<M>(a.x, H, nullptr, sh.tok, rows, H, Lw.post_ln, xs4, sh.ssq);
            dm_sync();
            const uint8_t* slot = take_slot();
            if (!alive) break;
            if (n > 0) {
                float rms[M];
#pragma unroll
                for (int m = 0; m < M; ++m) rms[m] = dec_rms(sh.ssq, m, H, true);
                dm_dots<2, M, 2>(slot, n, H, xs4, warp, lane, [&](int jj, float (&v)[2][M]) {
#pragma unroll
                    for (int m = 0; m < M; ++m)
                        if (m < rows) {
                            const float gg = __fdiv_rn(v[0][m], rms[m]), u = __fdiv_rn(v[1][m], rms[m]);
                            a.act[(size_t)m * I + ph.u0 + jj] = __fmul_rn(__fdiv_rn(gg, __fadd_rn(1.0f, expf(-gg))), u);
                        }
                });
            }
            finish(c_gu, n);
        }

        // ---- P5: down rows + residual (lib.rs:464-467, model.rs:186-197) ----
        {
            const DmPhase ph = dm_phase(3, nb, b, H, QW, I, a.kv_heads, G);
            const int n = ph.u1 - ph.u0;
            wait_count(c_gu, I);
            if (!alive) break;
            if (n > 0) dm_load_x<M>(a.act, I, nullptr, sh.tok, rows, I, nullptr, xs4, sh.ssq);
            dm_sync();
            const uint8_t* slot = take_slot();
            if (!alive) break;
            if (n > 0)
                dm_dots<1, M, 1>(slot, n, I, xs4, warp, lane, [&](int jj, float (&v)[1][M]) {
                    const int r = ph.u0 + jj;
#pragma unroll
                    for (int m = 0; m < M; ++m)
                        if (m < rows) a.x[(size_t)m * H + r] = __fadd_rn(__ldcg(a.x + (size_t)m * H + r), v[0][m]);
                });
            finish(c_dn, n);
        }
    }

    // ---- leave: copies still in flight land first; the last CTA resets the counters ----
    if (tid == 0) {
        if (!alive) {
            sh.stop = 1;
            for (uint32_t i = 0; i < DM_WAIT && !sh.loader_done; ++i) __nanosleep(100);
            const int issued = sh.loader_issued;
            for (int k = consumed; k < issued; ++k)
                ptx::mbar_wait(&sh.full[k % a.nslots], (k / a.nslots) & 1, DM_WAIT);
        }
        __threadfence();
        if (atomicAdd(exit_c, 1) == nb - 1) {
            __threadfence();
            for (int i = 0; i < a.L * NC; ++i) a.cnt[i] = 0;
            *abort_w = 0;
            __threadfence();
            *exit_c = 0;
        }
    }
}

}  // namespace

// Whether `m`'s draft steps run as k_draft_fused, and its ring and shared memory.
bool dm_supported(const jl_model* m, int* slot_bytes, int* nslots, size_t* smem) {
    if (!m->dec_ok || m->embed.kind != MAT_BF16 || m->lw.empty() || m->sms < 1) return false;
    const int H = m->hidden, QW = m->q_heads * HEAD, I = m->inter;
    const int G = m->q_heads / m->kv_heads;
    const int nb = m->sms;
    if (2 * G > 8 || m->kv_heads > nb || std::max(H, std::max(QW, I)) > DEC_XCHUNKS * 4 * DM_COMPUTE) return false;
    uint32_t most = 0;
    for (int b = 0; b < nb; ++b)
        for (int q = 0; q < 4; ++q) most = std::max(most, dm_phase(q, nb, b, H, QW, I, m->kv_heads, G).bytes);
    const int sb = (int)((most + 127) / 128 * 128);
    const size_t xs = (size_t)2 * std::max(H, std::max(QW, I)) * 4;
    int ns = DM_MAXSLOTS;
    while (ns > 2 && (size_t)ns * sb + xs > (size_t)DM_SMEM_MAX) --ns;
    if ((size_t)ns * sb + xs > (size_t)DM_SMEM_MAX) return false;
    if (slot_bytes) *slot_bytes = sb;
    if (nslots) *nslots = ns;
    if (smem) *smem = (size_t)ns * sb + xs;
    return true;
}

jl_status dm_configure() {
    JL_CUDA(cudaFuncSetAttribute(k_draft_fused<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, DM_SMEM_MAX));
    JL_CUDA(cudaFuncSetAttribute(k_draft_fused<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, DM_SMEM_MAX));
    return JL_OK;
}

jl_status dm_prepare(jl_model* m) {
    m->dm_ok = dm_supported(m, &m->dm_slot, &m->dm_nslots, &m->dm_smem);
    if (!m->dm_ok) return JL_OK;
    std::vector<DmLayer> h(m->layers);
    for (int l = 0; l < m->layers; ++l) {
        const LayerW& L = m->lw[l];
        const Mat* ws[7] = {&L.q, &L.k, &L.v, &L.o, &L.gate, &L.up, &L.down};
        for (int i = 0; i < 7; ++i) {
            h[l].codes[i] = (const uint8_t*)ws[i]->data;
            h[l].scales[i] = ws[i]->scales;
        }
        h[l].in_ln = L.in_ln;
        h[l].post_ln = L.post_ln;
        h[l].qn = L.q_norm;
        h[l].kn = L.k_norm;
    }
    const size_t nc = (size_t)m->layers * dm_layer_counters(m->kv_heads) + 2;
    if (cudaMalloc(&m->dm_layers, h.size() * sizeof(DmLayer)) != cudaSuccess ||
        cudaMalloc(&m->dm_cnt, nc * sizeof(int)) != cudaSuccess) {
        cudaGetLastError();
        set_error("cannot allocate the fused draft step's descriptors");
        return JL_ERR_OOM;
    }
    JL_CUDA(cudaMemcpy(m->dm_layers, h.data(), h.size() * sizeof(DmLayer), cudaMemcpyHostToDevice));
    JL_CUDA(cudaMemset(m->dm_cnt, 0, nc * sizeof(int)));
    return JL_OK;
}

// The draft-step pass of one or two rows as one launch (k_draft_fused); the
// output table's kernels follow it.
jl_status record_dm_pass(const PassCtx& c) {
    const jl_model* m = c.m;
    DmArgs a{};
    a.layers = (const DmLayer*)m->dm_layers;
    a.L = m->layers;
    a.H = m->hidden;
    a.QW = m->q_heads * HEAD;
    a.KVW = m->kv_heads * HEAD;
    a.I = m->inter;
    a.kv_heads = m->kv_heads;
    a.group = m->q_heads / m->kv_heads;
    a.embed = (const uint16_t*)m->embed.data;
    a.rope = m->rope;
    a.kv_base = (char*)m->kv.base;
    a.kv_layer_bytes = m->kv.pages * m->kv.page_elems * m->kv.elem;
    a.kv_f32 = m->kv.dtype == JL_KV_F32;
    a.kv_pages = (int)m->kv.pages;
    a.max_pos = m->max_positions;
    a.pb = c.pass();
    a.x = m->s.x;
    a.qkv = m->s.qkv;
    a.attn = m->s.attn;
    a.act = m->s.act;
    a.part = m->att_ws;
    a.cnt = m->dm_cnt;
    a.err = m->counters;
    a.slot_bytes = m->dm_slot;
    a.nslots = m->dm_nslots;
    const dim3 grid(m->sms), block(DM_THREADS);
    if (c.rows_cap == 1) return launch_pdl(k_draft_fused<1>, grid, block, m->dm_smem, c.stream, a);
    return launch_pdl(k_draft_fused<2>, grid, block, m->dm_smem, c.stream, a);
}

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
    if (m->dm_ok && layers == m->layers) return record_dm_pass(c);
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
