// MXFP4 projections on the 5th-generation tensor cores (tcgen05, sm_100a).
//
// y[m, r] = sum_k x[m, k] * W[r, k] with W in the checkpoint's MXFP4 format
// (E2M1 codes + one E8M0 scale per 32 weights) and x in f32.
//
// The weights go HBM -> shared memory (bulk copies on the TMA engine) ->
// tensor core with no CUDA-core work at all: tcgen05.mma kind::mxf4 applies
// both operands' E8M0 scales itself.  The f32 activations are written as a
// sum of PIECES E2M1 vectors with their own E8M0 block scales: piece p
// quantizes what pieces 0..p-1 left over (each subtraction is exact), so
// eight pieces carry an activation with error below f32 rounding.  The MMA's
// N dimension holds (token, piece) pairs; the epilogue adds a token's eight
// columns.
//
// Layouts, all built once at load time:
//  * weight tile (t, s): 128 weight rows x 256 K-elements (128 bytes per
//    row), 16 KB in the 128-byte-swizzled K-major layout the MMA reads,
//    followed by its scales: two 512-byte atoms (128 rows x 4 blocks of 32),
//    byte 16*(r%32) + 4*(r/32) + kb, which tcgen05.cp broadcasts into 4 TMEM
//    columns.  The stages of a tile are contiguous ([T][S][17 KB]);
//  * activation pieces for stage s: N rows x 128 bytes, same swizzle, then
//    their scale atoms (N <= 128), stages contiguous too.
// A bulk copy costs a few hundred nanoseconds of a CTA's copy engine
// whatever its size, so the ring moves GROUP stages of weights as one copy
// and their activation stages as a second one.
// Split-K partials go to a workspace; the last CTA of a tile (atomic ticket)
// adds them in a fixed order and runs the epilogue, so a row's result does
// not depend on timing or on how many tokens share the pass.
#include <cstdio>

#include <algorithm>

#include "jl_internal.h"
#include "kernels.cuh"
#include "launch.cuh"
#include "mx_pieces.cuh"
#include "ptx.cuh"
#include "timeline.cuh"

namespace jl {

namespace {

using mx::PIECES;
using mx::SF_STAGE;
using mx::STAGE_K;
using mx::sf_offset;
using mx::swz128;

constexpr int TILE_ROWS = 128;
constexpr int A_STAGE = 128 * 128;       // bytes of one weight tile stage
constexpr uint32_t WAIT_LIMIT = 1u << 22;  // polls before a wait reports failure (seconds)
constexpr int TMEM_COLS = 256;
constexpr int ACC_COL = 0, SFA_COL = 128, SFB_COL = 136;

// ---------------------------------------------------------------------------
// activation pieces

// One warp per (token, 32-element block): PIECES residual E2M1 pieces with
// their E8M0 exponents, written into the stage images the MMA streams.  Piece
// p of token m is row 8m+p of the B operand.
__global__ void __launch_bounds__(256) k_mx_pieces(const PassHdr* __restrict__ hdr, int use_head,
                                                   int mcap, const float* __restrict__ x, int ldx,
                                                   int K, int S, int N, uint8_t* __restrict__ bimg) {
    ptx::grid_dependency_wait();  // x comes from the previous kernel; bimg may still be read by it
    ptx::launch_dependents();
    const int lane = threadIdx.x & 31;
    const int item = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int nblocks = S * (STAGE_K / 32);
    if (item >= mcap * nblocks) return;
    const int m = item / nblocks, kb = item % nblocks;
    const int M = min(use_head ? hdr->head_rows : hdr->rows, mcap);
    const int k = kb * 32 + lane;
    float r = (m < M && k < K) ? x[(size_t)m * ldx + k] : 0.f;
    mx::emit_pieces(r, lane, m, kb * 32, N, bimg);
}

// Pieces of x * w for a projection that follows an RMSNorm, plus the
// per-tile sums of squares of x the projection's epilogue turns into the
// row's RMS: one CTA of 128 threads per (128-element tile, row).  Used where
// no projection epilogue produced them (after the embedding).
__global__ void __launch_bounds__(128) k_norm_pieces(const PassHdr* __restrict__ hdr, int mcap,
                                                     const float* __restrict__ x, int ldx,
                                                     const uint16_t* __restrict__ w, int width, int N,
                                                     uint8_t* __restrict__ bout, float* __restrict__ part,
                                                     size_t cs_bout, size_t cs_part) {
    __shared__ float red[4];
    ptx::grid_dependency_wait();
    ptx::launch_dependents();
    const int t = blockIdx.x, m = blockIdx.y, c = blockIdx.z;  // chunk c of a multi-chunk pass
    hdr += c;
    x += (size_t)c * SMALL_M * ldx;
    bout += c * cs_bout;
    part += c * cs_part;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int M = min(hdr->rows, mcap);
    const int k = t * 128 + threadIdx.x;
    const float v = (m < M && k < width) ? x[(size_t)m * ldx + k] : 0.f;
    const float wk = k < width ? bf16f(w[k]) : 0.f;
    mx::emit_pieces(__fmul_rn(v, wk), lane, m, t * 128 + warp * 32, N, bout);
    const float ss = warp_sum(__fmul_rn(v, v));
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    if (threadIdx.x == 0) part[t * MX_PART_STRIDE + m] = __fadd_rn(__fadd_rn(red[0], red[1]), __fadd_rn(red[2], red[3]));
}

// The final RMSNorm of the rows whose next token is predicted
// (model.rs:228, lib.rs:268-290, the same arithmetic as k_rmsnorm), written
// as the bf16 output table's input: four bf16 pieces per value (each the
// rounding of what the previous ones left; together about 32 significant
// bits, more than the f32 value holds), row n = 4 * r + piece of an image
// with N MMA columns and 64 K-elements (128 bytes) per stage.  CTA r < N/4;
// rows past the predicted ones are zero.
__global__ void __launch_bounds__(256) k_head_pieces(PassBuf pb, int head_cap, const float* __restrict__ x,
                                                     int hidden, const uint16_t* __restrict__ w, int N,
                                                     uint8_t* __restrict__ bimg, size_t cs_img) {
    __shared__ float red[32];
    ptx::grid_dependency_wait();
    ptx::launch_dependents();
    const int r = blockIdx.x, c = blockIdx.y;  // chunk c of a multi-chunk pass
    pb.hdr += c;
    pb.head_row += c * SMALL_M;
    x += (size_t)c * SMALL_M * hidden;
    bimg += c * cs_img;
    const bool live = r < min(pb.hdr->head_rows, head_cap);
    const float* xr = live ? x + (size_t)pb.head_row[r] * hidden : x;
    float size = 1.f;
    if (live) {  // uniform over the CTA
        float ss = 0.f;
        for (int j = threadIdx.x; j < hidden; j += blockDim.x) ss = fmaf(xr[j], xr[j], ss);
        ss = block_sum(ss, red);
        size = sqrtf(__fadd_rn(__fdiv_rn(ss, (float)hidden), 1e-6f));
    }
    for (int j2 = threadIdx.x; j2 < hidden / 2; j2 += blockDim.x) {
        const int j = 2 * j2;
        float v0 = 0.f, v1 = 0.f;
        if (live) {
            v0 = __fmul_rn(__fdiv_rn(xr[j], size), bf16f(w[j]));
            v1 = __fmul_rn(__fdiv_rn(xr[j + 1], size), bf16f(w[j + 1]));
        }
        uint8_t* img = bimg + (size_t)(j / 64) * N * 128;
        const uint32_t byte = (uint32_t)(j % 64) * 2;
#pragma unroll
        for (int p = 0; p < 4; ++p) {
            const uint32_t b0 = f2bf16(v0), b1 = f2bf16(v1);
            v0 = __fsub_rn(v0, bf16f(b0));  // exact: a value minus its rounding
            v1 = __fsub_rn(v1, bf16f(b1));
            *(uint32_t*)(img + swz128((uint32_t)(4 * r + p), byte)) = b0 | (b1 << 16);
        }
    }
}

// First maximum of each predicted row over the head tiles' partial maxima,
// in tile order (ties to the lower index, model.rs:288-296).
__global__ void __launch_bounds__(256) k_argmax_tiles(PassBuf pb, int T, const float* __restrict__ amax_v,
                                                      const int* __restrict__ amax_i, size_t cs_amax) {
    __shared__ float bv_s[8];
    __shared__ int bi_s[8];
    ptx::grid_dependency_wait();
    ptx::launch_dependents();
    const int r = blockIdx.x, c = blockIdx.y;  // chunk c of a multi-chunk pass
    pb.hdr += c;
    pb.out_ids += c * SMALL_M;
    amax_v += c * cs_amax;
    amax_i += c * cs_amax;
    if (r >= pb.hdr->head_rows) return;
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int t = threadIdx.x; t < T; t += blockDim.x) {
        const float v = amax_v[t * MX_PART_STRIDE + r];
        const int i = amax_i[t * MX_PART_STRIDE + r];
        if (v > bv || (v == bv && i < bi)) {
            bv = v;
            bi = i;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_down_sync(0xffffffffu, bv, o);
        const int oi = __shfl_down_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) {
            bv = ov;
            bi = oi;
        }
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) {
        bv_s[warp] = bv;
        bi_s[warp] = bi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int q = 1; q < (int)(blockDim.x >> 5); ++q)
            if (bv_s[q] > bv || (bv_s[q] == bv && bi_s[q] < bi)) {
                bv = bv_s[q];
                bi = bi_s[q];
            }
        pb.out_ids[r] = bi == 0x7fffffff ? 0u : (uint32_t)bi;
    }
}

// Load-time re-layout of a bf16 matrix [rows][K] into the tiled, swizzled
// stages of the bf16 projection: tile t, stage s = rows 128t.., elements
// 64s..64s+63 (128 bytes per row).  One thread per 16-byte chunk.
__global__ void k_bf16_tile(const uint16_t* __restrict__ src, int rows, int K, int T, int S,
                            uint8_t* __restrict__ dst) {
    const size_t chunks = (size_t)T * S * TILE_ROWS * 8;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < chunks;
         i += (size_t)gridDim.x * blockDim.x) {
        const int c16 = (int)(i % 8);
        const int r = (int)((i / 8) % TILE_ROWS);
        const int s = (int)((i / (8 * TILE_ROWS)) % S);
        const int t = (int)(i / ((size_t)8 * TILE_ROWS * S));
        const int gr = t * TILE_ROWS + r, k0 = s * 64 + c16 * 8;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (gr < rows && k0 < K) v = *reinterpret_cast<const uint4*>(src + (size_t)gr * K + k0);
        *reinterpret_cast<uint4*>(dst + ((size_t)t * S + s) * A_STAGE + swz128((uint32_t)r, (uint32_t)c16 * 16)) = v;
    }
}

// ---------------------------------------------------------------------------
// the projection

struct MxArgs {
    const uint8_t* a;      // [T][S][w_stage]: codes, then (MXFP4) scale atoms
    const uint8_t* b;      // [S][b_stage]: pieces, then (MXFP4) their scale atoms
    int T, S, ksplit, N, mcap;
    int nbuf, stages;      // TMEM accumulator buffers (1 or 2), ring slots
    int group;             // K stages per ring slot (1 or 2)
    const PassHdr* hdr;
    int use_head;
    float* y;
    int ldy;
    int out_rows;          // outputs past this (last tile's padding) are not written
    float* ws;             // [T][ksplit][mcap][128]
    int* tickets;          // [T]
    int* err;
    // Fused epilogue (decode pass).  Input RMSNorm: the projection reads the
    // pieces of x*w and divides its outputs by the row's RMS, computed from
    // per-tile sums of squares (part_in, part_tiles tiles of MX_MAXTOK).
    const float* part_in;
    int part_tiles, norm_width;
    // Output pieces for the next projection (bout, bN columns) and,
    // after a residual add, the sums of squares of the new x (part_out) and
    // the next RMSNorm weight (next_w) the pieces are scaled by.
    uint8_t* bout;
    int bN;
    float* part_out;
    const uint16_t* next_w;
    // q|k|v epilogue: QK-RMSNorm, RoPE, K/V appended to the paged cache.
    int q_heads, kv_heads;
    const uint16_t* qn;
    const uint16_t* kn;
    const float2* rope;
    const RowDesc* rows;
    const int32_t* const* page_table;
    KvView kv;
    // head: each tile's first maximum per row ([T][MX_PART_STRIDE])
    float* amax_v;
    int* amax_i;
    // Multi-chunk launches (grid y = chunk of MX_MAXTOK rows): chunk c reads
    // b + c*cs_b and writes bout + c*cs_bout (bytes), part_in/part_out/amax
    // + c*cs_* (elements); hdr, rows and y advance by one chunk.
    size_t cs_b, cs_bout, cs_part_in, cs_part_out, cs_amax;
    // TMEM columns between the two accumulator buffers: 64 (0 reads as 64)
    // in a 256-column allocation, or 256 in a 512-column one (two
    // accumulators of 128 columns; the launch then keeps one CTA per SM)
    int acc_step;
    // Ring slots whose weights are requested into L2 ahead of their copy
    // into shared memory (0: none)
    int l2_ahead;
    TlSlot tl;  // phase stamps (timeline build)
};

enum : int { MX_STORE = 0, MX_ADD = 1, MX_SWIGLU = 2, MX_QKV = 3, MX_HEAD = 4 };
// Weight formats: MXFP4 (kind::mxf4 block-scaled MMA, 8 E2M1 activation
// pieces per row) or bf16 (kind::f16 MMA, 4 bf16 activation pieces per row).
enum : int { KIND_MX = 0, KIND_BF = 1 };
constexpr int MX_MAXSTAGES = 6;
constexpr int MX_MAXCLUSTER = 8;  // portable cluster size: split-K at most 8 ways
constexpr int MX_MAXTOK = 16;       // tokens per pass on this path: N = 8 * tokens <= 128
constexpr int MX_THREADS = 192;     // warp 0 loads, warp 1 MMAs, warps 2-5 epilogue
static_assert(MX_PART_STRIDE >= MX_MAXTOK, "partials hold every row of a pass");
static_assert(MX_MAXTOK == 16, "emit_pieces_all takes 16 rows");

// Bytes of one K stage of a weight tile and of an activation image.
__host__ __device__ constexpr int w_stage(int kind) { return A_STAGE + (kind == KIND_MX ? SF_STAGE : 0); }
__host__ __device__ constexpr int b_stage(int N, int kind) {
    return N * 128 + (kind == KIND_MX ? SF_STAGE : 0);
}
// One ring slot: `group` weight stages, then their activation stages.
__host__ __device__ constexpr int mx_slot_bytes(int N, int kind, int group) {
    return group * (w_stage(kind) + b_stage(N, kind));
}
// First K stage of split kc of ks: splits start on a slot boundary.
__host__ __device__ inline int split_stage(int S, int group, int ks, int kc) {
    const int slots = (S + group - 1) / group;
    return min(S, group * (int)((long long)kc * slots / ks));
}
// MMA columns one row occupies (its pieces, then padding).
__host__ __device__ constexpr int cols_per_row(int kind) { return kind == KIND_MX ? 8 : 4; }

// Per-warp sums of v[m]^2 over the warp's 32 rows for rows m < mcap (MT a
// bucket >= mcap: the rows advance together), written to red[quarter][m].
// Each row's reduction tree is the same whatever the bucket.
template <int MT>
__device__ __forceinline__ void warp_sq_sums_t(const float (&v)[16], float (*red)[16], int quarter, int lane) {
    float s[MT];
#pragma unroll
    for (int m = 0; m < MT; ++m) s[m] = __fmul_rn(v[m], v[m]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int m = 0; m < MT; ++m) s[m] += __shfl_xor_sync(0xffffffffu, s[m], o);
    if (lane == 0)
#pragma unroll
        for (int m = 0; m < MT; ++m) red[quarter][m] = s[m];
}

__device__ __forceinline__ void warp_sq_sums(const float (&v)[16], int mcap, float (*red)[16], int quarter,
                                             int lane) {
    if (mcap <= 1) warp_sq_sums_t<1>(v, red, quarter, lane);
    else if (mcap <= 2) warp_sq_sums_t<2>(v, red, quarter, lane);
    else if (mcap <= 4) warp_sq_sums_t<4>(v, red, quarter, lane);
    else if (mcap <= 8) warp_sq_sums_t<8>(v, red, quarter, lane);
    else warp_sq_sums_t<16>(v, red, quarter, lane);
}

// The four epilogue warps synchronise among themselves only.
__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// Persistent, warp-specialised projection.  Split-K runs inside a thread-
// block cluster: the `ksplit` CTAs of a cluster take the same tiles (tile
// cid, cid + clusters, ...), CTA rank kc streaming K slice kc of each.
// Warp 0 lane 0 streams weight stages through a ring of shared-memory slots
// (the first slots are issued before the grid-dependency wait: weights never
// depend on the previous kernel); warp 1 lane 0 issues the MMAs into one of
// two TMEM accumulators; warps 2-5 drain the other accumulator, so one tile's
// epilogue overlaps the next tile's streaming.  Warp w reads TMEM lanes
// 32*(w%4).., weight rows 32*(w%4).. of the tile.
//
// Split-K reduction through distributed shared memory: ranks 1.. push their
// partial tile into the leader's reduction buffer with st.async, whose bytes
// complete the leader's red_full barrier; the leader (rank 0) adds the
// partials in rank order (a fixed order, so results do not depend on timing
// or on the row count) and runs the epilogue.  When the cluster has another
// tile, each leader warp frees the buffer with a 4-byte st.async onto every
// peer's slot_free barrier.  No thread waits on a remote acknowledgement.
// The arguments of chunk c of a multi-chunk launch.
__device__ __forceinline__ MxArgs chunk_args(const MxArgs& a0, int c) {
    MxArgs a = a0;
    if (c) {
        a.b += c * a.cs_b;
        a.hdr += c;
        if (a.y) a.y += (size_t)c * MX_MAXTOK * a.ldy;
        if (a.bout) a.bout += c * a.cs_bout;
        if (a.part_in) a.part_in += c * a.cs_part_in;
        if (a.part_out) a.part_out += c * a.cs_part_out;
        if (a.rows) a.rows += c * MX_MAXTOK;
        if (a.amax_v) {
            a.amax_v += c * a.cs_amax;
            a.amax_i += c * a.cs_amax;
        }
    }
    return a;
}

template <int EPI, int KIND>
__global__ void __launch_bounds__(MX_THREADS, 1) k_mx_gemv(const MxArgs a0) {
    const MxArgs a = chunk_args(a0, blockIdx.y);
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    __shared__ uint64_t full[MX_MAXSTAGES], empty[MX_MAXSTAGES], tfull[2], tempty[2];
    __shared__ uint64_t red_full, slot_free;
    __shared__ uint32_t free_sig;            // target of the leader's slot_free stores
    __shared__ uint32_t tmem_base_s;
    __shared__ float red_s[4][MX_MAXTOK];    // per-warp sums of squares / row maxima
    __shared__ int redi_s[4][MX_MAXTOK];     // per-warp arg maxima
    __shared__ float sz_s[MX_MAXTOK];        // 1 / input RMS per row
    __shared__ float qk_s[MX_MAXTOK];        // 1 / RMS of this head, per row
    __shared__ int kvpos_s[MX_MAXTOK];       // q|k|v: position of each row, -1 if invalid
    __shared__ int kvpage_s[MX_MAXTOK];      //   and its cache page

    const int N = a.N, ST = a.stages, NB = a.nbuf, G = a.group;
    constexpr int WS = w_stage(KIND);
    const int BS = b_stage(N, KIND);
    const int sbytes = mx_slot_bytes(N, KIND, G);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ks = a.ksplit;
    const int kc = ks > 1 ? (int)ptx::cluster_ctarank() : 0;
    const int cid = blockIdx.x / ks, NC = gridDim.x / ks;
    const int s0 = split_stage(a.S, G, ks, kc), s1 = split_stage(a.S, G, ks, kc + 1);
    if (threadIdx.x == 0) tl_stamp(a.tl, 0);
    // epilogue scratch (staged outputs [m][128], SwiGLU up halves and RoPE
    // partners xs[m][64]), then the leader's reduction buffer: for each peer
    // rank and group of four rows of the pass, [128 tile rows][4] floats
    const int RB = (a.mcap + 3) >> 2;
    float* slot = (float*)(smem + ST * sbytes);
    float(*xs)[64] = (float(*)[64])slot;
    float* red = slot + RB * 4 * 128;

    if (threadIdx.x == 0) {
        for (int i = 0; i < ST; ++i) {
            ptx::mbar_init(&full[i], 1);
            ptx::mbar_init(&empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            ptx::mbar_init(&tfull[i], 1);
            ptx::mbar_init(&tempty[i], 4);
        }
        ptx::mbar_init(&red_full, 1);   // the leader's expect_tx, then the peers' bytes
        ptx::mbar_init(&slot_free, 1);  // a peer's expect_tx, then the leader warps' bytes
        ptx::fence_barrier_init();
    }
    const int acc_step = a.acc_step > 64 ? 256 : 64;
    const uint32_t tcols = acc_step > 64 ? 512u : (uint32_t)TMEM_COLS;
    if (warp == 1) {
        ptx::tmem_alloc(&tmem_base_s, tcols);
        ptx::tmem_relinquish();
    }
    ptx::tc_fence_before();
    __syncthreads();
    ptx::tc_fence_after();
    if (ks > 1) {  // every CTA's barriers are initialised before any remote arrive
        ptx::cluster_arrive();
        ptx::cluster_wait();
    }
    const uint32_t tmem = tmem_base_s;
    bool ok = true;

    if (warp == 0) {
        if (lane == 0) {
            // Prefetch the first ring slots' weights, then wait for the
            // kernel that produces the activation pieces.  A slot holds the
            // stages [s, min(s + G, s1)) of one tile: one copy of their
            // weights, one of their activations.
            int pre = 0;
            {
                int g = 0;
                for (int t = cid; t < a.T && g < ST; t += NC) {
                    for (int s = s0; s < s1 && g < ST; s += G, ++g) {
                        const int n = min(G, s1 - s);
                        ptx::mbar_arrive_expect_tx(&full[g], (uint32_t)(n * (WS + BS)));
                        ptx::bulk_g2s(smem + g * sbytes, a.a + ((size_t)t * a.S + s) * WS, (uint32_t)(n * WS),
                                      &full[g]);
                    }
                }
                pre = g;
            }
            ptx::grid_dependency_wait();
            tl_stamp(a.tl, 1);
            // Slot h of this CTA is stage s0 + (h % spt) * G of its
            // (h / spt)-th tile.  Once the activation copies of the slots
            // loaded before the wait are out, each slot's copy is followed
            // by an L2 request for the weights of the slot l2_ahead + ST - 1
            // further on, so that copy later finds them in L2: more bytes
            // are on their way from HBM than the ring holds.
            const int spt = (s1 - s0 + G - 1) / G;
            int pf = pre;  // next slot whose weights go to L2
            auto l2_upto = [&](int last) {
                for (; a.l2_ahead > 0 && spt > 0 && pf <= last; ++pf) {
                    const int t = cid + (pf / spt) * NC;
                    if (t >= a.T) break;
                    const int s = s0 + (pf % spt) * G;
                    ptx::bulk_prefetch_l2(a.a + ((size_t)t * a.S + s) * WS, (uint32_t)(min(G, s1 - s) * WS));
                }
            };
            int g = 0;
            for (int t = cid; t < a.T && ok; t += NC) {
                for (int s = s0; s < s1; s += G, ++g) {
                    const int slot = g % ST, n = min(G, s1 - s);
                    uint8_t* base = smem + slot * sbytes;
                    if (g >= pre) {
                        if (g >= ST && !ptx::mbar_wait(&empty[slot], ((g / ST) - 1) & 1, WAIT_LIMIT)) {
                            ok = false;
                            break;
                        }
                        ptx::mbar_arrive_expect_tx(&full[slot], (uint32_t)(n * (WS + BS)));
                        ptx::bulk_g2s(base, a.a + ((size_t)t * a.S + s) * WS, (uint32_t)(n * WS), &full[slot]);
                    }
                    ptx::bulk_g2s(base + G * WS, a.b + (size_t)s * BS, (uint32_t)(n * BS), &full[slot]);
                    if (g + 1 >= pre) l2_upto(g + ST + a.l2_ahead - 1);
                }
            }
            // every load is issued: the next kernel may start prefetching
            ptx::launch_dependents();
        }
    } else if (warp == 1) {
        ptx::grid_dependency_wait();
        if (lane == 0) {
            int g = 0, j = 0;
            for (int t = cid; t < a.T && ok; t += NC, ++j) {
                const int buf = NB == 2 ? (j & 1) : 0;
                const int use = NB == 2 ? (j >> 1) : j;  // earlier uses of this accumulator
                if (use > 0 && !ptx::mbar_wait(&tempty[buf], (use - 1) & 1, WAIT_LIMIT)) {
                    ok = false;
                    break;
                }
                ptx::tc_fence_after();
                const uint32_t d_tmem = tmem + ACC_COL + buf * acc_step;
                for (int s = s0; s < s1; s += G, ++g) {
                    const int slot = g % ST;
                    if (!ptx::mbar_wait(&full[slot], (g / ST) & 1, WAIT_LIMIT)) {
                        ok = false;
                        break;
                    }
                    if (g == 0) tl_stamp(a.tl, 2);
                    ptx::tc_fence_after();
                    uint8_t* base = smem + slot * sbytes;
                    const int n = min(G, s1 - s);
                    for (int i = 0; i < n; ++i) {
                        const uint32_t a_addr = ptx::smem_u32(base + i * WS);
                        const uint32_t b_addr = ptx::smem_u32(base + G * WS + i * BS);
                        if (KIND == KIND_MX) {
                            const uint32_t sfa_addr = a_addr + A_STAGE;
                            const uint32_t sfb_addr = b_addr + N * 128;
                            ptx::tmem_cp_32x128b_warpx4(tmem + SFA_COL, ptx::smem_desc(sfa_addr, 16, 128, 0));
                            ptx::tmem_cp_32x128b_warpx4(tmem + SFA_COL + 4,
                                                        ptx::smem_desc(sfa_addr + 512, 16, 128, 0));
                            ptx::tmem_cp_32x128b_warpx4(tmem + SFB_COL, ptx::smem_desc(sfb_addr, 16, 128, 0));
                            ptx::tmem_cp_32x128b_warpx4(tmem + SFB_COL + 4,
                                                        ptx::smem_desc(sfb_addr + 512, 16, 128, 0));
                        }
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            // 32 bytes of K per instruction: 64 E2M1 codes or 16 bf16 values
                            const uint64_t ad = ptx::smem_desc(a_addr + 32 * q, 16, 1024, 2);
                            const uint64_t bd = ptx::smem_desc(b_addr + 32 * q, 16, 1024, 2);
                            const uint32_t acc = (s + i > s0 || q > 0) ? 1u : 0u;
                            if (KIND == KIND_MX) {
                                const uint32_t sf_id = (uint32_t)(q & 1) * 2;
                                const uint32_t sfa_t = (tmem + SFA_COL + (q >> 1) * 4) | (sf_id << 30);
                                const uint32_t sfb_t = (tmem + SFB_COL + (q >> 1) * 4) | (sf_id << 30);
                                ptx::mma_mxf4(d_tmem, ad, bd, ptx::mxf4_idesc(128, (uint32_t)N, sf_id, sf_id),
                                              sfa_t, sfb_t, acc);
                            } else {
                                ptx::mma_bf16(d_tmem, ad, bd, ptx::bf16_idesc(128, (uint32_t)N), acc);
                            }
                        }
                    }
                    ptx::tc_commit(&empty[slot]);
                }
                ptx::tc_commit(&tfull[buf]);
            }
        }
    } else {
        // epilogue warps
        ptx::grid_dependency_wait();
        const int quarter = warp & 3;
        const int row = quarter * 32 + lane;
        const int M = min(a.use_head ? a.hdr->head_rows : a.hdr->rows, a.mcap);
        if (a.part_in) {
            // RMS of each input row from the per-tile sums of squares, in tile order
            if (row < a.mcap) {
                float ss = 0.f;
                for (int i = 0; i < a.part_tiles; ++i) ss = __fadd_rn(ss, a.part_in[i * MX_PART_STRIDE + row]);
                sz_s[row] = __frcp_rn(sqrtf(__fadd_rn(__fdiv_rn(ss, (float)a.norm_width), 1e-6f)));
            }
        }
        // q|k|v: each row's position, cache page and RoPE factors, the same
        // for every head: fetched once, while the first tile's MMAs run
        float2 rope_cs[MX_MAXTOK];
        if (EPI == MX_QKV) {
            if (row < a.mcap) {
                int pos = -1, page = -1;
                if (row < M) {
                    const RowDesc rd = a.rows[row];
                    if (rd.pos >= 0 && rd.pos < a.kv.max_pos && (unsigned)rd.seq < (unsigned)MAX_SEQS) {
                        pos = rd.pos;
                        page = a.page_table[rd.seq][rd.pos / PAGE];
                    } else {
                        atomicOr(a.kv.err, 2);
                    }
                }
                kvpos_s[row] = pos;
                kvpage_s[row] = page;
            }
            epi_bar();
#pragma unroll
            for (int m = 0; m < MX_MAXTOK; ++m) {
                const int pos = m < a.mcap ? kvpos_s[m] : -1;
                rope_cs[m] = pos >= 0 ? a.rope[(size_t)pos * HALF + (row & 63)] : make_float2(1.f, 0.f);
            }
        }
        if (a.part_in) epi_bar();
        int j = 0;
        for (int t = cid; t < a.T; t += NC, ++j) {
            const int buf = NB == 2 ? (j & 1) : 0;
            const int use = NB == 2 ? (j >> 1) : j;
            // the residual this tile adds to: only this tile's epilogue writes
            // it, so load it while the MMAs run
            float xold[MX_MAXTOK];
            float wnext = 1.f;
            if (EPI == MX_ADD) {
                const int gr = t * TILE_ROWS + row;
#pragma unroll
                for (int m = 0; m < MX_MAXTOK; ++m)
                    xold[m] = (m < M && gr < a.out_rows) ? __ldcg(a.y + (size_t)m * a.ldy + gr) : 0.f;
                if (a.next_w) wnext = gr < a.out_rows ? bf16f(a.next_w[gr]) : 0.f;
            }
            if (!ptx::mbar_wait(&tfull[buf], use & 1, WAIT_LIMIT)) ok = false;
            ptx::tc_fence_after();
            if (j == 0 && threadIdx.x == 64) tl_stamp(a.tl, 3);
            float val[MX_MAXTOK];
            const uint32_t lanebase = tmem + ((uint32_t)(quarter * 32) << 16) + ACC_COL + buf * acc_step;
            constexpr int CPR = cols_per_row(KIND), RPL = 32 / CPR;  // rows per 32-column load
#pragma unroll
            for (int m0 = 0; m0 < MX_MAXTOK; m0 += RPL) {
                if (m0 < a.mcap) {  // uniform: the whole warp loads together
                    float v[32];
                    ptx::tmem_ld32(lanebase + m0 * CPR, v);
#pragma unroll
                    for (int i = 0; i < RPL; ++i) {
                        float acc = v[CPR * i + CPR - 1];  // smallest correction first
#pragma unroll
                        for (int p = CPR - 2; p >= 0; --p) acc = __fadd_rn(acc, v[CPR * i + p]);
                        val[m0 + i] = acc;
                    }
                } else {
#pragma unroll
                    for (int i = 0; i < RPL; ++i) val[m0 + i] = 0.f;
                }
            }
            ptx::tc_fence_before();
            __syncwarp();
            if (lane == 0) ptx::mbar_arrive(&tempty[buf]);

            if (ks > 1) {
                const bool more = t + NC < a.T;  // this cluster has another tile
                if (kc > 0) {
                    // push this K slice's partial into the leader's buffer
                    if (j > 0 && !ptx::mbar_wait_cluster(&slot_free, (j - 1) & 1, WAIT_LIMIT)) ok = false;
                    const uint32_t bar = ptx::mapa(ptx::smem_u32(&red_full), 0);
                    const uint32_t dst =
                        ptx::mapa(ptx::smem_u32(red + ((size_t)(kc - 1) * RB * 128 + row) * 4), 0);
#pragma unroll
                    for (int m4 = 0; m4 < MX_MAXTOK; m4 += 4)
                        if (m4 < a.mcap)
                            ptx::st_async_v4(dst + (uint32_t)(m4 / 4) * 128 * 16,
                                             make_float4(val[m4], val[m4 + 1], val[m4 + 2], val[m4 + 3]), bar);
                    // the leader's four warps free the buffer before the next tile
                    if (more && threadIdx.x == 64) ptx::mbar_arrive_expect_tx(&slot_free, 16);
                    continue;
                }
                if (threadIdx.x == 64) ptx::mbar_arrive_expect_tx(&red_full, (uint32_t)((ks - 1) * RB * 128 * 16));
                if (!ptx::mbar_wait_cluster(&red_full, j & 1, WAIT_LIMIT)) ok = false;
                if (j == 0 && threadIdx.x == 64) tl_stamp(a.tl, 4);
#pragma unroll
                for (int m4 = 0; m4 < MX_MAXTOK; m4 += 4) {
                    if (m4 >= a.mcap) continue;
                    // every rank's word first, then the sums in rank order
                    float4 part[MX_MAXCLUSTER - 1];
#pragma unroll
                    for (int r = 1; r < MX_MAXCLUSTER; ++r)
                        if (r < ks)
                            part[r - 1] = *(const float4*)(red + (((size_t)(r - 1) * RB + m4 / 4) * 128 + row) * 4);
#pragma unroll
                    for (int r = 1; r < MX_MAXCLUSTER; ++r) {
                        if (r >= ks) continue;
                        val[m4] = __fadd_rn(val[m4], part[r - 1].x);
                        val[m4 + 1] = __fadd_rn(val[m4 + 1], part[r - 1].y);
                        val[m4 + 2] = __fadd_rn(val[m4 + 2], part[r - 1].z);
                        val[m4 + 3] = __fadd_rn(val[m4 + 3], part[r - 1].w);
                    }
                }
                // this warp has read its rows: one 4-byte store per peer
                __syncwarp();
                if (more && lane >= 1 && lane < ks)
                    ptx::st_async_u32(ptx::mapa(ptx::smem_u32(&free_sig), (uint32_t)lane), 0u,
                                      ptx::mapa(ptx::smem_u32(&slot_free), (uint32_t)lane));
            }
            if (a.part_in) {  // input RMSNorm: scale by 1 / the row's RMS (lib.rs:268-290)
#pragma unroll
                for (int m = 0; m < MX_MAXTOK; ++m)
                    if (m < a.mcap) val[m] = __fmul_rn(val[m], sz_s[m]);
            }
            if (EPI == MX_SWIGLU) {
                // tile rows 0..63: gate rows 64t.., rows 64..127: the matching up rows
                if (row >= 64) {
#pragma unroll
                    for (int m = 0; m < MX_MAXTOK; ++m)
                        if (m < a.mcap) xs[m][row - 64] = val[m];
                }
                epi_bar();
                if (row < 64) {
                    const int k = t * 64 + row;
#pragma unroll
                    for (int m = 0; m < MX_MAXTOK; ++m) {
                        float act = 0.f;
                        if (m < M && k < a.out_rows) {
                            const float gt = val[m], up = xs[m][row];
                            act = __fmul_rn(__fdiv_rn(gt, __fadd_rn(1.0f, expf(-gt))), up);
                            if (a.y) a.y[(size_t)m * a.ldy + k] = act;
                        }
                        val[m] = act;
                    }
                }
                if (j == 0 && threadIdx.x == 64) tl_stamp(a.tl, 5);
                if (a.bout) {  // the tile's 64 activations: two 32-blocks of the down input
                    epi_bar();  // every up value has been read
                    if (row < 64) {
#pragma unroll
                        for (int m = 0; m < MX_MAXTOK; ++m)
                            if (m < a.mcap) xs[m][row] = val[m];
                    }
                    epi_bar();
                    mx::emit_pieces_smem(&xs[0][0], 64, 2, 0, a.mcap, a.mcap, row, 128, t * 64, a.bN, a.bout);
                }
                epi_bar();  // xs is reused by the next unit
            } else if (EPI == MX_QKV) {
                // tile t is head t: q heads, then k heads, then v heads (lib.rs:363-396)
                const int Hq = a.q_heads, Hkv = a.kv_heads;
                const bool is_q = t < Hq, is_k = !is_q && t < Hq + Hkv;
                if (is_q || is_k) {
                    const float w = bf16f((is_q ? a.qn : a.kn)[row]);
                    warp_sq_sums(val, a.mcap, red_s, quarter, lane);
                    epi_bar();
                    if (row < a.mcap) {
                        const float ss = __fadd_rn(__fadd_rn(red_s[0][row], red_s[1][row]),
                                                   __fadd_rn(red_s[2][row], red_s[3][row]));
                        qk_s[row] = __frcp_rn(sqrtf(__fadd_rn(__fdiv_rn(ss, 128.0f), 1e-6f)));
                    }
                    epi_bar();
#pragma unroll
                    for (int m = 0; m < MX_MAXTOK; ++m)
                        if (m < a.mcap) val[m] = __fmul_rn(__fmul_rn(val[m], qk_s[m]), w);
                    // RoPE pairs (i, i + 64) sit in rows i and i + 64: swap halves
                    // through shared memory, low half first
                    float other[MX_MAXTOK];
                    if (row < 64) {
#pragma unroll
                        for (int m = 0; m < MX_MAXTOK; ++m)
                            if (m < a.mcap) xs[m][row] = val[m];
                    }
                    epi_bar();
                    if (row >= 64) {
#pragma unroll
                        for (int m = 0; m < MX_MAXTOK; ++m) other[m] = m < a.mcap ? xs[m][row - 64] : 0.f;
                    }
                    epi_bar();
                    if (row >= 64) {
#pragma unroll
                        for (int m = 0; m < MX_MAXTOK; ++m)
                            if (m < a.mcap) xs[m][row - 64] = val[m];
                    }
                    epi_bar();
                    if (row < 64) {
#pragma unroll
                        for (int m = 0; m < MX_MAXTOK; ++m) other[m] = m < a.mcap ? xs[m][row] : 0.f;
                    }
#pragma unroll
                    for (int m = 0; m < MX_MAXTOK; ++m) {
                        // lib.rs:306-313: out[i] = a cos - b sin; out[i+64] = b cos + a sin
                        const float2 r = rope_cs[m];
                        const float v = row < 64 ? __fsub_rn(__fmul_rn(val[m], r.x), __fmul_rn(other[m], r.y))
                                                 : __fadd_rn(__fmul_rn(val[m], r.x), __fmul_rn(other[m], r.y));
                        if (m < M) val[m] = v;
                    }
                    epi_bar();  // xs and red_s are reused by the next unit
                }
                if (is_q) {
#pragma unroll
                    for (int m = 0; m < MX_MAXTOK; ++m)
                        if (m < M) a.y[(size_t)m * a.ldy + t * TILE_ROWS + row] = val[m];
                } else {
                    const int kvh = is_k ? t - Hq : t - Hq - Hkv;
                    void* dst = is_k ? a.kv.k : a.kv.v;
#pragma unroll
                    for (int m = 0; m < MX_MAXTOK; ++m) {
                        if (m >= M) continue;
                        const int pos = kvpos_s[m], page = kvpage_s[m];
                        if (pos < 0 || !page_ok(a.kv, page)) continue;  // bad positions were flagged
                        const size_t idx = kv_index(page, kvh, pos % PAGE, a.kv.kv_heads) + row;
                        if (a.kv.f32) ((float*)dst)[idx] = val[m];
                        else ((uint16_t*)dst)[idx] = f2bf16(val[m]);
                    }
                }
            } else if (EPI == MX_HEAD) {
                // logits, and this tile's first maximum per row (model.rs:288-296):
                // ties go to the lower vocabulary index
                const int gr = t * TILE_ROWS + row;
                const bool valid = gr < a.out_rows;
#pragma unroll
                for (int m = 0; m < MX_MAXTOK; ++m)
                    if (m < M && valid) a.y[(size_t)m * a.ldy + gr] = val[m];
#pragma unroll
                for (int m = 0; m < MX_MAXTOK; ++m) {
                    float bv = valid ? val[m] : -INFINITY;
                    int bi = gr;
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) {
                        const float ov = __shfl_down_sync(0xffffffffu, bv, o);
                        const int oi = __shfl_down_sync(0xffffffffu, bi, o);
                        if (ov > bv || (ov == bv && oi < bi)) {
                            bv = ov;
                            bi = oi;
                        }
                    }
                    if (lane == 0) {
                        red_s[quarter][m] = bv;
                        redi_s[quarter][m] = bi;
                    }
                }
                epi_bar();
                if (row < M) {  // quarters hold increasing indices: keep the first on ties
                    float bv = red_s[0][row];
                    int bi = redi_s[0][row];
                    for (int q = 1; q < 4; ++q)
                        if (red_s[q][row] > bv) {
                            bv = red_s[q][row];
                            bi = redi_s[q][row];
                        }
                    a.amax_v[t * MX_PART_STRIDE + row] = bv;
                    a.amax_i[t * MX_PART_STRIDE + row] = bi;
                }
                epi_bar();  // red_s is reused by the next tile
            } else {
                const int gr = t * TILE_ROWS + row;
                const bool valid = gr < a.out_rows;
#pragma unroll
                for (int m = 0; m < MX_MAXTOK; ++m) {
                    if (m < M && valid) {
                        const float v = EPI == MX_ADD ? __fadd_rn(xold[m], val[m]) : val[m];
                        a.y[(size_t)m * a.ldy + gr] = v;
                        val[m] = v;
                    } else {
                        val[m] = 0.f;
                    }
                }
                if (j == 0 && threadIdx.x == 64) tl_stamp(a.tl, 5);
                if (a.bout) {  // the next projection's input: pieces of x * w
#pragma unroll
                    for (int m = 0; m < MX_MAXTOK; ++m)
                        if (m < a.mcap) slot[m * 128 + row] = __fmul_rn(val[m], wnext);
                    epi_bar();
                    mx::emit_pieces_smem(slot, 128, 4, 0, a.mcap, a.mcap, row, 128, t * TILE_ROWS, a.bN,
                                         a.bout);
                    epi_bar();  // the staging area is reused by the next tile
                }
                if (a.part_out) {  // sum of squares of this tile's 128 outputs, per row
                    warp_sq_sums(val, a.mcap, red_s, quarter, lane);
                    epi_bar();
                    if (row < a.mcap)
                        a.part_out[t * MX_PART_STRIDE + row] = __fadd_rn(__fadd_rn(red_s[0][row], red_s[1][row]),
                                                                    __fadd_rn(red_s[2][row], red_s[3][row]));
                    epi_bar();
                }
            }
        }
    }
    if (threadIdx.x == 64) tl_stamp(a.tl, 6);
    ptx::launch_dependents();
    ptx::tc_fence_before();
    __syncthreads();
    if (ks > 1) {  // no CTA leaves while a store to or from it may be in flight
        ptx::cluster_arrive();
        ptx::cluster_wait();
    }
    if (warp == 1) ptx::tmem_dealloc(tmem, tcols);
    if (!ok && lane == 0) atomicOr(a.err, 4);  // a bounded wait gave up
    if (threadIdx.x == 0) tl_stamp(a.tl, 7);
}
}  // namespace

}  // namespace jl

namespace jl {

namespace {

// Load-time re-layout of up to three row-major MXFP4 matrices (stacked along
// the output dimension, or gate/up interleaved per 64 rows) into the tiled,
// swizzled images k_mx_mma streams.  One thread per 16-byte chunk.
struct TileSrc {
    const uint8_t* packed[3];
    const uint8_t* scales[3];
    int rows[3];
};

__device__ __forceinline__ bool tile_row(const TileSrc& src, int swiglu, int t, int r, int& mat,
                                         int& local) {
    if (swiglu) {
        mat = r < 64 ? 0 : 1;
        local = t * 64 + (r & 63);
        return local < src.rows[mat];
    }
    int g = t * TILE_ROWS + r;
    for (mat = 0; mat < 3; ++mat) {
        if (g < src.rows[mat]) {
            local = g;
            return true;
        }
        g -= src.rows[mat];
    }
    return false;
}

__global__ void k_mx_tile(TileSrc src, int swiglu, int K, int T, int S, uint8_t* __restrict__ a) {
    const size_t chunks = (size_t)T * S * TILE_ROWS * 8;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < chunks;
         i += (size_t)gridDim.x * blockDim.x) {
        const int c16 = (int)(i % 8);
        const int r = (int)((i / 8) % TILE_ROWS);
        const int s = (int)((i / (8 * TILE_ROWS)) % S);
        const int t = (int)(i / ((size_t)8 * TILE_ROWS * S));
        int mat, local;
        const bool have = tile_row(src, swiglu, t, r, mat, local);
        const int k0 = s * STAGE_K + c16 * 32;  // first element of this 16-byte chunk
        uint4 v = make_uint4(0, 0, 0, 0);
        uint8_t sc = 0;
        if (have && k0 < K) {
            v = *reinterpret_cast<const uint4*>(src.packed[mat] + (size_t)local * (K / 2) + k0 / 2);
            sc = src.scales[mat][(size_t)local * (K / 32) + k0 / 32];
        }
        uint8_t* tile = a + ((size_t)t * S + s) * w_stage(KIND_MX);
        *reinterpret_cast<uint4*>(tile + swz128((uint32_t)r, (uint32_t)c16 * 16)) = v;
        tile[A_STAGE + sf_offset((uint32_t)r, (uint32_t)c16)] = sc;
    }
}

constexpr int MX_MAXDEV = 64;
// Clusters of each size that fit at one CTA per SM, per device (the GPU's
// processing clusters decide how many SMs a cluster size can use).
int g_clusters[MX_MAXDEV][MX_MAXCLUSTER + 1];

int mx_clusters(int ks) {
    int dev = 0;
    cudaGetDevice(&dev);
    const int n = (dev >= 0 && dev < MX_MAXDEV) ? g_clusters[dev][ks] : 0;
    return n > 0 ? n : 1;
}

// K slices per tile, from an estimate in microseconds of the time after the
// dependency wait: a CTA's first MX_PREFETCH stages are loaded before the
// wait, the rest stream at its share of HBM bandwidth (at most what one SM
// pulls); a tile costs about a microsecond of epilogue, and a split the
// reduction through distributed shared memory.  The choice depends only on
// the matrix shape, never on the token count.  A split holds at least one
// two-stage slot.
constexpr int MX_PREFETCH = 4;           // ring stages issued before the dependency wait
constexpr double MX_STAGE_KB = 17.0;     // weight bytes of a stage (codes + scales)
constexpr double MX_HBM_GBS = 6000.0;
constexpr double MX_SM_GBS = 60.0;       // one CTA's copy rate with two-stage copies
constexpr double MX_EPI_US = 1.0;
constexpr double MX_REDUCE_US = 1.5;

int mx_ksplit(int T, int S) {
    int best = 1;
    double best_cost = 1e30;
    for (int ks = 1; ks <= std::min((S + 1) / 2, MX_MAXCLUSTER); ++ks) {
        const int nc = std::min(mx_clusters(ks), T);
        const int tiles = (T + nc - 1) / nc;            // per cluster
        const int stages = tiles * ((S + ks - 1) / ks);  // per CTA
        const double after_kb = std::max(0, stages - MX_PREFETCH) * MX_STAGE_KB;
        const double gbs = std::min(MX_SM_GBS, MX_HBM_GBS / (nc * ks));
        const double cost = after_kb / gbs + tiles * MX_EPI_US + (ks > 1 ? MX_REDUCE_US : 0.0);
        if (cost < best_cost - 1e-9) {
            best_cost = cost;
            best = ks;
        }
    }
    return best;
}

// Ring slots, stages per slot and accumulator buffers for N MMA columns:
// two accumulators of up to 64 columns and two slots of two stages, or one
// accumulator of up to 128 and three one-stage slots; at most about 105 KB
// of ring, so a CTA of the next projection fits on the same SM
// (programmatic dependent launch).
void mx_shape(int N, int* stages, int* nbuf, int* group) {
    *nbuf = N <= 64 ? 2 : 1;
    *stages = N <= 64 ? 2 : 3;
    *group = N <= 64 ? 2 : 1;
}

// Ring slots, epilogue scratch (mcap rows rounded up to 4, x 128 f32), the
// leader's split-K buffer (ks - 1 partials of the same size), then alignment
// slack.  At five rows and up to four-way splits this stays under half an SM.
size_t mx_smem(int N, int kind, int mcap, int ks) {
    int st, nb, gr;
    mx_shape(N, &st, &nb, &gr);
    const size_t part = (size_t)((mcap + 3) & ~3) * 512;
    return (size_t)st * mx_slot_bytes(N, kind, gr) + part * ks + 1024;
}

// Multi-chunk launches of N > 64 columns run several tiles per CTA and hold
// the SM alone (MX_ONE_PER_SM), so their ring takes the shared memory a CTA
// may have: slots of MX_MULTI_GROUP stages, as many (up to MX_MAXSTAGES) as
// fit beside the epilogue scratch.  Measured on a 4096-token Qwen3-8B
// prompt: three one-stage slots 398 ms, six one-stage slots 397 ms, three
// two-stage slots 332 ms, two three-stage slots 351 ms.
constexpr int MX_MULTI_GROUP = 2;
constexpr size_t MX_SMEM_LIMIT = 227 * 1024 - 2048;  // dynamic + this kernel's static shared memory
int mx_multi_slots(int N, int kind, int mcap, int ks) {
    const size_t part = (size_t)((mcap + 3) & ~3) * 512;
    const size_t slot = (size_t)mx_slot_bytes(N, kind, MX_MULTI_GROUP);
    int slots = 0;
    while (slots < MX_MAXSTAGES && (size_t)(slots + 1) * slot + part * ks + 1024 <= MX_SMEM_LIMIT) ++slots;
    return slots;
}
size_t mx_multi_smem(int N, int kind, int mcap, int ks) {
    const size_t part = (size_t)((mcap + 3) & ~3) * 512;
    return (size_t)mx_multi_slots(N, kind, mcap, ks) * mx_slot_bytes(N, kind, MX_MULTI_GROUP) + part * ks + 1024;
}

// Ring slots requested into L2 beyond the ring by k_mx_gemv's loader: on for
// the output table (measured on B200: the 8B's 1.245 GB table 220 -> 202 us
// per pass), off for the layer projections (slightly slower with it).
constexpr int MX_L2_AHEAD = 1;

constexpr int MX_PROBE_SMEM = 120 * 1024;  // more than half an SM: one CTA per SM
// Dynamic shared memory of a launch whose CTAs allocate all 512 TMEM
// columns: more than half an SM, so no two CTAs (of one cluster above all,
// which wait for each other) ever share an SM and its TMEM.
constexpr size_t MX_ONE_PER_SM = 116 * 1024;

template <int EPI, int KIND>
jl_status configure_mx() {
    const size_t most = std::max(std::max(mx_smem(64, KIND, MX_MAXTOK, MX_MAXCLUSTER),
                                          mx_smem(8 * MX_MAXTOK, KIND, MX_MAXTOK, MX_MAXCLUSTER)),
                                 MX_SMEM_LIMIT);
    JL_CUDA(cudaFuncSetAttribute(k_mx_gemv<EPI, KIND>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)std::max<size_t>(MX_PROBE_SMEM, most)));
    JL_CUDA(cudaFuncSetAttribute(k_mx_gemv<EPI, KIND>, cudaFuncAttributePreferredSharedMemoryCarveout, 100));
    return JL_OK;
}

template <int EPI, int KIND>
jl_status launch_gemv_t(const MxArgs& a, int sms, cudaStream_t stream, int chunks) {
    // One wave of CTAs (one per SM at these shapes): a multi-chunk launch
    // gives each chunk its share of the wave's clusters (at most one per
    // tile), so a CTA runs several tiles through its ring instead of each
    // chunk waiting for a wave of its own.  When the chunks' tiles are many
    // times the SMs, split-K is dropped: a CTA then runs whole tiles, one
    // epilogue each, with no partials to exchange.
    // (A 4096-token Qwen3-8B prompt: 398 ms with min(T, clusters) / chunks
    // clusters per chunk and the planned split-K, 301 ms with this share,
    // 255 ms with split-K dropped as well.)
    const int ks = (chunks > 1 && a.N > 64 && (long long)a.T * chunks >= 4LL * sms) ? 1 : a.ksplit;
    const int per = ks > 1 ? mx_clusters(ks) : sms;
    const int nc = std::max(1, std::min(a.T, per / chunks));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(nc * ks, chunks);
    cfg.blockDim = dim3(MX_THREADS);
    cfg.dynamicSmemBytes = mx_smem(a.N, KIND, a.mcap, ks);
    MxArgs b = a;
    b.ksplit = ks;
    b.l2_ahead = EPI == MX_HEAD ? MX_L2_AHEAD : 0;
    static const char* const names[] = {"k_mx_gemv<store>", "k_mx_gemv<add>", "k_mx_gemv<swiglu>",
                                        "k_mx_gemv<qkv>", "k_mx_gemv<head>"};
    b.tl = tl_launch(names[EPI]);
    if (chunks > 1 && a.N > 64) {
        // several tiles per CTA: two 128-column accumulators, so a tile's
        // epilogue overlaps the next tile's MMAs
        b.nbuf = 2;
        b.acc_step = 256;
        cfg.dynamicSmemBytes = std::max(cfg.dynamicSmemBytes, MX_ONE_PER_SM);
        const int slots = mx_multi_slots(a.N, KIND, a.mcap, ks);
        if (slots * MX_MULTI_GROUP > a.stages * a.group) {  // the deeper ring, where it fits
            b.stages = slots;
            b.group = MX_MULTI_GROUP;
            cfg.dynamicSmemBytes = std::max(mx_multi_smem(a.N, KIND, a.mcap, ks), MX_ONE_PER_SM);
        }
    }
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    int n = 1;
    if (ks > 1) {
        attr[1].id = cudaLaunchAttributeClusterDimension;
        attr[1].val.clusterDim.x = (unsigned)ks;
        attr[1].val.clusterDim.y = 1;
        attr[1].val.clusterDim.z = 1;
        n = 2;
    }
    cfg.attrs = attr;
    cfg.numAttrs = n;
    JL_CUDA(cudaLaunchKernelEx(&cfg, k_mx_gemv<EPI, KIND>, b));
    return JL_OK;
}

jl_status launch_gemv(int epi, const MxArgs& a, int sms, cudaStream_t stream, int chunks = 1) {
    if (a.ksplit < 1 || a.ksplit > MX_MAXCLUSTER) {
        set_error("tensor-core projection: split-K %d outside 1..%d", a.ksplit, MX_MAXCLUSTER);
        return JL_ERR_INVALID_ARG;
    }
    switch (epi) {
        case MX_ADD: return launch_gemv_t<MX_ADD, KIND_MX>(a, sms, stream, chunks);
        case MX_SWIGLU: return launch_gemv_t<MX_SWIGLU, KIND_MX>(a, sms, stream, chunks);
        case MX_QKV: return launch_gemv_t<MX_QKV, KIND_MX>(a, sms, stream, chunks);
        case MX_HEAD: return launch_gemv_t<MX_HEAD, KIND_BF>(a, sms, stream, chunks);
        default: return launch_gemv_t<MX_STORE, KIND_MX>(a, sms, stream, chunks);
    }
}

}  // namespace

jl_status mx_configure() {
    JL_TRY((configure_mx<MX_STORE, KIND_MX>()));
    JL_TRY((configure_mx<MX_ADD, KIND_MX>()));
    JL_TRY((configure_mx<MX_SWIGLU, KIND_MX>()));
    JL_TRY((configure_mx<MX_QKV, KIND_MX>()));
    JL_TRY((configure_mx<MX_HEAD, KIND_BF>()));
    cudaFuncAttributes fa;  // loads the piece encoder now rather than at its first launch
    JL_CUDA(cudaFuncGetAttributes(&fa, k_mx_pieces));
    int dev = 0, sms = 0;
    JL_CUDA(cudaGetDevice(&dev));
    JL_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    if (dev >= 0 && dev < MX_MAXDEV) {
        g_clusters[dev][1] = sms;
        for (int ks = 2; ks <= MX_MAXCLUSTER; ++ks) {
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3(ks * sms);
            cfg.blockDim = dim3(MX_THREADS);
            cfg.dynamicSmemBytes = MX_PROBE_SMEM;
            cudaLaunchAttribute attr[1];
            attr[0].id = cudaLaunchAttributeClusterDimension;
            attr[0].val.clusterDim.x = (unsigned)ks;
            attr[0].val.clusterDim.y = 1;
            attr[0].val.clusterDim.z = 1;
            cfg.attrs = attr;
            cfg.numAttrs = 1;
            int n = 0;
            JL_CUDA(cudaOccupancyMaxActiveClusters(&n, k_mx_gemv<MX_STORE, KIND_MX>, &cfg));
            g_clusters[dev][ks] = n;
        }
    }
    return JL_OK;
}

int mx_max_tokens() { return MX_MAXTOK; }

size_t mx_tile_bytes(int out_rows, int K, bool swiglu) {
    const int T = swiglu ? (out_rows + 63) / 64 : (out_rows + TILE_ROWS - 1) / TILE_ROWS;
    const int S = (K + STAGE_K - 1) / STAGE_K;
    return (size_t)T * S * (A_STAGE + SF_STAGE);
}

jl_status mx_build(const Mat* const* mats, int nmats, bool swiglu, uint8_t* dst, int sms,
                   MxProj* out, cudaStream_t stream) {
    TileSrc src{};
    int rows = 0;
    const int K = mats[0]->cols;
    for (int i = 0; i < nmats; ++i) {
        if (mats[i]->kind != MAT_MXFP4 || mats[i]->cols != K) {
            set_error("tensor-core projections need MXFP4 matrices of one width");
            return JL_ERR_INVALID_ARG;
        }
        src.packed[i] = (const uint8_t*)mats[i]->data;
        src.scales[i] = mats[i]->scales;
        src.rows[i] = mats[i]->rows;
        rows += mats[i]->rows;
    }
    const int out_rows = swiglu ? mats[0]->rows : rows;
    MxProj p;
    // the last tile is zero-padded; its padding rows are never written out
    p.T = swiglu ? (out_rows + 63) / 64 : (out_rows + TILE_ROWS - 1) / TILE_ROWS;
    p.S = (K + STAGE_K - 1) / STAGE_K;
    p.K = K;
    p.swiglu = swiglu;
    p.out_rows = out_rows;
    p.a = dst;
    p.ksplit = mx_ksplit(p.T, p.S);
    (void)sms;
    const size_t chunks = (size_t)p.T * p.S * TILE_ROWS * 8;
    const int grid = (int)std::min<size_t>((chunks + 255) / 256, (size_t)sms * 8);
    k_mx_tile<<<grid, 256, 0, stream>>>(src, swiglu ? 1 : 0, K, p.T, p.S, (uint8_t*)p.a);
    JL_CUDA(cudaGetLastError());
    *out = p;
    return JL_OK;
}

jl_status mx_project(const PassCtx& c, const MxProj& p, int epi, int use_head, const float* x,
                     int ldx, const uint16_t* norm, float* y, int ldy) {
    const jl_model* m = c.m;
    const int mcap = use_head ? c.head_cap : c.rows_cap;
    if (mcap < 1 || mcap > MX_MAXTOK) {
        set_error("tensor-core projection takes 1..%d rows per pass, got %d", MX_MAXTOK, mcap);
        return JL_ERR_INVALID_ARG;
    }
    const int N = PIECES * mcap;
    (void)norm;  // inputs arrive normalised; see launch_rmsnorm
    const int items = mcap * p.S * (STAGE_K / 32);
    JL_TRY(launch_pdl(k_mx_pieces, dim3((items + 7) / 8), dim3(256), 0, c.stream,
                      (const PassHdr*)c.pass().hdr, use_head, mcap, x, ldx, p.K, p.S, N, m->mx.bimg));
    MxArgs a = {};
    a.a = p.a;
    a.b = m->mx.bimg;
    a.T = p.T;
    a.S = p.S;
    a.ksplit = p.ksplit;
    a.N = N;
    a.mcap = mcap;
    mx_shape(N, &a.stages, &a.nbuf, &a.group);
    a.hdr = c.pass().hdr;
    a.use_head = use_head;
    a.y = y;
    a.ldy = ldy;
    a.out_rows = p.out_rows;
    a.ws = m->mx.ws;
    a.tickets = m->mx.tickets;
    a.err = m->counters;
    return launch_gemv(epi, a, m->sms, c.stream);
}

// Rows per chunk of a pass on the fused kernels, or 0 when it has none.
int chunk_rows(const PassCtx& c) {
    if (c.chunks > 1)
        return c.chunks <= c.m->mx.chunks && c.rows_cap == c.chunks * MX_MAXTOK ? MX_MAXTOK : 0;
    return c.rows_cap >= 1 && c.rows_cap <= MX_MAXTOK ? c.rows_cap : 0;
}

jl_status mx_norm_pieces(const PassCtx& c, const float* x, int ldx, const uint16_t* w, int width,
                         uint8_t* bout, float* part) {
    const int mcap = chunk_rows(c);
    if (!mcap || width % STAGE_K) {
        set_error("norm pieces take 1..%d rows (or %d chunks of %d) and a width that is a multiple of %d",
                  MX_MAXTOK, c.m->mx.chunks, MX_MAXTOK, STAGE_K);
        return JL_ERR_INVALID_ARG;
    }
    return launch_pdl(k_norm_pieces, dim3(width / 128, mcap, c.chunks), dim3(128), 0, c.stream,
                      (const PassHdr*)c.pass().hdr, mcap, x, ldx, w, width, PIECES * mcap, bout, part,
                      c.m->mx.sx, c.m->mx.spart);
}

jl_status mx_project_fused(const PassCtx& c, const MxProj& p, int epi, const MxFuse& f, float* y,
                           int ldy) {
    const jl_model* m = c.m;
    const int mcap = chunk_rows(c);
    if (!mcap) {
        set_error("tensor-core projection takes 1..%d rows per pass (or %d chunks of %d), got %d", MX_MAXTOK,
                  m->mx.chunks, MX_MAXTOK, c.rows_cap);
        return JL_ERR_INVALID_ARG;
    }
    const int N = PIECES * mcap;
    MxArgs a = {};
    a.a = p.a;
    a.b = f.b;
    a.T = p.T;
    a.S = p.S;
    a.ksplit = p.ksplit;
    a.N = N;
    a.mcap = mcap;
    mx_shape(N, &a.stages, &a.nbuf, &a.group);
    a.hdr = c.pass().hdr;
    a.use_head = 0;
    a.y = y;
    a.ldy = ldy;
    a.out_rows = p.out_rows;
    a.ws = m->mx.ws;
    a.tickets = m->mx.tickets;
    a.err = m->counters;
    a.part_in = f.part_in;
    a.part_tiles = f.part_tiles;
    a.norm_width = f.norm_width;
    a.bout = f.bout;
    a.bN = N;
    a.part_out = f.part_out;
    a.next_w = f.next_w;
    if (epi == MX_QKV) {
        a.q_heads = m->q_heads;
        a.kv_heads = m->kv_heads;
        a.qn = f.qn;
        a.kn = f.kn;
        a.rope = (const float2*)m->rope;
        a.rows = c.pass().row;
        a.page_table = c.pass().page_table;
        a.kv = kv_view(m, f.layer);
    }
    a.cs_b = f.cs_b;
    a.cs_bout = f.cs_bout;
    a.cs_part_in = m->mx.spart;
    a.cs_part_out = m->mx.spart;
    return launch_gemv(epi, a, m->sms, c.stream, c.chunks);
}

MxScratchPlan mx_scratch_plan(const MxProj& p, int mcap) {
    auto up = [](size_t b) { return (b + 255) & ~(size_t)255; };
    MxScratchPlan s;
    s.tickets = up((size_t)p.T * sizeof(int));
    s.bimg = up((size_t)p.S * mx::img_stage(PIECES * mcap));
    s.ws = p.ksplit > 1 ? up((size_t)p.T * p.ksplit * mcap * 128 * sizeof(float)) : 0;
    s.total = s.tickets + s.bimg + s.ws;
    return s;
}

jl_status mx_project_with(const MxProj& p, int epi, const PassHdr* hdr, int mcap, const float* x,
                          int ldx, float* y, int ldy, uint8_t* scratch, int* err, int sms,
                          cudaStream_t stream) {
    if (mcap < 1 || mcap > MX_MAXTOK) {
        set_error("tensor-core projection takes 1..%d rows per pass, got %d", MX_MAXTOK, mcap);
        return JL_ERR_INVALID_ARG;
    }
    const MxScratchPlan plan = mx_scratch_plan(p, mcap);
    int* tickets = (int*)scratch;
    uint8_t* bimg = scratch + plan.tickets;
    float* ws = (float*)(bimg + plan.bimg);
    const int N = PIECES * mcap;
    const int items = mcap * p.S * (STAGE_K / 32);
    JL_TRY(launch_pdl(k_mx_pieces, dim3((items + 7) / 8), dim3(256), 0, stream, hdr, 0, mcap, x, ldx,
                      p.K, p.S, N, bimg));
    MxArgs a = {};
    a.a = p.a;
    a.b = bimg;
    a.T = p.T;
    a.S = p.S;
    a.ksplit = p.ksplit;
    a.N = N;
    a.mcap = mcap;
    mx_shape(N, &a.stages, &a.nbuf, &a.group);
    a.hdr = hdr;
    a.use_head = 0;
    a.y = y;
    a.ldy = ldy;
    a.out_rows = p.out_rows;
    a.ws = ws;
    a.tickets = tickets;
    a.err = err;
    return launch_gemv(epi, a, sms, stream);
}

size_t bf16_tile_bytes(int rows, int K) {
    const int T = (rows + TILE_ROWS - 1) / TILE_ROWS, S = (K + 63) / 64;
    return (size_t)T * S * A_STAGE;
}

jl_status mx_build_bf16(const Mat& w, uint8_t* dst, MxProj* out, cudaStream_t stream) {
    if (w.kind != MAT_BF16 || w.cols % 64) {
        set_error("the bf16 tensor-core table needs bf16 rows of a multiple of 64 elements");
        return JL_ERR_INVALID_ARG;
    }
    MxProj p;
    p.T = (w.rows + TILE_ROWS - 1) / TILE_ROWS;
    p.S = w.cols / 64;
    p.K = w.cols;
    p.out_rows = w.rows;
    p.a = dst;
    p.ksplit = mx_ksplit(p.T, p.S);
    const size_t chunks = (size_t)p.T * p.S * TILE_ROWS * 8;
    const int grid = (int)std::min<size_t>((chunks + 255) / 256, 148 * 8);
    k_bf16_tile<<<grid, 256, 0, stream>>>((const uint16_t*)w.data, w.rows, w.cols, p.T, p.S, dst);
    JL_CUDA(cudaGetLastError());
    *out = p;
    return JL_OK;
}

jl_status mx_head_fused(const PassCtx& c, const MxProj& p, const uint16_t* norm, float* logits,
                        int ldy) {
    const jl_model* m = c.m;
    const int mcap = c.chunks > 1 ? chunk_rows(c) : c.head_cap;
    if (mcap < 1 || mcap > MX_MAXTOK || !m->mx.bhead) {
        set_error("tensor-core output table takes 1..%d rows per pass (or %d chunks of %d)", MX_MAXTOK,
                  m->mx.chunks, MX_MAXTOK);
        return JL_ERR_INVALID_ARG;
    }
    const int N = ((4 * mcap + 7) / 8) * 8;  // four pieces per row, a multiple of 8 columns
    JL_TRY(launch_pdl(k_head_pieces, dim3(N / 4, c.chunks), dim3(256), 0, c.stream, c.pass(), mcap,
                      (const float*)m->s.x, m->hidden, norm, N, m->mx.bhead, m->mx.shead));
    MxArgs a = {};
    a.a = p.a;
    a.b = m->mx.bhead;
    a.T = p.T;
    a.S = p.S;
    a.ksplit = p.ksplit;
    a.N = N;
    a.mcap = mcap;
    mx_shape(N, &a.stages, &a.nbuf, &a.group);
    a.hdr = c.pass().hdr;
    a.use_head = 1;
    a.y = logits;
    a.ldy = ldy;
    a.out_rows = p.out_rows;
    a.err = m->counters;
    a.amax_v = m->mx.amax_v;
    a.amax_i = m->mx.amax_i;
    a.cs_b = m->mx.shead;
    a.cs_amax = m->mx.samax;
    JL_TRY(launch_gemv(MX_HEAD, a, m->sms, c.stream, c.chunks));
    return launch_pdl(k_argmax_tiles, dim3(mcap, c.chunks), dim3(256), 0, c.stream, c.pass(), p.T,
                      (const float*)m->mx.amax_v, (const int*)m->mx.amax_i, m->mx.samax);
}

}  // namespace jl
