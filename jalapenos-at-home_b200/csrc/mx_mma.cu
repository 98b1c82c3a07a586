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
//    row), 16 KB in the 128-byte-swizzled K-major layout the MMA reads;
//  * its scales: two 512-byte atoms (128 rows x 4 blocks of 32), byte
//    16*(r%32) + 4*(r/32) + kb, which tcgen05.cp broadcasts into 4 TMEM
//    columns;
//  * activation pieces for stage s: N rows x 128 bytes, same swizzle, and
//    their scale atoms (N <= 128).
// Split-K partials go to a workspace; the last CTA of a tile (atomic ticket)
// adds them in a fixed order and runs the epilogue, so a row's result does
// not depend on timing or on how many tokens share the pass.
#include <cstdio>

#include <algorithm>

#include "jl_internal.h"
#include "kernels.cuh"
#include "launch.cuh"
#include "ptx.cuh"

namespace jl {

namespace {

constexpr int PIECES = 8;
constexpr int TILE_ROWS = 128;
constexpr int STAGE_K = 256;             // K elements per pipeline stage
constexpr int A_STAGE = 128 * 128;       // bytes of one weight tile stage
constexpr int SF_STAGE = 1024;           // two scale atoms
constexpr uint32_t WAIT_LIMIT = 1u << 22;  // polls before a wait reports failure (seconds)
constexpr int TMEM_COLS = 256;
constexpr int ACC_COL = 0, SFA_COL = 128, SFB_COL = 136;

__device__ __forceinline__ uint32_t swz128(uint32_t row, uint32_t byte) {
    // byte offset of (row, byte-in-row) in a 128B-swizzled K-major image
    return (row >> 3) * 1024 + (row & 7) * 128 + ((((byte >> 4) ^ (row & 7)) & 7) << 4) + (byte & 15);
}

__device__ __forceinline__ uint32_t sf_offset(uint32_t row, uint32_t kb) {
    // kb: scale block within the stage (0..7); row < 128
    return (kb >> 2) * 512 + 16 * (row & 31) + 4 * (row >> 5) + (kb & 3);
}

// ---------------------------------------------------------------------------
// activation pieces

// 2^e as an exact f32 for e in [-127, 127].
__device__ __forceinline__ float pow2i(int e) {
    return e >= -126 ? __uint_as_float((uint32_t)(e + 127) << 23) : __uint_as_float(0x00400000u);
}

// Smallest E8M0 exponent e with amax <= 6 * 2^e (amax >= 0), clamped to the
// E8M0 range; -127 for an all-zero block.
__device__ __forceinline__ int piece_exponent(float amax) {
    const uint32_t b = __float_as_uint(amax);
    const int eb = (int)((b >> 23) & 0xFF);
    if (eb == 0) return -127;  // zero or subnormal: 6 * 2^-127 covers it
    // amax = 1.f * 2^(eb-127): 6 * 2^(eb-130) = 0.75 * 2^(eb-127) suffices when
    // the significand is at most 1.5
    const int e = (b & 0x7FFFFFu) <= 0x400000u ? eb - 129 : eb - 128;
    return max(-127, min(127, e));
}

// One warp per (token, 32-element block): PIECES residual E2M1 pieces with
// their E8M0 exponents, written into the stage images the MMA streams.  Piece
// p of token m is row 8m+p of the B operand.
__global__ void __launch_bounds__(256) k_mx_pieces(const PassHdr* __restrict__ hdr, int use_head,
                                                   int mcap, const float* __restrict__ x, int ldx,
                                                   int K, int S, int N, uint8_t* __restrict__ bimg,
                                                   uint8_t* __restrict__ sfb) {
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
    const int s = kb / (STAGE_K / 32), kbl = kb % (STAGE_K / 32);
    uint8_t* img = bimg + (size_t)s * N * 128;
    uint8_t* sf = sfb + (size_t)s * SF_STAGE;
    const uint32_t byte = (uint32_t)(kbl * 16 + (lane >> 1));
#pragma unroll
    for (int p = 0; p < PIECES; ++p) {
        const int e = piece_exponent(warp_max(fabsf(r)));
        const float sc = __fmul_rn(fabsf(r), pow2i(-e));  // exact power-of-two scaling
        // nearest level, ties to the even code (python/quantize_mxfp4.py:32-34)
        uint32_t c = (sc > 0.25f) + (sc > 0.75f) + (sc > 1.25f) + (sc > 1.75f) + (sc > 2.5f) +
                     (sc > 3.5f) + (sc > 5.0f);
        c += (c == 1 && sc == 0.75f) || (c == 3 && sc == 1.75f) || (c == 5 && sc == 3.5f);
        const float level = __fmul_rn(__uint_as_float(c << 22), 0x1p126f);
        const float q = __fmul_rn(level, pow2i(e));
        const uint32_t code = (c && r < 0.f) ? (c | 8u) : c;
        r = r < 0.f ? __fadd_rn(r, q) : __fsub_rn(r, q);  // exact (Sterbenz)
        const uint32_t other = __shfl_down_sync(0xffffffffu, code, 1);
        const uint32_t n = (uint32_t)(m * PIECES + p);
        if ((lane & 1) == 0) img[swz128(n, byte)] = (uint8_t)(code | (other << 4));
        if (lane == 0) sf[sf_offset(n, (uint32_t)kbl)] = (uint8_t)(e + 127);
    }
}

// ---------------------------------------------------------------------------
// the projection

struct MxArgs {
    const uint8_t* a;      // [T][S][A_STAGE]
    const uint8_t* sfa;    // [T][S][SF_STAGE]
    const uint8_t* b;      // [S][N*128]
    const uint8_t* sfb;    // [S][SF_STAGE]
    int T, S, ksplit, N, mcap;
    int nbuf, stages;      // TMEM accumulator buffers (1 or 2), ring depth
    const PassHdr* hdr;
    int use_head;
    float* y;
    int ldy;
    int out_rows;          // outputs past this (last tile's padding) are not written
    float* ws;             // [T][ksplit][mcap][128]
    int* tickets;          // [T]
    int* err;
};

enum : int { MX_STORE = 0, MX_ADD = 1, MX_SWIGLU = 2 };
constexpr int MX_MAXSTAGES = 6;
constexpr int MX_MAXTOK = 16;       // tokens per pass on this path: N = 8 * tokens <= 128
constexpr int MX_THREADS = 192;     // warp 0 loads, warp 1 MMAs, warps 2-5 epilogue

__host__ __device__ constexpr int mx_stage_bytes(int N) { return A_STAGE + N * 128 + 2 * SF_STAGE; }

// The four epilogue warps synchronise among themselves only.
__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// Units of work: (tile, K slice), unit u = t * ksplit + kc, handed to the
// persistent CTAs round robin.
__device__ __forceinline__ void unit_range(const MxArgs& a, int u, int& t, int& s0, int& s1) {
    t = u / a.ksplit;
    const int kc = u - t * a.ksplit;
    s0 = (int)((long long)kc * a.S / a.ksplit);
    s1 = (int)((long long)(kc + 1) * a.S / a.ksplit);
}

// Persistent, warp-specialised projection.  Warp 0 lane 0 streams weight
// stages through a ring of shared-memory slots (the first slots are issued
// before the grid-dependency wait: weights never depend on the previous
// kernel); warp 1 lane 0 issues the MMAs into one of two TMEM accumulators;
// warps 2-5 drain the other accumulator, so one unit's epilogue overlaps the
// next unit's streaming.  Warp w reads TMEM lanes 32*(w%4).., weight rows
// 32*(w%4).. of the tile.
template <int EPI>
__global__ void __launch_bounds__(MX_THREADS, 1) k_mx_gemv(MxArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    __shared__ uint64_t full[MX_MAXSTAGES], empty[MX_MAXSTAGES], tfull[2], tempty[2];
    __shared__ uint32_t tmem_base_s;
    __shared__ int last_s;
    __shared__ float up_s[MX_MAXTOK][64];

    const int N = a.N, ST = a.stages, NB = a.nbuf;
    const int sbytes = mx_stage_bytes(N);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int units = a.T * a.ksplit;
    const int G = gridDim.x;

    if (threadIdx.x == 0) {
        for (int i = 0; i < ST; ++i) {
            ptx::mbar_init(&full[i], 1);
            ptx::mbar_init(&empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            ptx::mbar_init(&tfull[i], 1);
            ptx::mbar_init(&tempty[i], 4);
        }
        ptx::fence_barrier_init();
    }
    if (warp == 1) {
        ptx::tmem_alloc(&tmem_base_s, TMEM_COLS);
        ptx::tmem_relinquish();
    }
    ptx::tc_fence_before();
    __syncthreads();
    ptx::tc_fence_after();
    const uint32_t tmem = tmem_base_s;
    bool ok = true;

    if (warp == 0) {
        if (lane == 0) {
            // Prefetch the first ring slots' weights, then wait for the
            // kernel that produces the activation pieces.
            int pre = 0;
            {
                int g = 0;
                for (int u = blockIdx.x; u < units && g < ST; u += G) {
                    int t, s0, s1;
                    unit_range(a, u, t, s0, s1);
                    for (int s = s0; s < s1 && g < ST; ++s, ++g) {
                        uint8_t* base = smem + g * sbytes;
                        ptx::mbar_arrive_expect_tx(&full[g], (uint32_t)sbytes);
                        ptx::bulk_g2s(base, a.a + ((size_t)t * a.S + s) * A_STAGE, A_STAGE, &full[g]);
                        ptx::bulk_g2s(base + A_STAGE + N * 128, a.sfa + ((size_t)t * a.S + s) * SF_STAGE,
                                      SF_STAGE, &full[g]);
                    }
                }
                pre = g;
            }
            ptx::grid_dependency_wait();
            int g = 0;
            for (int u = blockIdx.x; u < units && ok; u += G) {
                int t, s0, s1;
                unit_range(a, u, t, s0, s1);
                for (int s = s0; s < s1; ++s, ++g) {
                    const int slot = g % ST;
                    uint8_t* base = smem + slot * sbytes;
                    if (g >= pre) {
                        if (g >= ST && !ptx::mbar_wait(&empty[slot], ((g / ST) - 1) & 1, WAIT_LIMIT)) {
                            ok = false;
                            break;
                        }
                        ptx::mbar_arrive_expect_tx(&full[slot], (uint32_t)sbytes);
                        ptx::bulk_g2s(base, a.a + ((size_t)t * a.S + s) * A_STAGE, A_STAGE, &full[slot]);
                        ptx::bulk_g2s(base + A_STAGE + N * 128, a.sfa + ((size_t)t * a.S + s) * SF_STAGE,
                                      SF_STAGE, &full[slot]);
                    }
                    ptx::bulk_g2s(base + A_STAGE, a.b + (size_t)s * N * 128, (uint32_t)(N * 128), &full[slot]);
                    ptx::bulk_g2s(base + A_STAGE + N * 128 + SF_STAGE, a.sfb + (size_t)s * SF_STAGE,
                                  SF_STAGE, &full[slot]);
                }
            }
            // every load is issued: the next kernel may start prefetching
            ptx::launch_dependents();
        }
    } else if (warp == 1) {
        ptx::grid_dependency_wait();
        if (lane == 0) {
            int g = 0, j = 0;
            for (int u = blockIdx.x; u < units && ok; u += G, ++j) {
                int t, s0, s1;
                unit_range(a, u, t, s0, s1);
                const int buf = NB == 2 ? (j & 1) : 0;
                const int use = NB == 2 ? (j >> 1) : j;  // earlier uses of this accumulator
                if (use > 0 && !ptx::mbar_wait(&tempty[buf], (use - 1) & 1, WAIT_LIMIT)) {
                    ok = false;
                    break;
                }
                ptx::tc_fence_after();
                const uint32_t d_tmem = tmem + ACC_COL + buf * 64;
                for (int s = s0; s < s1; ++s, ++g) {
                    const int slot = g % ST;
                    if (!ptx::mbar_wait(&full[slot], (g / ST) & 1, WAIT_LIMIT)) {
                        ok = false;
                        break;
                    }
                    ptx::tc_fence_after();
                    uint8_t* base = smem + slot * sbytes;
                    const uint32_t a_addr = ptx::smem_u32(base);
                    const uint32_t b_addr = ptx::smem_u32(base + A_STAGE);
                    const uint32_t sfa_addr = ptx::smem_u32(base + A_STAGE + N * 128);
                    const uint32_t sfb_addr = sfa_addr + SF_STAGE;
                    ptx::tmem_cp_32x128b_warpx4(tmem + SFA_COL, ptx::smem_desc(sfa_addr, 16, 128, 0));
                    ptx::tmem_cp_32x128b_warpx4(tmem + SFA_COL + 4, ptx::smem_desc(sfa_addr + 512, 16, 128, 0));
                    ptx::tmem_cp_32x128b_warpx4(tmem + SFB_COL, ptx::smem_desc(sfb_addr, 16, 128, 0));
                    ptx::tmem_cp_32x128b_warpx4(tmem + SFB_COL + 4, ptx::smem_desc(sfb_addr + 512, 16, 128, 0));
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const uint64_t ad = ptx::smem_desc(a_addr + 32 * q, 16, 1024, 2);
                        const uint64_t bd = ptx::smem_desc(b_addr + 32 * q, 16, 1024, 2);
                        const uint32_t sf_id = (uint32_t)(q & 1) * 2;
                        const uint32_t sfa_t = (tmem + SFA_COL + (q >> 1) * 4) | (sf_id << 30);
                        const uint32_t sfb_t = (tmem + SFB_COL + (q >> 1) * 4) | (sf_id << 30);
                        ptx::mma_mxf4(d_tmem, ad, bd, ptx::mxf4_idesc(128, (uint32_t)N, sf_id, sf_id), sfa_t,
                                      sfb_t, (s > s0 || q > 0) ? 1u : 0u);
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
        const bool lead = threadIdx.x == 64;
        int j = 0;
        for (int u = blockIdx.x; u < units; u += G, ++j) {
            int t, s0, s1;
            unit_range(a, u, t, s0, s1);
            const int buf = NB == 2 ? (j & 1) : 0;
            const int use = NB == 2 ? (j >> 1) : j;
            if (!ptx::mbar_wait(&tfull[buf], use & 1, WAIT_LIMIT)) ok = false;
            ptx::tc_fence_after();
            float val[MX_MAXTOK];
            const uint32_t lanebase = tmem + ((uint32_t)(quarter * 32) << 16) + ACC_COL + buf * 64;
#pragma unroll
            for (int m0 = 0; m0 < MX_MAXTOK; m0 += 4) {
                if (m0 < a.mcap) {  // uniform: the whole warp loads together
                    float v[32];
                    ptx::tmem_ld32(lanebase + m0 * 8, v);
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        float acc = v[8 * i + 7];  // smallest correction first
#pragma unroll
                        for (int p = 6; p >= 0; --p) acc = __fadd_rn(acc, v[8 * i + p]);
                        val[m0 + i] = acc;
                    }
                } else {
#pragma unroll
                    for (int i = 0; i < 4; ++i) val[m0 + i] = 0.f;
                }
            }
            ptx::tc_fence_before();
            __syncwarp();
            if (lane == 0) ptx::mbar_arrive(&tempty[buf]);

            if (a.ksplit > 1) {
                const int kc = u - t * a.ksplit;
                float* ws = a.ws + (((size_t)t * a.ksplit + kc) * a.mcap) * 128;
#pragma unroll
                for (int m = 0; m < MX_MAXTOK; ++m)
                    if (m < a.mcap) __stcg(ws + (size_t)m * 128 + row, val[m]);
                __threadfence();
                epi_bar();
                if (lead) {
                    const int ticket = atomicAdd(&a.tickets[t], 1);
                    last_s = ticket == a.ksplit - 1;
                    if (last_s) a.tickets[t] = 0;  // every slice arrived: ready for the next launch
                }
                epi_bar();
                if (!last_s) continue;
                __threadfence();
                const float* w0 = a.ws + ((size_t)t * a.ksplit * a.mcap) * 128;
#pragma unroll
                for (int m = 0; m < MX_MAXTOK; ++m)
                    if (m < a.mcap) val[m] = __ldcg(w0 + (size_t)m * 128 + row);
                for (int k = 1; k < a.ksplit; ++k) {
                    float part[MX_MAXTOK];
#pragma unroll
                    for (int m = 0; m < MX_MAXTOK; ++m)
                        part[m] = m < a.mcap ? __ldcg(w0 + ((size_t)k * a.mcap + m) * 128 + row) : 0.f;
#pragma unroll
                    for (int m = 0; m < MX_MAXTOK; ++m) val[m] = __fadd_rn(val[m], part[m]);
                }
            }
            if (EPI == MX_SWIGLU) {
                // tile rows 0..63: gate rows 64t.., rows 64..127: the matching up rows
                if (row >= 64) {
#pragma unroll
                    for (int m = 0; m < MX_MAXTOK; ++m)
                        if (m < a.mcap) up_s[m][row - 64] = val[m];
                }
                epi_bar();
                if (row < 64 && t * 64 + row < a.out_rows) {
#pragma unroll
                    for (int m = 0; m < MX_MAXTOK; ++m) {
                        if (m >= M) continue;
                        const float gt = val[m], up = up_s[m][row];
                        a.y[(size_t)m * a.ldy + t * 64 + row] =
                            __fmul_rn(__fdiv_rn(gt, __fadd_rn(1.0f, expf(-gt))), up);
                    }
                }
                epi_bar();  // up_s is reused by the next unit
            } else if (t * TILE_ROWS + row < a.out_rows) {
#pragma unroll
                for (int m = 0; m < MX_MAXTOK; ++m) {
                    if (m >= M) continue;
                    float* out = a.y + (size_t)m * a.ldy + t * TILE_ROWS + row;
                    if (EPI == MX_ADD) *out = __fadd_rn(*out, val[m]);
                    else *out = val[m];
                }
            }
        }
    }
    ptx::launch_dependents();
    ptx::tc_fence_before();
    __syncthreads();
    if (warp == 1) ptx::tmem_dealloc(tmem, TMEM_COLS);
    if (!ok && lane == 0) atomicOr(a.err, 4);  // a bounded wait gave up
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

__global__ void k_mx_tile(TileSrc src, int swiglu, int K, int T, int S, uint8_t* __restrict__ a,
                          uint8_t* __restrict__ sfa) {
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
        uint8_t* tile = a + ((size_t)t * S + s) * A_STAGE;
        *reinterpret_cast<uint4*>(tile + swz128((uint32_t)r, (uint32_t)c16 * 16)) = v;
        sfa[((size_t)t * S + s) * SF_STAGE + sf_offset((uint32_t)r, (uint32_t)c16)] = sc;
    }
}

// K slices per tile for one persistent CTA per SM: the busiest CTA streams
// ceil(T*ks / sms) units of ceil(S/ks) stages; a unit also costs about one
// stage of epilogue and a split costs a partial-sum round trip.  The choice
// depends only on the matrix shape, never on the token count.
int mx_ksplit(int T, int S, int sms) {
    int best = 1;
    double best_cost = 1e30;
    for (int ks = 1; ks <= S; ++ks) {
        const int per_cta = (T * ks + sms - 1) / sms;
        const int per_unit = (S + ks - 1) / ks;
        const double cost = (double)per_cta * (per_unit + 1.0) + (ks > 1 ? 1.0 : 0.0);
        if (cost < best_cost - 1e-9) {
            best_cost = cost;
            best = ks;
        }
    }
    return best;
}

// Ring depth and accumulator buffers for N MMA columns: two accumulators of
// up to 64 columns, or one of up to 128; about 105 KB of stages, so a CTA of
// the next projection fits on the same SM (programmatic dependent launch).
void mx_shape(int N, int* stages, int* nbuf) {
    *nbuf = N <= 64 ? 2 : 1;
    *stages = N <= 64 ? 4 : 3;
}

size_t mx_smem(int N) {
    int st, nb;
    mx_shape(N, &st, &nb);
    return (size_t)st * mx_stage_bytes(N) + 1024;  // + alignment slack
}

template <int EPI>
jl_status configure_mx() {
    JL_CUDA(cudaFuncSetAttribute(k_mx_gemv<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)std::max(mx_smem(64), mx_smem(8 * MX_MAXTOK))));
    JL_CUDA(cudaFuncSetAttribute(k_mx_gemv<EPI>, cudaFuncAttributePreferredSharedMemoryCarveout, 100));
    return JL_OK;
}

}  // namespace

jl_status mx_configure() {
    JL_TRY(configure_mx<MX_STORE>());
    JL_TRY(configure_mx<MX_ADD>());
    JL_TRY(configure_mx<MX_SWIGLU>());
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
    p.sfa = dst + (size_t)p.T * p.S * A_STAGE;
    p.ksplit = mx_ksplit(p.T, p.S, sms);
    const size_t chunks = (size_t)p.T * p.S * TILE_ROWS * 8;
    const int grid = (int)std::min<size_t>((chunks + 255) / 256, (size_t)sms * 8);
    k_mx_tile<<<grid, 256, 0, stream>>>(src, swiglu ? 1 : 0, K, p.T, p.S, (uint8_t*)p.a,
                                        (uint8_t*)p.sfa);
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
                      (const PassHdr*)m->pass.hdr, use_head, mcap, x, ldx, p.K, p.S, N, m->mx.bimg,
                      m->mx.sfb));
    MxArgs a;
    a.a = p.a;
    a.sfa = p.sfa;
    a.b = m->mx.bimg;
    a.sfb = m->mx.sfb;
    a.T = p.T;
    a.S = p.S;
    a.ksplit = p.ksplit;
    a.N = N;
    a.mcap = mcap;
    mx_shape(N, &a.stages, &a.nbuf);
    a.hdr = m->pass.hdr;
    a.use_head = use_head;
    a.y = y;
    a.ldy = ldy;
    a.out_rows = p.out_rows;
    a.ws = m->mx.ws;
    a.tickets = m->mx.tickets;
    a.err = m->counters;
    const dim3 grid(std::min(p.T * p.ksplit, m->sms));
    const size_t smem = mx_smem(N);
    if (epi == MX_ADD) return launch_pdl(k_mx_gemv<MX_ADD>, grid, dim3(MX_THREADS), smem, c.stream, a);
    if (epi == MX_SWIGLU) return launch_pdl(k_mx_gemv<MX_SWIGLU>, grid, dim3(MX_THREADS), smem, c.stream, a);
    return launch_pdl(k_mx_gemv<MX_STORE>, grid, dim3(MX_THREADS), smem, c.stream, a);
}

MxScratchPlan mx_scratch_plan(const MxProj& p, int mcap) {
    auto up = [](size_t b) { return (b + 255) & ~(size_t)255; };
    MxScratchPlan s;
    s.tickets = up((size_t)p.T * sizeof(int));
    s.sfb = up((size_t)p.S * SF_STAGE);
    s.bimg = up((size_t)p.S * PIECES * mcap * 128);
    s.ws = p.ksplit > 1 ? up((size_t)p.T * p.ksplit * mcap * 128 * sizeof(float)) : 0;
    s.total = s.tickets + s.sfb + s.bimg + s.ws;
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
    uint8_t* sfb = scratch + plan.tickets;
    uint8_t* bimg = sfb + plan.sfb;
    float* ws = (float*)(bimg + plan.bimg);
    const int N = PIECES * mcap;
    const int items = mcap * p.S * (STAGE_K / 32);
    JL_TRY(launch_pdl(k_mx_pieces, dim3((items + 7) / 8), dim3(256), 0, stream, hdr, 0, mcap, x, ldx,
                      p.K, p.S, N, bimg, sfb));
    MxArgs a;
    a.a = p.a;
    a.sfa = p.sfa;
    a.b = bimg;
    a.sfb = sfb;
    a.T = p.T;
    a.S = p.S;
    a.ksplit = p.ksplit;
    a.N = N;
    a.mcap = mcap;
    mx_shape(N, &a.stages, &a.nbuf);
    a.hdr = hdr;
    a.use_head = 0;
    a.y = y;
    a.ldy = ldy;
    a.out_rows = p.out_rows;
    a.ws = ws;
    a.tickets = tickets;
    a.err = err;
    const dim3 grid(std::min(p.T * p.ksplit, sms));
    const size_t smem = mx_smem(N);
    if (epi == MX_ADD) return launch_pdl(k_mx_gemv<MX_ADD>, grid, dim3(MX_THREADS), smem, stream, a);
    if (epi == MX_SWIGLU) return launch_pdl(k_mx_gemv<MX_SWIGLU>, grid, dim3(MX_THREADS), smem, stream, a);
    return launch_pdl(k_mx_gemv<MX_STORE>, grid, dim3(MX_THREADS), smem, stream, a);
}

}  // namespace jl
