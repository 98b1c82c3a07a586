// Tensor-core prompt attention (lib.rs:401-441 for the prompt rows of
// predict): causal GQA flash attention over the paged bf16 KV cache with
// tcgen05 MMAs, for multi-chunk passes over one sequence's prompt.
//
// A CTA takes PT = 128 / group consecutive positions of one KV head: its 128
// MMA rows are (position, query head) pairs, row m = position (m / group),
// head (m % group), so the group's heads share every K/V tile.  Per tile of
// 128 keys (two pages):
//   * K and V come in by TMA from a 2-D tensor map over the pool ([page, kv
//     head, slot] rows x 128 dims), as two 64-dim boxes per page in the
//     128-byte-swizzled layout the MMA reads: K as a K-major operand, V as an
//     MN-major one.
//   * S = Q K^T in TMEM, with Q as two bf16 pieces (hi + lo, exact to 2^-17
//     of each element), both MMAs accumulating into one f32 tile.
//   * Softmax on CUDA cores: thread (row m, part t) reads keys 32t..32t+31 of
//     row m from TMEM; the four parts exchange their maxima through shared
//     memory, and the running max and sum are kept online as in k_attn_prefill.
//   * P goes back to shared memory as two bf16 pieces (hi + lo) and
//     O_tile = P V lands in TMEM; each thread folds its 32 output dims into
//     registers (o = o * correction + O_tile).
// The scores of tile j + 1 are issued right behind P V of tile j, so that MMA
// runs while the threads fold O.  Keys past a row's position, and keys of
// pages that were not copied, get zero weight; V rows no position of the CTA
// may see (never written, so possibly not finite) are zeroed before P V.
// The output goes out like k_attn_prefill's: f32 rows and the o projection's
// activation pieces, from a staging copy in shared memory.
//
// The result is within the f32 kernel's rounding of it, not bit-equal
// (different summation order, 2^-17 pieces); the parity tests hold it to the
// oracle's tolerance.  f32 pools and GQA groups other than 1, 2, 4 and 8 keep
// the CUDA-core k_attn_prefill.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cudaTypedefs.h>

#include <cmath>

#include "jl_internal.h"
#include "kernels.cuh"
#include "launch.cuh"
#include "mx_pieces.cuh"
#include "ptx.cuh"

namespace jl {
namespace {

using mx::swz128;

constexpr int TC_M = 128;        // MMA rows of a CTA
constexpr int TC_KEYS = 128;     // keys per tile (two pages)
constexpr int TC_PARTS = 4;                // threads per MMA row
constexpr int TC_THREADS = 128 * TC_PARTS;
constexpr int TC_KP = TC_KEYS / TC_PARTS;  // keys of a tile per thread
constexpr int TC_DP = HEAD / TC_PARTS;     // output dims per thread
static_assert(TC_KP == 32 && TC_DP == 32, "one 32-column TMEM load per thread and tile");
constexpr uint32_t TC_IMG = 16384;  // one 128-row x 128-byte swizzled image
constexpr uint32_t TC_PAGE_IMG = PAGE * 128;  // one page's rows of an image
// shared-memory images (1024-byte aligned): Q and P as [64-element K block]
// [row][128 B]; K and V as [64-dim block][key][128 B]
constexpr uint32_t OFF_QH = 0, OFF_QL = 2 * TC_IMG, OFF_K = 4 * TC_IMG, OFF_V = 6 * TC_IMG,
                   OFF_PH = 8 * TC_IMG, OFF_PL = 10 * TC_IMG;
constexpr size_t TC_SMEM = 12 * (size_t)TC_IMG + 1024;  // + alignment slack
constexpr uint32_t TC_WAIT = 1u << 22;  // polls before a wait reports failure
constexpr uint32_t TC_TMEM_COLS = 256;  // S: columns 0..127, O: 128..255
static_assert(PAGE == 64 && HEAD == 128, "a page is one 64-row box, a head two 64-dim boxes");

struct TcPrefillArgs {
    PassBuf pb;
    const float* qkv;  // q rows, QK-normalised and rotated by the q|k|v kernel
    int ld;
    int group;
    int rows_cap;      // rows of the pass (16 per chunk)
    KvView kv;
    float* out;        // attention output rows [row][q_heads * HEAD]
    int out_ld;
    uint8_t* bout;     // the o projection's activation pieces, or null
    int bN;
    size_t cs_bout;    // bytes between the pieces of consecutive chunks
};

// x as bf16 hi + lo (x - hi rounded again): the pair carries x to 2^-17.
__device__ __forceinline__ void split_bf16(float x, uint32_t& hi, uint32_t& lo) {
    const __nv_bfloat16 h = __float2bfloat16_rn(x);
    const __nv_bfloat16 l = __float2bfloat16_rn(__fsub_rn(x, __bfloat162float(h)));
    hi = __bfloat16_as_ushort(h);
    lo = __bfloat16_as_ushort(l);
}

// The same for a pair: (x, y) as packed bf16x2 hi and lo words (x low).
__device__ __forceinline__ void split_bf16x2(float x, float y, uint32_t& hi, uint32_t& lo) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(x, y);
    const float2 hf = __bfloat1622float2(h);
    const __nv_bfloat162 l = __floats2bfloat162_rn(__fsub_rn(x, hf.x), __fsub_rn(y, hf.y));
    hi = *reinterpret_cast<const uint32_t*>(&h);
    lo = *reinterpret_cast<const uint32_t*>(&l);
}

// 2^x by the hardware's approximation (ex2.approx.ftz: relative error about
// 2^-22 for the x <= 0 the softmax weights take, results below 2^-126 flushed
// to zero).
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// The MMAs of one tile, issued by one thread.  Not inlined: their 64-bit
// descriptors would otherwise be hoisted out of the tile loop and held in
// every thread's registers.
// S = Qh K^T + Ql K^T (both K-major), into TMEM columns 0..127.
__device__ __noinline__ void tc_issue_scores(uint32_t sbase, uint32_t tmem, uint64_t* bar) {
    const uint32_t idesc = ptx::bf16_idesc(TC_M, TC_KEYS);
#pragma unroll
    for (int pc = 0; pc < 2; ++pc)
#pragma unroll
        for (int kb = 0; kb < 2; ++kb)
#pragma unroll
            for (int q = 0; q < 4; ++q) {  // dims 64 kb + 16 q ..
                const uint32_t qa = sbase + (pc ? OFF_QL : OFF_QH) + kb * TC_IMG + 32 * q;
                const uint32_t ka = sbase + OFF_K + kb * TC_IMG + 32 * q;
                ptx::mma_bf16(tmem, ptx::smem_desc(qa, 16, 1024, 2), ptx::smem_desc(ka, 16, 1024, 2), idesc,
                              (pc | kb | q) ? 1u : 0u);
            }
    ptx::tc_commit(bar);
}

// O_tile = Ph V + Pl V into TMEM columns 128..255: P K-major, V MN-major
// (64-dim blocks TC_IMG apart, groups of 8 keys 1024 bytes apart).
__device__ __noinline__ void tc_issue_pv(uint32_t sbase, uint32_t tmem, uint64_t* bar) {
    const uint32_t idesc = ptx::bf16_idesc(TC_M, HEAD) | (1u << 16);  // B MN-major
#pragma unroll
    for (int pc = 0; pc < 2; ++pc)
#pragma unroll
        for (int kb = 0; kb < 2; ++kb)
#pragma unroll
            for (int q = 0; q < 4; ++q) {  // keys 64 kb + 16 q ..
                const uint32_t pa = sbase + (pc ? OFF_PL : OFF_PH) + kb * TC_IMG + 32 * q;
                const uint32_t va = sbase + OFF_V + kb * TC_PAGE_IMG + q * 2048;
                ptx::mma_bf16(tmem + 128, ptx::smem_desc(pa, 16, 1024, 2), ptx::smem_desc(va, TC_IMG, 1024, 2), idesc,
                              (pc | kb | q) ? 1u : 0u);
            }
    ptx::tc_commit(bar);
}

__global__ void __launch_bounds__(TC_THREADS, 1)
    k_attn_prefill_tc(TcPrefillArgs a, const __grid_constant__ CUtensorMap kmap,
                      const __grid_constant__ CUtensorMap vmap) {
    extern __shared__ uint8_t tc_raw[];
    uint8_t* sm = (uint8_t*)(((uintptr_t)tc_raw + 1023) & ~(uintptr_t)1023);
    __shared__ uint64_t bar_k, bar_v, bar_s, bar_o;
    __shared__ uint32_t tmem_s;
    __shared__ float xchg[TC_PARTS][TC_M];  // the parts of a row: tile maxima, then sums
    __shared__ int live_s;           // rows 0..live_s-1 of the CTA are live
    __shared__ int pvalid[2][2];     // [tile parity][page of the tile]: copied

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int quarter = warp & 3, part = warp >> 2;
    const int m = quarter * 32 + lane;  // MMA row = TMEM lane
    const int group = a.group, PT = TC_M / group;
    const int g = blockIdx.x, r0 = blockIdx.y * PT;
    if (tid == 0) {
        ptx::mbar_init(&bar_k, 1);
        ptx::mbar_init(&bar_v, 1);
        ptx::mbar_init(&bar_s, 1);
        ptx::mbar_init(&bar_o, 1);
        ptx::fence_barrier_init();
        ptx::prefetch_tensormap(&kmap);
        ptx::prefetch_tensormap(&vmap);
        live_s = PT;
    }
    if (warp == 0) {
        ptx::tmem_alloc(&tmem_s, TC_TMEM_COLS);
        ptx::tmem_relinquish();
    }
    ptx::tc_fence_before();
    __syncthreads();
    ptx::tc_fence_after();
    const uint32_t tmem = tmem_s;
    const uint32_t t_row = tmem + ((uint32_t)(quarter * 32) << 16);  // this warp's 32 lanes
    ptx::grid_dependency_wait();  // q and this pass's K/V come from the q|k|v kernel
    ptx::launch_dependents();

    // Live rows: the pass's rows r0, r0 + 1, ... while they are one sequence
    // at consecutive positions (as predict builds a prompt pass).
    const RowDesc first = a.pb.row[r0];
    if (tid < PT) {
        const int r = r0 + tid;
        const bool dead = r >= a.rows_cap || (r % SMALL_M) >= a.pb.hdr[r / SMALL_M].rows;
        bool bad = false;
        if (!dead) {
            const RowDesc rd = a.pb.row[r];
            bad = (unsigned)first.seq >= (unsigned)MAX_SEQS || rd.seq != first.seq || rd.pos != first.pos + tid ||
                  rd.pos < 0 || rd.pos >= a.kv.max_pos;
        }
        if (bad) atomicOr(a.kv.err, 2);
        if (dead || bad) atomicMin(&live_s, tid);
    }
    __syncthreads();
    const int live = live_s;
    const int last_pos = live > 0 ? first.pos + live - 1 : -1;
    const int npages = live > 0 ? last_pos / PAGE + 1 : 0;
    const int nt = (npages + 1) / 2;
    const int32_t* pt = live > 0 ? a.pb.page_table[first.seq] : nullptr;
    const int prow = m / group;
    const int pos_m = prow < live ? first.pos + prow : -1;  // -1: a dead row sees no key

    // Q as hi and lo bf16 images; a warp reads one 512-byte q row per step
    {
        const float* qb = a.qkv + (size_t)r0 * a.ld + (size_t)g * group * HEAD;
        for (int idx = tid; idx < TC_M * 32; idx += TC_THREADS) {
            const int mr = idx >> 5, c = idx & 31;  // row, float4 of the row
            const int i = mr / group, h = mr % group;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (i < live) v = *(const float4*)(qb + (size_t)i * a.ld + h * HEAD + 4 * c);
            uint32_t h0, h1, h2, h3, l0, l1, l2, l3;
            split_bf16(v.x, h0, l0);
            split_bf16(v.y, h1, l1);
            split_bf16(v.z, h2, l2);
            split_bf16(v.w, h3, l3);
            const uint32_t off = (uint32_t)(c >> 4) * TC_IMG + swz128((uint32_t)mr, (uint32_t)(c & 15) * 8);
            *(uint2*)(sm + OFF_QH + off) = make_uint2(h0 | (h1 << 16), h2 | (h3 << 16));
            *(uint2*)(sm + OFF_QL + off) = make_uint2(l0 | (l1 << 16), l2 | (l3 << 16));
        }
        ptx::fence_proxy_async_smem();
    }

    // thread 0: copies and MMAs, with counts of what it issued and saw complete
    int k_iss = 0, k_done = 0, v_iss = 0, v_done = 0, s_iss = 0, s_done = 0, o_iss = 0, o_done = 0;
    auto issue_tile = [&](int j, const CUtensorMap* map, uint32_t off, uint64_t* bar, bool record) {
        uint32_t bytes = 0;
        int pg[2];
        for (int ph = 0; ph < 2; ++ph) {
            const int p = 2 * j + ph;
            pg[ph] = -1;
            if (p < npages) {
                const int id = pt[p];
                if (page_ok(a.kv, id)) {
                    pg[ph] = id;
                    bytes += 2 * TC_PAGE_IMG;
                }
            }
            if (record) pvalid[j & 1][ph] = pg[ph] >= 0;
        }
        ptx::mbar_arrive_expect_tx(bar, bytes);
        for (int ph = 0; ph < 2; ++ph) {
            if (pg[ph] < 0) continue;
            const int y = (pg[ph] * a.kv.kv_heads + g) * PAGE;
#pragma unroll
            for (int db = 0; db < 2; ++db) ptx::tma_load_2d(sm + off + db * TC_IMG + ph * TC_PAGE_IMG, map, 64 * db, y, bar);
        }
    };
    const uint32_t sbase = ptx::smem_u32(sm);
    auto issue_scores = [&]() {
        tc_issue_scores(sbase, tmem, &bar_s);
        ++s_iss;
    };
    auto issue_pv = [&]() {
        tc_issue_pv(sbase, tmem, &bar_o);
        ++o_iss;
    };
    auto wait0 = [&](uint64_t* bar, int& done, bool& okv) {  // thread 0's bounded wait for the next phase
        if (ptx::mbar_wait(bar, (uint32_t)(done & 1), TC_WAIT)) ++done;
        else okv = false;
    };

    float o[TC_DP];  // output dims TC_DP * part .. of row m, unnormalised
#pragma unroll
    for (int i = 0; i < TC_DP; ++i) o[i] = 0.f;
    float mrun = -INFINITY, lpart = 0.f;  // running max of raw scores; this part's running sum
    const float c2 = (float)(1.4426950408889634 / 11.313708498984761);  // log2(e) / sqrt(HEAD)
    bool ok = true;
    if (tid == 0 && nt > 0) {
        issue_tile(0, &kmap, OFF_K, &bar_k, true);
        ++k_iss;
        issue_tile(0, &vmap, OFF_V, &bar_v, false);
        ++v_iss;
    }
    __syncthreads();  // Q images written and fenced; pages of tile 0 recorded
    if (tid == 0 && nt > 0) {
        wait0(&bar_k, k_done, ok);
        ptx::tc_fence_after();
        issue_scores();
    }
    for (int j = 0; j < nt; ++j) {
        const uint32_t par = (uint32_t)(j & 1);
        if (ptx::mbar_wait(&bar_s, par, TC_WAIT)) {
            if (tid == 0) ++s_done;
        } else {
            ok = false;
        }
        ptx::tc_fence_after();
        if (tid == 0 && j + 1 < nt) {  // the scores are done with K: the next tile's K
            issue_tile(j + 1, &kmap, OFF_K, &bar_k, true);
            ++k_iss;
        }
        // keys k0 + c, c < nvis, are this row's (causal, page copied); S is
        // read from TMEM twice (maximum, then weights) rather than held
        const int k0 = j * TC_KEYS + TC_KP * part;
        const int nvis = pvalid[par][part >> 1] ? max(0, min(TC_KP, pos_m - k0 + 1)) : 0;
        const bool whole = nvis == TC_KP;  // no masking (every tile but a CTA's last one or two)
        float s[TC_KP];
        ptx::tmem_ld32(t_row + TC_KP * part, s);
        float tmax = -INFINITY;
        if (whole) {
#pragma unroll
            for (int c = 0; c < TC_KP; ++c) tmax = fmaxf(tmax, s[c]);
        } else {
#pragma unroll
            for (int c = 0; c < TC_KP; ++c)
                if (c < nvis) tmax = fmaxf(tmax, s[c]);
        }
        xchg[part][m] = tmax;
        __syncthreads();  // every part's maximum
        const float mnew = fmaxf(mrun, fmaxf(fmaxf(xchg[0][m], xchg[1][m]), fmaxf(xchg[2][m], xchg[3][m])));
        const float corr = mrun == -INFINITY ? 0.f : ex2(__fmul_rn(__fsub_rn(mrun, mnew), c2));
        mrun = mnew;
        const float mc = __fmul_rn(mnew, c2);
        float psum = 0.f;
        // keys 32 part .. of the row: P image part / 2, chunks 4 (part & 1) ..
        uint8_t* ph_img = sm + OFF_PH + (part >> 1) * TC_IMG;
        uint8_t* pl_img = sm + OFF_PL + (part >> 1) * TC_IMG;
#pragma unroll
        for (int ch = 0; ch < 4; ++ch) {  // 8 keys = one 16-byte chunk of the row
            uint32_t wh[4], wl[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int c = 8 * ch + 2 * e;
                // 2^(s c2 - m c2): one multiply-add per weight
                float p0 = ex2(__fmaf_rn(s[c], c2, -mc)), p1 = ex2(__fmaf_rn(s[c + 1], c2, -mc));
                if (!whole) {
                    p0 = c < nvis ? p0 : 0.f;
                    p1 = c + 1 < nvis ? p1 : 0.f;
                }
                psum = __fadd_rn(psum, __fadd_rn(p0, p1));
                split_bf16x2(p0, p1, wh[e], wl[e]);
            }
            const uint32_t off = swz128((uint32_t)m, (uint32_t)(16 * (4 * (part & 1) + ch)));
            *(uint4*)(ph_img + off) = make_uint4(wh[0], wh[1], wh[2], wh[3]);
            *(uint4*)(pl_img + off) = make_uint4(wl[0], wl[1], wl[2], wl[3]);
        }
        lpart = __fmaf_rn(lpart, corr, psum);
        ptx::fence_proxy_async_smem();
        // V rows that no position of the CTA sees (past the last position, or
        // of a page not copied) may hold anything: zero weight times them
        // must stay zero, so they are cleared first
        const bool tail = j == nt - 1 || !pvalid[par][0] || !pvalid[par][1];
        if (tail) {
            if (!ptx::mbar_wait(&bar_v, par, TC_WAIT)) ok = false;
            else if (tid == 0) ++v_done;
            const int kz = last_pos - j * TC_KEYS;  // last key of the tile anyone sees
            for (int idx = tid; idx < 2 * TC_KEYS * 8; idx += TC_THREADS) {
                const int db = idx >> 10, k = (idx >> 3) & (TC_KEYS - 1), ch = idx & 7;
                if (k > kz || !pvalid[par][k >> 6])
                    *(uint4*)(sm + OFF_V + db * TC_IMG + (k >> 6) * TC_PAGE_IMG + (k & 63) * 128 + ch * 16) =
                        make_uint4(0u, 0u, 0u, 0u);
            }
            ptx::fence_proxy_async_smem();
        }
        ptx::tc_fence_before();
        if (!__syncthreads_and(ok)) break;  // P written; V rows cleared
        if (tid == 0) {
            if (!tail) wait0(&bar_v, v_done, ok);
            ptx::tc_fence_after();
            issue_pv();
            if (j + 1 < nt) {  // the next scores run while the threads fold O
                wait0(&bar_k, k_done, ok);
                ptx::tc_fence_after();
                issue_scores();
            }
        }
        if (ptx::mbar_wait(&bar_o, par, TC_WAIT)) {
            if (tid == 0) ++o_done;
        } else {
            ok = false;
        }
        ptx::tc_fence_after();
        if (tid == 0 && j + 1 < nt) {  // P V is done with V: the next tile's V
            issue_tile(j + 1, &vmap, OFF_V, &bar_v, false);
            ++v_iss;
        }
        float t[TC_DP];
        ptx::tmem_ld32(t_row + 128 + TC_DP * part, t);
#pragma unroll
        for (int i = 0; i < TC_DP; ++i) o[i] = __fmaf_rn(o[i], corr, t[i]);
        ptx::tc_fence_before();
    }
    // after a failed wait: let every copy and MMA this CTA issued finish
    // (bounded) before its shared memory and TMEM are released
    if (tid == 0) {
        while (k_done < k_iss && ptx::mbar_wait(&bar_k, (uint32_t)(k_done & 1), TC_WAIT)) ++k_done;
        while (v_done < v_iss && ptx::mbar_wait(&bar_v, (uint32_t)(v_done & 1), TC_WAIT)) ++v_done;
        while (s_done < s_iss && ptx::mbar_wait(&bar_s, (uint32_t)(s_done & 1), TC_WAIT)) ++s_done;
        while (o_done < o_iss && ptx::mbar_wait(&bar_o, (uint32_t)(o_done & 1), TC_WAIT)) ++o_done;
    }
    if (__syncthreads_or(!ok) && tid == 0) atomicOr(a.kv.err, 4);  // a copy or MMA did not finish in time
    ptx::tc_fence_after();
    if (warp == 0) ptx::tmem_dealloc(tmem, TC_TMEM_COLS);

    // outputs: o / l for live rows, zero for the others, staged as
    // [position][group * HEAD + 4] f32 over the Q and K images (the pad
    // spreads positions over the banks)
    xchg[part][m] = lpart;
    __syncthreads();
    const float l = __fadd_rn(__fadd_rn(xchg[0][m], xchg[1][m]), __fadd_rn(xchg[2][m], xchg[3][m]));
    const int st = group * HEAD + 4;
    float* ost = (float*)sm;
    {
        float* dst = ost + (size_t)prow * st + (m % group) * HEAD + TC_DP * part;
        const bool lv = pos_m >= 0 && l > 0.f;
#pragma unroll
        for (int i = 0; i < TC_DP; i += 4)
            *(float4*)(dst + i) = lv ? make_float4(__fdiv_rn(o[i], l), __fdiv_rn(o[i + 1], l),
                                                   __fdiv_rn(o[i + 2], l), __fdiv_rn(o[i + 3], l))
                                     : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    __syncthreads();
    const int rowf4 = group * HEAD / 4;  // float4s of one position's heads
    for (int idx = tid; idx < PT * rowf4; idx += TC_THREADS) {
        const int i = idx / rowf4, c = idx % rowf4;
        const int r = r0 + i;
        if (r >= a.rows_cap || (r % SMALL_M) >= a.pb.hdr[r / SMALL_M].rows) continue;
        *(float4*)(a.out + (size_t)r * a.out_ld + (size_t)g * group * HEAD + 4 * c) =
            *(const float4*)(ost + (size_t)i * st + 4 * c);
    }
    if (a.bout) {  // every row of the CTA's chunks (zero pieces for dead rows)
        for (int cc = 0; cc < PT / SMALL_M; ++cc) {
            const int r = r0 + cc * SMALL_M;
            if (r >= a.rows_cap) break;
            const int count = min(max(live - cc * SMALL_M, 0), SMALL_M);
            mx::emit_pieces_smem(ost + (size_t)cc * SMALL_M * st, st, group * (HEAD / 32), 0, count, SMALL_M, tid,
                                 TC_THREADS, g * group * HEAD, a.bN, a.bout + (size_t)(r / SMALL_M) * a.cs_bout);
        }
    }
}

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static bool looked = false;
    if (!looked) {
        looked = true;
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (PFN_cuTensorMapEncodeTiled_v12000)p;
        cudaGetLastError();
    }
    return fn;
}

}  // namespace

bool prefill_tc_supported(const jl_model* m) {
    if (m->prompt_attn_cuda_cores || m->kv_tmaps.empty() || m->kv_heads <= 0 || m->q_heads % m->kv_heads)
        return false;
    if (!m->mx.fused) return false;  // prompts of other models take k_attention
    const int group = m->q_heads / m->kv_heads;
    return group == 1 || group == 2 || group == 4 || group == 8;
}

// Two tensor maps per layer over its K and V pages: rows (page, kv head,
// slot) of HEAD bf16, boxes of 64 dims x one page, 128-byte swizzle.
jl_status kv_tensor_maps(jl_model* m) {
    m->kv_tmaps.clear();
    if (m->kv.dtype != JL_KV_BF16) return JL_OK;
    const uint64_t rows = (uint64_t)m->kv.pages * m->kv_heads * PAGE;
    if (rows >= (1ull << 31)) return JL_OK;  // row coordinates are 32-bit
    PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
    if (!enc) {
        set_error("cuTensorMapEncodeTiled is not available from the driver");
        return JL_ERR_CUDA;
    }
    std::vector<CUtensorMap> maps((size_t)2 * m->layers);
    for (int l = 0; l < m->layers; ++l) {
        const KvView v = kv_view(m, l);
        for (int which = 0; which < 2; ++which) {
            const cuuint64_t dims[2] = {(cuuint64_t)HEAD, (cuuint64_t)rows};
            const cuuint64_t strides[1] = {(cuuint64_t)HEAD * 2};
            const cuuint32_t box[2] = {64, (cuuint32_t)PAGE};
            const cuuint32_t es[2] = {1, 1};
            const CUresult r = enc(&maps[(size_t)2 * l + which], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                                   which ? v.v : v.k, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
            if (r != CUDA_SUCCESS) {
                set_error("cuTensorMapEncodeTiled failed (%d) for the KV pages of layer %d", (int)r, l);
                return JL_ERR_CUDA;
            }
        }
    }
    m->kv_tmaps.swap(maps);
    return JL_OK;
}

jl_status configure_prefill_tc() {
    JL_CUDA(cudaFuncSetAttribute(k_attn_prefill_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)TC_SMEM));
    return JL_OK;
}

jl_status launch_attention_prefill_tc(const PassCtx& c, int layer, uint8_t* bout, int bN) {
    const jl_model* m = c.m;
    if (!prefill_tc_supported(m) || layer < 0 || layer >= m->layers || c.rows_cap % SMALL_M) {
        set_error("tensor-core prompt attention: unsupported model or pass");
        return JL_ERR_INVALID_ARG;
    }
    const int group = m->q_heads / m->kv_heads, PT = TC_M / group;
    TcPrefillArgs a;
    a.pb = c.pass();
    a.qkv = m->s.qkv;
    a.ld = qkv_ld(m);
    a.group = group;
    a.rows_cap = c.rows_cap;
    a.kv = kv_view(m, layer);
    a.out = m->s.attn;
    a.out_ld = m->q_heads * HEAD;
    a.bout = bout;
    a.bN = bN;
    a.cs_bout = m->mx.sattn;
    const dim3 grid(m->kv_heads, (c.rows_cap + PT - 1) / PT);
    return launch_pdl(k_attn_prefill_tc, grid, dim3(TC_THREADS), TC_SMEM, c.stream, a, m->kv_tmaps[(size_t)2 * layer],
                      m->kv_tmaps[(size_t)2 * layer + 1]);
}

}  // namespace jl
