// Activation pieces: the B operand of the block-scaled MXFP4 projections.
//
// An f32 activation vector is written as the sum of PIECES E2M1 vectors, each
// with its own E8M0 scale per 32-element block.  Piece p quantizes what
// pieces 0..p-1 left over; every subtraction is exact (Sterbenz), so eight
// pieces carry an activation with relative error about 3e-8.
//
// Image layout for a projection with K input elements and N = PIECES * rows
// MMA columns: S = K / STAGE_K stages of img_stage(N) bytes each, stage s
// holding
//   * N rows x 128 bytes of E2M1 codes (two per byte, even element in the
//     low nibble), row n = PIECES * token + piece, in the 128-byte-swizzled
//     K-major layout the MMA descriptor reads (swz128);
//   * right after them, one 1 KB scale region: two 512-byte atoms, byte
//     sf_offset(n, kb) = the E8M0 exponent of block kb (0..7) of row n, the
//     layout tcgen05.cp 32x128b.warpx4 broadcasts into TMEM.
// Consecutive stages are contiguous, so a run of them is one bulk copy.
// Any kernel holding one 32-element block in a warp (one element per lane)
// emits its pieces with emit_pieces / emit_pieces_all.
#pragma once

#include <cuda_fp16.h>
#include <cuda_fp4.h>

#include <cstdint>

namespace jl {
namespace mx {

constexpr int PIECES = 8;
constexpr int STAGE_K = 256;   // K elements per pipeline stage
constexpr int SF_STAGE = 1024;  // two scale atoms

// Bytes of one stage of an activation image with N MMA columns (N % 8 == 0
// keeps every stage 1024-byte aligned, as the swizzled layout needs).
__host__ __device__ constexpr int img_stage(int N) { return N * 128 + SF_STAGE; }

__device__ __forceinline__ uint32_t swz128(uint32_t row, uint32_t byte) {
    // byte offset of (row, byte-in-row) in a 128B-swizzled K-major image
    return (row >> 3) * 1024 + (row & 7) * 128 + ((((byte >> 4) ^ (row & 7)) & 7) << 4) + (byte & 15);
}

__device__ __forceinline__ uint32_t sf_offset(uint32_t row, uint32_t kb) {
    // kb: scale block within the stage (0..7); row < 128
    return (kb >> 2) * 512 + 16 * (row & 31) + 4 * (row >> 5) + (kb & 3);
}

// 2^e as an exact f32 for e in [-127, 127].
__device__ __forceinline__ float pow2i(int e) {
    return e >= -126 ? __uint_as_float((uint32_t)(e + 127) << 23) : __uint_as_float(0x00400000u);
}

// Smallest E8M0 exponent e with amax <= 6 * 2^e (amax >= 0, finite),
// clamped below at -127; -127 for an all-zero block.  amax = 1.f * 2^(eb-127):
// 6 * 2^(eb-129) = 1.5 * 2^(eb-127) suffices when the significand is at most
// 1.5, else 2^(eb-128) * 6 = 3 * 2^(eb-127) does.  Zero and subnormal amax
// (eb = 0) land below -127 and are clamped: 6 * 2^-127 covers them.
__device__ __forceinline__ int piece_exponent(float amax) {
    const uint32_t b = __float_as_uint(amax);
    const int e = (int)(b >> 23) - 129 + ((b & 0x7FFFFFu) > 0x400000u ? 1 : 0);
    return max(e, -127);
}

// 2^-e for e from piece_exponent (e <= 126, so 2^-e is a normal float).
__device__ __forceinline__ float pow2_neg(int e) { return __uint_as_float((uint32_t)(127 - e) << 23); }

// max |v| over the warp: non-negative floats order like their bit patterns,
// so one redux.sync does it.
__device__ __forceinline__ float warp_absmax(float v) {
    return __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(fabsf(v))));
}

// E2M1 code (sign in bit 3) of v rounded to nearest, ties to the even code
// (python/quantize_mxfp4.py:32-34 rounds the same way), saturating at 6.
__device__ __forceinline__ uint32_t e2m1_code(float v) {
    return (uint32_t)__nv_cvt_float2_to_fp4x2(make_float2(v, 0.f), __NV_E2M1, cudaRoundNearest) & 0xFu;
}

// Signed E2M1 level of a code: magnitude bits placed at [22,25) read as
// level * 2^-126 (code 1 is the subnormal 2^-127), times 2^126 exactly.
__device__ __forceinline__ float e2m1_level(uint32_t c) {
    const float mag = __fmul_rn(__uint_as_float((c & 7u) << 22), 0x1p126f);
    return __uint_as_float(__float_as_uint(mag) | ((c & 8u) << 28));
}

// The pieces of one 32-element block (lane i holds element k0 + i) for MT
// tokens at once: token m0 + m has its values in r[m] and is written when
// m < count.  Output goes to the image at bimg for N MMA columns.
// Tokens advance through the pieces together, so their dependent chains
// overlap.  k0 is a multiple of 32.  The whole warp calls it.
template <int MT>
__device__ __forceinline__ void emit_pieces_rows(float (&r)[MT], int m0, int count, int lane, int k0,
                                                 int N, uint8_t* __restrict__ bimg) {
    const int s = k0 / STAGE_K, kbl = (k0 % STAGE_K) / 32;
    uint8_t* img = bimg + (size_t)s * img_stage(N);
    uint8_t* sf = img + N * 128;
    const uint32_t byte = (uint32_t)(kbl * 16 + (lane >> 1));
#pragma unroll 1
    for (int p = 0; p < PIECES; ++p) {
#pragma unroll
        for (int m = 0; m < MT; ++m) {
            const int e = piece_exponent(warp_absmax(r[m]));
            // |r| * 2^-e <= 6: the scaled value rounds to an E2M1 level
            const uint32_t code = e2m1_code(__fmul_rn(r[m], pow2i(-e)));
            r[m] = __fsub_rn(r[m], __fmul_rn(e2m1_level(code), pow2i(e)));  // exact (Sterbenz)
            const uint32_t other = __shfl_down_sync(0xffffffffu, code, 1);
            const uint32_t n = (uint32_t)((m0 + m) * PIECES + p);
            if (m < count) {
                if ((lane & 1) == 0) img[swz128(n, byte)] = (uint8_t)(code | (other << 4));
                if (lane == 0) sf[sf_offset(n, (uint32_t)kbl)] = (uint8_t)(e + 127);
            }
        }
    }
}

// One token's block.
__device__ __forceinline__ void emit_pieces(float r, int lane, int m, int k0, int N,
                                            uint8_t* __restrict__ bimg) {
    float rr[1] = {r};
    emit_pieces_rows<1>(rr, m, 1, lane, k0, N, bimg);
}

// Token buckets: the pieces of tokens 0..count-1 (count <= 16) of one block,
// with the token loop unrolled to the smallest bucket of 1, 2, 4, 8 or 16.
__device__ __forceinline__ void emit_pieces_all(const float (&v)[16], int count, int lane, int k0, int N,
                                                uint8_t* __restrict__ bimg) {
    if (count <= 1) {
        float r[1] = {v[0]};
        emit_pieces_rows<1>(r, 0, count, lane, k0, N, bimg);
    } else if (count <= 2) {
        float r[2] = {v[0], v[1]};
        emit_pieces_rows<2>(r, 0, count, lane, k0, N, bimg);
    } else if (count <= 4) {
        float r[4] = {v[0], v[1], v[2], v[3]};
        emit_pieces_rows<4>(r, 0, count, lane, k0, N, bimg);
    } else if (count <= 8) {
        float r[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) r[i] = v[i];
        emit_pieces_rows<8>(r, 0, count, lane, k0, N, bimg);
    } else {
        float r[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) r[i] = v[i];
        emit_pieces_rows<16>(r, 0, count, lane, k0, N, bimg);
    }
}

// Tokens m0 .. m0+count-1 of one block whose values sit in shared memory,
// vals[m][col] (row stride `ld` floats), bucketed like emit_pieces_all.
__device__ __forceinline__ void emit_pieces_range(const float* vals, int ld, int col, int m0, int count,
                                                  int lane, int k0, int N, uint8_t* __restrict__ bimg) {
    if (count <= 0) return;
    if (count <= 1) {
        float r[1] = {vals[m0 * ld + col]};
        emit_pieces_rows<1>(r, m0, count, lane, k0, N, bimg);
    } else if (count <= 2) {
        float r[2];
#pragma unroll
        for (int i = 0; i < 2; ++i) r[i] = vals[(m0 + i) * ld + col];
        emit_pieces_rows<2>(r, m0, count, lane, k0, N, bimg);
    } else if (count <= 4) {
        float r[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) r[i] = i < count ? vals[(m0 + i) * ld + col] : 0.f;
        emit_pieces_rows<4>(r, m0, count, lane, k0, N, bimg);
    } else {
        float r[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) r[i] = i < count ? vals[(m0 + i) * ld + col] : 0.f;
        emit_pieces_rows<8>(r, m0, count, lane, k0, N, bimg);
    }
}

// Two elements as one E2M1 byte (x in the low nibble, y in the high one),
// rounded to nearest, ties to the even code, saturating at 6; and the two
// levels that byte holds, exactly.
__device__ __forceinline__ uint32_t e2m1x2(float x, float y) {
    return (uint32_t)__nv_cvt_float2_to_fp4x2(make_float2(x, y), __NV_E2M1, cudaRoundNearest);
}
__device__ __forceinline__ float2 e2m1x2_levels(uint32_t byte) {
    const __half2_raw h = __nv_cvt_fp4x2_to_halfraw2((__nv_fp4x2_storage_t)byte, __NV_E2M1);
    __half_raw lo, hi;
    lo.x = h.x;
    hi.x = h.y;
    return make_float2(__half2float(__half(lo)), __half2float(__half(hi)));
}

// Pieces of blocks staged in shared memory, four threads per (token, block):
// thread q of a group owns elements 8q..8q+7, so the block maximum takes two
// shuffles inside the group and each piece is one 4-byte store.
//   vals[m * stride + 32 * b + i]: element i of block b of token m0 + m
//   (m < mcap, b < nblocks); tokens m >= count are encoded as zero.
//   Block b sits at K index k0 + 32 * b of an image with N MMA columns.
// Called by `nthreads` threads (tid = 0..nthreads-1, a multiple of 32 of
// them, all of each warp).
__device__ __forceinline__ void emit_pieces_smem(const float* vals, int stride, int nblocks, int m0,
                                                 int count, int mcap, int tid, int nthreads, int k0,
                                                 int N, uint8_t* __restrict__ bimg) {
    const int groups = mcap * nblocks;
    const int q = tid & 3;
    const int rounds = (groups + nthreads / 4 - 1) / (nthreads / 4);
    for (int it = 0; it < rounds; ++it) {
        const int g = it * (nthreads / 4) + (tid >> 2);
        const bool live = g < groups;
        const int m = live ? g / nblocks : 0, b = live ? g % nblocks : 0;
        float r[8];
        if (live && m < count) {
            const float4* src = (const float4*)(vals + m * stride + 32 * b + 8 * q);
            const float4 v0 = src[0], v1 = src[1];
            r[0] = v0.x; r[1] = v0.y; r[2] = v0.z; r[3] = v0.w;
            r[4] = v1.x; r[5] = v1.y; r[6] = v1.z; r[7] = v1.w;
        } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) r[i] = 0.f;
        }
        const int kk = k0 + 32 * b;
        const int s = kk / STAGE_K, kbl = (kk % STAGE_K) / 32;
        float amax = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(r[i]));
        // the piece words stay in registers until the chain is done, so no
        // store sits between one piece's residual and the next maximum
        uint32_t words[PIECES];
        int exps[PIECES];
#pragma unroll
        for (int p = 0; p < PIECES; ++p) {
            amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
            amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
            const int e = piece_exponent(amax);
            const float down = pow2_neg(e), up = pow2i(e);
            uint32_t word = 0;
            float next = 0.f;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                // |r| * 2^-e <= 6 (exact power-of-two scaling)
                const uint32_t byte = e2m1x2(__fmul_rn(r[2 * i], down), __fmul_rn(r[2 * i + 1], down));
                const float2 lv = e2m1x2_levels(byte);
                r[2 * i] = __fmaf_rn(-lv.x, up, r[2 * i]);  // exact: the difference is representable
                r[2 * i + 1] = __fmaf_rn(-lv.y, up, r[2 * i + 1]);
                next = fmaxf(next, fmaxf(fabsf(r[2 * i]), fabsf(r[2 * i + 1])));
                word |= byte << (8 * i);
            }
            amax = next;
            words[p] = word;
            exps[p] = e;
        }
        if (live) {
            uint8_t* img = bimg + (size_t)s * img_stage(N);
            uint8_t* sf = img + N * 128;
#pragma unroll
            for (int p = 0; p < PIECES; ++p) {
                const uint32_t n = (uint32_t)((m0 + m) * PIECES + p);
                *(uint32_t*)(img + swz128(n, (uint32_t)(kbl * 16 + 4 * q))) = words[p];
                if (q == 0) sf[sf_offset(n, (uint32_t)kbl)] = (uint8_t)(exps[p] + 127);
            }
        }
    }
}

}  // namespace mx
}  // namespace jl
