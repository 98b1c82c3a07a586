// Device helpers shared by the kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "jl_internal.h"

namespace jl {

__device__ __forceinline__ float bf16f(uint32_t bits) { return __uint_as_float(bits << 16); }

// Round-to-nearest-even f32 -> bf16 bits (NaN kept quiet).
__device__ __forceinline__ uint16_t f2bf16(float f) {
    uint32_t u = __float_as_uint(f);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

// E8M0 scale byte -> 2^(s-127) exactly (s == 0 is the subnormal 2^-127;
// 255 is rejected at load time).
__device__ __forceinline__ float e8m0(uint32_t s) {
    return s ? __uint_as_float(s << 23) : __uint_as_float(0x00400000u);
}

// One E2M1 code (low 4 bits of c) as f32: level {0,.5,1,1.5,2,3,4,6}, sign
// in bit 3.  The magnitude bits placed at [22,25) read as level * 2^-126
// (c == 1 lands on the subnormal 2^-127); the exact product by 2^126 restores
// the level.
__device__ __forceinline__ float e2m1(uint32_t c) {
    float mag = __fmul_rn(__uint_as_float((c & 7u) << 22), 0x1p126f);
    return __uint_as_float(__float_as_uint(mag) | ((c & 8u) << 28));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Block-wide sum for blockDim.x a multiple of 32 (<= 1024); `red` holds 32
// floats.  Every thread gets the total.
__device__ __forceinline__ float block_sum(float v, float* red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = 0.f;
    for (int i = 0; i < nw; ++i) t += red[i];
    return t;
}

__device__ __forceinline__ float block_max(float v, float* red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    v = warp_max(v);
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = -INFINITY;
    for (int i = 0; i < nw; ++i) t = fmaxf(t, red[i]);
    return t;
}

// Streaming 16-byte load of weights: read once per pass, so keep them out of L1.
__device__ __forceinline__ uint4 ldg_stream(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

// One layer's view of the paged KV pool ([page][kv_head][PAGE][HEAD]).
struct KvView {
    void* k;       // this layer's K pages
    void* v;       // this layer's V pages
    int kv_heads;
    int f32;       // 1: f32 elements, 0: bf16
    int pages;     // pool size: page ids outside [0, pages) are never dereferenced
    int max_pos;   // RoPE table rows (context limit)
    int* err;      // device error flag: bit 0 page id out of range, bit 1 bad position
};

__device__ __forceinline__ bool page_ok(const KvView& kv, int page) {
    if ((unsigned)page < (unsigned)kv.pages) return true;
    atomicOr(kv.err, 1);
    return false;
}

__device__ __forceinline__ size_t kv_index(int page, int kvh, int t, int kv_heads) {
    return (((size_t)page * kv_heads + kvh) * PAGE + t) * HEAD;
}

// Host side: the view of `layer` and the row stride of the fused q|k|v buffer.
inline KvView kv_view(const jl_model* m, int layer) {
    KvView v;
    const size_t bytes_layer = m->kv.pages * m->kv.page_elems * m->kv.elem;
    char* base = (char*)m->kv.base + (size_t)layer * 2 * bytes_layer;
    v.k = base;
    v.v = base + bytes_layer;
    v.kv_heads = m->kv_heads;
    v.f32 = m->kv.dtype == JL_KV_F32;
    v.pages = (int)m->kv.pages;
    v.max_pos = m->max_positions;
    v.err = m->counters;
    return v;
}

inline int qkv_ld(const jl_model* m) { return (m->q_heads + 2 * m->kv_heads) * HEAD; }

// What the QK-RMSNorm and RoPE of one head need besides the head itself:
// lane l's norm weights for dims (l, l+32, l+64, l+96) and rotation factors
// for dims l and l+32 at position pos.  None of it depends on the previous
// kernel, so it is fetched before the dependency wait.
struct NormRope {
    float w[4];
    float2 c0, c1;
};
__device__ __forceinline__ NormRope norm_rope_args(const uint16_t* gw, const float2* rope, int pos, int lane) {
    NormRope r;
#pragma unroll
    for (int i = 0; i < 4; ++i) r.w[i] = bf16f(gw[lane + 32 * i]);
    r.c0 = rope[(size_t)pos * HALF + lane];
    r.c1 = rope[(size_t)pos * HALF + lane + 32];
    return r;
}

// QK-RMSNorm and RoPE of one head held as dims (l, l+32, l+64, l+96) by lane
// l (lib.rs:306-313, 372-388; the arithmetic of k_qk_rope_kv).
__device__ __forceinline__ void norm_rope4(float& a0, float& a1, float& a2, float& a3, const NormRope& nr) {
    float ss = fmaf(a0, a0, fmaf(a1, a1, fmaf(a2, a2, a3 * a3)));
    ss = warp_sum(ss);
    const float size = sqrtf(__fadd_rn(__fdiv_rn(ss, 128.0f), 1e-6f));
    const float2 c0 = nr.c0, c1 = nr.c1;
    a0 = __fmul_rn(__fdiv_rn(a0, size), nr.w[0]);
    a1 = __fmul_rn(__fdiv_rn(a1, size), nr.w[1]);
    a2 = __fmul_rn(__fdiv_rn(a2, size), nr.w[2]);
    a3 = __fmul_rn(__fdiv_rn(a3, size), nr.w[3]);
    const float b0 = __fsub_rn(__fmul_rn(a0, c0.x), __fmul_rn(a2, c0.y));
    const float b2 = __fadd_rn(__fmul_rn(a2, c0.x), __fmul_rn(a0, c0.y));
    const float b1 = __fsub_rn(__fmul_rn(a1, c1.x), __fmul_rn(a3, c1.y));
    const float b3 = __fadd_rn(__fmul_rn(a3, c1.x), __fmul_rn(a1, c1.y));
    a0 = b0; a1 = b1; a2 = b2; a3 = b3;
}


}  // namespace jl
