// A/B benchmark (not part of the library): an MXFP4 projection on CUDA cores
// for M <= 8 input rows, to compare with the tensor-core projection the
// library runs (k_mx_gemv) at the verify pass's M = k + 1 = 5.
//
// One lane per weight row, so no reduction across lanes: weights in a
// transposed tile layout (a tile is 32 rows; per 32-element block, codes
// [4 words][32 rows] -- word w of row r holds elements 8w..8w+7 -- then 32
// E8M0 scale bytes), each lane decoding E2M1 pairs in hardware
// (cvt.rn.f16x2.e2m1x2) and multiplying them into M f32 accumulators; the
// activations of a stage are read by every lane at the same address
// (broadcast).  A CTA of NW warps owns NW tiles; one producer thread streams
// stages of SB blocks of every tile, plus the stage's activation slice,
// through a shared-memory ring with bulk copies.  Random codes and scales;
// three rows are checked against a double-precision host sum.
//
// Build and run (B200): make -C jalapenos-at-home_b200 ab && jalapenos-at-home_b200/ab/cuda_core_projection [case]
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_fp4.h>
#include <cstdio>
#include <cstdlib>
#include <vector>
#include <cstdint>

#define CK(x) do { cudaError_t e = (x); if (e != cudaSuccess) { printf("%s: %s\n", #x, cudaGetErrorString(e)); exit(1); } } while (0)

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void mbar_init(uint64_t* b, uint32_t c) { asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(c)); }
__device__ __forceinline__ void mbar_expect(uint64_t* b, uint32_t bytes) { asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)), "r"(bytes) : "memory"); }
__device__ __forceinline__ void mbar_arrive(uint64_t* b) { asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(b)) : "memory"); }
__device__ __forceinline__ bool mbar_try(uint64_t* b, uint32_t par) {
    uint32_t ok; asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}" : "=r"(ok) : "r"(smem_u32(b)), "r"(par) : "memory"); return ok; }
__device__ __forceinline__ void mbar_wait(uint64_t* b, uint32_t par) { for (uint32_t i = 0; i < (1u << 24); ++i) if (mbar_try(b, par)) return; }
__device__ __forceinline__ void bulk(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)) : "memory"); }

__device__ __forceinline__ float2 lv2(uint32_t byte) {
    __half2_raw h = __nv_cvt_fp4x2_to_halfraw2((__nv_fp4x2_storage_t)byte, __NV_E2M1);
    __half_raw lo, hi; lo.x = h.x; hi.x = h.y;
    return make_float2(__half2float(__half(lo)), __half2float(__half(hi)));
}
__device__ __forceinline__ float e8m0(uint32_t s) { return s ? __uint_as_float(s << 23) : __uint_as_float(0x00400000u); }

constexpr int NW = 4;            // warps (tiles of 32 rows) per CTA
constexpr int SB = 8;            // 32-element blocks per stage
constexpr int NST = 6;           // ring stages
constexpr int BLK_BYTES = 32 * 16 + 32;   // one block of one tile: codes + scales
constexpr int WST_BYTES = NW * SB * BLK_BYTES;  // weights of a stage
template <int M> constexpr int stage_bytes() { return WST_BYTES + M * SB * 32 * 4; }

// w: [tiles][K/32][BLK_BYTES]; x: [M][K]; y: [M][rows]
template <int M>
__global__ void __launch_bounds__(NW * 32 + 32) k_lanerow(const uint8_t* __restrict__ w, const float* __restrict__ x,
                                                         float* __restrict__ y, int K, int tiles) {
    extern __shared__ __align__(128) uint8_t sm[];
    __shared__ uint64_t full[NST], empty[NST];
    constexpr int STAGE_BYTES = stage_bytes<M>();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nblk = K / 32, nst = nblk / SB;
    const int t0 = blockIdx.x * NW;
    if (threadIdx.x == 0) { for (int s = 0; s < NST; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], NW); } asm volatile("fence.mbarrier_init.release.cluster;"); }
    __syncthreads();
    if (warp == NW) {
        if (lane == 0) {
            for (int st = 0; st < nst; ++st) {
                const int s = st % NST, it = st / NST;
                if (st >= NST) mbar_wait(&empty[s], (it - 1) & 1);
                mbar_expect(&full[s], STAGE_BYTES);
                for (int t = 0; t < NW; ++t)
                    bulk(sm + s * STAGE_BYTES + t * SB * BLK_BYTES, w + ((size_t)(t0 + t) * nblk + st * SB) * BLK_BYTES,
                         SB * BLK_BYTES, &full[s]);
                for (int m = 0; m < M; ++m)
                    bulk(sm + s * STAGE_BYTES + WST_BYTES + m * SB * 128, x + (size_t)m * K + st * SB * 32, SB * 128, &full[s]);
            }
        }
        return;
    }
    float acc[M];
#pragma unroll
    for (int m = 0; m < M; ++m) acc[m] = 0.f;
    for (int st = 0; st < nst; ++st) {
        const int s = st % NST, it = st / NST;
        mbar_wait(&full[s], it & 1);
        const uint8_t* tile = sm + s * STAGE_BYTES + warp * SB * BLK_BYTES;
        const float* xst = reinterpret_cast<const float*>(sm + s * STAGE_BYTES + WST_BYTES);  // [M][SB * 32]
#pragma unroll 2
        for (int b = 0; b < SB; ++b) {
            const uint8_t* blk = tile + b * BLK_BYTES;
            const float sc = e8m0(blk[512 + lane]);
            float part[M];
#pragma unroll
            for (int m = 0; m < M; ++m) part[m] = 0.f;
            const int kb = b * 32;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const uint32_t word = reinterpret_cast<const uint32_t*>(blk)[q * 32 + lane];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const float2 l = lv2((word >> (8 * j)) & 0xffu);
                    const int k = kb + 8 * q + 2 * j;
#pragma unroll
                    for (int m = 0; m < M; ++m) {
                        const float2 xv = *reinterpret_cast<const float2*>(xst + m * SB * 32 + k);
                        part[m] = fmaf(l.x, xv.x, part[m]);
                        part[m] = fmaf(l.y, xv.y, part[m]);
                    }
                }
            }
#pragma unroll
            for (int m = 0; m < M; ++m) acc[m] = fmaf(part[m], sc, acc[m]);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }
    const int row = (t0 + warp) * 32 + lane;
#pragma unroll
    for (int m = 0; m < M; ++m) y[(size_t)m * tiles * 32 + row] = acc[m];
}

template <int M>
void run(int rows, int K, int iters) {
    const int tiles = rows / 32, nblk = K / 32;
    std::vector<uint8_t> hw((size_t)tiles * nblk * BLK_BYTES);
    for (size_t i = 0; i < hw.size(); ++i) hw[i] = (uint8_t)(rand() & 0x77);
    for (int t = 0; t < tiles; ++t) for (int b = 0; b < nblk; ++b) for (int r = 0; r < 32; ++r) hw[((size_t)t * nblk + b) * BLK_BYTES + 512 + r] = 120 + (rand() % 8);
    uint8_t* dw; float *dx, *dy;
    const size_t copies = std::max<size_t>(1, (size_t)(600u << 20) / hw.size());  // > L2
    CK(cudaMalloc(&dw, hw.size() * copies)); CK(cudaMalloc(&dx, (size_t)M * K * 4)); CK(cudaMalloc(&dy, (size_t)M * rows * 4));
    for (size_t c = 0; c < copies; ++c) CK(cudaMemcpy(dw + c * hw.size(), hw.data(), hw.size(), cudaMemcpyHostToDevice));
    std::vector<float> hx((size_t)M * K); for (auto& v : hx) v = (rand() % 2000 - 1000) / 1000.f;
    CK(cudaMemcpy(dx, hx.data(), hx.size() * 4, cudaMemcpyHostToDevice));
    const size_t smem = NST * stage_bytes<M>();
    CK(cudaFuncSetAttribute(k_lanerow<M>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    const int grid = tiles / NW;
    k_lanerow<M><<<grid, NW * 32 + 32, smem>>>(dw, dx, dy, K, tiles);
    CK(cudaDeviceSynchronize());
    // check one row against a host dot
    std::vector<float> hy((size_t)M * rows); CK(cudaMemcpy(hy.data(), dy, hy.size() * 4, cudaMemcpyDeviceToHost));
    double maxerr = 0;
    for (int row : {0, 33, rows - 1}) {
        const int t = row / 32, r = row % 32;
        for (int m = 0; m < M; ++m) {
            double acc = 0;
            for (int b = 0; b < nblk; ++b) {
                const uint8_t* blk = &hw[((size_t)t * nblk + b) * BLK_BYTES];
                const double sc = ldexp(1.0, blk[512 + r] - 127);
                for (int q = 0; q < 4; ++q) {
                    uint32_t word; memcpy(&word, blk + (q * 32 + r) * 4, 4);
                    for (int e = 0; e < 8; ++e) {
                        const uint32_t c = (word >> (4 * e)) & 15;
                        static const float L[8] = {0, .5f, 1, 1.5f, 2, 3, 4, 6};
                        const double v = (c & 8 ? -1 : 1) * L[c & 7];
                        acc += v * sc * hx[(size_t)m * K + b * 32 + q * 8 + e];
                    }
                }
            }
            maxerr = std::max(maxerr, fabs(acc - hy[(size_t)m * rows + row]) / (fabs(acc) + 1e-3));
        }
    }
    cudaEvent_t e0, e1; cudaEventCreate(&e0); cudaEventCreate(&e1);
    cudaEventRecord(e0);
    for (int i = 0; i < iters; ++i) k_lanerow<M><<<grid, NW * 32 + 32, smem>>>(dw + (i % copies) * hw.size(), dx, dy, K, tiles);
    cudaEventRecord(e1); CK(cudaEventSynchronize(e1));
    float ms; cudaEventElapsedTime(&ms, e0, e1);
    const double per = ms / iters * 1e-3;
    printf("M=%d rows=%d K=%d grid=%d: %.2f us/launch, %.0f GB/s, rel err %.2e\n", M, rows, K, grid, per * 1e6,
           hw.size() / per / 1e9, maxerr);
    cudaFree(dw); cudaFree(dx); cudaFree(dy);
}

// Qwen3-8B shapes: gate/up (24576 x 4096), down (4096 x 12288), q|k|v
// (6144 x 4096).  With an argument, only that case (for a profiler).
int main(int argc, char** argv) {
    const int only = argc > 1 ? atoi(argv[1]) : -1;
    int c = 0;
    if (only < 0 || only == c) run<1>(24576, 4096, 50);
    if (only < 0 || only == ++c) run<5>(24576, 4096, 50);
    if (only < 0 || only == ++c) run<8>(24576, 4096, 50);
    if (only < 0 || only == ++c) run<5>(4096, 12288, 50);
    if (only < 0 || only == ++c) run<5>(6144, 4096, 50);
    if (only < 0 || only == ++c) run<1>(6144, 4096, 50);
    return 0;
}
