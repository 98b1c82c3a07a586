// A/B benchmark (not part of the library): the activation-piece encoder.
//
// The tensor-core projections take their f32 inputs as eight E2M1 "pieces"
// with E8M0 block scales (csrc/mx_pieces.cuh); each projection's epilogue
// encodes its outputs for the next one, so the encoder sits on the critical
// path of every decode kernel.  This times the library's encoder
// (emit_pieces_smem: four threads per (row, 32-element block), hardware
// cvt.rn.satfinite.e2m1x2.f32 rounding) against a variant that rounds to the
// E2M1 grid with float arithmetic (adding 2^22 * max(1, 2^floor(log2 |y|))
// leaves the grid step as the ulp, ties to even), on 1, 5, 8 and 16 rows of
// 4 blocks by 128 threads, 20 calls per launch, clock64 per call, on one CTA
// and on 148.  It first checks over 200 seeds of adversarial inputs (exact
// ties, zeros of both signs, subnormals, dense mantissas) that both write
// identical images.
//
// Build and run (B200): make -C jalapenos-at-home_b200 ab && jalapenos-at-home_b200/ab/piece_encoder
#include <cuda_runtime.h>
#include <cstdio>
#include <cstdlib>
#include <vector>
#include "../csrc/mx_pieces.cuh"
using namespace jl;
using namespace jl::mx;

// four threads per (token, block) as emit_pieces_smem; E2M1 rounding by float arithmetic
__device__ __forceinline__ void emit_float(const float* vals, int stride, int nblocks, int m0, int count, int mcap,
                                          int tid, int nthreads, int k0, int N, uint8_t* __restrict__ bimg) {
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
        float a4[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) a4[i] = fmaxf(fabsf(r[2 * i]), fabsf(r[2 * i + 1]));
        float amax = fmaxf(fmaxf(a4[0], a4[1]), fmaxf(a4[2], a4[3]));
        uint32_t words[PIECES];
        int exps[PIECES];
#pragma unroll
        for (int p = 0; p < PIECES; ++p) {
            amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
            amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
            const int e = piece_exponent(amax);
            const float down = pow2_neg(e), up = pow2i(e);
            uint32_t word = 0;
            float ab[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const float y = __fmul_rn(r[i], down);  // |y| <= 6
                const uint32_t yb = __float_as_uint(y);
                // round |y| to the E2M1 grid (steps 0.5 below 2, then 1, then 2), ties to even:
                // adding 2^22 * max(1, 2^floor(log2|y|)) leaves exactly that step as the ulp
                const float big = __uint_as_float(max(yb & 0x7F800000u, 0x3F800000u) + (22u << 23));
                const float mag = __fsub_rn(__fadd_rn(__uint_as_float(yb & 0x7FFFFFFFu), big), big);
                const uint32_t code = (__float_as_uint(__fmul_rn(mag, 0x1p-126f)) >> 22) | ((yb >> 28) & 8u);
                const float lv = __uint_as_float(__float_as_uint(mag) | (yb & 0x80000000u));
                r[i] = __fmaf_rn(-lv, up, r[i]);
                ab[i] = fabsf(r[i]);
                word |= code << (4 * i);
            }
            amax = fmaxf(fmaxf(fmaxf(ab[0], ab[1]), fmaxf(ab[2], ab[3])), fmaxf(fmaxf(ab[4], ab[5]), fmaxf(ab[6], ab[7])));
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

template <int V>
__global__ void k_bench(const float* in, int mcap, uint8_t* out, long long* cyc, int reps) {
    __shared__ __align__(16) float vals[16 * 128];
    for (int i = threadIdx.x; i < 16 * 128; i += blockDim.x) vals[i] = in[i];
    __syncthreads();
    uint8_t* img = out + (size_t)blockIdx.x * 128 * 1024;
    long long t0 = clock64();
    for (int r = 0; r < reps; ++r) {
        if (V == 0) emit_pieces_smem(vals, 128, 4, 0, mcap, mcap, threadIdx.x, 128, 128 * (r & 7), 8 * mcap, img);
        else emit_float(vals, 128, 4, 0, mcap, mcap, threadIdx.x, 128, 128 * (r & 7), 8 * mcap, img);
        __syncthreads();
    }
    long long t1 = clock64();
    if (threadIdx.x == 0) cyc[blockIdx.x] = (t1 - t0) / reps;
}


static float adversarial(int i, int seed) {
    unsigned h = (unsigned)(i * 2654435761u) ^ (unsigned)(seed * 40503u + 17u);
    h ^= h >> 13; h *= 0x5bd1e995u; h ^= h >> 15;
    const int kind = h % 8;
    const float sign = (h >> 8) & 1 ? -1.f : 1.f;
    const int ex = (int)((h >> 9) % 60) - 30;
    switch (kind) {
        case 0: return 0.f;
        case 1: return -0.f;
        case 2: return sign * ldexpf(0.25f * (float)((h >> 16) % 25), ex);         // grid points and exact ties
        case 3: return sign * ldexpf(1.f + (float)((h >> 16) % 4096) / 4096.f, ex); // dense mantissas
        case 4: return sign * ldexpf((float)((h >> 16) % 1000), -149 + (int)((h >> 3) % 20));  // subnormals
        case 5: return sign * (float)((h >> 16) % 7);
        default: return sign * ldexpf((float)((h >> 12) & 0xFFFFF) / 1048576.f, ex);
    }
}

int main() {
    std::vector<float> h(16 * 128);
    float* din; uint8_t* dout; long long* dc;
    cudaMalloc(&din, h.size() * 4); cudaMalloc(&dout, 148 * 128 * 1024); cudaMalloc(&dc, 148 * 8);
    int bad = 0;
    for (int seed = 0; seed < 200; ++seed) {
        for (size_t i = 0; i < h.size(); ++i) h[i] = adversarial((int)i, seed);
        if (seed % 5 == 4) for (size_t i = 0; i < h.size(); ++i) h[i] = (rand() % 20001 - 10000) / 777.0f;
        cudaMemcpy(din, h.data(), h.size() * 4, cudaMemcpyHostToDevice);
        for (int mcap : {1, 5, 16}) {
            std::vector<uint8_t> a(80 * 1024), b(80 * 1024);
            cudaMemset(dout, 0, 80 * 1024); k_bench<0><<<1, 128>>>(din, mcap, dout, dc, 8); cudaMemcpy(a.data(), dout, a.size(), cudaMemcpyDeviceToHost);
            cudaMemset(dout, 0, 80 * 1024); k_bench<1><<<1, 128>>>(din, mcap, dout, dc, 8); cudaMemcpy(b.data(), dout, b.size(), cudaMemcpyDeviceToHost);
            if (a != b) { if (bad < 5) printf("seed %d mcap %d: images differ\n", seed, mcap); ++bad; }
        }
    }
    cudaError_t e = cudaDeviceSynchronize();
    printf("identical images over 200 seeds x 3 row counts: %d mismatches (%s)\n", bad, cudaGetErrorString(e));
    for (int mcap : {1, 5, 8, 16}) {
        for (int v : {0, 1}) {
            for (int grid : {1, 148}) {
                if (v == 0) k_bench<0><<<grid, 128>>>(din, mcap, dout, dc, 20);
                else k_bench<1><<<grid, 128>>>(din, mcap, dout, dc, 20);
                cudaError_t e2 = cudaDeviceSynchronize();
                if (e2 != cudaSuccess) { printf("err %s\n", cudaGetErrorString(e2)); return 1; }
                long long c; cudaMemcpy(&c, dc, 8, cudaMemcpyDeviceToHost);
                printf("rows %2d %-22s grid %3d: %lld cycles per call (%.2f us at 1.9 GHz)\n", mcap, v ? "float rounding" : "library (cvt rounding)", grid, c, c / 1900.0);
            }
        }
    }
    return bad ? 1 : 0;
}
