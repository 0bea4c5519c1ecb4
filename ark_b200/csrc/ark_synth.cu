// ark_synth.cu -- seeded synthetic optimizer inputs generated on the device.
//
// splitmix64 counter RNG keyed by (seed, stream, global flat index) and an
// Irwin-Hall(12) normal: the sum of twelve 24-bit uniforms is formed as an
// exact integer, converted to float once (round to nearest even) and scaled
// by 2^-24 (exact).  Every later rounding is an explicit _rn intrinsic, so
// the values are bit-identical to the CPU generator used by the tests, for
// any sharding of the flat index space.
#include <cuda_runtime.h>

#include "ark_device.cuh"
#include "ark_internal.h"

namespace ark {

__device__ __forceinline__ uint64_t splitmix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

__device__ __forceinline__ float irwin_hall_normal(uint64_t key, uint64_t idx) {
    int32_t s = 0;
#pragma unroll
    for (uint64_t j = 0; j < 6; ++j) {
        const uint64_t r = splitmix64(key + idx * 6u + j);
        s += (int32_t)(r >> 40);
        s += (int32_t)((r >> 16) & 0xFFFFFFu);
    }
    return __fmul_rn(__int2float_rn(s - 6 * (1 << 24)), 0x1p-24f);
}

constexpr int kST = 256;

__global__ void __launch_bounds__(kST) synth_f16_kernel(uint16_t* out, uint64_t n, uint64_t offset,
                                                       uint64_t seed, uint64_t key, float sigma,
                                                       float mult, uint32_t heavy_every,
                                                       float heavy_mult) {
    const uint64_t stride = (uint64_t)gridDim.x * kST;
    for (uint64_t i = (uint64_t)blockIdx.x * kST + threadIdx.x; i < n; i += stride) {
        const uint64_t gi = offset + i;
        float x = __fmul_rn(irwin_hall_normal(key, gi), sigma);
        if (heavy_every && splitmix64(seed ^ gi ^ 0xA5A5A5A5A5A5A5A5ull) % heavy_every == 0)
            x = __fmul_rn(x, heavy_mult);
        x = __fmul_rn(x, mult);
        out[i] = f2h(x);
    }
}

__global__ void __launch_bounds__(kST) synth_f32_kernel(float* out, uint64_t n, uint64_t offset,
                                                       uint64_t key, float sigma, int square) {
    const uint64_t stride = (uint64_t)gridDim.x * kST;
    for (uint64_t i = (uint64_t)blockIdx.x * kST + threadIdx.x; i < n; i += stride) {
        const float x = __fmul_rn(irwin_hall_normal(key, offset + i), sigma);
        out[i] = square ? __fmul_rn(x, x) : x;
    }
}

static uint64_t host_splitmix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

}  // namespace ark

using namespace ark;

extern "C" {

int ark_synth_f16(uint16_t* out, uint64_t n, uint64_t offset, uint64_t seed, uint64_t stream,
                  float sigma, float mult, uint32_t heavy_every, float heavy_mult,
                  void* cuda_stream) {
    if (n == 0) return ARK_OK;
    if (!out) return ARK_E_INVALID_ARG;
    const uint64_t key = host_splitmix64(seed ^ host_splitmix64(stream));
    const int blocks = streaming_grid(reinterpret_cast<const void*>(synth_f16_kernel), kST, 0, n);
    synth_f16_kernel<<<blocks, kST, 0, reinterpret_cast<cudaStream_t>(cuda_stream)>>>(
        out, n, offset, seed, key, sigma, mult, heavy_every, heavy_mult);
    return cudaGetLastError() == cudaSuccess ? ARK_OK : ARK_E_CUDA;
}

int ark_synth_f32(float* out, uint64_t n, uint64_t offset, uint64_t seed, uint64_t stream,
                  float sigma, int square, void* cuda_stream) {
    if (n == 0) return ARK_OK;
    if (!out) return ARK_E_INVALID_ARG;
    const uint64_t key = host_splitmix64(seed ^ host_splitmix64(stream));
    const int blocks = streaming_grid(reinterpret_cast<const void*>(synth_f32_kernel), kST, 0, n);
    synth_f32_kernel<<<blocks, kST, 0, reinterpret_cast<cudaStream_t>(cuda_stream)>>>(
        out, n, offset, key, sigma, square);
    return cudaGetLastError() == cudaSuccess ? ARK_OK : ARK_E_CUDA;
}

}  // extern "C"
