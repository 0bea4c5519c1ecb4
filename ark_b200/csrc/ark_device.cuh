// ark_device.cuh -- device-side building blocks shared by the optimizer
// kernels.  Every floating-point operation that must match the reference is
// written with an explicit-rounding intrinsic (__fmul_rn, __fadd_rn,
// __fsub_rn, __fdiv_rn, __fsqrt_rn, __fmaf_rn) so nvcc can neither contract
// nor approximate it; the library is built without --use_fast_math and with
// -ftz=false so subnormals are kept, as on the reference's FPU (default FPCR).
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

namespace ark {

__device__ __forceinline__ float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }
__device__ __forceinline__ uint16_t f2h(float f) { return __half_as_ushort(__float2half_rn(f)); }

// AdamW per-call scalars (asm/opti.s:210-271).
struct AdamK {
    float b1, b2, omb1, omb2, eps, lr_eff, decay;
};

__device__ __forceinline__ float pow_binary(float base, uint32_t t) {
    // opti.s:223-237 -- res=1; while t: if t&1: res*=base; base*=base; t>>=1
    float res = 1.0f;
    for (uint32_t e = t; e; e >>= 1) {
        if (e & 1u) res = __fmul_rn(res, base);
        base = __fmul_rn(base, base);
    }
    return res;
}

__device__ __forceinline__ AdamK adam_scalars(float lr, float b1, float b2, float eps, float wd,
                                              uint32_t t) {
    if (t == 0) t = 1;                                           // opti.s:211-212
    AdamK k;
    k.decay = __fsub_rn(1.0f, __fmul_rn(lr, wd));                // :219-221
    const float bc1 = __fsub_rn(1.0f, pow_binary(b1, t));        // :223-237
    const float bc2 = __fsub_rn(1.0f, pow_binary(b2, t));        // :239-253
    k.lr_eff = __fmul_rn(__fdiv_rn(__fsqrt_rn(bc2), bc1), lr);   // :256-258
    k.b1 = b1;
    k.b2 = b2;
    k.omb1 = __fsub_rn(1.0f, b1);                                // :263-265
    k.omb2 = __fsub_rn(1.0f, b2);                                // :266-268
    k.eps = eps;
    return k;
}

// One element of the update, opti.s:285-304 (== tail :324-343):
//   m = fma(1-b1, g, m*b1); v = fma(1-b2, g*g, v*b2)
//   w = w*decay - (m / (sqrt(v) + eps)) * lr_eff      (mul and sub separate)
__device__ __forceinline__ float adam_elem(float w, float g, float& m, float& v, const AdamK& k,
                                           float decay) {
    const float mm = __fmaf_rn(k.omb1, g, __fmul_rn(m, k.b1));
    const float vv = __fmaf_rn(k.omb2, __fmul_rn(g, g), __fmul_rn(v, k.b2));
    const float den = __fadd_rn(__fsqrt_rn(vv), k.eps);
    const float upd = __fmul_rn(__fdiv_rn(mm, den), k.lr_eff);
    m = mm;
    v = vv;
    return __fsub_rn(__fmul_rn(w, decay), upd);
}

// ---- streaming memory access ----------------------------------------
// Read-once data: bypass L1, mark for early eviction in L2.
__device__ __forceinline__ uint4 ld_stream(const uint4* p) { return __ldcs(p); }
__device__ __forceinline__ float4 ld_stream(const float4* p) { return __ldcs(p); }
__device__ __forceinline__ void st_stream(uint4* p, uint4 x) { __stcs(p, x); }
__device__ __forceinline__ void st_stream(float4* p, float4 x) { __stcs(p, x); }
// Data another kernel reads soon (pass-1 gradients re-read by pass 2).
__device__ __forceinline__ uint4 ld_keep(const uint4* p) { return __ldcg(p); }

__device__ __forceinline__ uint16_t lo16(uint32_t x) { return (uint16_t)(x & 0xFFFFu); }
__device__ __forceinline__ uint16_t hi16(uint32_t x) { return (uint16_t)(x >> 16); }
__device__ __forceinline__ uint32_t pack16(uint16_t lo, uint16_t hi) {
    return (uint32_t)lo | ((uint32_t)hi << 16);
}

// ---- block reductions (fixed shape => deterministic for a fixed grid) --
template <int THREADS>
__device__ __forceinline__ double block_sum(double x, double* smem) {
    static_assert(THREADS % 32 == 0 && THREADS <= 1024, "block size");
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xFFFFFFFFu, x, o);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) smem[warp] = x;
    __syncthreads();
    double r = 0.0;
    if (warp == 0) {
        r = lane < THREADS / 32 ? smem[lane] : 0.0;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) r += __shfl_xor_sync(0xFFFFFFFFu, r, o);
    }
    __syncthreads();
    return r;  // valid in thread 0
}

template <int THREADS>
__device__ __forceinline__ unsigned long long block_sum_u64(unsigned long long x,
                                                            unsigned long long* smem) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xFFFFFFFFu, x, o);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) smem[warp] = x;
    __syncthreads();
    unsigned long long r = 0;
    if (warp == 0) {
        r = lane < THREADS / 32 ? smem[lane] : 0ull;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) r += __shfl_xor_sync(0xFFFFFFFFu, r, o);
    }
    __syncthreads();
    return r;
}

// "Last block done" ticket: returns true in every thread of the block that
// arrives last.  The partials written before the call are visible to that
// block (release fence before the ticket, acquire fence after it).
__device__ __forceinline__ bool last_block_arrived(unsigned int* ticket, int* flag_smem) {
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned int prev = atomicAdd(ticket, 1u);
        const bool last = (prev == gridDim.x - 1);
        if (last) *ticket = 0u;  // re-armed for the next launch / graph replay
        *flag_smem = last;
    }
    __syncthreads();
    const bool last = *flag_smem != 0;
    if (last) __threadfence();
    return last;
}

}  // namespace ark
