// ark_legacy.cu -- the five symbols ARK's Rust code binds today
// (proyecto_ark/ark01/src/optimizer.rs:20-23, src/ffi.rs:88-115), as CUDA
// kernels over device pointers, plus the library-wide controls.
//
//   ark_asm_adam_step_f16 / ark_asm_adam_step  (asm/opti.s:192-360, :20-177)
//   ark_asm_grad_clip                          (asm/opti.s:369-432)
//   ark_quant_f32_to_f16 / ark_dequant_f16_to_f32 (asm/kern.s:879-913, :835-869)
//
// All are HBM-streaming kernels: 16-byte vector loads/stores when every
// pointer is 16-byte aligned, a scalar grid-stride path otherwise (any
// element alignment works).  Calls run on the legacy default stream (so they
// are ordered after other default-stream work) and are synchronous by
// default, so the reference's "returns when done" contract holds for a
// caller that reads the buffers right after the call.
#include <cuda_runtime.h>
#include <stdlib.h>
#include <string.h>

#include <atomic>
#include <mutex>

#include "ark_device.cuh"
#include "ark_internal.h"
#include "ark_sync.cuh"

namespace ark {

// ------------------------------------------------------------ errors
static thread_local int t_last_error = ARK_OK;
static std::atomic<uint32_t> g_reported{0};

void set_last_error(int code) { t_last_error = code; }

void legacy_fail(const char* fn, int code, const char* detail) {
    t_last_error = code;
    const uint32_t bit = 1u << ((-code) & 31);
    if (!(g_reported.fetch_or(bit) & bit))
        fprintf(stderr, "[ark_cuda] %s failed: %s%s%s\n", fn, status_string(code),
                detail ? ": " : "", detail ? detail : "");
}

const char* status_string(int s) {
    switch (s) {
        case ARK_OK: return "ok";
        case ARK_E_INVALID_ARG: return "invalid argument";
        case ARK_E_MISALIGNED: return "buffer not 16-byte aligned";
        case ARK_E_CUDA: return "CUDA runtime error";
        case ARK_E_NCCL: return "NCCL error";
        case ARK_E_TIMEOUT: return "device-side wait timed out";
        case ARK_E_EARLY_STOP: return "early stop: too many consecutive overflow steps";
        case ARK_E_NO_DEVICE: return "no usable CUDA device";
        case ARK_E_UNSUPPORTED: return "unsupported";
        default: return "unknown status";
    }
}

// Resident-block capacity (SMs x blocks per SM) per kernel and device,
// looked up once: the legacy entry points are called hundreds of times per
// optimizer step (one call per tensor), and the occupancy query costs more
// host time than launching a small kernel.
struct GridCacheEntry {
    const void* kernel;
    int dev, threads;
    size_t smem;
    uint64_t full;
};
static std::mutex g_grid_mu;
static GridCacheEntry g_grid_cache[128];
static int g_grid_used = 0;

static uint64_t resident_capacity(const void* kernel, int threads, size_t dyn_smem) {
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lk(g_grid_mu);
    for (int i = 0; i < g_grid_used; ++i) {
        const GridCacheEntry& e = g_grid_cache[i];
        if (e.kernel == kernel && e.dev == dev && e.threads == threads && e.smem == dyn_smem)
            return e.full;
    }
    int sms = 148, per_sm = 1;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, dyn_smem);
    if (per_sm < 1) per_sm = 1;
    const uint64_t full = (uint64_t)sms * (uint64_t)per_sm;
    if (g_grid_used < (int)(sizeof(g_grid_cache) / sizeof(g_grid_cache[0])))
        g_grid_cache[g_grid_used++] = GridCacheEntry{kernel, dev, threads, dyn_smem, full};
    return full;
}

// SMs of the current device (looked up once per device).
static int sm_count() {
    static std::atomic<int> cache[64];
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) dev = 0;
    int v = cache[dev].load();
    if (v <= 0) {
        v = 148;
        cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
        cache[dev].store(v);
    }
    return v;
}

int streaming_grid(const void* kernel, int threads, size_t dyn_smem, uint64_t work_items) {
    const uint64_t full = resident_capacity(kernel, threads, dyn_smem);
    uint64_t need = (work_items + threads - 1) / threads;
    if (need < 1) need = 1;
    return (int)(need < full ? need : full);
}

// ------------------------------------------------------------ legacy context
struct LegacyCtx {
    std::mutex mu;
    void* scratch = nullptr;            // grad-clip partials + ticket + result
    int scratch_blocks = 0;
};

static LegacyCtx g_ctx[64];
static std::atomic<int> g_async{0};
static std::atomic<uint32_t> g_compat{0};
static std::atomic<cudaStream_t> g_stream{nullptr};   // NULL: legacy default stream

struct ClipResult {
    float norm;
    float scale;
    int apply;
    int pad;
};

static int current_ctx(LegacyCtx** out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return ARK_E_NO_DEVICE;
    if (dev < 0 || dev >= 64) return ARK_E_NO_DEVICE;
    *out = &g_ctx[dev];
    return ARK_OK;
}

static cudaStream_t legacy_stream(LegacyCtx*) { return g_stream.load(); }

static int finish(LegacyCtx* c) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return ARK_E_CUDA;
    if (!g_async.load()) {
        e = cudaStreamSynchronize(legacy_stream(c));
        if (e != cudaSuccess) return ARK_E_CUDA;
    }
    return ARK_OK;
}

constexpr int kT = 256;

// ------------------------------------------------------------ AdamW kernels
template <typename WT>
struct WTraits;
template <>
struct WTraits<uint16_t> {
    static __device__ __forceinline__ float load(const uint16_t* p, uint64_t i) { return h2f(p[i]); }
    static __device__ __forceinline__ void store(uint16_t* p, uint64_t i, float x) { p[i] = f2h(x); }
};
template <>
struct WTraits<float> {
    static __device__ __forceinline__ float load(const float* p, uint64_t i) { return p[i]; }
    static __device__ __forceinline__ void store(float* p, uint64_t i, float x) { p[i] = x; }
};

struct AdamArgs {
    uint64_t n;
    float lr, b1, b2, eps, wd;
    uint32_t t;
};

// Vector path: 4 elements per item (g, m, v as float4; w as 4 halves or a float4).
template <typename WT>
__global__ void __launch_bounds__(kT) adam_vec_kernel(WT* __restrict__ w, const float* __restrict__ g,
                                                     float* __restrict__ m, float* __restrict__ v,
                                                     AdamArgs a) {
    __shared__ AdamK s_k;
    if (threadIdx.x == 0) s_k = adam_scalars(a.lr, a.b1, a.b2, a.eps, a.wd, a.t);
    __syncthreads();
    const AdamK k = s_k;
    const uint64_t nq = a.n >> 2;
    const uint64_t stride = (uint64_t)gridDim.x * kT;
    const float4* g4 = reinterpret_cast<const float4*>(g);
    float4* m4 = reinterpret_cast<float4*>(m);
    float4* v4 = reinterpret_cast<float4*>(v);
    for (uint64_t i = (uint64_t)blockIdx.x * kT + threadIdx.x; i < nq; i += stride) {
        const float4 gg = ld_stream(g4 + i);
        float4 mm = ld_stream(m4 + i);
        float4 vv = ld_stream(v4 + i);
        float wf[4];
        if constexpr (sizeof(WT) == 2) {
            const uint2 wq = __ldcs(reinterpret_cast<const uint2*>(w) + i);
            wf[0] = h2f(lo16(wq.x)); wf[1] = h2f(hi16(wq.x));
            wf[2] = h2f(lo16(wq.y)); wf[3] = h2f(hi16(wq.y));
        } else {
            const float4 wq = ld_stream(reinterpret_cast<const float4*>(w) + i);
            wf[0] = wq.x; wf[1] = wq.y; wf[2] = wq.z; wf[3] = wq.w;
        }
        wf[0] = adam_elem(wf[0], gg.x, mm.x, vv.x, k, k.decay);
        wf[1] = adam_elem(wf[1], gg.y, mm.y, vv.y, k, k.decay);
        wf[2] = adam_elem(wf[2], gg.z, mm.z, vv.z, k, k.decay);
        wf[3] = adam_elem(wf[3], gg.w, mm.w, vv.w, k, k.decay);
        st_stream(m4 + i, mm);
        st_stream(v4 + i, vv);
        if constexpr (sizeof(WT) == 2) {
            uint2 o;
            o.x = pack16(f2h(wf[0]), f2h(wf[1]));
            o.y = pack16(f2h(wf[2]), f2h(wf[3]));
            __stcs(reinterpret_cast<uint2*>(w) + i, o);
        } else {
            st_stream(reinterpret_cast<float4*>(w) + i, make_float4(wf[0], wf[1], wf[2], wf[3]));
        }
    }
    // ragged tail (n % 4): same arithmetic as the reference's scalar tail
    if (blockIdx.x == 0 && threadIdx.x < (a.n & 3u)) {
        const uint64_t i = (nq << 2) + threadIdx.x;
        float mi = m[i], vi = v[i];
        const float wn = adam_elem(WTraits<WT>::load(w, i), g[i], mi, vi, k, k.decay);
        m[i] = mi;
        v[i] = vi;
        WTraits<WT>::store(w, i, wn);
    }
}

// Main vector path (every pointer 16-byte aligned): 8-element groups, U of
// them per thread per round, every load of a round issued before the first
// update -- g, m, v as two float4 each and w as one 16-byte vector of halves
// (or two float4).  Launch bounds keep it at <= 128 registers (2 blocks of
// 256 per SM), the shape of the fused step's update kernel.
template <typename WT, int U>
__global__ void __launch_bounds__(kT, 2) adam_vec8_kernel(WT* __restrict__ w,
                                                         const float* __restrict__ g,
                                                         float* __restrict__ m,
                                                         float* __restrict__ v, AdamArgs a) {
    __shared__ AdamK s_k;
    if (threadIdx.x == 0) s_k = adam_scalars(a.lr, a.b1, a.b2, a.eps, a.wd, a.t);
    __syncthreads();
    const AdamK k = s_k;
    const uint64_t n8 = a.n >> 3;
    const uint64_t stride = (uint64_t)gridDim.x * kT;
    const float4* g4 = reinterpret_cast<const float4*>(g);
    float4* m4 = reinterpret_cast<float4*>(m);
    float4* v4 = reinterpret_cast<float4*>(v);
    for (uint64_t base = (uint64_t)blockIdx.x * kT + threadIdx.x; base < n8;
         base += stride * U) {
        float4 gq[U][2], mq[U][2], vq[U][2], wq[U][2];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const uint64_t i = base + u * stride;
            if (i < n8) {
                gq[u][0] = ld_stream(g4 + 2 * i);
                gq[u][1] = ld_stream(g4 + 2 * i + 1);
                mq[u][0] = ld_stream(m4 + 2 * i);
                mq[u][1] = ld_stream(m4 + 2 * i + 1);
                vq[u][0] = ld_stream(v4 + 2 * i);
                vq[u][1] = ld_stream(v4 + 2 * i + 1);
                if constexpr (sizeof(WT) == 2) {
                    const uint4 h = ld_stream(reinterpret_cast<const uint4*>(w) + i);
                    wq[u][0] = make_float4(h2f(lo16(h.x)), h2f(hi16(h.x)), h2f(lo16(h.y)),
                                           h2f(hi16(h.y)));
                    wq[u][1] = make_float4(h2f(lo16(h.z)), h2f(hi16(h.z)), h2f(lo16(h.w)),
                                           h2f(hi16(h.w)));
                } else {
                    wq[u][0] = ld_stream(reinterpret_cast<const float4*>(w) + 2 * i);
                    wq[u][1] = ld_stream(reinterpret_cast<const float4*>(w) + 2 * i + 1);
                }
            }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const uint64_t i = base + u * stride;
            if (i >= n8) continue;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                float4& ww = wq[u][h];
                float4& mm = mq[u][h];
                float4& vv = vq[u][h];
                const float4 gg = gq[u][h];
                ww.x = adam_elem(ww.x, gg.x, mm.x, vv.x, k, k.decay);
                ww.y = adam_elem(ww.y, gg.y, mm.y, vv.y, k, k.decay);
                ww.z = adam_elem(ww.z, gg.z, mm.z, vv.z, k, k.decay);
                ww.w = adam_elem(ww.w, gg.w, mm.w, vv.w, k, k.decay);
                st_stream(m4 + 2 * i + h, mm);
                st_stream(v4 + 2 * i + h, vv);
            }
            if constexpr (sizeof(WT) == 2) {
                uint4 o;
                o.x = pack16(f2h(wq[u][0].x), f2h(wq[u][0].y));
                o.y = pack16(f2h(wq[u][0].z), f2h(wq[u][0].w));
                o.z = pack16(f2h(wq[u][1].x), f2h(wq[u][1].y));
                o.w = pack16(f2h(wq[u][1].z), f2h(wq[u][1].w));
                st_stream(reinterpret_cast<uint4*>(w) + i, o);
            } else {
                st_stream(reinterpret_cast<float4*>(w) + 2 * i, wq[u][0]);
                st_stream(reinterpret_cast<float4*>(w) + 2 * i + 1, wq[u][1]);
            }
        }
    }
    // ragged tail (n % 8): the reference's scalar tail arithmetic
    if (blockIdx.x == 0 && threadIdx.x < (a.n & 7u)) {
        const uint64_t i = (n8 << 3) + threadIdx.x;
        float mi = m[i], vi = v[i];
        const float wn = adam_elem(WTraits<WT>::load(w, i), g[i], mi, vi, k, k.decay);
        m[i] = mi;
        v[i] = vi;
        WTraits<WT>::store(w, i, wn);
    }
}

// Scalar path for arbitrarily aligned pointers.
template <typename WT>
__global__ void __launch_bounds__(kT) adam_scalar_kernel(WT* w, const float* g, float* m, float* v,
                                                        AdamArgs a) {
    __shared__ AdamK s_k;
    if (threadIdx.x == 0) s_k = adam_scalars(a.lr, a.b1, a.b2, a.eps, a.wd, a.t);
    __syncthreads();
    const AdamK k = s_k;
    const uint64_t stride = (uint64_t)gridDim.x * kT;
    for (uint64_t i = (uint64_t)blockIdx.x * kT + threadIdx.x; i < a.n; i += stride) {
        float mi = m[i], vi = v[i];
        const float wn = adam_elem(WTraits<WT>::load(w, i), g[i], mi, vi, k, k.decay);
        m[i] = mi;
        v[i] = vi;
        WTraits<WT>::store(w, i, wn);
    }
}

template <typename WT>
static int adam_launch(WT* w, const float* g, float* m, float* v, uint64_t n, float lr, float b1,
                       float b2, float eps, float wd, uint32_t t) {
    if (n == 0) return ARK_OK;                                  // opti.s:314-315 (n=0: no work)
    if (!w || !g || !m || !v) return ARK_E_INVALID_ARG;
    LegacyCtx* c = nullptr;
    int rc = current_ctx(&c);
    if (rc) return rc;
    AdamArgs a{n, lr, b1, b2, eps, wd, t};
    cudaStream_t s = legacy_stream(c);
    const bool gmv16 = aligned16(g) && aligned16(m) && aligned16(v);
    bool launched = false;
    if (gmv16 && aligned16(w)) {
        constexpr int U = 2;
        const int blocks = streaming_grid(reinterpret_cast<const void*>(adam_vec8_kernel<WT, U>),
                                          kT, 0, (n >> 3) / U + 1);
        adam_vec8_kernel<WT, U><<<blocks, kT, 0, s>>>(w, g, m, v, a);
        launched = true;
    }
    if constexpr (sizeof(WT) == 2) {   // FP16 weights 8- but not 16-byte aligned
        if (!launched && gmv16 && (reinterpret_cast<uintptr_t>(w) & 7u) == 0) {
            const int blocks = streaming_grid(reinterpret_cast<const void*>(adam_vec_kernel<WT>),
                                              kT, 0, (n >> 2) + 1);
            adam_vec_kernel<WT><<<blocks, kT, 0, s>>>(w, g, m, v, a);
            launched = true;
        }
    }
    if (!launched) {
        const int blocks = streaming_grid(reinterpret_cast<const void*>(adam_scalar_kernel<WT>), kT,
                                          0, n);
        adam_scalar_kernel<WT><<<blocks, kT, 0, s>>>(w, g, m, v, a);
    }
    return finish(c);
}

// ------------------------------------------------------------ grad clip
// Pass A: per-block sum of squares in double; the last block turns it into
// {norm, scale, apply}.  Pass B: in-place scale when apply.
struct ClipScratch {
    double* blk;
    unsigned int* ticket;
    ClipResult* res;
};

constexpr int kClipU = 4;   // float4 loads in flight per thread (norm and scale kernels)

__global__ void __launch_bounds__(kT) clip_norm_kernel(const float* __restrict__ g, uint64_t n,
                                                      float thr, ClipScratch sc) {
    __shared__ double s_sum[kT / 32];
    __shared__ int s_last;
    griddep_launch_dependents();   // the scale kernel may start loading g
    double acc = 0.0, acc1 = 0.0;
    const uint64_t stride = (uint64_t)gridDim.x * kT;
    if (aligned16(g)) {
        // rounds of kClipU float4 loads per thread, all issued before any is
        // squared; two accumulators halve the dependent chain of double FMAs
        const uint64_t nq = n >> 2;
        const float4* g4 = reinterpret_cast<const float4*>(g);
        for (uint64_t base = (uint64_t)blockIdx.x * kT + threadIdx.x; base < nq;
             base += stride * kClipU) {
            float4 x[kClipU];
#pragma unroll
            for (int u = 0; u < kClipU; ++u) {
                const uint64_t i = base + u * stride;
                x[u] = i < nq ? __ldcg(g4 + i) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int u = 0; u < kClipU; ++u) {
                acc = __fma_rn((double)x[u].x, (double)x[u].x, acc);
                acc1 = __fma_rn((double)x[u].y, (double)x[u].y, acc1);
                acc = __fma_rn((double)x[u].z, (double)x[u].z, acc);
                acc1 = __fma_rn((double)x[u].w, (double)x[u].w, acc1);
            }
        }
        acc += acc1;
        if (blockIdx.x == 0 && threadIdx.x < (n & 3u)) {
            const double x = g[(nq << 2) + threadIdx.x];
            acc = __fma_rn(x, x, acc);
        }
    } else {
        for (uint64_t i = (uint64_t)blockIdx.x * kT + threadIdx.x; i < n; i += stride) {
            const double x = g[i];
            acc = __fma_rn(x, x, acc);
        }
    }
    const double b = block_sum<kT>(acc, s_sum);
    if (threadIdx.x == 0) sc.blk[blockIdx.x] = b;
    if (!last_block_arrived(sc.ticket, &s_last)) return;
    double a = 0.0;
    for (unsigned int i = threadIdx.x; i < gridDim.x; i += kT) a += __ldcg(sc.blk + i);
    a = block_sum<kT>(a, s_sum);
    if (threadIdx.x == 0) {
        const float norm = __double2float_rn(__dsqrt_rn(a));
        const int apply = norm > thr;                     // opti.s:402-403 (unordered: no scale)
        sc.res->norm = norm;
        sc.res->apply = apply;
        sc.res->scale = apply ? __fdiv_rn(thr, norm) : 1.0f;  // opti.s:405
    }
}

// ARK_COMPAT_CLIP_NEON_FOLD: the reference's exact accumulation order --
// four f32 lanes, lane l folding fma(x,x,acc) over i = 4k+l (opti.s:383-389),
// (a0+a1)+(a2+a3) (:391-392), then the sequential tail (:393-398).  One warp;
// the fold is serial by definition.
__global__ void clip_neon_fold_kernel(const float* __restrict__ g, uint64_t n, float thr,
                                      ClipResult* res) {
    const int lane = threadIdx.x;
    float acc = 0.0f;
    const uint64_t n4 = n & ~uint64_t(3);
    if (lane < 4)
        for (uint64_t i = lane; i < n4; i += 4) acc = __fmaf_rn(g[i], g[i], acc);
    const float a1 = __shfl_sync(0xFFFFFFFFu, acc, 1);
    const float a2 = __shfl_sync(0xFFFFFFFFu, acc, 2);
    const float a3 = __shfl_sync(0xFFFFFFFFu, acc, 3);
    if (lane == 0) {
        float s = __fadd_rn(__fadd_rn(acc, a1), __fadd_rn(a2, a3));
        for (uint64_t i = n4; i < n; ++i) s = __fmaf_rn(g[i], g[i], s);
        const float norm = __fsqrt_rn(s);
        const int apply = norm > thr;
        res->norm = norm;
        res->apply = apply;
        res->scale = apply ? __fdiv_rn(thr, norm) : 1.0f;
    }
}

// The scale pass, launched as a programmatic dependent of the norm kernel
// (or the compat fold kernel): its blocks start as the norm kernel's retire,
// load their first round of g (which the norm pass only reads), then wait
// for the norm pass's result.  It walks g in reverse so that the first
// lines it touches are the last ones the norm pass read, still in L2.
// `res` is written by the kernel this one overlaps: it is read only after
// griddep_wait, through a volatile pointer (a const __restrict__ pointer
// would let the compiler treat it as unchanging and load it early).
__global__ void __launch_bounds__(kT) clip_scale_kernel(float* __restrict__ g, uint64_t n,
                                                       const ClipResult* res_ptr) {
    const volatile ClipResult* res = res_ptr;
    const uint64_t stride = (uint64_t)gridDim.x * kT;
    if (aligned16(g)) {
        const uint64_t nq = n >> 2;
        float4* g4 = reinterpret_cast<float4*>(g);
        uint64_t base = (uint64_t)blockIdx.x * kT + threadIdx.x;
        float4 x[kClipU];
#pragma unroll
        for (int u = 0; u < kClipU; ++u) {
            const uint64_t j = base + u * stride;
            if (j < nq) x[u] = ld_stream(g4 + (nq - 1 - j));
        }
        griddep_wait();
        if (!res->apply) return;
        const float s = res->scale;
        while (base < nq) {
#pragma unroll
            for (int u = 0; u < kClipU; ++u) {
                const uint64_t j = base + u * stride;
                if (j >= nq) continue;
                x[u].x = __fmul_rn(x[u].x, s);
                x[u].y = __fmul_rn(x[u].y, s);
                x[u].z = __fmul_rn(x[u].z, s);
                x[u].w = __fmul_rn(x[u].w, s);
                st_stream(g4 + (nq - 1 - j), x[u]);
            }
            base += stride * kClipU;
            if (base >= nq) break;
#pragma unroll
            for (int u = 0; u < kClipU; ++u) {
                const uint64_t j = base + u * stride;
                if (j < nq) x[u] = ld_stream(g4 + (nq - 1 - j));
            }
        }
        if (blockIdx.x == 0 && threadIdx.x < (n & 3u)) {
            const uint64_t i = (nq << 2) + threadIdx.x;
            g[i] = __fmul_rn(g[i], s);
        }
    } else {
        griddep_wait();
        if (!res->apply) return;
        const float s = res->scale;
        for (uint64_t i = (uint64_t)blockIdx.x * kT + threadIdx.x; i < n; i += stride)
            g[i] = __fmul_rn(g[i], s);
    }
}

// The scale pass as a programmatic dependent of the kernel before it.
static cudaError_t launch_clip_scale(int blocks, cudaStream_t s, float* g, uint64_t n,
                                     const ClipResult* res) {
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t lc = {};
    lc.gridDim = dim3((unsigned)blocks);
    lc.blockDim = dim3(kT);
    lc.stream = s;
    lc.attrs = attr;
    lc.numAttrs = 1;
    return cudaLaunchKernelEx(&lc, clip_scale_kernel, g, n, res);
}

// Grids of the two clip kernels (norm, scale) for n elements: one
// definition for the allocating and the allocation-free entry points, whose
// norms must agree bit for bit (the double sum's order depends on the grid).
static void clip_grids(uint64_t n, int* norm_blocks, int* scale_blocks) {
    *norm_blocks = streaming_grid(reinterpret_cast<const void*>(clip_norm_kernel), kT, 0,
                                  (n >> 2) / kClipU + 1);
    *scale_blocks = streaming_grid(reinterpret_cast<const void*>(clip_scale_kernel), kT, 0,
                                   (n >> 2) / kClipU + 1);
}

static int clip_scratch(LegacyCtx* c, int blocks, ClipScratch* sc) {
    std::lock_guard<std::mutex> lk(c->mu);
    if (!c->scratch || c->scratch_blocks < blocks) {
        if (c->scratch) {
            cudaStreamSynchronize(legacy_stream(c));
            cudaFree(c->scratch);
            c->scratch = nullptr;
        }
        const size_t bytes = 256 + 256 + sizeof(double) * (size_t)blocks;
        if (cudaMalloc(&c->scratch, bytes) != cudaSuccess) return ARK_E_CUDA;
        if (cudaMemset(c->scratch, 0, bytes) != cudaSuccess) return ARK_E_CUDA;
        c->scratch_blocks = blocks;
    }
    char* b = static_cast<char*>(c->scratch);
    sc->ticket = reinterpret_cast<unsigned int*>(b);
    sc->res = reinterpret_cast<ClipResult*>(b + 256);
    sc->blk = reinterpret_cast<double*>(b + 512);
    return ARK_OK;
}

static int clip_launch(float* g, uint64_t n, float thr, float* norm_out) {
    *norm_out = 0.0f;
    if (n == 0) return ARK_OK;        // empty: norm 0, no scale
    if (!g) return ARK_E_INVALID_ARG;
    LegacyCtx* c = nullptr;
    int rc = current_ctx(&c);
    if (rc) return rc;
    cudaStream_t s = legacy_stream(c);
    int blocks = 0, sblocks = 0;
    clip_grids(n, &blocks, &sblocks);
    ClipScratch sc;
    rc = clip_scratch(c, blocks, &sc);
    if (rc) return rc;
    if (g_compat.load() & ARK_COMPAT_CLIP_NEON_FOLD)
        clip_neon_fold_kernel<<<1, 32, 0, s>>>(g, n, thr, sc.res);
    else
        clip_norm_kernel<<<blocks, kT, 0, s>>>(g, n, thr, sc);
    if (launch_clip_scale(sblocks, s, g, n, sc.res) != cudaSuccess) return ARK_E_CUDA;
    if (cudaGetLastError() != cudaSuccess) return ARK_E_CUDA;
    ClipResult r;
    // the norm is the return value: this entry point always waits
    if (cudaMemcpyAsync(&r, sc.res, sizeof(r), cudaMemcpyDeviceToHost, s) != cudaSuccess)
        return ARK_E_CUDA;
    if (cudaStreamSynchronize(s) != cudaSuccess) return ARK_E_CUDA;
    *norm_out = r.norm;
    return ARK_OK;
}

// ------------------------------------------------------------ grad clip, no allocation
// Scratch of ark_cuda_grad_clip_noalloc, in the module image instead of a
// cudaMalloc'd buffer: bytes [0, 256) hold the last-block ticket, [256, 512)
// the {norm, scale, apply} result, then one double partial per thread block.
// Every GPU that loads this library holds these 16.5 KiB until the process
// exits.  All calls share it.
constexpr int kNoAllocMaxBlocks = 2048;
constexpr size_t kNoAllocScratchBytes = 512 + sizeof(double) * kNoAllocMaxBlocks;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

static std::mutex g_noalloc_mu;
static void* g_noalloc_addr[64];   // device address of g_noalloc_scratch, per device

// Set-up, once per device, with that device current: the host-side name of a
// __device__ array is only a stand-in, so its device address is looked up.
static int noalloc_scratch(int dev, ClipScratch* sc) {
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_addr[dev]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) {
            fprintf(stderr, "[ark_cuda] ark_cuda_grad_clip_noalloc: cudaGetSymbolAddress: %s\n",
                    cudaGetErrorString(e));
            return ARK_E_CUDA;
        }
        g_noalloc_addr[dev] = p;
    }
    char* b = static_cast<char*>(g_noalloc_addr[dev]);
    sc->ticket = reinterpret_cast<unsigned int*>(b);
    sc->res = reinterpret_cast<ClipResult*>(b + 256);
    sc->blk = reinterpret_cast<double*>(b + 512);
    return ARK_OK;
}

static int clip_noalloc_launch(float* g, uint64_t n, float thr, float* norm_dev,
                               cudaStream_t s) {
    if (!norm_dev || (n && !g)) return ARK_E_INVALID_ARG;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return ARK_E_NO_DEVICE;
    ClipScratch sc;
    int rc = noalloc_scratch(dev, &sc);
    if (rc) return rc;
    if (n == 0)   // empty: norm 0, nothing to scale (as ark_asm_grad_clip)
        return cudaMemsetAsync(norm_dev, 0, sizeof(float), s) == cudaSuccess ? ARK_OK : ARK_E_CUDA;
    // the same grids and kernels as ark_asm_grad_clip (the compat flag
    // included), so both give the same norm bit for bit
    int blocks = 0, sblocks = 0;
    clip_grids(n, &blocks, &sblocks);
    if (g_compat.load() & ARK_COMPAT_CLIP_NEON_FOLD) {
        clip_neon_fold_kernel<<<1, 32, 0, s>>>(g, n, thr, sc.res);   // no block partials
    } else {
        if (blocks > kNoAllocMaxBlocks) {
            fprintf(stderr,
                    "[ark_cuda] ark_cuda_grad_clip_noalloc: needs %d block partials, the static "
                    "scratch holds %d\n", blocks, kNoAllocMaxBlocks);
            return ARK_E_UNSUPPORTED;
        }
        // the ticket must start at zero; a call that stopped early could have left it set
        if (cudaMemsetAsync(sc.ticket, 0, sizeof(unsigned int), s) != cudaSuccess)
            return ARK_E_CUDA;
        clip_norm_kernel<<<blocks, kT, 0, s>>>(g, n, thr, sc);
    }
    if (launch_clip_scale(sblocks, s, g, n, sc.res) != cudaSuccess) return ARK_E_CUDA;
    if (cudaGetLastError() != cudaSuccess) return ARK_E_CUDA;
    if (cudaMemcpyAsync(norm_dev, &sc.res->norm, sizeof(float), cudaMemcpyDeviceToDevice, s) !=
        cudaSuccess)
        return ARK_E_CUDA;
    return ARK_OK;
}

// ------------------------------------------------------------ conversions
constexpr int kConvU = 2;   // quant: 8-element vectors in flight per thread
// dequant (2 B read, 4 B written per element): one vector per thread per
// iteration at 5 blocks of 256 per SM measured fastest on B200 (2^27
// elements: 6.24 TB/s; 2 in flight at 4 blocks/SM 4.80, at 3 blocks/SM 6.21;
// one at 4 or 6 blocks/SM 5.85 / 4.83)
constexpr int kDeqU = 1;
constexpr int kDeqBlocksPerSM = 5;
__global__ void __launch_bounds__(kT) quant_kernel(const float* __restrict__ src,
                                                  uint16_t* __restrict__ dst, uint64_t n, int vec) {
    const uint64_t stride = (uint64_t)gridDim.x * kT;
    uint64_t done = 0;
    if (vec) {
        const uint64_t n8 = n >> 3;
        const float4* s4 = reinterpret_cast<const float4*>(src);
        uint4* d4 = reinterpret_cast<uint4*>(dst);
        for (uint64_t base = (uint64_t)blockIdx.x * kT + threadIdx.x; base < n8;
             base += stride * kConvU) {
            float4 a[kConvU], b[kConvU];
#pragma unroll
            for (int u = 0; u < kConvU; ++u) {
                const uint64_t i = base + u * stride;
                if (i < n8) {
                    a[u] = ld_stream(s4 + 2 * i);
                    b[u] = ld_stream(s4 + 2 * i + 1);
                }
            }
#pragma unroll
            for (int u = 0; u < kConvU; ++u) {
                const uint64_t i = base + u * stride;
                if (i >= n8) continue;
                uint4 o;
                o.x = pack16(f2h(a[u].x), f2h(a[u].y));
                o.y = pack16(f2h(a[u].z), f2h(a[u].w));
                o.z = pack16(f2h(b[u].x), f2h(b[u].y));
                o.w = pack16(f2h(b[u].z), f2h(b[u].w));
                st_stream(d4 + i, o);
            }
        }
        done = n8 << 3;
    }
    for (uint64_t i = done + (uint64_t)blockIdx.x * kT + threadIdx.x; i < n; i += stride)
        dst[i] = f2h(src[i]);
}

__global__ void __launch_bounds__(kT) dequant_kernel(const uint16_t* __restrict__ src,
                                                    float* __restrict__ dst, uint64_t n, int vec) {
    const uint64_t stride = (uint64_t)gridDim.x * kT;
    uint64_t done = 0;
    if (vec) {
        const uint64_t n8 = n >> 3;
        const uint4* s4 = reinterpret_cast<const uint4*>(src);
        float4* d4 = reinterpret_cast<float4*>(dst);
        for (uint64_t base = (uint64_t)blockIdx.x * kT + threadIdx.x; base < n8;
             base += stride * kDeqU) {
            uint4 q[kDeqU];
#pragma unroll
            for (int u = 0; u < kDeqU; ++u) {
                const uint64_t i = base + u * stride;
                if (i < n8) q[u] = ld_stream(s4 + i);
            }
#pragma unroll
            for (int u = 0; u < kDeqU; ++u) {
                const uint64_t i = base + u * stride;
                if (i >= n8) continue;
                st_stream(d4 + 2 * i, make_float4(h2f(lo16(q[u].x)), h2f(hi16(q[u].x)),
                                                  h2f(lo16(q[u].y)), h2f(hi16(q[u].y))));
                st_stream(d4 + 2 * i + 1, make_float4(h2f(lo16(q[u].z)), h2f(hi16(q[u].z)),
                                                      h2f(lo16(q[u].w)), h2f(hi16(q[u].w))));
            }
        }
        done = n8 << 3;
    }
    for (uint64_t i = done + (uint64_t)blockIdx.x * kT + threadIdx.x; i < n; i += stride)
        dst[i] = h2f(src[i]);
}

static int convert_launch(const void* src, void* dst, uint64_t n, bool quant) {
    if (n == 0) return ARK_OK;
    if (!src || !dst) return ARK_E_INVALID_ARG;
    LegacyCtx* c = nullptr;
    int rc = current_ctx(&c);
    if (rc) return rc;
    const int vec = aligned16(src) && aligned16(dst);
    cudaStream_t s = legacy_stream(c);
    if (quant) {
        const int blocks = streaming_grid(reinterpret_cast<const void*>(quant_kernel), kT, 0,
                                          vec ? (n >> 3) / kConvU + 1 : n);
        quant_kernel<<<blocks, kT, 0, s>>>(static_cast<const float*>(src),
                                            static_cast<uint16_t*>(dst), n, vec);
    } else {
        int blocks = streaming_grid(reinterpret_cast<const void*>(dequant_kernel), kT, 0,
                                    vec ? (n >> 3) / kDeqU + 1 : n);
        const int cap = sm_count() * kDeqBlocksPerSM;
        if (blocks > cap) blocks = cap;
        dequant_kernel<<<blocks, kT, 0, s>>>(static_cast<const uint16_t*>(src),
                                              static_cast<float*>(dst), n, vec);
    }
    return finish(c);
}

}  // namespace ark

using namespace ark;

extern "C" {

void ark_asm_adam_step_f16(uint16_t* w, const float* g, float* m, float* v, uint64_t n, float lr,
                           float beta1, float beta2, float eps, float wd, uint32_t t) {
    const int rc = adam_launch<uint16_t>(w, g, m, v, n, lr, beta1, beta2, eps, wd, t);
    if (rc) legacy_fail("ark_asm_adam_step_f16", rc, nullptr); else set_last_error(ARK_OK);
}

void ark_asm_adam_step(float* w, const float* g, float* m, float* v, uint64_t n, float lr,
                       float beta1, float beta2, float eps, float wd, uint32_t t) {
    const int rc = adam_launch<float>(w, g, m, v, n, lr, beta1, beta2, eps, wd, t);
    if (rc) legacy_fail("ark_asm_adam_step", rc, nullptr); else set_last_error(ARK_OK);
}

float ark_asm_grad_clip(float* grads, uint64_t n, float threshold) {
    float norm = 0.0f;
    const int rc = clip_launch(grads, n, threshold, &norm);
    if (rc) {
        legacy_fail("ark_asm_grad_clip", rc, nullptr);
        return __builtin_nanf("");
    }
    set_last_error(ARK_OK);
    return norm;
}

void ark_quant_f32_to_f16(const float* src, uint16_t* dst, uint64_t n) {
    const int rc = convert_launch(src, dst, n, true);
    if (rc) legacy_fail("ark_quant_f32_to_f16", rc, nullptr); else set_last_error(ARK_OK);
}

void ark_dequant_f16_to_f32(const uint16_t* src, float* dst, uint64_t n) {
    const int rc = convert_launch(src, dst, n, false);
    if (rc) legacy_fail("ark_dequant_f16_to_f32", rc, nullptr); else set_last_error(ARK_OK);
}

int ark_cuda_grad_clip_noalloc(float* grads, uint64_t n, float threshold, float* norm_out,
                               void* cuda_stream) {
    return clip_noalloc_launch(grads, n, threshold, norm_out,
                               reinterpret_cast<cudaStream_t>(cuda_stream));
}

int ark_cuda_last_error(void) { return t_last_error; }

const char* ark_cuda_strerror(int status) { return status_string(status); }

int ark_cuda_set_compat(uint32_t flags) {
    if (flags & ~ARK_COMPAT_CLIP_NEON_FOLD) return ARK_E_INVALID_ARG;
    g_compat.store(flags);
    return ARK_OK;
}

int ark_cuda_legacy_set_stream(void* stream) {
    g_stream.store(reinterpret_cast<cudaStream_t>(stream));
    return ARK_OK;
}

int ark_cuda_legacy_set_async(int async) {
    g_async.store(async ? 1 : 0);
    return ARK_OK;
}

int ark_cuda_legacy_sync(void) {
    LegacyCtx* c = nullptr;
    int rc = current_ctx(&c);
    if (rc) return rc;
    return cudaStreamSynchronize(legacy_stream(c)) == cudaSuccess ? ARK_OK : ARK_E_CUDA;
}

uint32_t ark_cuda_abi_version(void) { return ARK_OPT_ABI_VERSION; }

}  // extern "C"
