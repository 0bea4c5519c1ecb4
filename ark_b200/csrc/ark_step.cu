// ark_step.cu -- the fused optimizer step for one flat ZeRO-1 shard.
//
// One step = two streaming kernels (plus one 16-byte NCCL all-gather per
// rank when the optimizer state is sharded over several GPUs):
//
//   pass 1  reads the FP16 loss-scaled gradients once (2 B/param): counts
//           non-finite values (training.rs:291) and accumulates the sum of
//           squares of the UNSCALED gradient (training.rs:308 then
//           optimizer.rs:126-145) in double; per-block partials are reduced
//           in a fixed order by the last block to finish.
//   [all-gather of {sumsq, nonfinite} over ranks -- rank order, deterministic]
//   pass 2  every block derives the step plan from device memory (no host
//           sync): skip on overflow (training.rs:293-305), else t = step+1,
//           lr(t), clip coefficient (optimizer.rs:145-149), AdamW scalars
//           (opti.s:210-271).  Then the fused element update (20 B/param):
//           g = fp16(g) * inv_scale * clip ; m, v, w as opti.s:285-308.  The
//           last block to finish advances the loss-scale state machine
//           (training.rs:316-326) in device memory.
#include <cuda_runtime.h>
#include <nccl.h>
#include <stdlib.h>
#include <string.h>

#include <vector>

#include "ark_device.cuh"
#include "ark_fused.cuh"
#include "ark_internal.h"

namespace ark {

// Device state: identical layout to ark_opt_status so a status read is one
// 64-byte copy.
static_assert(sizeof(ark_opt_status) == 64, "status layout");

// Per-rank pass-1 result exchanged between ranks (16 bytes).
struct Partial {
    double sumsq;
    unsigned long long nonfinite;
};

struct StepParams {
    const uint16_t* g16;
    uint64_t n;          // shard elements
    uint64_t offset;     // global index of element 0
    uint64_t n_decay;
    uint64_t keep_lo, keep_hi;
    ark_opt_status* st;  // device state
    const float* lr_table;
    uint32_t lr_len;
    float beta1, beta2, eps, wd, clip;
    float scale_backoff, scale_growth, scale_min, scale_max;
    uint32_t scale_every, max_nans;
    int world;
    double* blk_sum;                 // pass-1 per-block partials
    unsigned long long* blk_bad;
    unsigned int* ticket1;
    unsigned int* ticket2;
    Partial* part_local;             // this rank's partial (all-gather send buffer)
    const Partial* part_all;         // [world] gathered partials
};

constexpr int kThreads = 256;
constexpr int kUnroll1 = 4;   // 16-byte gradient vectors in flight per thread, pass 1
constexpr int kUnroll2 = 2;   // 8-element groups in flight per thread, pass 2

// --------------------------------------------------------------- pass 1
// Exact FP16 -> FP64 widening (one conversion instruction).
__device__ __forceinline__ double h2d(uint16_t h) {
    double d;
    asm("cvt.f64.f16 %0, %1;" : "=d"(d) : "h"(h));
    return d;
}

// Max of |h| over the packed halves seen so far (SIMD on 2 x 16 bits); a
// value >= 0x7C00 in either half means an inf or NaN was present.
__device__ __forceinline__ uint32_t absmax2(uint32_t acc, uint32_t w) {
    return __vmaxu2(acc, w & 0x7FFF7FFFu);
}

// General path: u = fp32(h) * inv rounded to f32, exactly as training.rs:308
// computes the unscaled gradient, then u*u accumulated in double.
__device__ __forceinline__ void accum8_general(uint4 q, uint64_t gi0, float inv, uint64_t keep_lo,
                                               uint64_t keep_hi, double& acc) {
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
    const bool keep_any = (gi0 + 8 > keep_lo) && (gi0 < keep_hi);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const uint16_t h = (j & 1) ? hi16(w[j >> 1]) : lo16(w[j >> 1]);
        const float f = h2f(h);
        const bool keep = keep_any && (gi0 + j >= keep_lo) && (gi0 + j < keep_hi);
        const float u = keep ? f : __fmul_rn(f, inv);
        const double d = (double)u;
        acc = __fma_rn(d, d, acc);
    }
}

// Power-of-two loss scale (the only kind the state machine produces from a
// power-of-two init, backoff and growth): fp32(h) * inv is exact, so the sum
// of squared unscaled gradients is inv^2 * sum(h^2), with h^2 exact in
// double.  Elements in the kept range (compat mode) go to acc_k unscaled.
__device__ __forceinline__ void accum8_pow2(uint4 q, uint64_t gi0, uint64_t keep_lo,
                                            uint64_t keep_hi, double& acc_s, double& acc_k) {
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
    if (gi0 + 8 > keep_lo && gi0 < keep_hi) {           // rare: straddles the kept range
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const double d = h2d((j & 1) ? hi16(w[j >> 1]) : lo16(w[j >> 1]));
            if (gi0 + j >= keep_lo && gi0 + j < keep_hi) acc_k = __fma_rn(d, d, acc_k);
            else acc_s = __fma_rn(d, d, acc_s);
        }
        return;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const double d = h2d((j & 1) ? hi16(w[j >> 1]) : lo16(w[j >> 1]));
        acc_s = __fma_rn(d, d, acc_s);
    }
}

__global__ void __launch_bounds__(kThreads) pass1_kernel(StepParams p) {
    __shared__ double s_sum[kThreads / 32];
    __shared__ unsigned long long s_bad[kThreads / 32];
    __shared__ int s_last;
    const float inv = __fdiv_rn(1.0f, p.st->loss_scale);   // training.rs:244
    const uint32_t ib = __float_as_uint(inv);
    const bool pow2 = (ib & 0x7FFFFFu) == 0 && (ib & 0x7F800000u) != 0 &&
                      (ib & 0x7F800000u) != 0x7F800000u;
    double acc_s = 0.0, acc_k = 0.0;
    uint32_t amax = 0;
    const uint4* g = reinterpret_cast<const uint4*>(p.g16);
    const uint64_t nvec = p.n >> 3;
    const uint64_t stride = (uint64_t)gridDim.x * kThreads;
    for (uint64_t base = (uint64_t)blockIdx.x * kThreads + threadIdx.x; base < nvec;
         base += stride * kUnroll1) {
        uint4 q[kUnroll1];
#pragma unroll
        for (int u = 0; u < kUnroll1; ++u) {
            const uint64_t i = base + u * stride;
            q[u] = i < nvec ? ld_keep(g + i) : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int u = 0; u < kUnroll1; ++u) {
            amax = absmax2(amax, q[u].x);
            amax = absmax2(amax, q[u].y);
            amax = absmax2(amax, q[u].z);
            amax = absmax2(amax, q[u].w);
            const uint64_t i = base + u * stride;
            if (i < nvec) {
                if (pow2) accum8_pow2(q[u], p.offset + (i << 3), p.keep_lo, p.keep_hi, acc_s, acc_k);
                else accum8_general(q[u], p.offset + (i << 3), inv, p.keep_lo, p.keep_hi, acc_s);
            }
        }
    }
    // ragged tail (n % 8 elements)
    if (blockIdx.x == 0 && threadIdx.x < (p.n & 7u)) {
        const uint64_t i = (nvec << 3) + threadIdx.x;
        const uint16_t h = p.g16[i];
        amax = absmax2(amax, h);
        const uint64_t gi = p.offset + i;
        const bool keep = gi >= p.keep_lo && gi < p.keep_hi;
        if (pow2) {
            const double d = h2d(h);
            if (keep) acc_k = __fma_rn(d, d, acc_k);
            else acc_s = __fma_rn(d, d, acc_s);
        } else {
            const float f = h2f(h);
            const double d = (double)(keep ? f : __fmul_rn(f, inv));
            acc_s = __fma_rn(d, d, acc_s);
        }
    }
    // fold the power-of-two scaling in per thread (exact): sum of u^2
    const double inv_d = (double)inv;
    const double acc = pow2 ? __fma_rn(acc_s, inv_d * inv_d, acc_k) : acc_s;
    const unsigned long long bad = ((amax & 0xFFFFu) >= 0x7C00u) || ((amax >> 16) >= 0x7C00u);
    const double bsum = block_sum<kThreads>(acc, s_sum);
    const unsigned long long bbad = block_sum_u64<kThreads>(bad, s_bad);
    if (threadIdx.x == 0) {
        p.blk_sum[blockIdx.x] = bsum;
        p.blk_bad[blockIdx.x] = bbad;
    }
    if (!last_block_arrived(p.ticket1, &s_last)) return;
    // Last block: fixed-order reduction of the per-block partials.
    double a = 0.0;
    unsigned long long b = 0;
    for (unsigned int i = threadIdx.x; i < gridDim.x; i += kThreads) {
        a += __ldcg(p.blk_sum + i);
        b += __ldcg(p.blk_bad + i);
    }
    a = block_sum<kThreads>(a, s_sum);
    b = block_sum_u64<kThreads>(b, s_bad);
    if (threadIdx.x == 0) {
        p.part_local->sumsq = a;
        p.part_local->nonfinite = b;   // threads that saw an inf/NaN (> 0 iff any)
    }
}

// --------------------------------------------------------------- pass 2
struct Plan {
    AdamK k;
    float inv, s, norm, lr;
    double sumsq;
    uint32_t t;
    int skip;       // overflow, early stop or error: no element work
    int clip;
    int overflow;
    int error;      // ARK_E_* raised while forming the plan (0 = none)
};

// The step plan from the device state and the global {sum, non-finite}.
__device__ void make_plan_from(const ark_opt_status& st, double sumsq, unsigned long long bad,
                               const StepParams& p, Plan& pl) {
    pl.sumsq = sumsq;
    pl.overflow = bad != 0;
    pl.error = 0;
    pl.skip = pl.overflow || st.early_stop;
    pl.inv = __fdiv_rn(1.0f, st.loss_scale);          // training.rs:244
    pl.t = st.opt_step + 1u;                          // optimizer.rs:172
    const uint32_t li = pl.t < p.lr_len ? pl.t : p.lr_len - 1u;
    pl.lr = p.lr_table[li];                           // optimizer.rs:173
    pl.norm = __double2float_rn(__dsqrt_rn(sumsq));   // optimizer.rs:145
    pl.clip = (pl.norm > p.clip) && (pl.norm > 0.0f); // optimizer.rs:148
    pl.s = pl.clip ? __fdiv_rn(p.clip, pl.norm) : 1.0f;
    pl.k = adam_scalars(pl.lr, p.beta1, p.beta2, p.eps, p.wd, pl.t);
}

__device__ void make_plan(const StepParams& p, Plan& pl) {
    const ark_opt_status st = *p.st;
    double sumsq = 0.0;
    unsigned long long bad = 0;
    for (int r = 0; r < p.world; ++r) {               // rank order: deterministic
        sumsq += p.part_all[r].sumsq;
        bad += p.part_all[r].nonfinite;
    }
    make_plan_from(st, sumsq, bad, p, pl);
}

// State machine update (training.rs:293-305 on overflow, :316-326 after a
// clean step); runs once per step in the last pass-2 block.
__device__ void advance_state(const StepParams& p, const Plan& pl) {
    ark_opt_status st = *p.st;
    st.steps_called += 1;
    if (pl.error) st.error = pl.error;
    if (st.early_stop || pl.error) {
        *p.st = st;
        return;
    }
    if (pl.overflow) {
        st.loss_scale = fmaxf(__fmul_rn(st.loss_scale, p.scale_backoff), p.scale_min);
        st.clean_steps = 0;
        st.skipped_steps += 1;
        st.consecutive_nans += 1;
        st.last_overflow = 1;
        if (st.consecutive_nans > p.max_nans) st.early_stop = 1;
    } else {
        st.opt_step = pl.t;
        st.last_overflow = 0;
        st.last_norm = pl.norm;
        st.last_sumsq = pl.sumsq;
        st.last_clip_coef = pl.s;
        st.last_lr = pl.lr;
        st.clean_steps += 1;
        st.consecutive_nans = 0;
        if (st.clean_steps >= p.scale_every) {
            const float nueva = fminf(__fmul_rn(st.loss_scale, p.scale_growth), p.scale_max);
            if (nueva > st.loss_scale) st.loss_scale = nueva;
            st.clean_steps = 0;
        }
    }
    *p.st = st;
}

__device__ __forceinline__ void update8(uint4& wq, const uint4 gq, float4& m0, float4& m1,
                                        float4& v0, float4& v1, uint64_t gi0, const Plan& pl,
                                        const StepParams& p) {
    const uint32_t gw[4] = {gq.x, gq.y, gq.z, gq.w};
    uint32_t ww[4] = {wq.x, wq.y, wq.z, wq.w};
    float mm[8] = {m0.x, m0.y, m0.z, m0.w, m1.x, m1.y, m1.z, m1.w};
    float vv[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
    const bool keep_any = (gi0 + 8 > p.keep_lo) && (gi0 < p.keep_hi);
    const bool dec_all = gi0 + 8 <= p.n_decay;
    const bool dec_none = gi0 >= p.n_decay;
    uint16_t wout[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const uint16_t gh = (j & 1) ? hi16(gw[j >> 1]) : lo16(gw[j >> 1]);
        const uint16_t wh = (j & 1) ? hi16(ww[j >> 1]) : lo16(ww[j >> 1]);
        float gf = h2f(gh);
        const bool keep = keep_any && (gi0 + j >= p.keep_lo) && (gi0 + j < p.keep_hi);
        if (!keep) gf = __fmul_rn(gf, pl.inv);                       // training.rs:308
        if (pl.clip) gf = __fmul_rn(gf, pl.s);                       // optimizer.rs:151-166
        const bool dec = dec_all || (!dec_none && gi0 + j < p.n_decay);
        const float decay = dec ? pl.k.decay : 1.0f;                 // wd = 0: 1 - lr*0
        wout[j] = f2h(adam_elem(h2f(wh), gf, mm[j], vv[j], pl.k, decay));
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) ww[i] = pack16(wout[2 * i], wout[2 * i + 1]);
    wq = make_uint4(ww[0], ww[1], ww[2], ww[3]);
    m0 = make_float4(mm[0], mm[1], mm[2], mm[3]);
    m1 = make_float4(mm[4], mm[5], mm[6], mm[7]);
    v0 = make_float4(vv[0], vv[1], vv[2], vv[3]);
    v1 = make_float4(vv[4], vv[5], vv[6], vv[7]);
}

__global__ void __launch_bounds__(kThreads) pass2_kernel(StepParams p, uint16_t* __restrict__ w16,
                                                        float* __restrict__ m,
                                                        float* __restrict__ v) {
    __shared__ Plan s_plan;
    __shared__ int s_last;
    if (threadIdx.x == 0) make_plan(p, s_plan);
    __syncthreads();
    const Plan pl = s_plan;
    if (!pl.skip) {
        const uint4* g4 = reinterpret_cast<const uint4*>(p.g16);
        uint4* w4 = reinterpret_cast<uint4*>(w16);
        float4* m4 = reinterpret_cast<float4*>(m);
        float4* v4 = reinterpret_cast<float4*>(v);
        const uint64_t nvec = p.n >> 3;
        const uint64_t stride = (uint64_t)gridDim.x * kThreads;
        for (uint64_t base = (uint64_t)blockIdx.x * kThreads + threadIdx.x; base < nvec;
             base += stride * kUnroll2) {
            uint4 gq[kUnroll2], wq[kUnroll2];
            float4 ma[kUnroll2], mb[kUnroll2], va[kUnroll2], vb[kUnroll2];
#pragma unroll
            for (int u = 0; u < kUnroll2; ++u) {
                const uint64_t i = base + u * stride;
                if (i < nvec) {
                    gq[u] = ld_stream(g4 + i);
                    wq[u] = ld_stream(w4 + i);
                    ma[u] = ld_stream(m4 + 2 * i);
                    mb[u] = ld_stream(m4 + 2 * i + 1);
                    va[u] = ld_stream(v4 + 2 * i);
                    vb[u] = ld_stream(v4 + 2 * i + 1);
                }
            }
#pragma unroll
            for (int u = 0; u < kUnroll2; ++u) {
                const uint64_t i = base + u * stride;
                if (i < nvec) {
                    update8(wq[u], gq[u], ma[u], mb[u], va[u], vb[u], p.offset + (i << 3), pl, p);
                    st_stream(w4 + i, wq[u]);
                    st_stream(m4 + 2 * i, ma[u]);
                    st_stream(m4 + 2 * i + 1, mb[u]);
                    st_stream(v4 + 2 * i, va[u]);
                    st_stream(v4 + 2 * i + 1, vb[u]);
                }
            }
        }
        if (blockIdx.x == 0 && threadIdx.x < (p.n & 7u)) {
            const uint64_t i = (nvec << 3) + threadIdx.x;
            const uint64_t gi = p.offset + i;
            float gf = h2f(p.g16[i]);
            if (!(gi >= p.keep_lo && gi < p.keep_hi)) gf = __fmul_rn(gf, pl.inv);
            if (pl.clip) gf = __fmul_rn(gf, pl.s);
            const float decay = gi < p.n_decay ? pl.k.decay : 1.0f;
            float mi = m[i], vi = v[i];
            w16[i] = f2h(adam_elem(h2f(w16[i]), gf, mi, vi, pl.k, decay));
            m[i] = mi;
            v[i] = vi;
        }
    }
    if (!last_block_arrived(p.ticket2, &s_last)) return;
    if (threadIdx.x == 0) advance_state(p, pl);
}

// ======================================================================
// The persistent single-kernel step (default when cooperative launch is
// available): every CTA of a co-resident grid owns a contiguous range of
// 2048-element tiles.  Phase 1 streams its gradients through a 4-stage
// shared-memory ring filled by 1-D bulk copies (TMA engine); a grid barrier
// (last-arriving CTA) reduces the CTA partials in a fixed order, exchanges
// the 16-byte rank partials with the peers over NVLink (P2P stores into
// their receive slots, world > 1) and publishes the plan; phase 2 walks the
// same tiles in reverse, so the gradient tiles read last in phase 1 are
// still in L2, with g, w, m, v brought in by bulk copies and w, m, v
// written back with streaming stores.  Every wait is bounded by the global
// timer; a timeout turns the step into a no-op and raises ARK_E_TIMEOUT in
// the device state.
// ======================================================================
constexpr int kFT = 256;                       // threads per CTA
constexpr int kStages = 4;
constexpr int kTile2Vec = kFT;                 // phase-2 tile: 256 x 8 = 2048 elements
constexpr int kTile1Vec = 4 * kFT;             // phase-1 tile: 1024 x 8 = 8192 elements (16 KB)
constexpr int kStage2Bytes = kTile2Vec * 8 * 12;   // g 4 KB | w 4 KB | m 8 KB | v 8 KB
constexpr int kStage1Bytes = kTile1Vec * 16;
constexpr int kFusedSmem = kStages * kStage2Bytes; // 96 KB, phase 1 uses the first 64 KB
constexpr int kMaxP2PRanks = 32;
static_assert(kStages * kStage1Bytes <= kFusedSmem, "phase-1 ring fits");

struct FusedParams {
    uint16_t* w16;
    float* m;
    float* v;
    Plan* plan;                     // published by the last CTA of phase 1
    uint64_t* release;              // == epoch once the plan is published
    unsigned int* arrive;           // phase-1 arrival counter
    unsigned int* err;              // CTA-local failures (bulk-copy wait timeouts)
    uint64_t* xchg;                 // this rank's receive slots [2][world][4] x u64
    uint64_t* const* peers;         // receive-slot bases of every rank (peers[rank] == xchg)
    int rank;
    int keep_g_in_l2;               // phase-1 gradient loads with L2 evict_last
    uint64_t local_timeout_ns, peer_timeout_ns;
};

// 4 elements of phase 2 (one half of a thread's 8): same arithmetic as update8.
__device__ __forceinline__ void update4(uint2& wq, const uint2 gq, float4& mm, float4& vv,
                                        uint64_t gi0, const Plan& pl, const StepParams& p) {
    const uint32_t gw[2] = {gq.x, gq.y};
    const uint32_t ww[2] = {wq.x, wq.y};
    float mv[4] = {mm.x, mm.y, mm.z, mm.w};
    float vv4[4] = {vv.x, vv.y, vv.z, vv.w};
    const bool keep_any = (gi0 + 4 > p.keep_lo) && (gi0 < p.keep_hi);
    const bool dec_all = gi0 + 4 <= p.n_decay;
    const bool dec_none = gi0 >= p.n_decay;
    uint16_t wout[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint16_t gh = (j & 1) ? hi16(gw[j >> 1]) : lo16(gw[j >> 1]);
        const uint16_t wh = (j & 1) ? hi16(ww[j >> 1]) : lo16(ww[j >> 1]);
        float gf = h2f(gh);
        const bool keep = keep_any && (gi0 + j >= p.keep_lo) && (gi0 + j < p.keep_hi);
        if (!keep) gf = __fmul_rn(gf, pl.inv);                       // training.rs:308
        if (pl.clip) gf = __fmul_rn(gf, pl.s);                       // optimizer.rs:151-166
        const bool dec = dec_all || (!dec_none && gi0 + j < p.n_decay);
        const float decay = dec ? pl.k.decay : 1.0f;
        wout[j] = f2h(adam_elem(h2f(wh), gf, mv[j], vv4[j], pl.k, decay));
    }
    wq = make_uint2(pack16(wout[0], wout[1]), pack16(wout[2], wout[3]));
    mm = make_float4(mv[0], mv[1], mv[2], mv[3]);
    vv = make_float4(vv4[0], vv4[1], vv4[2], vv4[3]);
}

__device__ __forceinline__ void copy_plan_from_global(Plan& dst, const Plan* src) {
    static_assert(sizeof(Plan) % 4 == 0, "plan words");
    const unsigned int* s = reinterpret_cast<const unsigned int*>(src);
    unsigned int* d = reinterpret_cast<unsigned int*>(&dst);
#pragma unroll
    for (int i = 0; i < (int)(sizeof(Plan) / 4); ++i) d[i] = __ldcg(s + i);
}

__global__ void __launch_bounds__(kFT) fused_step_kernel(StepParams p, FusedParams f) {
    extern __shared__ __align__(128) unsigned char ring[];
    __shared__ __align__(8) uint64_t bar1[kStages];
    __shared__ __align__(8) uint64_t bar2[kStages];
    __shared__ double s_sum[kFT / 32];
    __shared__ unsigned long long s_bad[kFT / 32];
    __shared__ double s_rsum[kMaxP2PRanks];
    __shared__ unsigned long long s_rbad[kMaxP2PRanks];
    __shared__ int s_rok[kMaxP2PRanks];
    __shared__ Plan s_plan;
    __shared__ int s_flag, s_err;
    const int tid = threadIdx.x;
    // Step sequence number; the state is only advanced after every CTA has
    // passed the final ticket, so all CTAs read the same value here.
    const unsigned long long epoch = p.st->steps_called + 1ull;
    if (tid == 0) {
        for (int i = 0; i < kStages; ++i) {
            mbar_init(&bar1[i], 1);
            mbar_init(&bar2[i], 1);
        }
        fence_barrier_init();
        s_err = 0;
    }
    __syncthreads();

    const uint64_t nvec = p.n >> 3;
    const uint64_t ntiles = (nvec + kTile2Vec - 1) / kTile2Vec;
    const uint64_t t_lo = ntiles * blockIdx.x / gridDim.x;
    const uint64_t t_hi = ntiles * (blockIdx.x + 1) / gridDim.x;
    const uint64_t v_lo = t_lo * kTile2Vec;
    const uint64_t v_hi = t_hi * kTile2Vec < nvec ? t_hi * kTile2Vec : nvec;

    // ------------------------------------------------ phase 1
    const float inv = __fdiv_rn(1.0f, p.st->loss_scale);   // training.rs:244
    const uint32_t ib = __float_as_uint(inv);
    const bool pow2 = (ib & 0x7FFFFFu) == 0 && (ib & 0x7F800000u) != 0 &&
                      (ib & 0x7F800000u) != 0x7F800000u;
    double acc_s = 0.0, acc_k = 0.0;
    uint32_t amax = 0;
    {
        const uint64_t pol = f.keep_g_in_l2 ? policy_evict_last() : policy_evict_first();
        const int n1 = v_hi > v_lo ? (int)((v_hi - v_lo + kTile1Vec - 1) / kTile1Vec) : 0;
        int issued = 0, done = 0;
        auto issue = [&](int k) {
            const uint64_t a = v_lo + (uint64_t)k * kTile1Vec;
            const uint32_t cnt = (uint32_t)(v_hi - a < (uint64_t)kTile1Vec ? v_hi - a : kTile1Vec);
            const int st = k % kStages;
            mbar_arrive_expect_tx(&bar1[st], cnt * 16u);
            bulk_load(ring + st * kStage1Bytes, p.g16 + a * 8, cnt * 16u, &bar1[st], pol);
        };
        if (tid == 0)
            for (; issued < kStages - 1 && issued < n1; ++issued) issue(issued);
        for (int k = 0; k < n1; ++k) {
            if (tid == 0 && issued < n1) issue(issued++);
            const int st = k % kStages;
            if (!mbar_wait(&bar1[st], (uint32_t)(k / kStages) & 1u, f.local_timeout_ns)) s_err = 1;
            __syncthreads();
            if (s_err) break;
            done = k + 1;
            const uint64_t a = v_lo + (uint64_t)k * kTile1Vec;
            const uint32_t cnt = (uint32_t)(v_hi - a < (uint64_t)kTile1Vec ? v_hi - a : kTile1Vec);
            const uint4* tile = reinterpret_cast<const uint4*>(ring + st * kStage1Bytes);
            for (uint32_t j = tid; j < cnt; j += kFT) {
                const uint4 q = tile[j];
                amax = absmax2(amax, q.x);
                amax = absmax2(amax, q.y);
                amax = absmax2(amax, q.z);
                amax = absmax2(amax, q.w);
                const uint64_t gi0 = p.offset + ((a + j) << 3);
                if (pow2) accum8_pow2(q, gi0, p.keep_lo, p.keep_hi, acc_s, acc_k);
                else accum8_general(q, gi0, inv, p.keep_lo, p.keep_hi, acc_s);
            }
            __syncthreads();   // the stage may be refilled
        }
        if (s_err && tid == 0) {
            // drain copies still in flight into this CTA's ring before it is reused or left
            for (int k = done; k < issued; ++k)
                mbar_wait(&bar1[k % kStages], (uint32_t)(k / kStages) & 1u, f.local_timeout_ns);
            atomicExch(f.err, (unsigned int)ARK_E_TIMEOUT);
        }
    }
    if (blockIdx.x == 0 && tid < (p.n & 7u)) {          // ragged tail (n % 8)
        const uint64_t i = (nvec << 3) + tid;
        const uint16_t h = p.g16[i];
        amax = absmax2(amax, h);
        const uint64_t gi = p.offset + i;
        const bool keep = gi >= p.keep_lo && gi < p.keep_hi;
        if (pow2) {
            const double d = h2d(h);
            if (keep) acc_k = __fma_rn(d, d, acc_k);
            else acc_s = __fma_rn(d, d, acc_s);
        } else {
            const float fl = h2f(h);
            const double d = (double)(keep ? fl : __fmul_rn(fl, inv));
            acc_s = __fma_rn(d, d, acc_s);
        }
    }
    {
        const double inv_d = (double)inv;
        const double acc = pow2 ? __fma_rn(acc_s, inv_d * inv_d, acc_k) : acc_s;
        const unsigned long long bad = ((amax & 0xFFFFu) >= 0x7C00u) || ((amax >> 16) >= 0x7C00u);
        const double bsum = block_sum<kFT>(acc, s_sum);
        const unsigned long long bbad = block_sum_u64<kFT>(bad, s_bad);
        if (tid == 0) {
            p.blk_sum[blockIdx.x] = bsum;
            p.blk_bad[blockIdx.x] = bbad;
        }
    }
    // ------------------------------------------------ grid barrier + exchange
    __threadfence();
    __syncthreads();
    if (tid == 0) s_flag = atomicAdd(f.arrive, 1u) == gridDim.x - 1;
    __syncthreads();
    if (s_flag) {
        __threadfence();
        double a = 0.0;
        unsigned long long b = 0;
        for (unsigned int i = tid; i < gridDim.x; i += kFT) {
            a += __ldcg(p.blk_sum + i);
            b += __ldcg(p.blk_bad + i);
        }
        a = block_sum<kFT>(a, s_sum);
        b = block_sum_u64<kFT>(b, s_bad);
        if (tid == 0) {
            *f.arrive = 0u;   // re-armed for the next step
            s_sum[0] = a;     // broadcast this rank's partial
            s_bad[0] = b;
        }
        __syncthreads();
        if (tid < kMaxP2PRanks) {
            const int r = tid;
            double rs = 0.0;
            unsigned long long rb = 0;
            int ok = 1;
            if (p.world == 1) {
                if (r == 0) {
                    rs = s_sum[0];
                    rb = s_bad[0];
                }
            } else if (r < p.world) {
                // my partial -> rank r's slot [epoch & 1][my rank], payload before epoch
                uint64_t* dst = f.peers[r] + (((epoch & 1ull) * p.world + f.rank) * 4);
                st_relaxed_sys_v2(dst, (uint64_t)__double_as_longlong(s_sum[0]), s_bad[0]);
                st_release_sys(dst + 2, epoch);
                // rank r's partial <- my slot [epoch & 1][r]
                const uint64_t* src = f.xchg + (((epoch & 1ull) * p.world + r) * 4);
                const uint64_t t0 = global_ns();
                while (ld_acquire_sys(src + 2) != epoch) {
                    if (global_ns() - t0 > f.peer_timeout_ns) {
                        ok = 0;
                        break;
                    }
                    __nanosleep(32);
                }
                if (ok) {
                    uint64_t x, y;
                    ld_relaxed_sys_v2(src, x, y);
                    rs = __longlong_as_double((long long)x);
                    rb = y;
                }
            }
            s_rsum[r] = rs;
            s_rbad[r] = rb;
            s_rok[r] = ok;
        }
        __syncthreads();
        if (tid == 0) {
            double sum = 0.0;
            unsigned long long bad = 0;
            int ok = 1;
            for (int r = 0; r < p.world; ++r) {           // rank order: deterministic
                sum += s_rsum[r];
                bad += s_rbad[r];
                ok &= s_rok[r];
            }
            Plan pl;
            const ark_opt_status st = *p.st;
            make_plan_from(st, sum, bad, p, pl);
            const unsigned int e = atomicAdd(f.err, 0u);
            if (!ok || e) {
                pl.skip = 1;
                pl.error = ARK_E_TIMEOUT;
            }
            *f.plan = pl;
            __threadfence();
            st_release_gpu(f.release, epoch);
        }
    }
    if (tid == 0) {
        const uint64_t t0 = global_ns();
        const uint64_t limit = f.peer_timeout_ns + f.local_timeout_ns;
        bool ok = true;
        while (ld_acquire_gpu(f.release) != epoch) {
            if (global_ns() - t0 > limit) {
                ok = false;
                break;
            }
            __nanosleep(64);
        }
        if (ok) {
            copy_plan_from_global(s_plan, f.plan);
        } else {
            s_plan.skip = 1;
            s_plan.error = ARK_E_TIMEOUT;
            s_plan.overflow = 0;
        }
    }
    __syncthreads();
    const Plan pl = s_plan;

    // ------------------------------------------------ phase 2 (reverse tile order)
    if (!pl.skip) {
        const uint64_t pol_g = policy_evict_first();
        const uint64_t pol_s = policy_evict_first();
        const int n2 = (int)(t_hi - t_lo);
        int issued = 0, done = 0;
        auto tile_of = [&](int k) { return t_hi - 1 - (uint64_t)k; };
        auto issue = [&](int k) {
            const uint64_t a = tile_of(k) * kTile2Vec;
            const uint32_t cnt = (uint32_t)(nvec - a < (uint64_t)kTile2Vec ? nvec - a : kTile2Vec);
            const int st = k % kStages;
            unsigned char* base = ring + st * kStage2Bytes;
            mbar_arrive_expect_tx(&bar2[st], cnt * 96u);
            bulk_load(base, p.g16 + a * 8, cnt * 16u, &bar2[st], pol_g);
            bulk_load(base + 4096, f.w16 + a * 8, cnt * 16u, &bar2[st], pol_s);
            bulk_load(base + 8192, f.m + a * 8, cnt * 32u, &bar2[st], pol_s);
            bulk_load(base + 16384, f.v + a * 8, cnt * 32u, &bar2[st], pol_s);
        };
        if (tid == 0)
            for (; issued < kStages - 1 && issued < n2; ++issued) issue(issued);
        for (int k = 0; k < n2; ++k) {
            if (tid == 0 && issued < n2) issue(issued++);
            const int st = k % kStages;
            if (!mbar_wait(&bar2[st], (uint32_t)(k / kStages) & 1u, f.local_timeout_ns)) s_err = 1;
            __syncthreads();
            if (s_err) break;
            done = k + 1;
            const uint64_t a = tile_of(k) * kTile2Vec;
            const uint32_t nel = (uint32_t)((nvec - a < (uint64_t)kTile2Vec ? nvec - a : kTile2Vec) * 8);
            const unsigned char* base = ring + st * kStage2Bytes;
            const uint2* gs = reinterpret_cast<const uint2*>(base);
            const uint2* ws = reinterpret_cast<const uint2*>(base + 4096);
            const float4* ms = reinterpret_cast<const float4*>(base + 8192);
            const float4* vs = reinterpret_cast<const float4*>(base + 16384);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const uint32_t q = (uint32_t)tid + h * kFT;   // 4-element group within the tile
                if (q * 4 < nel) {
                    uint2 wq = ws[q];
                    float4 mm = ms[q], vv = vs[q];
                    const uint64_t e0 = a * 8 + (uint64_t)q * 4;   // shard element index
                    update4(wq, gs[q], mm, vv, p.offset + e0, pl, p);
                    __stcs(reinterpret_cast<uint2*>(f.w16 + e0), wq);
                    __stcs(reinterpret_cast<float4*>(f.m + e0), mm);
                    __stcs(reinterpret_cast<float4*>(f.v + e0), vv);
                }
            }
            __syncthreads();
        }
        if (s_err && tid == 0) {
            for (int k = done; k < issued; ++k)
                mbar_wait(&bar2[k % kStages], (uint32_t)(k / kStages) & 1u, f.local_timeout_ns);
            atomicExch(f.err, (unsigned int)ARK_E_TIMEOUT);
        }
        if (blockIdx.x == 0 && tid < (p.n & 7u)) {       // ragged tail
            const uint64_t i = (nvec << 3) + tid;
            const uint64_t gi = p.offset + i;
            float gf = h2f(p.g16[i]);
            if (!(gi >= p.keep_lo && gi < p.keep_hi)) gf = __fmul_rn(gf, pl.inv);
            if (pl.clip) gf = __fmul_rn(gf, pl.s);
            const float decay = gi < p.n_decay ? pl.k.decay : 1.0f;
            float mi = f.m[i], vi = f.v[i];
            f.w16[i] = f2h(adam_elem(h2f(f.w16[i]), gf, mi, vi, pl.k, decay));
            f.m[i] = mi;
            f.v[i] = vi;
        }
    }
    // ------------------------------------------------ state machine
    if (!last_block_arrived(p.ticket2, &s_flag)) return;
    if (tid == 0) {
        Plan fin = pl;
        const unsigned int e = atomicExch(f.err, 0u);
        if (e && !fin.error) {
            fin.error = (int)e;
        }
        advance_state(p, fin);
    }
}

}  // namespace ark

// ======================================================================
// host side
// ======================================================================
using namespace ark;

struct ark_opt_state {
    ark_opt_cfg cfg;
    int device = 0;
    cudaStream_t stream = nullptr;
    ncclComm_t comm = nullptr;
    // device allocations (one block, carved)
    void* dmem = nullptr;
    ark_opt_status* d_state = nullptr;
    float* d_lr = nullptr;
    double* d_blk_sum = nullptr;
    unsigned long long* d_blk_bad = nullptr;
    unsigned int* d_tickets = nullptr;
    Partial* d_part_local = nullptr;
    Partial* d_part_all = nullptr;
    ark_opt_status* h_status = nullptr;  // pinned
    int blocks1 = 0, blocks2 = 0;
    // persistent single-kernel step
    bool fused = false;
    int fused_blocks = 0;
    Plan* d_plan = nullptr;
    uint64_t* d_release = nullptr;
    unsigned int* d_arrive = nullptr;
    unsigned int* d_err = nullptr;
    // P2P exchange slots (world > 1)
    bool p2p = false;
    uint64_t* xchg = nullptr;                 // own receive slots (cudaMalloc, IPC-exported)
    std::vector<uint64_t*> peer_slots;        // every rank's slots, mapped here
    uint64_t** d_peers = nullptr;             // device copy of peer_slots
    uint64_t timeout_ns = 0;
    // graph replay
    cudaGraphExec_t graph = nullptr;
    cudaStream_t capture_stream = nullptr;
    const void* graph_key[4] = {nullptr, nullptr, nullptr, nullptr};
    // profiling
    std::vector<cudaEvent_t> prof_events;
    uint32_t prof_cap = 0, prof_used = 0;
};

namespace {

int check_cfg(const ark_opt_cfg* c) {
    if (!c || c->abi_version != ARK_OPT_ABI_VERSION) return ARK_E_INVALID_ARG;
    if (!c->lr_table || c->lr_table_len == 0) return ARK_E_INVALID_ARG;
    if (c->world_size < 1 || c->rank < 0 || c->rank >= c->world_size) return ARK_E_INVALID_ARG;
    if (c->world_size > 1 && !c->nccl_comm) return ARK_E_INVALID_ARG;
    if (!(c->scale_init > 0.0f) || !(c->scale_min > 0.0f) || !(c->scale_max >= c->scale_min))
        return ARK_E_INVALID_ARG;
    if (c->scale_every == 0) return ARK_E_INVALID_ARG;
    if (c->keep_scaled_hi < c->keep_scaled_lo) return ARK_E_INVALID_ARG;
    if (c->flags & ~(ARK_OPT_COMPAT_GAMMA_FINAL_UNSCALED | ARK_OPT_USE_GRAPH | ARK_OPT_TWO_PASS))
        return ARK_E_INVALID_ARG;
    return ARK_OK;
}

FusedParams make_fused(const ark_opt_state* s, uint16_t* w16, float* m, float* v) {
    FusedParams f;
    f.w16 = w16;
    f.m = m;
    f.v = v;
    f.plan = s->d_plan;
    f.release = s->d_release;
    f.arrive = s->d_arrive;
    f.err = s->d_err;
    f.xchg = s->xchg;
    f.peers = s->d_peers;
    f.rank = s->cfg.rank;
    // keep the shard's gradients in L2 between the phases when they fit comfortably
    f.keep_g_in_l2 = s->cfg.n * 2 <= (uint64_t)64 << 20;
    f.local_timeout_ns = 2000000000ull;
    f.peer_timeout_ns = s->timeout_ns;
    return f;
}

// Exchange-slot set-up for the fused step on world > 1: each rank exports
// its receive slots through CUDA IPC, the handles are all-gathered over the
// rank's NCCL communicator, and every rank maps its peers' slots.  All ranks
// then agree (NCCL min-reduction) whether every mapping succeeded; if not,
// every rank uses the two-kernel step with the NCCL exchange instead.
int setup_p2p(ark_opt_state* s) {
    const int W = s->cfg.world_size, R = s->cfg.rank;
    if (W < 2 || W > kMaxP2PRanks || !s->comm) return ARK_OK;
    const size_t slot_bytes = sizeof(uint64_t) * 4 * 2 * (size_t)W;
    int ok = 1;
    char* d_tmp = nullptr;   // [W] handles | ok flag
    if (cudaMalloc(&s->xchg, slot_bytes) != cudaSuccess) ok = 0;
    if (ok && cudaMemset(s->xchg, 0, slot_bytes) != cudaSuccess) ok = 0;
    cudaIpcMemHandle_t mine;
    memset(&mine, 0, sizeof(mine));
    if (ok && cudaIpcGetMemHandle(&mine, s->xchg) != cudaSuccess) ok = 0;
    const size_t hb = sizeof(cudaIpcMemHandle_t);
    if (cudaMalloc(&d_tmp, hb * W + 256) != cudaSuccess) return ARK_E_CUDA;
    int* d_ok = reinterpret_cast<int*>(d_tmp + hb * W);
    std::vector<cudaIpcMemHandle_t> all(W);
    cudaMemcpy(d_tmp + hb * R, &mine, hb, cudaMemcpyHostToDevice);
    if (ncclAllGather(d_tmp + hb * R, d_tmp, hb, ncclUint8, s->comm, s->stream) != ncclSuccess)
        return ARK_E_NCCL;
    if (cudaStreamSynchronize(s->stream) != cudaSuccess) return ARK_E_CUDA;
    cudaMemcpy(all.data(), d_tmp, hb * W, cudaMemcpyDeviceToHost);
    s->peer_slots.assign(W, nullptr);
    for (int r = 0; r < W && ok; ++r) {
        if (r == R) {
            s->peer_slots[r] = s->xchg;
            continue;
        }
        void* p = nullptr;
        if (cudaIpcOpenMemHandle(&p, all[r], cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
            cudaGetLastError();
            ok = 0;
            break;
        }
        s->peer_slots[r] = static_cast<uint64_t*>(p);
    }
    if (ok) {
        if (cudaMalloc(&s->d_peers, sizeof(uint64_t*) * W) != cudaSuccess ||
            cudaMemcpy(s->d_peers, s->peer_slots.data(), sizeof(uint64_t*) * W,
                       cudaMemcpyHostToDevice) != cudaSuccess)
            ok = 0;
    }
    cudaMemcpy(d_ok, &ok, sizeof(int), cudaMemcpyHostToDevice);
    if (ncclAllReduce(d_ok, d_ok, 1, ncclInt32, ncclMin, s->comm, s->stream) != ncclSuccess)
        return ARK_E_NCCL;
    if (cudaStreamSynchronize(s->stream) != cudaSuccess) return ARK_E_CUDA;
    int all_ok = 0;
    cudaMemcpy(&all_ok, d_ok, sizeof(int), cudaMemcpyDeviceToHost);
    cudaFree(d_tmp);
    s->p2p = all_ok != 0;
    return ARK_OK;
}

void teardown_p2p(ark_opt_state* s) {
    for (size_t r = 0; r < s->peer_slots.size(); ++r)
        if (s->peer_slots[r] && s->peer_slots[r] != s->xchg) cudaIpcCloseMemHandle(s->peer_slots[r]);
    s->peer_slots.clear();
    if (s->d_peers) cudaFree(s->d_peers);
    if (s->xchg) cudaFree(s->xchg);
    s->d_peers = nullptr;
    s->xchg = nullptr;
    s->p2p = false;
}

StepParams make_params(const ark_opt_state* s, const uint16_t* g16) {
    const ark_opt_cfg& c = s->cfg;
    StepParams p;
    p.g16 = g16;
    p.n = c.n;
    p.offset = c.shard_offset;
    p.n_decay = c.n_decay;
    const bool compat = (c.flags & ARK_OPT_COMPAT_GAMMA_FINAL_UNSCALED) != 0;
    p.keep_lo = compat ? c.keep_scaled_lo : 0;
    p.keep_hi = compat ? c.keep_scaled_hi : 0;
    p.st = s->d_state;
    p.lr_table = s->d_lr;
    p.lr_len = c.lr_table_len;
    p.beta1 = c.beta1;
    p.beta2 = c.beta2;
    p.eps = c.eps;
    p.wd = c.weight_decay;
    p.clip = c.grad_clip;
    p.scale_backoff = c.scale_backoff;
    p.scale_growth = c.scale_growth;
    p.scale_min = c.scale_min;
    p.scale_max = c.scale_max;
    p.scale_every = c.scale_every;
    p.max_nans = c.max_consecutive_nans;
    p.world = c.world_size;
    p.blk_sum = s->d_blk_sum;
    p.blk_bad = s->d_blk_bad;
    p.ticket1 = s->d_tickets;
    p.ticket2 = s->d_tickets + 1;
    p.part_local = s->d_part_local;
    p.part_all = s->d_part_all;
    return p;
}

int enqueue_step(ark_opt_state* s, cudaStream_t stream, uint16_t* w16, const uint16_t* g16,
                 float* m, float* v, bool profile) {
    StepParams p = make_params(s, g16);
    cudaEvent_t* ev = nullptr;
    if (profile) ev = &s->prof_events[4 * s->prof_used];
    if (s->fused) {
        FusedParams f = make_fused(s, w16, m, v);
        cudaLaunchConfig_t lc;
        memset(&lc, 0, sizeof(lc));
        lc.gridDim = dim3((unsigned)s->fused_blocks);
        lc.blockDim = dim3(kFT);
        lc.dynamicSmemBytes = kFusedSmem;
        lc.stream = stream;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeCooperative;   // all CTAs co-resident (grid barrier)
        attr[0].val.cooperative = 1;
        lc.attrs = attr;
        lc.numAttrs = 1;
        if (ev) ARK_CUDA_TRY(cudaEventRecord(ev[2], stream));
        ARK_CUDA_TRY(cudaLaunchKernelEx(&lc, fused_step_kernel, p, f));
        if (ev) {
            ARK_CUDA_TRY(cudaEventRecord(ev[3], stream));
            s->prof_used++;
        }
        return ARK_OK;
    }
    if (ev) ARK_CUDA_TRY(cudaEventRecord(ev[0], stream));
    pass1_kernel<<<s->blocks1, kThreads, 0, stream>>>(p);
    ARK_CUDA_TRY(cudaGetLastError());
    if (ev) ARK_CUDA_TRY(cudaEventRecord(ev[1], stream));
    if (s->cfg.world_size > 1) {
        ncclResult_t r = ncclAllGather(s->d_part_local, s->d_part_all, sizeof(Partial), ncclUint8,
                                       s->comm, stream);
        if (r != ncclSuccess) {
            fprintf(stderr, "[ark_cuda] ncclAllGather failed: %s\n", ncclGetErrorString(r));
            return ARK_E_NCCL;
        }
    }
    if (ev) ARK_CUDA_TRY(cudaEventRecord(ev[2], stream));
    pass2_kernel<<<s->blocks2, kThreads, 0, stream>>>(p, w16, m, v);
    ARK_CUDA_TRY(cudaGetLastError());
    if (ev) {
        ARK_CUDA_TRY(cudaEventRecord(ev[3], stream));
        s->prof_used++;
    }
    return ARK_OK;
}

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        cudaGetDevice(&prev);
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        int cur = -1;
        cudaGetDevice(&cur);
        if (prev >= 0 && cur != prev) cudaSetDevice(prev);
    }
};

}  // namespace

extern "C" {

int ark_cuda_opt_init(const ark_opt_cfg* cfg, ark_opt_state** out) {
    if (!out) return ARK_E_INVALID_ARG;
    *out = nullptr;
    int rc = check_cfg(cfg);
    if (rc) return rc;
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) return ARK_E_NO_DEVICE;
    if (cfg->device < 0 || cfg->device >= ndev) return ARK_E_INVALID_ARG;
    DeviceGuard dg(cfg->device);
    ark_opt_state* s = new ark_opt_state();
    s->cfg = *cfg;
    s->device = cfg->device;
    s->comm = reinterpret_cast<ncclComm_t>(cfg->nccl_comm);
    // The caller's stream (NULL: the legacy default stream), so the step is
    // ordered after whatever produced the gradients on that stream.
    s->stream = reinterpret_cast<cudaStream_t>(cfg->stream);
    s->blocks1 = streaming_grid(reinterpret_cast<const void*>(pass1_kernel), kThreads, 0,
                                (cfg->n >> 3) / kUnroll1 + 1);
    s->blocks2 = streaming_grid(reinterpret_cast<const void*>(pass2_kernel), kThreads, 0,
                                (cfg->n >> 3) / kUnroll2 + 1);
    const int W = cfg->world_size;
    s->timeout_ns = (uint64_t)(cfg->wait_timeout_ms ? cfg->wait_timeout_ms : 5000u) * 1000000ull;
    // persistent single-kernel step: every SM filled with co-resident CTAs
    int coop = 0, sms = 0, per_sm = 0;
    cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, cfg->device);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, cfg->device);
    if (coop && !(cfg->flags & ARK_OPT_TWO_PASS) && W <= kMaxP2PRanks &&
        cudaFuncSetAttribute(fused_step_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kFusedSmem) == cudaSuccess &&
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fused_step_kernel, kFT,
                                                      kFusedSmem) == cudaSuccess &&
        per_sm > 0) {
        s->fused = true;
        s->fused_blocks = sms * per_sm;
    }
    cudaGetLastError();
    const int nblk = s->blocks1 > s->fused_blocks ? s->blocks1 : s->fused_blocks;
    // carve one allocation: state | lr table | block partials | tickets | partials
    size_t off = 0;
    auto take = [&](size_t bytes) {
        size_t o = (off + 255) & ~size_t(255);
        off = o + bytes;
        return o;
    };
    const size_t o_state = take(sizeof(ark_opt_status));
    const size_t o_lr = take(sizeof(float) * cfg->lr_table_len);
    const size_t o_bs = take(sizeof(double) * nblk);
    const size_t o_bb = take(sizeof(unsigned long long) * nblk);
    const size_t o_tk = take(sizeof(unsigned int) * 4);
    const size_t o_pl = take(sizeof(Partial));
    const size_t o_pa = take(sizeof(Partial) * W);
    const size_t o_plan = take(sizeof(Plan));
    const size_t o_rel = take(sizeof(uint64_t));
    if (cudaMalloc(&s->dmem, off) != cudaSuccess) {
        ark_cuda_opt_destroy(s);
        return ARK_E_CUDA;
    }
    char* base = static_cast<char*>(s->dmem);
    s->d_state = reinterpret_cast<ark_opt_status*>(base + o_state);
    s->d_lr = reinterpret_cast<float*>(base + o_lr);
    s->d_blk_sum = reinterpret_cast<double*>(base + o_bs);
    s->d_blk_bad = reinterpret_cast<unsigned long long*>(base + o_bb);
    s->d_tickets = reinterpret_cast<unsigned int*>(base + o_tk);
    s->d_part_local = reinterpret_cast<Partial*>(base + o_pl);
    s->d_part_all = reinterpret_cast<Partial*>(base + o_pa);
    s->d_arrive = s->d_tickets + 2;
    s->d_err = s->d_tickets + 3;
    s->d_plan = reinterpret_cast<Plan*>(base + o_plan);
    s->d_release = reinterpret_cast<uint64_t*>(base + o_rel);
    // single-GPU: pass 1 writes the rank partial straight into the gathered slot
    if (W == 1) s->d_part_local = s->d_part_all;
    if (cudaMallocHost(&s->h_status, sizeof(ark_opt_status)) != cudaSuccess) {
        ark_cuda_opt_destroy(s);
        return ARK_E_CUDA;
    }
    ark_opt_status init;
    memset(&init, 0, sizeof(init));
    init.loss_scale = cfg->scale_init;
    init.opt_step = cfg->initial_step;
    init.last_clip_coef = 1.0f;
    bool ok = cudaMemsetAsync(s->dmem, 0, off, s->stream) == cudaSuccess &&
              cudaMemcpyAsync(s->d_state, &init, sizeof(init), cudaMemcpyHostToDevice,
                              s->stream) == cudaSuccess &&
              cudaMemcpyAsync(s->d_lr, cfg->lr_table, sizeof(float) * cfg->lr_table_len,
                              cudaMemcpyHostToDevice, s->stream) == cudaSuccess &&
              cudaStreamSynchronize(s->stream) == cudaSuccess;
    if (!ok) {
        ark_cuda_opt_destroy(s);
        return ARK_E_CUDA;
    }
    s->cfg.lr_table = nullptr;  // host table not retained
    if (W > 1 && s->fused) {
        rc = setup_p2p(s);
        if (rc) {
            ark_cuda_opt_destroy(s);
            return rc;
        }
        if (!s->p2p) {            // every rank agreed to fall back
            teardown_p2p(s);
            s->fused = false;
        }
    }
    *out = s;
    return ARK_OK;
}

int ark_cuda_opt_step(ark_opt_state* s, uint16_t* w16, const uint16_t* g16, float* m, float* v) {
    if (!s) return ARK_E_INVALID_ARG;
    if (s->cfg.n && (!w16 || !g16 || !m || !v)) return ARK_E_INVALID_ARG;
    if (!aligned16(w16) || !aligned16(g16) || !aligned16(m) || !aligned16(v))
        return ARK_E_MISALIGNED;
    DeviceGuard dg(s->device);
    const bool profile = s->prof_used < s->prof_cap;
    const bool use_graph = (s->cfg.flags & ARK_OPT_USE_GRAPH) && !profile;
    if (!use_graph) return enqueue_step(s, s->stream, w16, g16, m, v, profile);
    const void* key[4] = {w16, g16, m, v};
    if (!s->graph || memcmp(key, s->graph_key, sizeof(key)) != 0) {
        if (s->graph) {
            cudaGraphExecDestroy(s->graph);
            s->graph = nullptr;
        }
        // Capture on a private stream (the legacy default stream cannot be
        // captured); the graph is then launched on the state's stream.
        if (!s->capture_stream)
            ARK_CUDA_TRY(cudaStreamCreateWithFlags(&s->capture_stream, cudaStreamNonBlocking));
        cudaGraph_t g = nullptr;
        ARK_CUDA_TRY(cudaStreamBeginCapture(s->capture_stream, cudaStreamCaptureModeThreadLocal));
        int rc = enqueue_step(s, s->capture_stream, w16, g16, m, v, false);
        cudaError_t e = cudaStreamEndCapture(s->capture_stream, &g);
        if (rc != ARK_OK) {
            if (g) cudaGraphDestroy(g);
            return rc;
        }
        ARK_CUDA_TRY(e);
        e = cudaGraphInstantiate(&s->graph, g, 0);
        cudaGraphDestroy(g);
        ARK_CUDA_TRY(e);
        memcpy(s->graph_key, key, sizeof(key));
    }
    ARK_CUDA_TRY(cudaGraphLaunch(s->graph, s->stream));
    return ARK_OK;
}

int ark_cuda_opt_read_status(ark_opt_state* s, ark_opt_status* out) {
    if (!s || !out) return ARK_E_INVALID_ARG;
    DeviceGuard dg(s->device);
    ARK_CUDA_TRY(cudaMemcpyAsync(s->h_status, s->d_state, sizeof(ark_opt_status),
                                 cudaMemcpyDeviceToHost, s->stream));
    ARK_CUDA_TRY(cudaStreamSynchronize(s->stream));
    *out = *s->h_status;
    if (out->error) return out->error;
    if (out->early_stop) return ARK_E_EARLY_STOP;
    return ARK_OK;
}

int ark_cuda_opt_set_status(ark_opt_state* s, const ark_opt_status* in) {
    if (!s || !in) return ARK_E_INVALID_ARG;
    DeviceGuard dg(s->device);
    *s->h_status = *in;
    ARK_CUDA_TRY(cudaMemcpyAsync(s->d_state, s->h_status, sizeof(ark_opt_status),
                                 cudaMemcpyHostToDevice, s->stream));
    ARK_CUDA_TRY(cudaStreamSynchronize(s->stream));
    return ARK_OK;
}

int ark_cuda_opt_upload_grads(ark_opt_state* s, uint16_t* g16_dev, const uint16_t* g16_host,
                              uint64_t n) {
    if (!s || (n && (!g16_dev || !g16_host))) return ARK_E_INVALID_ARG;
    DeviceGuard dg(s->device);
    if (n) {
        ARK_CUDA_TRY(cudaMemcpyAsync(g16_dev, g16_host, n * sizeof(uint16_t),
                                     cudaMemcpyHostToDevice, s->stream));
    }
    return ARK_OK;
}

int ark_cuda_allgather_weights(ark_opt_state* s, const uint16_t* shard, uint16_t* full,
                               uint64_t stride) {
    if (!s || !shard || !full || stride < s->cfg.n) return ARK_E_INVALID_ARG;
    DeviceGuard dg(s->device);
    if (s->cfg.world_size == 1) {
        if (s->cfg.n && (const void*)full != (const void*)shard)
            ARK_CUDA_TRY(cudaMemcpyAsync(full, shard, s->cfg.n * 2, cudaMemcpyDeviceToDevice,
                                         s->stream));
        return ARK_OK;
    }
    // every rank contributes `stride` elements (its shard plus padding)
    ncclResult_t r = ncclAllGather(shard, full, stride, ncclHalf, s->comm, s->stream);
    if (r != ncclSuccess) {
        fprintf(stderr, "[ark_cuda] ncclAllGather(weights) failed: %s\n", ncclGetErrorString(r));
        return ARK_E_NCCL;
    }
    return ARK_OK;
}

int ark_cuda_opt_profile_begin(ark_opt_state* s, uint32_t max_steps) {
    if (!s) return ARK_E_INVALID_ARG;
    DeviceGuard dg(s->device);
    for (cudaEvent_t e : s->prof_events) cudaEventDestroy(e);
    s->prof_events.assign(4 * (size_t)max_steps, nullptr);
    for (auto& e : s->prof_events) ARK_CUDA_TRY(cudaEventCreate(&e));
    s->prof_cap = max_steps;
    s->prof_used = 0;
    return ARK_OK;
}

int ark_cuda_opt_profile_read(ark_opt_state* s, float* out, uint32_t capacity, uint32_t* steps) {
    if (!s || !steps) return ARK_E_INVALID_ARG;
    DeviceGuard dg(s->device);
    ARK_CUDA_TRY(cudaStreamSynchronize(s->stream));
    const uint32_t k = s->prof_used < capacity ? s->prof_used : capacity;
    for (uint32_t i = 0; i < k; ++i) {
        cudaEvent_t* ev = &s->prof_events[4 * i];
        ARK_CUDA_TRY(cudaEventElapsedTime(&out[3 * i + 0], ev[0], ev[1]));
        ARK_CUDA_TRY(cudaEventElapsedTime(&out[3 * i + 1], ev[1], ev[2]));
        ARK_CUDA_TRY(cudaEventElapsedTime(&out[3 * i + 2], ev[2], ev[3]));
    }
    if (s->fused)
        for (uint32_t i = 0; i < k; ++i) out[3 * i] = out[3 * i + 1] = 0.0f;
    *steps = k;
    s->prof_cap = 0;
    s->prof_used = 0;
    return ARK_OK;
}

int ark_cuda_opt_geometry(ark_opt_state* s, uint32_t* b1, uint32_t* b2, uint32_t* threads) {
    if (!s) return ARK_E_INVALID_ARG;
    if (b1) *b1 = s->fused ? 0u : (uint32_t)s->blocks1;
    if (b2) *b2 = s->fused ? (uint32_t)s->fused_blocks : (uint32_t)s->blocks2;
    if (threads) *threads = (uint32_t)(s->fused ? kFT : kThreads);
    return ARK_OK;
}

int ark_cuda_opt_destroy(ark_opt_state* s) {
    if (!s) return ARK_OK;
    DeviceGuard dg(s->device);
    cudaStreamSynchronize(s->stream);
    if (s->graph) cudaGraphExecDestroy(s->graph);
    if (s->capture_stream) cudaStreamDestroy(s->capture_stream);
    teardown_p2p(s);
    for (cudaEvent_t e : s->prof_events) cudaEventDestroy(e);
    if (s->dmem) cudaFree(s->dmem);
    if (s->h_status) cudaFreeHost(s->h_status);
    delete s;
    return ARK_OK;
}

int ark_cuda_lr_schedule(float* table, uint32_t len, float lr, uint32_t warmup) {
    if (!table || len == 0) return ARK_E_INVALID_ARG;
    // optimizer.rs:80-92, evaluated in f32 in the order written there (the
    // library is compiled with -ffp-contract=off, SSE scalar math).
    for (uint32_t step = 0; step < len; ++step) {
        float out;
        if (step < warmup) {
            out = lr * ((float)step + 1.0f) / (float)warmup;
        } else {
            const float decay_steps = (float)(step - warmup);
            const float progress = fminf(decay_steps / 800000.0f, 1.0f);
            const float cosine = 0.5f * (1.0f + cosf(3.14159274101257324f * progress));
            const float lr_min = lr * 0.1f;
            out = lr_min + (lr - lr_min) * cosine;
        }
        table[step] = out;
    }
    return ARK_OK;
}

int ark_cuda_nccl_unique_id(void* id_out) {
    if (!id_out) return ARK_E_INVALID_ARG;
    ncclUniqueId id;
    if (ncclGetUniqueId(&id) != ncclSuccess) return ARK_E_NCCL;
    memcpy(id_out, &id, sizeof(id));
    return ARK_OK;
}

int ark_cuda_nccl_comm_init(int world, int rank, const void* id_in, int device, void** comm_out) {
    if (!id_in || !comm_out || world < 1 || rank < 0 || rank >= world) return ARK_E_INVALID_ARG;
    DeviceGuard dg(device);
    ncclUniqueId id;
    memcpy(&id, id_in, sizeof(id));
    ncclComm_t comm = nullptr;
    ncclResult_t r = ncclCommInitRank(&comm, world, id, rank);
    if (r != ncclSuccess) {
        fprintf(stderr, "[ark_cuda] ncclCommInitRank failed: %s\n", ncclGetErrorString(r));
        return ARK_E_NCCL;
    }
    *comm_out = comm;
    return ARK_OK;
}

int ark_cuda_nccl_comm_destroy(void* comm) {
    if (!comm) return ARK_OK;
    return ncclCommDestroy(reinterpret_cast<ncclComm_t>(comm)) == ncclSuccess ? ARK_OK : ARK_E_NCCL;
}

}  // extern "C"
