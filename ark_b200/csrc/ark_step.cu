// ark_step.cu -- the fused optimizer step for one flat ZeRO-1 shard.
//
// One step = two streaming kernels on the caller's stream, no host sync:
//
//   pass 1  reads the FP16 loss-scaled gradients once (2 B/param): detects
//           non-finite values (training.rs:291) and accumulates the sum of
//           squares of the UNSCALED gradient (training.rs:308 then
//           optimizer.rs:126-145) in double; the per-block partials are
//           reduced in a fixed order by the last block to finish, which (on
//           several GPUs) also exchanges the 16-byte rank partial with every
//           peer over NVLink: P2P stores into the peers' receive slots and a
//           bounded wait for theirs.  Where the peers' slots cannot be
//           mapped, an NCCL all-gather between the passes does the exchange.
//   pass 2  every block derives the step plan from device memory: skip on
//           overflow (training.rs:293-305), else t = step+1, lr(t), clip
//           coefficient (optimizer.rs:145-149), AdamW scalars
//           (opti.s:210-271).  Then the fused element update (22 B/param:
//           g, w, m, v read, w, m, v written): g = fp16(g) * inv_scale *
//           clip ; m, v, w as opti.s:285-308, walking the shard in REVERSE
//           so the gradient lines pass 1 read last are still in L2.  The
//           last block to finish advances the loss-scale state machine
//           (training.rs:316-326).  Launched as a programmatic dependent of
//           pass 1: its blocks start as pass 1's retire, form the parts of
//           the plan that only need the state, load their first vectors,
//           and wait in the kernel for pass 1's results.
#include <cuda_runtime.h>
#include <nccl.h>
#include <stdlib.h>
#include <string.h>

#include <vector>

#include "ark_device.cuh"
#include "ark_internal.h"
#include "ark_sync.cuh"

namespace ark {

// Device state: identical layout to ark_opt_status so a status read is one
// 64-byte copy.
static_assert(sizeof(ark_opt_status) == 64, "status layout");

// Per-rank pass-1 result exchanged between ranks (16 bytes).
struct Partial {
    double sumsq;
    unsigned long long nonfinite;   // > 0 iff an inf/NaN was seen; kPartialTimeout: no data
};
constexpr unsigned long long kPartialTimeout = ~0ull;
constexpr int kMaxP2PRanks = 32;
constexpr int kSlotWords = 8;
enum SlotWord { kSlotSum = 0, kSlotBad = 1, kSlotEpoch = 2, kSlotGradsReady = 3,
                kSlotWeightsReady = 4 };

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
    int rank;
    int p2p;                         // exchange in pass 1 over mapped peer slots
    double* blk_sum;                 // pass-1 per-block partials
    unsigned long long* blk_bad;
    unsigned int* ticket1;
    unsigned int* ticket2;
    int p1_last;                     // pass 1's last block forms the rank partial (NCCL exchange)
    unsigned int nblk1;              // pass-1 blocks (partials pass 2 reduces otherwise)
    Partial* part_local;             // this rank's partial (NCCL all-gather send buffer)
    Partial* part_all;               // [world] partials of every rank, rank order
    uint64_t* xchg;                  // own receive slots [2][world] x kSlotWords (slot_of)
    uint64_t* const* peers;          // every rank's receive slots (peers[rank] == xchg)
    uint64_t peer_timeout_ns;
    unsigned long long* verdict;     // pass 2: (epoch << 1) | every partial arrived
    unsigned long long* logits_bad;  // non-finite logits gradients counted since the last step
    // reduce-scatter step: every rank's full FP16 gradient buffer (mapped here)
    const uint16_t* const* gsrc;
    uint16_t* g16_out;               // this rank's reduced shard
    float* w32_out;                  // optional FP32 copy of the updated weights
    // weight all-gather fused with pass 2: every rank's full FP16 weight
    // buffer (mapped here); the updated shard is stored into each of them,
    // into this rank's own too when wself (w16 is not that buffer's slice)
    uint16_t* const* wdst;           // [world], device memory
    int wself;
};

constexpr int kThreads = 256;

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
                                               uint64_t keep_hi, double& acc0, double& acc1) {
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
    const bool keep_any = (gi0 + 8 > keep_lo) && (gi0 < keep_hi);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const uint16_t h = (j & 1) ? hi16(w[j >> 1]) : lo16(w[j >> 1]);
        const float f = h2f(h);
        const bool keep = keep_any && (gi0 + j >= keep_lo) && (gi0 + j < keep_hi);
        const double d = (double)(keep ? f : __fmul_rn(f, inv));
        if (j & 1) acc1 = __fma_rn(d, d, acc1);
        else acc0 = __fma_rn(d, d, acc0);
    }
}

// Power-of-two loss scale (the only kind the state machine produces from a
// power-of-two init, backoff and growth): fp32(h) * inv is exact, so the sum
// of squared unscaled gradients is inv^2 * sum(h^2), with h^2 exact in
// double.  With KEEP, elements in the kept range (compat mode) go to acc_k
// unscaled; without it the range is empty and no index is compared.  Two
// accumulators halve the dependent chain of double FMAs.  An inf or NaN
// gradient makes its square, and from then on the accumulator, non-finite;
// a finite h^2 is at most 2^32, so a finite sum never overflows: the
// accumulators double as the non-finite check.
template <bool KEEP>
__device__ __forceinline__ void accum8_pow2(uint4 q, uint64_t gi0, uint64_t keep_lo,
                                            uint64_t keep_hi, double& acc0, double& acc1,
                                            double& acc_k) {
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
    if (KEEP && gi0 + 8 > keep_lo && gi0 < keep_hi) {   // rare: straddles the kept range
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const double d = h2d((j & 1) ? hi16(w[j >> 1]) : lo16(w[j >> 1]));
            if (gi0 + j >= keep_lo && gi0 + j < keep_hi) acc_k = __fma_rn(d, d, acc_k);
            else acc0 = __fma_rn(d, d, acc0);
        }
        return;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const double d = h2d((j & 1) ? hi16(w[j >> 1]) : lo16(w[j >> 1]));
        if (j & 1) acc1 = __fma_rn(d, d, acc1);
        else acc0 = __fma_rn(d, d, acc0);
    }
}

// Receive slot of rank q in rank r's buffer, for one epoch parity:
// kSlotWords x u64 {sum of squares, non-finite, partial epoch,
// gradients-ready epoch, weights-ready epoch, unused...} (one 64-byte line).
__device__ __forceinline__ uint64_t* slot_of(uint64_t* base, unsigned long long epoch, int world,
                                             int q) {
    return base + (((epoch & 1ull) * (unsigned long long)world + (unsigned long long)q) *
                   kSlotWords);
}

// Pass 2, block 0, world > 1 over mapped peer slots: lane r (< world) of
// warp 0 stores this rank's partial into rank r's slot [epoch & 1][rank]
// (payload, then the epoch with release semantics).  Slots alternate with
// the epoch parity: a rank publishes epoch e + 2 into the slot of epoch e
// only after its pass 2 of step e + 1 has seen every rank's partial e + 1,
// which every rank publishes only after its own pass 2 of step e (the last
// reader of epoch e) has completed.
__device__ void publish_partial_p2p(const StepParams& p, unsigned long long epoch,
                                    const Partial& mine) {
    const int r = threadIdx.x;
    if (r >= p.world || r == p.rank) return;
    uint64_t* dst = slot_of(p.peers[r], epoch, p.world, p.rank);
    st_relaxed_sys_v2(dst + kSlotSum, (uint64_t)__double_as_longlong(mine.sumsq), mine.nonfinite);
    st_release_sys(dst + kSlotEpoch, epoch);
}

// Bounded wait of one lane for rank q's partial of `epoch` in this rank's
// slots.  Returns false if it did not arrive within the limit.
__device__ bool wait_partial(const StepParams& p, unsigned long long epoch, int q, Partial* out) {
    const uint64_t* src = slot_of(p.xchg, epoch, p.world, q);
    const uint64_t t0 = global_ns();
    while (ld_acquire_sys(src + kSlotEpoch) != epoch) {
        if (global_ns() - t0 > p.peer_timeout_ns) return false;
        __nanosleep(32);
    }
    uint64_t x, y;
    ld_relaxed_sys_v2(src + kSlotSum, x, y);
    out->sumsq = __longlong_as_double((long long)x);
    out->nonfinite = y;
    return true;
}

// Pass 2, every block, warp 0: every rank's partial of this step into
// out[0, world) (shared memory); out[rank] is this rank's own partial, which
// every block has reduced itself, so only the peers' are waited for (in this
// rank's receive slots, bounded by the global timer).  The outcome is made
// uniform across the grid's blocks: the first block to decide (every
// partial arrived, or a wait ran out) records (epoch << 1 | ok) in
// p.verdict with a compare-and-swap and every block follows it, so no block
// updates while another skips.  A block that timed out while the verdict
// says every partial arrived reads them again (they are in this GPU's memory
// by then); if even that wait runs out it marks its partials as missing (its
// vectors are not updated) and the state reports ARK_E_TIMEOUT.
__device__ void gather_partials_p2p(const StepParams& p, unsigned long long epoch,
                                    const Partial& mine, Partial* out) {
    const int lane = threadIdx.x;
    bool ok = true;
    if (lane == p.rank) out[lane] = mine;
    else if (lane < p.world) ok = wait_partial(p, epoch, lane, &out[lane]);
    const bool all_ok = __all_sync(0xFFFFFFFFu, ok);
    unsigned long long v = 0;
    if (lane == 0) {
        const unsigned long long want = (epoch << 1) | (all_ok ? 1ull : 0ull);
        v = *reinterpret_cast<volatile unsigned long long*>(p.verdict);
        while ((v >> 1) != epoch) {
            const unsigned long long w = atomicCAS(p.verdict, v, want);
            if (w == v) {
                v = want;
                break;
            }
            v = w;
        }
    }
    v = __shfl_sync(0xFFFFFFFFu, v, 0);
    const bool verdict_ok = (v & 1ull) != 0;
    if (verdict_ok && !ok && lane < p.world) ok = wait_partial(p, epoch, lane, &out[lane]);
    if (lane < p.world && (!verdict_ok || !ok)) {
        out[lane].sumsq = 0.0;
        out[lane].nonfinite = kPartialTimeout;
    }
    __syncwarp();
}

// Per-thread pass-1 accumulators.
struct P1Acc {
    double acc0 = 0.0, acc1 = 0.0, acc_k = 0.0;
    uint32_t amax = 0;
};

struct P1Scale {
    float inv;
    bool pow2;
};

// pow2: inv is a power of two for which fp32(h) * inv is exact for every
// finite FP16 h (2^-102 <= inv <= 2^111: no f32 underflow or overflow);
// any other scale takes the general path, which rounds like the reference.
__device__ __forceinline__ P1Scale p1_scale(const StepParams& p) {
    P1Scale sc;
    sc.inv = __fdiv_rn(1.0f, p.st->loss_scale);   // training.rs:244
    const uint32_t ib = __float_as_uint(sc.inv);
    const uint32_t e = (ib >> 23) & 0xFFu;
    sc.pow2 = (ib & 0x807FFFFFu) == 0 && e >= 127u - 102u && e <= 127u + 111u;
    return sc;
}

// One 8-element vector.  POW2 takes its non-finite check from the
// accumulators (accum8_pow2); the general path, where fp32(h) * inv may
// overflow for a finite h, checks the FP16 bit patterns.
template <bool KEEP, bool POW2>
__device__ __forceinline__ void p1_consume(P1Acc& a, const uint4 q, uint64_t vec,
                                           const P1Scale& sc, const StepParams& p) {
    const uint64_t gi0 = p.offset + (vec << 3);
    if (POW2) {
        accum8_pow2<KEEP>(q, gi0, p.keep_lo, p.keep_hi, a.acc0, a.acc1, a.acc_k);
    } else {
        a.amax = absmax2(a.amax, q.x);
        a.amax = absmax2(a.amax, q.y);
        a.amax = absmax2(a.amax, q.z);
        a.amax = absmax2(a.amax, q.w);
        accum8_general(q, gi0, sc.inv, p.keep_lo, p.keep_hi, a.acc0, a.acc1);
    }
}

__device__ __forceinline__ void p1_consume1(P1Acc& a, uint16_t h, uint64_t i, const P1Scale& sc,
                                            const StepParams& p) {
    a.amax = absmax2(a.amax, h);
    const uint64_t gi = p.offset + i;
    const bool keep = gi >= p.keep_lo && gi < p.keep_hi;
    if (sc.pow2) {
        const double d = h2d(h);
        if (keep) a.acc_k = __fma_rn(d, d, a.acc_k);
        else a.acc0 = __fma_rn(d, d, a.acc0);
    } else {
        const float f = h2f(h);
        const double d = (double)(keep ? f : __fmul_rn(f, sc.inv));
        a.acc0 = __fma_rn(d, d, a.acc0);
    }
}

// A block whose partial is unusable (its gradients-ready wait ran out) adds
// kFailBit to the block's non-finite count; real counts stay below 2^40.
constexpr unsigned long long kFailBit = 1ull << 40;

// Fixed-order reduction of pass 1's per-block partials into this rank's
// partial (valid in thread 0; every thread of the block must call it).  The
// same code in every block gives the same value bit for bit, so pass 2 runs
// it in every block instead of a last pass-1 block running it once.
__device__ Partial reduce_block_partials(const StepParams& p, unsigned int nblk) {
    __shared__ double s_sum[kThreads / 32];
    __shared__ unsigned long long s_bad[kThreads / 32];
    double s = 0.0;
    unsigned long long b = 0;
    for (unsigned int i = threadIdx.x; i < nblk; i += kThreads) {
        s += __ldcg(p.blk_sum + i);
        const unsigned long long x = __ldcg(p.blk_bad + i);
        b += x == kPartialTimeout ? kFailBit : x;
    }
    s = block_sum<kThreads>(s, s_sum);
    b = block_sum_u64<kThreads>(b, s_bad);
    Partial r;
    r.sumsq = s;
    r.nonfinite = b >= kFailBit ? kPartialTimeout : b;   // threads that saw an inf/NaN
    return r;
}

// End of pass 1 in every block: the block's sum of squares and non-finite
// count (`failed` in any thread marks the block's partial unusable).  With
// p.p1_last (the NCCL exchange between the kernels) the last block to
// finish also reduces the block partials into this rank's partial, folds in
// the logits count and writes it for the all-gather; otherwise pass 2 does
// that reduction and pass 1 retires here.
__device__ void p1_finish(const P1Acc& a, const P1Scale& sc, bool failed, const StepParams& p) {
    __shared__ double s_sum[kThreads / 32];
    __shared__ unsigned long long s_bad[kThreads / 32];
    __shared__ int s_last;
    // fold the power-of-two scaling in per thread (exact): sum of u^2
    const double inv_d = (double)sc.inv;
    const double acc_s = a.acc0 + a.acc1;
    const double acc = sc.pow2 ? __fma_rn(acc_s, inv_d * inv_d, a.acc_k) : acc_s;
    const bool raw_nonfinite = sc.pow2 && !isfinite(acc_s + a.acc_k);
    const unsigned long long bad =
        (raw_nonfinite || ((a.amax & 0xFFFFu) >= 0x7C00u) || ((a.amax >> 16) >= 0x7C00u) ? 1ull
                                                                                       : 0ull) +
        (failed ? kFailBit : 0ull);
    const double bsum = block_sum<kThreads>(acc, s_sum);
    const unsigned long long bbad = block_sum_u64<kThreads>(bad, s_bad);
    if (threadIdx.x == 0) {
        p.blk_sum[blockIdx.x] = bsum;
        p.blk_bad[blockIdx.x] = bbad >= kFailBit ? kPartialTimeout : bbad;
    }
    if (!p.p1_last) return;
    if (!last_block_arrived(p.ticket1, &s_last)) return;
    const Partial r = reduce_block_partials(p, gridDim.x);
    __shared__ Partial s_rank;
    if (threadIdx.x == 0) {
        // Non-finite logits gradients counted by the logits check since the
        // last step (training.rs:228-241) skip this step like non-finite
        // gradients: the reference applies the same transitions on both
        // paths (:232-236, :294-298).  Folding the count into the rank
        // partial makes every rank skip when any rank's logits were bad.
        const unsigned long long lb = atomicExch(p.logits_bad, 0ull);
        Partial out = r;
        if (out.nonfinite != kPartialTimeout) out.nonfinite += lb;
        *p.part_local = out;
        s_rank = out;
    }
    if (p.p2p) {   // publish to the peers now; pass 2 does the waiting
        __syncthreads();
        if (threadIdx.x < kMaxP2PRanks) publish_partial_p2p(p, p.st->steps_called + 1ull, s_rank);
    }
}

// The grid-stride stream of pass 1: rounds of U vectors per thread, loads
// issued before any is consumed; rounds entirely in range run without
// per-vector bounds checks, and the one partial round after them with.
// LD 0: L2 only (ld.global.cg); LD 1: the non-coherent path without L1
// allocation (the gradients are read-only while pass 1 runs).
template <int LD>
__device__ __forceinline__ uint4 p1_load(const uint4* p) {
    if (LD == 0) return ld_keep(p);
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

template <int U, int LD>
__device__ __forceinline__ void p1_load_round(uint4 (&q)[U], const uint4* g, uint64_t base,
                                              uint64_t stride, uint64_t nvec) {
#pragma unroll
    for (int u = 0; u < U; ++u) {
        const uint64_t i = base + u * stride;
        q[u] = i < nvec ? p1_load<LD>(g + i) : make_uint4(0, 0, 0, 0);
    }
}

// q holds this thread's first round, loaded before the loss scale was read.
template <int U, bool KEEP, bool POW2, int LD>
__device__ __forceinline__ void p1_stream(P1Acc& a, const P1Scale& sc, const StepParams& p,
                                          uint4 (&q)[U]) {
    const uint4* g = reinterpret_cast<const uint4*>(p.g16);
    const uint64_t nvec = p.n >> 3;
    const uint64_t stride = (uint64_t)gridDim.x * kThreads;
    uint64_t base = (uint64_t)blockIdx.x * kThreads + threadIdx.x;
#pragma unroll
    for (int u = 0; u < U; ++u) {
        const uint64_t i = base + u * stride;
        if (i < nvec) p1_consume<KEEP, POW2>(a, q[u], i, sc, p);
    }
    base += stride * U;
    for (; base + stride * (U - 1) < nvec; base += stride * U) {
#pragma unroll
        for (int u = 0; u < U; ++u) q[u] = p1_load<LD>(g + base + u * stride);
#pragma unroll
        for (int u = 0; u < U; ++u) p1_consume<KEEP, POW2>(a, q[u], base + u * stride, sc, p);
    }
    if (base < nvec) {
        p1_load_round<U, LD>(q, g, base, stride, nvec);
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const uint64_t i = base + u * stride;
            if (i < nvec) p1_consume<KEEP, POW2>(a, q[u], i, sc, p);
        }
    }
}

// KEEP: the compat kept range is non-empty (chosen on the host).
template <int U, int MINB, bool KEEP, int LD>
__global__ void __launch_bounds__(kThreads, MINB) pass1_kernel(StepParams p) {
    griddep_launch_dependents();
    uint4 q[U];   // the first round goes out before the loss scale is read
    p1_load_round<U, LD>(q, reinterpret_cast<const uint4*>(p.g16),
                         (uint64_t)blockIdx.x * kThreads + threadIdx.x,
                         (uint64_t)gridDim.x * kThreads, p.n >> 3);
    const P1Scale sc = p1_scale(p);
    P1Acc a;
    if (sc.pow2) p1_stream<U, KEEP, true, LD>(a, sc, p, q);
    else p1_stream<U, KEEP, false, LD>(a, sc, p, q);
    if (blockIdx.x == 0 && threadIdx.x < (p.n & 7u)) {   // ragged tail (n % 8)
        const uint64_t i = (p.n & ~7ull) + threadIdx.x;
        p1_consume1(a, p.g16[i], i, sc, p);
    }
    p1_finish(a, sc, false, p);
}

// The gradient hand-off fused with pass 1: this rank's shard of the sum over
// ranks of every rank's full FP16 gradient buffer, read straight from the
// peers' memory over NVLink.  The reference zeroes its FP32 gradients and
// accumulates the backward's output with += (src/memory.rs:338-342,
// objc/bridge.m:907-949); here the contributions of the ranks are
// accumulated in FP32 in rank order starting from 0, rounded once to FP16
// (RNE) into the local shard, and finite-checked / squared from the same
// registers.  Before reading, each rank announces that its buffer is
// complete (gradients-ready epoch in every peer's slot) and waits, bounded,
// for every peer's announcement; the partial exchange at the end of pass 1
// then proves that every peer has finished reading this rank's buffer.
// Gradients-ready barrier of the reduce-scatter step: block 0 publishes
// this rank's epoch into every peer's slot; every block waits (bounded) for
// every peer's.  Returns true (in all threads) if a peer never showed up.
__device__ bool reduce_ready_barrier(const StepParams& p) {
    __shared__ int s_fail;
    const unsigned long long epoch = p.st->steps_called + 1ull;
    if (threadIdx.x == 0) s_fail = 0;
    if (p.world > 1) {
        if (blockIdx.x == 0 && threadIdx.x < p.world) {
            __threadfence_system();
            st_release_sys(slot_of(p.peers[threadIdx.x], epoch, p.world, p.rank) + kSlotGradsReady,
                           epoch);
        }
        if (threadIdx.x == 0) {
            const uint64_t t0 = global_ns();
            for (int q = 0; q < p.world && !s_fail; ++q) {
                const uint64_t* ready = slot_of(p.xchg, epoch, p.world, q) + kSlotGradsReady;
                while (ld_acquire_sys(ready) != epoch) {
                    if (global_ns() - t0 > p.peer_timeout_ns) {
                        s_fail = 1;
                        break;
                    }
                    __nanosleep(64);
                }
            }
        }
    }
    __syncthreads();
    return s_fail != 0;
}

// Any rank count: U vectors of every rank per round, rank by rank.
template <int U, bool KEEP, bool POW2>
__device__ __forceinline__ void reduce_stream(P1Acc& a, const P1Scale& sc, const StepParams& p) {
    const uint64_t nvec = p.n >> 3;
    const uint64_t stride = (uint64_t)gridDim.x * kThreads;
    uint4* out = reinterpret_cast<uint4*>(p.g16_out);
    for (uint64_t base = (uint64_t)blockIdx.x * kThreads + threadIdx.x; base < nvec;
         base += stride * U) {
        float acc[U][8];
#pragma unroll
        for (int u = 0; u < U; ++u)
#pragma unroll
            for (int j = 0; j < 8; ++j) acc[u][j] = 0.0f;
        for (int r = 0; r < p.world; ++r) {                 // rank order
            const uint4* src = reinterpret_cast<const uint4*>(p.gsrc[r] + p.offset);
            uint4 q[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const uint64_t i = base + u * stride;
                q[u] = i < nvec ? __ldcg(src + i) : make_uint4(0, 0, 0, 0);
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const uint32_t w[4] = {q[u].x, q[u].y, q[u].z, q[u].w};
#pragma unroll
                for (int j = 0; j < 8; ++j)
                    acc[u][j] = __fadd_rn(acc[u][j],
                                          h2f((j & 1) ? hi16(w[j >> 1]) : lo16(w[j >> 1])));
            }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const uint64_t i = base + u * stride;
            if (i < nvec) {
                uint32_t w[4];
#pragma unroll
                for (int k = 0; k < 4; ++k) w[k] = pack16(f2h(acc[u][2 * k]), f2h(acc[u][2 * k + 1]));
                const uint4 rq = make_uint4(w[0], w[1], w[2], w[3]);
                out[i] = rq;
                p1_consume<KEEP, POW2>(a, rq, i, sc, p);
            }
        }
    }
}

// Ragged tail (n % 8) of the reduce-scatter step, block 0.
__device__ __forceinline__ void reduce_tail(P1Acc& a, const P1Scale& sc, const StepParams& p) {
    if (blockIdx.x == 0 && threadIdx.x < (p.n & 7u)) {
        const uint64_t i = (p.n & ~7ull) + threadIdx.x;
        float f = 0.0f;
        for (int r = 0; r < p.world; ++r) f = __fadd_rn(f, h2f(p.gsrc[r][p.offset + i]));
        const uint16_t h = f2h(f);
        p.g16_out[i] = h;
        p1_consume1(a, h, i, sc, p);
    }
}

// KEEP: the compat kept range is non-empty (chosen on the host); the
// power-of-two path is chosen per step by the loss scale, as in pass 1.
template <int U, int MINB, bool KEEP>
__global__ void __launch_bounds__(kThreads, MINB) pass1_reduce_kernel(StepParams p) {
    griddep_launch_dependents();
    const bool failed = reduce_ready_barrier(p);
    const P1Scale sc = p1_scale(p);
    P1Acc a;
    if (!failed) {
        if (sc.pow2) reduce_stream<U, KEEP, true>(a, sc, p);
        else reduce_stream<U, KEEP, false>(a, sc, p);
        reduce_tail(a, sc, p);
    }
    p1_finish(a, sc, failed, p);
}

// --------------------------------------------------------------- pass 2
struct Plan {
    AdamK k;
    float inv, s, norm, lr;
    double sumsq;
    uint32_t t;
    int skip;       // overflow, early stop or error: no element work
    int early_stop;
    int clip;
    int overflow;
    int error;      // ARK_E_* raised while forming the plan (0 = none)
    unsigned long long epoch;   // this step's number (steps_called + 1)
};

// The step plan, in two parts.  plan_from_state reads only the state (last
// written by the previous step's pass 2) and the lr table, so pass 2 may
// form it before pass 1 of this step has completed; plan_from_partials reads
// every rank's {sum, non-finite}, which pass 1 writes.
__device__ void plan_from_state(const StepParams& p, Plan& pl) {
    const ark_opt_status st = *p.st;
    pl.epoch = st.steps_called + 1ull;
    pl.early_stop = st.early_stop != 0;
    pl.inv = __fdiv_rn(1.0f, st.loss_scale);          // training.rs:244
    pl.t = st.opt_step + 1u;                          // optimizer.rs:172
    const uint32_t li = pl.t < p.lr_len ? pl.t : p.lr_len - 1u;
    pl.lr = p.lr_table[li];                           // optimizer.rs:173
    pl.k = adam_scalars(pl.lr, p.beta1, p.beta2, p.eps, p.wd, pl.t);
}

__device__ void plan_from_partials(const StepParams& p, const Partial* parts, Plan& pl) {
    double sumsq = 0.0;
    unsigned long long bad = 0;
    bool timeout = false;
    for (int r = 0; r < p.world; ++r) {               // rank order: deterministic
        const Partial q = parts[r];
        if (q.nonfinite == kPartialTimeout) timeout = true;
        else {
            sumsq += q.sumsq;
            bad += q.nonfinite;
        }
    }
    pl.sumsq = sumsq;
    pl.overflow = bad != 0;
    pl.error = timeout ? ARK_E_TIMEOUT : 0;
    pl.skip = pl.overflow || pl.early_stop || timeout;
    pl.norm = __double2float_rn(__dsqrt_rn(sumsq));   // optimizer.rs:145
    pl.clip = (pl.norm > p.clip) && (pl.norm > 0.0f); // optimizer.rs:148
    pl.s = pl.clip ? __fdiv_rn(p.clip, pl.norm) : 1.0f;
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

// The norm part of pass 2's plan, once per block after the grid-dependency
// wait; every thread of the block calls it and on return the plan is in
// s_plan for every thread.  P2RED: this rank's partial comes from reducing
// pass 1's block partials here (a fixed order, the same value in every
// block, plus the non-finite logits count), and block 0 publishes it to the
// peers; otherwise pass 1's last block formed (and published) it.  With the
// peer-to-peer exchange every block then reads the peers' partials from this
// rank's slots (bounded); with the NCCL exchange they were all-gathered into
// part_all.  P2RED is a template parameter so that the update kernel without
// it keeps its register allocation (120 instead of 125 registers).
template <bool P2RED>
__device__ __forceinline__ void pass2_plan(const StepParams& p, Plan& s_plan, Partial* s_part) {
    if (!P2RED && !p.p2p) {   // one GPU, or the NCCL all-gather into part_all
        if (threadIdx.x == 0) plan_from_partials(p, p.part_all, s_plan);
        __syncthreads();
        return;
    }
    if (P2RED) {
        Partial mine = reduce_block_partials(p, p.nblk1);
        if (threadIdx.x == 0) {
            if (mine.nonfinite != kPartialTimeout)
                mine.nonfinite += *reinterpret_cast<volatile unsigned long long*>(p.logits_bad);
            s_part[p.rank] = mine;
        }
    } else if (threadIdx.x == 0) {
        s_part[p.rank] = *p.part_local;
    }
    __syncthreads();
    if (!p.p2p) {
        if (threadIdx.x == 0) plan_from_partials(p, s_part, s_plan);
    } else if (threadIdx.x < 32) {   // the peers' partials from this rank's slots
        const Partial own = s_part[p.rank];
        if (P2RED && blockIdx.x == 0) publish_partial_p2p(p, s_plan.epoch, own);
        gather_partials_p2p(p, s_plan.epoch, own, s_part);
        if (threadIdx.x == 0) {
            plan_from_partials(p, s_part, s_plan);
            // a block that could not read a partial reports it (the last
            // block folds it into the state); see gather_partials_p2p
            if (s_plan.error) atomicExch(&p.st->error, s_plan.error);
        }
    }
    __syncthreads();
}

// Eight elements of the update.  Without KEEP the compat kept range is
// empty and no element index is compared for it.  DEC 1 turns the
// weight-decay boundary n_decay into a count of decayed elements in this
// vector (0-8) once, so each element costs one 32-bit compare; DEC 0
// compares each element's 64-bit index with the boundary.
template <bool KEEP, int DEC>
__device__ __forceinline__ void update8(uint4& wq, const uint4 gq, float4& m0, float4& m1,
                                        float4& v0, float4& v1, uint64_t gi0, const Plan& pl,
                                        const StepParams& p) {
    const uint32_t gw[4] = {gq.x, gq.y, gq.z, gq.w};
    uint32_t ww[4] = {wq.x, wq.y, wq.z, wq.w};
    float mm[8] = {m0.x, m0.y, m0.z, m0.w, m1.x, m1.y, m1.z, m1.w};
    float vv[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
    const bool keep_any = KEEP && (gi0 + 8 > p.keep_lo) && (gi0 < p.keep_hi);
    const uint32_t ndec = gi0 >= p.n_decay ? 0u
                          : (p.n_decay - gi0 >= 8 ? 8u : (uint32_t)(p.n_decay - gi0));
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
        const bool dec = DEC ? (uint32_t)j < ndec
                             : (dec_all || (!dec_none && gi0 + j < p.n_decay));
        const float decay = dec ? pl.k.decay : 1.0f;  // wd = 0: 1 - lr*0
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

// One round of pass 2: U vectors per thread, all loads before any update.
template <int U>
struct P2Round {
    uint4 gq[U], wq[U];
    float4 ma[U], mb[U], va[U], vb[U];
};

template <int U>
__device__ __forceinline__ void p2_load(P2Round<U>& r, uint64_t base, uint64_t stride,
                                        uint64_t nvec, const uint4* g4, const uint4* w4,
                                        const float4* m4, const float4* v4, bool with_g) {
#pragma unroll
    for (int u = 0; u < U; ++u) {
        const uint64_t j = base + u * stride;
        if (j < nvec) {
            const uint64_t i = nvec - 1 - j;
            if (with_g) r.gq[u] = ld_stream(g4 + i);
            r.wq[u] = ld_stream(w4 + i);
            r.ma[u] = ld_stream(m4 + 2 * i);
            r.mb[u] = ld_stream(m4 + 2 * i + 1);
            r.va[u] = ld_stream(v4 + 2 * i);
            r.vb[u] = ld_stream(v4 + 2 * i + 1);
        }
    }
}

template <int U>
__device__ __forceinline__ void p2_load_g(P2Round<U>& r, uint64_t base, uint64_t stride,
                                          uint64_t nvec, const uint4* g4) {
#pragma unroll
    for (int u = 0; u < U; ++u) {
        const uint64_t j = base + u * stride;
        if (j < nvec) r.gq[u] = ld_stream(g4 + (nvec - 1 - j));
    }
}

template <int U, bool kW32, bool KEEP, int DEC, bool GATHER>
__device__ __forceinline__ void p2_update(P2Round<U>& r, uint64_t base, uint64_t stride,
                                          uint64_t nvec, uint4* w4, float4* m4, float4* v4,
                                          const Plan& pl, const StepParams& p) {
#pragma unroll
    for (int u = 0; u < U; ++u) {
        const uint64_t j = base + u * stride;
        if (j < nvec) {
            const uint64_t i = nvec - 1 - j;
            update8<KEEP, DEC>(r.wq[u], r.gq[u], r.ma[u], r.mb[u], r.va[u], r.vb[u],
                          p.offset + (i << 3), pl, p);
            st_stream(w4 + i, r.wq[u]);
            if (GATHER) {   // every rank's full weight buffer: plain (peer) stores
                const uint64_t gv = (p.offset >> 3) + i;
                // the peer order starts at a different rank in each block, so
                // the blocks of all ranks spread over every destination
                int q = (int)(blockIdx.x % (unsigned)p.world);
                for (int k = 0; k < p.world; ++k) {
                    if (q != p.rank || p.wself) reinterpret_cast<uint4*>(p.wdst[q])[gv] = r.wq[u];
                    if (++q == p.world) q = 0;
                }
            }
            if (kW32) {   // the forward's FP32 weights (training.rs:165-186)
                float4* o = reinterpret_cast<float4*>(p.w32_out) + 2 * i;
                const uint4 wq = r.wq[u];
                st_stream(o, make_float4(h2f(lo16(wq.x)), h2f(hi16(wq.x)), h2f(lo16(wq.y)),
                                         h2f(hi16(wq.y))));
                st_stream(o + 1, make_float4(h2f(lo16(wq.z)), h2f(hi16(wq.z)), h2f(lo16(wq.w)),
                                             h2f(hi16(wq.w))));
            }
            st_stream(m4 + 2 * i, r.ma[u]);
            st_stream(m4 + 2 * i + 1, r.mb[u]);
            st_stream(v4 + 2 * i, r.va[u]);
            st_stream(v4 + 2 * i + 1, r.vb[u]);
        }
    }
}

// Grid-stride over 8-element vectors in reverse (vector i = nvec-1-j for the
// j-th in forward order): consecutive threads still touch consecutive
// vectors, and the first vectors updated are the last ones pass 1 read.
// Launched as a programmatic dependent of pass 1, the blocks start as pass
// 1's retire: before griddep_wait they form the state part of the plan and
// load their first round of w, m, v (and g, unless pass 1 writes it: the
// reduce-scatter step), none of which pass 1 writes.
template <int kUnroll2, int MINB, bool kW32, bool KEEP, int DEC = 1, bool GATHER = false,
          bool P2RED = false>
__global__ void __launch_bounds__(kThreads, MINB) pass2_kernel(StepParams p,
                                                              uint16_t* __restrict__ w16,
                                                              float* __restrict__ m,
                                                              float* __restrict__ v) {
    __shared__ Plan s_plan;
    __shared__ int s_last;
    __shared__ Partial s_part[kMaxP2PRanks];
    const uint4* g4 = reinterpret_cast<const uint4*>(p.g16);
    uint4* w4 = reinterpret_cast<uint4*>(w16);
    float4* m4 = reinterpret_cast<float4*>(m);
    float4* v4 = reinterpret_cast<float4*>(v);
    const uint64_t nvec = p.n >> 3;
    const uint64_t stride = (uint64_t)gridDim.x * kThreads;
    const bool g_early = p.g16_out == nullptr;
    uint64_t base = (uint64_t)blockIdx.x * kThreads + threadIdx.x;
    if (threadIdx.x == 0) plan_from_state(p, s_plan);
    P2Round<kUnroll2> r;
    p2_load<kUnroll2>(r, base, stride, nvec, g4, w4, m4, v4, g_early);
    griddep_wait();
    pass2_plan<P2RED>(p, s_plan, s_part);
    const Plan pl = s_plan;
    if (!pl.skip) {
        if (!g_early) p2_load_g<kUnroll2>(r, base, stride, nvec, g4);
        while (base < nvec) {
            p2_update<kUnroll2, kW32, KEEP, DEC, GATHER>(r, base, stride, nvec, w4, m4, v4, pl, p);
            base += stride * kUnroll2;
            if (base >= nvec) break;
            p2_load<kUnroll2>(r, base, stride, nvec, g4, w4, m4, v4, true);
        }
        if (blockIdx.x == 0 && threadIdx.x < (p.n & 7u)) {
            const uint64_t i = (nvec << 3) + threadIdx.x;
            const uint64_t gi = p.offset + i;
            float gf = h2f(p.g16[i]);
            if (!(gi >= p.keep_lo && gi < p.keep_hi)) gf = __fmul_rn(gf, pl.inv);
            if (pl.clip) gf = __fmul_rn(gf, pl.s);
            const float decay = gi < p.n_decay ? pl.k.decay : 1.0f;
            float mi = m[i], vi = v[i];
            const uint16_t wn = f2h(adam_elem(h2f(w16[i]), gf, mi, vi, pl.k, decay));
            w16[i] = wn;
            if (kW32) p.w32_out[i] = h2f(wn);
            if (GATHER)
                for (int q = 0; q < p.world; ++q)
                    if (q != p.rank || p.wself) p.wdst[q][gi] = wn;
            m[i] = mi;
            v[i] = vi;
        }
    }
    // peer stores of this block visible system-wide before it is counted
    if (GATHER) __threadfence_system();
    if (!last_block_arrived(p.ticket2, &s_last)) return;
    if (threadIdx.x == 0) {
        advance_state(p, pl);
        // every block has read the logits count (before the ticket)
        if (P2RED) *p.logits_bad = 0ull;
    }
    if (GATHER && p.p2p && threadIdx.x < p.world) {
        // weights-ready epoch into every rank's slot: every block's stores
        // into that rank's weight buffer precede it
        __threadfence_system();
        st_release_sys(slot_of(p.peers[threadIdx.x], pl.epoch, p.world, p.rank) +
                           kSlotWeightsReady,
                       pl.epoch);
    }
}

// The same for a fixed rank count NR: all NR x U loads of a thread are in
// flight before any addition (remote loads over NVLink have long latency).
template <int NR, int U, bool KEEP, bool POW2>
__device__ __forceinline__ void reduce_stream_nr(P1Acc& a, const P1Scale& sc,
                                                 const StepParams& p) {
    const uint64_t nvec = p.n >> 3;
    const uint64_t stride = (uint64_t)gridDim.x * kThreads;
    uint4* out = reinterpret_cast<uint4*>(p.g16_out);
    const uint4* src[NR];
#pragma unroll
    for (int r = 0; r < NR; ++r) src[r] = reinterpret_cast<const uint4*>(p.gsrc[r] + p.offset);
    for (uint64_t base = (uint64_t)blockIdx.x * kThreads + threadIdx.x; base < nvec;
         base += stride * U) {
        uint4 q[NR][U];
#pragma unroll
        for (int r = 0; r < NR; ++r)
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const uint64_t i = base + u * stride;
                q[r][u] = i < nvec ? __ldcg(src[r] + i) : make_uint4(0, 0, 0, 0);
            }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const uint64_t i = base + u * stride;
            if (i >= nvec) continue;
            float acc[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) acc[j] = 0.0f;
#pragma unroll
            for (int r = 0; r < NR; ++r) {                 // rank order
                const uint32_t w[4] = {q[r][u].x, q[r][u].y, q[r][u].z, q[r][u].w};
#pragma unroll
                for (int j = 0; j < 8; ++j)
                    acc[j] = __fadd_rn(acc[j], h2f((j & 1) ? hi16(w[j >> 1]) : lo16(w[j >> 1])));
            }
            uint32_t w[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) w[k] = pack16(f2h(acc[2 * k]), f2h(acc[2 * k + 1]));
            const uint4 rq = make_uint4(w[0], w[1], w[2], w[3]);
            out[i] = rq;
            p1_consume<KEEP, POW2>(a, rq, i, sc, p);
        }
    }
}

template <int NR, int U, int MINB, bool KEEP>
__global__ void __launch_bounds__(kThreads, MINB) pass1_reduce_nr_kernel(StepParams p) {
    griddep_launch_dependents();
    const bool failed = reduce_ready_barrier(p);
    const P1Scale sc = p1_scale(p);
    P1Acc a;
    if (!failed) {
        if (sc.pow2) reduce_stream_nr<NR, U, KEEP, true>(a, sc, p);
        else reduce_stream_nr<NR, U, KEEP, false>(a, sc, p);
        reduce_tail(a, sc, p);
    }
    p1_finish(a, sc, failed, p);
}

// ark_cuda_opt_weights_wait: one warp; lane r waits, bounded, for rank r's
// weights-ready epoch of the last step (published by the last block of its
// pass 2 after its stores into this rank's weight buffer).  On a timeout
// the state reports ARK_E_TIMEOUT.
__global__ void weights_wait_kernel(StepParams p) {
    const int lane = threadIdx.x;
    const unsigned long long epoch = p.st->steps_called;   // the step just run
    bool ok = true;
    if (lane < p.world && epoch > 0) {
        const uint64_t* w = slot_of(p.xchg, epoch, p.world, lane) + kSlotWeightsReady;
        const uint64_t t0 = global_ns();
        while (ld_acquire_sys(w) != epoch) {
            if (global_ns() - t0 > p.peer_timeout_ns) {
                ok = false;
                break;
            }
            __nanosleep(64);
        }
    }
    if (!__all_sync(0xFFFFFFFFu, ok) && lane == 0) p.st->error = ARK_E_TIMEOUT;
}

// The logits-gradient check and loss scaling (training.rs:228-245): counts
// the non-finite values of the unscaled logits gradients and multiplies
// every element by the current loss scale in place (x *= loss_scale, one
// f32 multiply, :244-245).  The count goes into the state's logits_bad word,
// which the next step's pass 1 folds into its non-finite partial.  One pass
// (4 B read + 4 B written per element): on a step the check rejects, the
// reference returns before scaling and discards the buffer, so its contents
// are not part of the result.
constexpr int kLogitsU = 4;
__device__ __forceinline__ unsigned int f32_nonfinite(float f) {
    return (__float_as_uint(f) & 0x7F800000u) == 0x7F800000u;
}

__global__ void __launch_bounds__(kThreads) logits_kernel(float* __restrict__ x, uint64_t n,
                                                          const ark_opt_status* __restrict__ st,
                                                          unsigned long long* bad_out) {
    __shared__ unsigned long long s_bad[kThreads / 32];
    const float scale = st->loss_scale;
    const uint64_t stride = (uint64_t)gridDim.x * kThreads;
    unsigned int bad = 0;
    if (((uintptr_t)x & 15u) == 0) {
        const uint64_t nq = n >> 2;
        float4* x4 = reinterpret_cast<float4*>(x);
        for (uint64_t base = (uint64_t)blockIdx.x * kThreads + threadIdx.x; base < nq;
             base += stride * kLogitsU) {
            float4 q[kLogitsU];
#pragma unroll
            for (int u = 0; u < kLogitsU; ++u) {
                const uint64_t i = base + u * stride;
                if (i < nq) q[u] = ld_stream(x4 + i);
            }
#pragma unroll
            for (int u = 0; u < kLogitsU; ++u) {
                const uint64_t i = base + u * stride;
                if (i >= nq) continue;
                bad += f32_nonfinite(q[u].x) + f32_nonfinite(q[u].y) + f32_nonfinite(q[u].z) +
                       f32_nonfinite(q[u].w);
                q[u].x = __fmul_rn(q[u].x, scale);
                q[u].y = __fmul_rn(q[u].y, scale);
                q[u].z = __fmul_rn(q[u].z, scale);
                q[u].w = __fmul_rn(q[u].w, scale);
                st_stream(x4 + i, q[u]);
            }
        }
        if (blockIdx.x == 0 && threadIdx.x < (n & 3u)) {
            const uint64_t i = (nq << 2) + threadIdx.x;
            bad += f32_nonfinite(x[i]);
            x[i] = __fmul_rn(x[i], scale);
        }
    } else {
        for (uint64_t i = (uint64_t)blockIdx.x * kThreads + threadIdx.x; i < n; i += stride) {
            bad += f32_nonfinite(x[i]);
            x[i] = __fmul_rn(x[i], scale);
        }
    }
    const unsigned long long b = block_sum_u64<kThreads>(bad, s_bad);
    if (threadIdx.x == 0 && b) atomicAdd(bad_out, b);
}

// Launch-shape variants, selected at init by shard size (or by index through
// ARK_PASS1_VARIANT / ARK_PASS2_VARIANT / ARK_PASS2W_VARIANT).  Pass 1:
// vectors in flight per thread x minimum resident blocks per SM x load path
// (0: L2 only, 1: non-coherent); pass 2: 8-element groups in flight per
// thread x minimum resident blocks per SM.
using Pass1Fn = void (*)(StepParams);
using Pass2Fn = void (*)(StepParams, uint16_t*, float*, float*);
struct Pass1Variant {
    int unroll, min_blocks;
    Pass1Fn fn, fn_keep;   // empty / non-empty compat kept range
};
struct Pass2Variant {
    int unroll, min_blocks;
    // [pass 2 reduces pass 1's block partials][kept range non-empty]:
    // plain / also writing FP32 weights
    Pass2Fn fn[2][2], fn_w32[2][2];
};
#define ARK_P1(U, B, L) {U, B, pass1_kernel<U, B, false, L>, pass1_kernel<U, B, true, L>}
static const Pass1Variant kPass1Variants[] = {
    ARK_P1(4, 4, 0), ARK_P1(4, 6, 0), ARK_P1(2, 8, 0), ARK_P1(8, 4, 0), ARK_P1(16, 2, 0),
    ARK_P1(6, 6, 0), ARK_P1(8, 4, 1), ARK_P1(4, 6, 1), ARK_P1(8, 8, 1), ARK_P1(4, 8, 1),
};
#undef ARK_P1
// reduce-scatter pass 1 by rank count (any other count: the generic kernel)
template <bool KEEP>
static Pass1Fn pass1_reduce_for(int world) {
    switch (world) {
        case 1: return pass1_reduce_nr_kernel<1, 8, 4, KEEP>;
        case 2: return pass1_reduce_nr_kernel<2, 4, 4, KEEP>;
        case 4: return pass1_reduce_nr_kernel<4, 2, 4, KEEP>;
        case 8: return pass1_reduce_nr_kernel<8, 1, 4, KEEP>;
        default: return pass1_reduce_kernel<2, 4, KEEP>;
    }
}
#define ARK_P2S(U, B, W, K, D)                                                           \
    {{pass2_kernel<U, B, W, K, D, false, false>, pass2_kernel<U, B, W, true, D, false, false>}, \
     {pass2_kernel<U, B, W, K, D, false, true>, pass2_kernel<U, B, W, true, D, false, true>}}
#define ARK_P2(U, B) {U, B, ARK_P2S(U, B, false, false, 1), ARK_P2S(U, B, true, false, 1)}
#define ARK_P2X(U, B, K, D) {U, B, ARK_P2S(U, B, false, K, D), ARK_P2S(U, B, true, K, D)}
// 5 and 6: the 2 x 2 shape with the kept-range check compiled in even when
// the range is empty (5: decay chosen by two 64-bit boundary compares, 6: by
// the per-vector count).  On B200 these are faster than 4 when the SM clock
// is not power-capped (EKO step 0.900 vs 0.925 ms at 1965 MHz) and slower
// when it is (0.918-0.921 vs 0.907 ms at ~1670 MHz, the usual state of a
// long run under the 1 kW cap), which is why 4 is the default.
static const Pass2Variant kPass2Variants[] = {
    ARK_P2(2, 1), ARK_P2(1, 3), ARK_P2(1, 4), ARK_P2(3, 1), ARK_P2(2, 2),
    ARK_P2X(2, 2, true, 0), ARK_P2X(2, 2, true, 1),
};
#undef ARK_P2X
#undef ARK_P2
#undef ARK_P2S
// Pass 2 with the fused weight all-gather, [shape][pass-2 reduction][kept
// range non-empty]: shape 0 is 1 group x 3 blocks/SM (shards below 100M
// params), shape 1 is 2 groups x 2 blocks/SM, as for the plain kernel.
#define ARK_P2G(U, B, R) \
    {pass2_kernel<U, B, false, false, 1, true, R>, pass2_kernel<U, B, false, true, 1, true, R>}
static const Pass2Fn kPass2Gather[2][2][2] = {
    {ARK_P2G(1, 3, false), ARK_P2G(1, 3, true)},
    {ARK_P2G(2, 2, false), ARK_P2G(2, 2, true)},
};
#undef ARK_P2G

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
    unsigned long long* d_verdict = nullptr;     // pass-2 exchange verdict word
    unsigned long long* d_logits_bad = nullptr;  // non-finite logits count since the last step
    ark_opt_status* h_status = nullptr;  // pinned
    int blocks1 = 0, blocks2 = 0, blocks1r = 0;
    Pass1Fn pass1 = nullptr, pass1r = nullptr;   // chosen launch-shape variants
    Pass2Fn pass2 = nullptr, pass2_w32 = nullptr, pass2_gather = nullptr;
    int blocks2g = 0;
    bool pdl = false;  // pass 2 launched as a programmatic dependent of pass 1
    bool p1_last = true;   // pass 1's last block forms the rank partial (else pass 2 does)
    int blocks2w = 0;
    // P2P exchange slots (world > 1)
    bool p2p = false;
    uint64_t* xchg = nullptr;                 // own receive slots (cudaMalloc, IPC-exported)
    std::vector<uint64_t*> peer_slots;        // every rank's slots, mapped here
    uint64_t** d_peers = nullptr;             // device copy of peer_slots
    // full-gradient buffers of the reduce-scatter step (world >= 1)
    void* gbuf = nullptr;                     // this rank's buffer (cudaMalloc, IPC-exported)
    uint64_t gbuf_n = 0;
    std::vector<void*> gpeer;                 // every rank's buffer, mapped here
    const uint16_t** d_gsrc = nullptr;        // device copy of gpeer
    // full-weight buffers of the fused weight all-gather (world >= 1)
    void* wbuf = nullptr;                     // this rank's buffer (cudaMalloc, IPC-exported)
    uint64_t wbuf_n = 0;
    std::vector<void*> wpeer;                 // every rank's buffer, mapped here
    uint16_t** d_wdst = nullptr;              // device copy of wpeer
    uint64_t timeout_ns = 0;
    // graph replay
    // graph replay: slot 0 plain, slot 1 with four event-record nodes that are
    // pointed at the profiling events of each replay
    // (slots 2 and 3: the same for the reduce-scatter step)
    cudaGraph_t gsrc[4] = {nullptr, nullptr, nullptr, nullptr};
    cudaGraphExec_t gexec[4] = {nullptr, nullptr, nullptr, nullptr};
    const void* gkey[4][6] = {};
    cudaGraphNode_t ev_node[2][4] = {};     // per profiled slot (1, 3)
    cudaEvent_t ph_ev[4] = {nullptr, nullptr, nullptr, nullptr};   // capture placeholders
    cudaStream_t capture_stream = nullptr;
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
    if (c->flags &
        ~(ARK_OPT_COMPAT_GAMMA_FINAL_UNSCALED | ARK_OPT_USE_GRAPH | ARK_OPT_NCCL_EXCHANGE))
        return ARK_E_INVALID_ARG;
    return ARK_OK;
}

// Exchange-slot set-up for world > 1: each rank exports its receive slots
// through CUDA IPC, the handles are all-gathered over the rank's NCCL
// communicator, and every rank maps its peers' slots.  All ranks then agree
// (NCCL min-reduction) whether every mapping succeeded; if not, every rank
// exchanges the partials with an NCCL all-gather instead.
// Collective over the rank's NCCL communicator: export `local` (the base
// of a cudaMalloc allocation) through CUDA IPC, all-gather the handles, map
// every peer's allocation here (mapped[rank] = local), and agree with an
// NCCL min-reduction whether every rank mapped every peer.  On disagreement
// the mappings made here are closed again and *all_ok is false on every rank.
int share_ipc(ark_opt_state* s, void* local, std::vector<void*>& mapped, bool* all_ok) {
    const int W = s->cfg.world_size, R = s->cfg.rank;
    *all_ok = false;
    mapped.assign(W, nullptr);
    int ok = local != nullptr;
    cudaIpcMemHandle_t mine;
    memset(&mine, 0, sizeof(mine));
    if (ok && cudaIpcGetMemHandle(&mine, local) != cudaSuccess) {
        cudaGetLastError();
        ok = 0;
    }
    const size_t hb = sizeof(cudaIpcMemHandle_t);
    char* d_tmp = nullptr;   // [W] handles | agreement flag
    if (cudaMalloc(&d_tmp, hb * W + 256) != cudaSuccess) return ARK_E_CUDA;
    int* d_ok = reinterpret_cast<int*>(d_tmp + hb * W);
    int rc = ARK_OK;
    std::vector<cudaIpcMemHandle_t> all(W);
    cudaMemcpy(d_tmp + hb * R, &mine, hb, cudaMemcpyHostToDevice);
    if (ncclAllGather(d_tmp + hb * R, d_tmp, hb, ncclUint8, s->comm, s->stream) != ncclSuccess)
        rc = ARK_E_NCCL;
    else if (cudaStreamSynchronize(s->stream) != cudaSuccess)
        rc = ARK_E_CUDA;
    if (rc == ARK_OK) {
        cudaMemcpy(all.data(), d_tmp, hb * W, cudaMemcpyDeviceToHost);
        for (int r = 0; r < W && ok; ++r) {
            if (r == R) {
                mapped[r] = local;
                continue;
            }
            if (cudaIpcOpenMemHandle(&mapped[r], all[r], cudaIpcMemLazyEnablePeerAccess) !=
                cudaSuccess) {
                cudaGetLastError();
                mapped[r] = nullptr;
                ok = 0;
            }
        }
        cudaMemcpy(d_ok, &ok, sizeof(int), cudaMemcpyHostToDevice);
        if (ncclAllReduce(d_ok, d_ok, 1, ncclInt32, ncclMin, s->comm, s->stream) != ncclSuccess)
            rc = ARK_E_NCCL;
        else if (cudaStreamSynchronize(s->stream) != cudaSuccess)
            rc = ARK_E_CUDA;
        int agreed = 0;
        if (rc == ARK_OK) cudaMemcpy(&agreed, d_ok, sizeof(int), cudaMemcpyDeviceToHost);
        *all_ok = rc == ARK_OK && agreed != 0;
    }
    cudaFree(d_tmp);
    if (!*all_ok) {
        for (int r = 0; r < W; ++r)
            if (mapped[r] && mapped[r] != local) cudaIpcCloseMemHandle(mapped[r]);
        mapped.assign(W, nullptr);
    }
    return rc;
}

// Exchange-slot set-up for world > 1: each rank's receive slots are shared
// through share_ipc; if any rank cannot map its peers, every rank exchanges
// the partials with an NCCL all-gather instead.
int setup_p2p(ark_opt_state* s) {
    const int W = s->cfg.world_size;
    if (W < 2 || W > kMaxP2PRanks || !s->comm) return ARK_OK;
    const size_t slot_bytes = sizeof(uint64_t) * kSlotWords * 2 * (size_t)W;
    if (cudaMalloc(&s->xchg, slot_bytes) != cudaSuccess) s->xchg = nullptr;
    else if (cudaMemset(s->xchg, 0, slot_bytes) != cudaSuccess) return ARK_E_CUDA;
    std::vector<void*> mapped;
    bool all_ok = false;
    const int rc = share_ipc(s, s->xchg, mapped, &all_ok);
    if (rc) return rc;
    s->peer_slots.assign(W, nullptr);
    if (all_ok) {
        for (int r = 0; r < W; ++r) s->peer_slots[r] = static_cast<uint64_t*>(mapped[r]);
        if (cudaMalloc(&s->d_peers, sizeof(uint64_t*) * W) != cudaSuccess ||
            cudaMemcpy(s->d_peers, s->peer_slots.data(), sizeof(uint64_t*) * W,
                       cudaMemcpyHostToDevice) != cudaSuccess)
            return ARK_E_CUDA;
    }
    s->p2p = all_ok;
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

// A buffer of every rank mapped into every other rank: close the peers'
// mappings, free this rank's allocation and the device pointer table.
template <typename T>
void release_shared(void*& local, std::vector<void*>& mapped, T**& d_table) {
    for (size_t r = 0; r < mapped.size(); ++r)
        if (mapped[r] && mapped[r] != local) cudaIpcCloseMemHandle(mapped[r]);
    mapped.clear();
    if (d_table) cudaFree(d_table);
    if (local) cudaFree(local);
    d_table = nullptr;
    local = nullptr;
}

// Collective over the rank's communicator (every rank calls it): allocate
// `bytes` here (zeroed), map every rank's allocation into this process
// (world > 1: CUDA IPC, needs the mapped exchange slots) and copy the
// rank-ordered pointer table to the device.  On failure nothing is kept.
template <typename T>
int make_shared(ark_opt_state* s, size_t bytes, void*& local, std::vector<void*>& mapped,
                T**& d_table) {
    const int W = s->cfg.world_size;
    if (W > 1 && !s->p2p) return ARK_E_UNSUPPORTED;
    release_shared(local, mapped, d_table);
    bytes = (bytes + 255) & ~size_t(255);
    if (cudaMalloc(&local, bytes) != cudaSuccess) {
        local = nullptr;
        if (W == 1) return ARK_E_CUDA;   // else share_ipc reports it to every rank
    } else if (cudaMemset(local, 0, bytes) != cudaSuccess) {
        return ARK_E_CUDA;
    }
    if (W == 1) {
        mapped.assign(1, local);
    } else {
        bool all_ok = false;
        const int rc = share_ipc(s, local, mapped, &all_ok);
        if (rc || !all_ok) {
            release_shared(local, mapped, d_table);
            return rc ? rc : ARK_E_UNSUPPORTED;
        }
    }
    if (cudaMalloc(&d_table, sizeof(T*) * W) != cudaSuccess ||
        cudaMemcpy(d_table, mapped.data(), sizeof(T*) * W, cudaMemcpyHostToDevice) !=
            cudaSuccess) {
        release_shared(local, mapped, d_table);
        return ARK_E_CUDA;
    }
    return ARK_OK;
}

void teardown_grads(ark_opt_state* s) {
    release_shared(s->gbuf, s->gpeer, s->d_gsrc);
    s->gbuf_n = 0;
}

void teardown_weights(ark_opt_state* s) {
    release_shared(s->wbuf, s->wpeer, s->d_wdst);
    s->wbuf_n = 0;
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
    p.rank = c.rank;
    p.p2p = s->p2p ? 1 : 0;
    p.xchg = s->xchg;
    p.peers = s->d_peers;
    p.peer_timeout_ns = s->timeout_ns;
    p.gsrc = s->d_gsrc;
    p.g16_out = nullptr;
    p.w32_out = nullptr;
    p.blk_sum = s->d_blk_sum;
    p.blk_bad = s->d_blk_bad;
    p.ticket1 = s->d_tickets;
    p.ticket2 = s->d_tickets + 1;
    p.part_local = s->d_part_local;
    p.part_all = s->d_part_all;
    p.verdict = s->d_verdict;
    p.p1_last = s->p1_last ? 1 : 0;
    p.nblk1 = 0;
    p.logits_bad = s->d_logits_bad;
    p.wdst = s->d_wdst;
    p.wself = 1;
    return p;
}

// Under stream capture, events are recorded "external" so that they become
// event-record nodes of the graph (a plain record would only order streams);
// the external flag is only valid while capturing.
#define ARK_RECORD(e, st)                                                                   \
    ARK_CUDA_TRY(capturing ? cudaEventRecordWithFlags((e), (st), cudaEventRecordExternal) \
                           : cudaEventRecord((e), (st)))

// Pass 2, as a programmatic dependent of pass 1 when `pdl` (it then directly
// follows pass 1 in the stream: no event record or collective between).
cudaError_t launch_pass2(Pass2Fn fn, int blocks, cudaStream_t stream, bool pdl,
                         const StepParams& p, uint16_t* w16, float* m, float* v) {
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t lc = {};
    lc.gridDim = dim3((unsigned)blocks);
    lc.blockDim = dim3(kThreads);
    lc.dynamicSmemBytes = 0;
    lc.stream = stream;
    lc.attrs = attr;
    lc.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&lc, fn, p, w16, m, v);
}

int enqueue_step(ark_opt_state* s, cudaStream_t stream, uint16_t* w16, const uint16_t* g16,
                 float* m, float* v, float* w32, cudaEvent_t* ev, bool capturing = false,
                 bool reduce = false, bool gather = false) {
    StepParams p = make_params(s, g16);
    if (reduce) p.g16_out = const_cast<uint16_t*>(g16);
    p.w32_out = w32;
    // the caller's shard may live inside this rank's full weight buffer
    p.wself = !(gather && w16 == static_cast<uint16_t*>(s->wbuf) + s->cfg.shard_offset);
    if (ev) ARK_RECORD(ev[0], stream);
    p.nblk1 = (unsigned int)(reduce ? s->blocks1r : s->blocks1);
    if (reduce) s->pass1r<<<s->blocks1r, kThreads, 0, stream>>>(p);
    else s->pass1<<<s->blocks1, kThreads, 0, stream>>>(p);
    ARK_CUDA_TRY(cudaGetLastError());
    if (ev) ARK_RECORD(ev[1], stream);
    if (s->cfg.world_size > 1 && !s->p2p) {
        ncclResult_t r = ncclAllGather(s->d_part_local, s->d_part_all, sizeof(Partial), ncclUint8,
                                       s->comm, stream);
        if (r != ncclSuccess) {
            fprintf(stderr, "[ark_cuda] ncclAllGather failed: %s\n", ncclGetErrorString(r));
            return ARK_E_NCCL;
        }
    }
    if (ev) ARK_RECORD(ev[2], stream);
    const bool pdl = s->pdl && !ev && (s->cfg.world_size == 1 || s->p2p);
    if (w32) ARK_CUDA_TRY(launch_pass2(s->pass2_w32, s->blocks2w, stream, pdl, p, w16, m, v));
    else if (gather)
        ARK_CUDA_TRY(launch_pass2(s->pass2_gather, s->blocks2g, stream, pdl, p, w16, m, v));
    else ARK_CUDA_TRY(launch_pass2(s->pass2, s->blocks2, stream, pdl, p, w16, m, v));
    if (ev) ARK_RECORD(ev[3], stream);
    return ARK_OK;
}

void drop_graph(ark_opt_state* s, int slot) {
    if (s->gexec[slot]) cudaGraphExecDestroy(s->gexec[slot]);
    if (s->gsrc[slot]) cudaGraphDestroy(s->gsrc[slot]);
    s->gexec[slot] = nullptr;
    s->gsrc[slot] = nullptr;
}

// Capture one step into graph slot 0 (plain) or 1 (with event-record nodes
// on placeholder events, whose nodes are then located for retargeting).
int capture_graph(ark_opt_state* s, int slot, uint16_t* w16, const uint16_t* g16, float* m,
                  float* v, float* w32, bool gather) {
    const bool profiled = slot & 1, reduce = slot >= 2;
    drop_graph(s, slot);
    // capture on a private stream (the legacy default stream cannot be
    // captured); the graph is then launched on the state's stream
    if (!s->capture_stream)
        ARK_CUDA_TRY(cudaStreamCreateWithFlags(&s->capture_stream, cudaStreamNonBlocking));
    if (profiled && !s->ph_ev[0])
        for (auto& e : s->ph_ev) ARK_CUDA_TRY(cudaEventCreate(&e));
    cudaGraph_t g = nullptr;
    ARK_CUDA_TRY(cudaStreamBeginCapture(s->capture_stream, cudaStreamCaptureModeThreadLocal));
    const int rc = enqueue_step(s, s->capture_stream, w16, g16, m, v, w32,
                                profiled ? s->ph_ev : nullptr, true, reduce, gather);
    const cudaError_t e = cudaStreamEndCapture(s->capture_stream, &g);
    if (rc != ARK_OK) {
        if (g) cudaGraphDestroy(g);
        return rc;
    }
    ARK_CUDA_TRY(e);
    s->gsrc[slot] = g;
    if (profiled) {
        cudaGraphNode_t* evn = s->ev_node[slot >> 1];
        size_t nn = 0;
        ARK_CUDA_TRY(cudaGraphGetNodes(g, nullptr, &nn));
        std::vector<cudaGraphNode_t> nodes(nn);
        ARK_CUDA_TRY(cudaGraphGetNodes(g, nodes.data(), &nn));
        for (cudaGraphNode_t node : nodes) {
            cudaGraphNodeType t;
            ARK_CUDA_TRY(cudaGraphNodeGetType(node, &t));
            if (t != cudaGraphNodeTypeEventRecord) continue;
            cudaEvent_t ev = nullptr;
            ARK_CUDA_TRY(cudaGraphEventRecordNodeGetEvent(node, &ev));
            for (int j = 0; j < 4; ++j)
                if (ev == s->ph_ev[j]) evn[j] = node;
        }
        for (int j = 0; j < 4; ++j)
            if (!evn[j]) return ARK_E_CUDA;
    }
    ARK_CUDA_TRY(cudaGraphInstantiate(&s->gexec[slot], g, 0));
    const void* key[6] = {w16, g16, m, v, w32, gather ? s->wbuf : nullptr};
    memcpy(s->gkey[slot], key, sizeof(key));
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
    // pass-1 variant: vectors in flight per thread x resident blocks per SM x
    // load path.  B200 sweeps (EKO and EKO/8 shards): 4 x 6 through the
    // non-coherent path for large shards (pass 2 after it also runs faster:
    // EKO step 0.912 ms vs 0.926 ms for 8 x 4 through L2-only loads), 4 x 6
    // L2-only below 100M params
    const int nvar1 = (int)(sizeof(kPass1Variants) / sizeof(kPass1Variants[0]));
    int var = cfg->n < 100000000ull ? 1 : 7;
    if (const char* e = getenv("ARK_PASS1_VARIANT")) var = atoi(e);
    if (var < 0 || var >= nvar1) var = 1;
    // pass 2 as a programmatic dependent of pass 1: its prologue overlaps
    // pass 1's tail.  B200, ms per step without / with: EKO/8 shard 0.1214 /
    // 0.1188, EKO/2 shards on 2 GPUs 0.4731 / 0.4717, full EKO 0.9007 /
    // 0.9018 (within run-to-run spread)
    s->pdl = true;
    if (const char* e = getenv("ARK_PDL")) s->pdl = atoi(e) != 0;
    const bool keep = (cfg->flags & ARK_OPT_COMPAT_GAMMA_FINAL_UNSCALED) &&
                      cfg->keep_scaled_hi > cfg->keep_scaled_lo;
    s->pass1 = keep ? kPass1Variants[var].fn_keep : kPass1Variants[var].fn;
    s->blocks1 = streaming_grid(reinterpret_cast<const void*>(s->pass1), kThreads, 0,
                                (cfg->n >> 3) / kPass1Variants[var].unroll + 1);
    s->pass1r = keep ? pass1_reduce_for<true>(cfg->world_size)
                     : pass1_reduce_for<false>(cfg->world_size);
    s->blocks1r = streaming_grid(reinterpret_cast<const void*>(s->pass1r), kThreads, 0,
                                 (cfg->n >> 3) + 1);
    const int W = cfg->world_size;
    s->timeout_ns = (uint64_t)(cfg->wait_timeout_ms ? cfg->wait_timeout_ms : 5000u) * 1000000ull;
    const int nblk = s->blocks1 > s->blocks1r ? s->blocks1 : s->blocks1r;
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
    const size_t o_tk = take(sizeof(unsigned int) * 2);
    const size_t o_pl = take(sizeof(Partial));
    const size_t o_pa = take(sizeof(Partial) * W);
    const size_t o_vd = take(sizeof(unsigned long long));
    const size_t o_lb = take(sizeof(unsigned long long));
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
    s->d_verdict = reinterpret_cast<unsigned long long*>(base + o_vd);
    s->d_logits_bad = reinterpret_cast<unsigned long long*>(base + o_lb);
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
    if (W > 1 && !(cfg->flags & ARK_OPT_NCCL_EXCHANGE)) {
        rc = setup_p2p(s);
        if (rc) {
            ark_cuda_opt_destroy(s);
            return rc;
        }
        if (!s->p2p) teardown_p2p(s);   // every rank agreed to use the NCCL exchange
    }
    // Who reduces pass 1's block partials into the rank partial.  Below 100M
    // params per shard every pass-2 block does (pass 1 then has no serial
    // last-block tail: 8-way EKO shard on B200, step 0.1265 -> 0.1211 ms);
    // above, pass 1's last block does, overlapped by pass 2's prologue (the
    // pass-2 reduction widens the update kernel's register allocation, 120
    // -> 125, and measured 0.4 % slower on the 1.3B step).  The NCCL
    // exchange always needs it in pass 1.  ARK_P1_LAST=0/1 forces either.
    s->p1_last = cfg->n >= 100000000ull;
    if (const char* e = getenv("ARK_P1_LAST")) s->p1_last = atoi(e) != 0;
    if (W > 1 && !s->p2p) s->p1_last = true;
    const int red = s->p1_last ? 0 : 1;
    // pass 2: 2 groups in flight x 2 blocks/SM (<= 128 registers) for large
    // shards, 1 group x 3 blocks/SM below 100M params (shorter tail); from the
    // B200 sweeps at the EKO, EKO/4 and EKO/8 shard sizes
    int var2 = cfg->n < 100000000ull ? 1 : 4;
    if (const char* e = getenv("ARK_PASS2_VARIANT")) var2 = atoi(e);
    if (var2 < 0 || var2 >= (int)(sizeof(kPass2Variants) / sizeof(kPass2Variants[0]))) var2 = 0;
    s->pass2 = kPass2Variants[var2].fn[red][keep];
    s->blocks2 = streaming_grid(reinterpret_cast<const void*>(s->pass2), kThreads, 0,
                                (cfg->n >> 3) / kPass2Variants[var2].unroll + 1);
    // with the FP32 weight copy: 2 groups x 2 blocks/SM (<= 128 registers)
    // is the fastest shape on B200 (EKO: 1.161 ms vs 1.237 ms for 1 x 3)
    int varw = 4;
    if (const char* e = getenv("ARK_PASS2W_VARIANT")) varw = atoi(e);
    if (varw < 0 || varw >= (int)(sizeof(kPass2Variants) / sizeof(kPass2Variants[0]))) varw = 4;
    s->pass2_w32 = kPass2Variants[varw].fn_w32[red][keep];
    s->blocks2w = streaming_grid(reinterpret_cast<const void*>(s->pass2_w32), kThreads, 0,
                                 (cfg->n >> 3) / kPass2Variants[varw].unroll + 1);
    // fused weight all-gather: the plain kernel's shape by shard size (or
    // by index through ARK_PASS2G_SHAPE: 0 = 1 group x 3 blocks/SM, 1 = 2 x 2)
    int shape_g = cfg->n < 100000000ull ? 0 : 1;
    if (const char* e = getenv("ARK_PASS2G_SHAPE")) shape_g = atoi(e) ? 1 : 0;
    s->pass2_gather = kPass2Gather[shape_g][red][keep];
    s->blocks2g = streaming_grid(reinterpret_cast<const void*>(s->pass2_gather), kThreads, 0,
                                 (cfg->n >> 3) / (shape_g ? 2 : 1) + 1);
    *out = s;
    return ARK_OK;
}

static int run_step(ark_opt_state* s, uint16_t* w16, const uint16_t* g16, float* m, float* v,
                    float* w32, bool reduce, bool gather = false) {
    if (!s) return ARK_E_INVALID_ARG;
    if (s->cfg.n && (!w16 || !g16 || !m || !v)) return ARK_E_INVALID_ARG;
    if (!aligned16(w16) || !aligned16(g16) || !aligned16(m) || !aligned16(v) || !aligned16(w32))
        return ARK_E_MISALIGNED;
    if (reduce) {
        if (!s->gbuf) return ARK_E_INVALID_ARG;          // no ark_cuda_opt_grad_buffer yet
        if (s->cfg.shard_offset + s->cfg.n > s->gbuf_n) return ARK_E_INVALID_ARG;
        if ((s->cfg.shard_offset & 7u) != 0) return ARK_E_MISALIGNED;
    }
    if (gather) {
        if (!s->wbuf) return ARK_E_INVALID_ARG;          // no ark_cuda_opt_weight_buffer yet
        if (s->cfg.shard_offset + s->cfg.n > s->wbuf_n) return ARK_E_INVALID_ARG;
        if ((s->cfg.shard_offset & 7u) != 0) return ARK_E_MISALIGNED;
        if (w32) return ARK_E_UNSUPPORTED;               // one option or the other
    }
    DeviceGuard dg(s->device);
    const bool profile = s->prof_used < s->prof_cap;
    cudaEvent_t* ev = profile ? &s->prof_events[4 * s->prof_used] : nullptr;
    if (!(s->cfg.flags & ARK_OPT_USE_GRAPH)) {
        const int rc = enqueue_step(s, s->stream, w16, g16, m, v, w32, ev, false, reduce, gather);
        if (rc == ARK_OK && profile) s->prof_used++;
        return rc;
    }
    const int slot = (reduce ? 2 : 0) + (profile ? 1 : 0);
    const void* key[6] = {w16, g16, m, v, w32, gather ? s->wbuf : nullptr};
    if (!s->gexec[slot] || memcmp(key, s->gkey[slot], sizeof(key)) != 0) {
        const int rc = capture_graph(s, slot, w16, g16, m, v, w32, gather);
        if (rc != ARK_OK) {
            drop_graph(s, slot);
            return rc;
        }
    }
    if (profile)   // this replay records into this step's profiling events
        for (int j = 0; j < 4; ++j)
            ARK_CUDA_TRY(cudaGraphExecEventRecordNodeSetEvent(s->gexec[slot],
                                                              s->ev_node[slot >> 1][j], ev[j]));
    ARK_CUDA_TRY(cudaGraphLaunch(s->gexec[slot], s->stream));
    if (profile) s->prof_used++;
    return ARK_OK;
}

int ark_cuda_opt_step(ark_opt_state* s, uint16_t* w16, const uint16_t* g16, float* m, float* v) {
    return run_step(s, w16, g16, m, v, nullptr, false);
}

int ark_cuda_opt_step_reduce(ark_opt_state* s, uint16_t* w16, uint16_t* g16_shard, float* m,
                             float* v) {
    return run_step(s, w16, g16_shard, m, v, nullptr, true);
}

int ark_cuda_opt_step_ex(ark_opt_state* s, uint16_t* w16, uint16_t* g16, float* m, float* v,
                         float* w32_out, uint32_t options) {
    if (options & ~(ARK_STEP_REDUCE | ARK_STEP_GATHER_WEIGHTS)) return ARK_E_INVALID_ARG;
    return run_step(s, w16, g16, m, v, w32_out, (options & ARK_STEP_REDUCE) != 0,
                    (options & ARK_STEP_GATHER_WEIGHTS) != 0);
}

int ark_cuda_opt_grad_buffer(ark_opt_state* s, uint64_t n_full, uint16_t** out) {
    if (!s || !out || n_full == 0) return ARK_E_INVALID_ARG;
    *out = nullptr;
    if (s->cfg.shard_offset + s->cfg.n > n_full) return ARK_E_INVALID_ARG;
    DeviceGuard dg(s->device);
    teardown_grads(s);
    const int rc = make_shared(s, n_full * sizeof(uint16_t), s->gbuf, s->gpeer, s->d_gsrc);
    if (rc) return rc;
    s->gbuf_n = n_full;
    *out = static_cast<uint16_t*>(s->gbuf);
    return ARK_OK;
}

int ark_cuda_opt_weight_buffer(ark_opt_state* s, uint64_t n_full, uint16_t** out) {
    if (!s || !out || n_full == 0) return ARK_E_INVALID_ARG;
    *out = nullptr;
    if (s->cfg.shard_offset + s->cfg.n > n_full) return ARK_E_INVALID_ARG;
    DeviceGuard dg(s->device);
    teardown_weights(s);
    const int rc = make_shared(s, n_full * sizeof(uint16_t), s->wbuf, s->wpeer, s->d_wdst);
    if (rc) return rc;
    s->wbuf_n = n_full;
    *out = static_cast<uint16_t*>(s->wbuf);
    return ARK_OK;
}

int ark_cuda_opt_zero_grads(ark_opt_state* s) {
    if (!s) return ARK_E_INVALID_ARG;
    if (!s->gbuf) return ARK_E_INVALID_ARG;   // no ark_cuda_opt_grad_buffer yet
    DeviceGuard dg(s->device);
    ARK_CUDA_TRY(cudaMemsetAsync(s->gbuf, 0, s->gbuf_n * sizeof(uint16_t), s->stream));
    return ARK_OK;
}

int ark_cuda_opt_weights_wait(ark_opt_state* s) {
    if (!s) return ARK_E_INVALID_ARG;
    if (!s->wbuf) return ARK_E_INVALID_ARG;   // no ark_cuda_opt_weight_buffer yet
    if (s->cfg.world_size == 1) return ARK_OK;   // stream order suffices
    DeviceGuard dg(s->device);
    const StepParams p = make_params(s, nullptr);
    weights_wait_kernel<<<1, 32, 0, s->stream>>>(p);
    ARK_CUDA_TRY(cudaGetLastError());
    return ARK_OK;
}

int ark_cuda_opt_logits_check(ark_opt_state* s, float* logits_grad, uint64_t n) {
    if (!s || (n && !logits_grad)) return ARK_E_INVALID_ARG;
    if (n == 0) return ARK_OK;
    DeviceGuard dg(s->device);
    const int blocks = streaming_grid(reinterpret_cast<const void*>(logits_kernel), kThreads, 0,
                                      (n >> 2) / kLogitsU + 1);
    logits_kernel<<<blocks, kThreads, 0, s->stream>>>(logits_grad, n, s->d_state,
                                                      s->d_logits_bad);
    ARK_CUDA_TRY(cudaGetLastError());
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
    *steps = k;
    s->prof_cap = 0;
    s->prof_used = 0;
    return ARK_OK;
}

}  // extern "C"

int ark::opt_view(const ark_opt_state* s, OptView* out) {
    if (!s || !out) return ARK_E_INVALID_ARG;
    out->device = s->device;
    out->rank = s->cfg.rank;
    out->world = s->cfg.world_size;
    out->n = s->cfg.n;
    out->shard_offset = s->cfg.shard_offset;
    out->scale_init = s->cfg.scale_init;
    return ARK_OK;
}

extern "C" {

int ark_cuda_opt_geometry(ark_opt_state* s, uint32_t* b1, uint32_t* b2, uint32_t* threads) {
    if (!s) return ARK_E_INVALID_ARG;
    if (b1) *b1 = (uint32_t)s->blocks1;
    if (b2) *b2 = (uint32_t)s->blocks2;
    if (threads) *threads = (uint32_t)kThreads;
    return ARK_OK;
}

int ark_cuda_opt_destroy(ark_opt_state* s) {
    if (!s) return ARK_OK;
    DeviceGuard dg(s->device);
    cudaStreamSynchronize(s->stream);
    for (int slot = 0; slot < 4; ++slot) drop_graph(s, slot);
    teardown_grads(s);
    teardown_weights(s);
    for (cudaEvent_t e : s->ph_ev)
        if (e) cudaEventDestroy(e);
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
