/*
 * ark_opt.h -- C ABI of the B200 optimizer library (libark_cuda.so / .a).
 *
 * Drop-in for ARK's native optimizer kernels (proyecto_ark/ark01, linked
 * today as libark_asm.a by build.rs:59-74) plus a fused, asynchronous
 * whole-step API.  Plain C: pointers, sizes and integer status codes only.
 *
 * Pointer convention: every buffer argument is CUDA DEVICE memory (or
 * managed memory) unless the name says host.  The caller owns all buffers;
 * no entry point frees a caller buffer.
 */
#ifndef ARK_OPT_H
#define ARK_OPT_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define ARK_API __attribute__((visibility("default")))
#else
#define ARK_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define ARK_OPT_ABI_VERSION 2u

/* ---- status codes (0 = success; negative = error) --------------------- */
#define ARK_OK               0
#define ARK_E_INVALID_ARG   -1  /* null pointer, bad size or bad config value */
#define ARK_E_MISALIGNED    -2  /* a buffer is not 16-byte aligned where required */
#define ARK_E_CUDA          -3  /* a CUDA runtime call failed */
#define ARK_E_NCCL          -4  /* an NCCL call failed */
#define ARK_E_TIMEOUT       -5  /* a bounded device-side wait gave up */
#define ARK_E_EARLY_STOP    -6  /* more than max_consecutive_nans overflow steps in a row */
#define ARK_E_NO_DEVICE     -7  /* no CUDA device / wrong architecture */
#define ARK_E_UNSUPPORTED   -8  /* feature not built into this library */

/* ======================================================================
 * 1. Legacy entry points -- same names and signatures as the symbols
 *    proyecto_ark/ark01 binds today.  Pointers are device pointers.
 *    Each call is enqueued on the legacy default CUDA stream (or the stream
 *    given to ark_cuda_legacy_set_stream) and, by default, waited for
 *    before returning, so the void/no-error contract of the reference
 *    holds.  Failures are recorded for ark_cuda_last_error() and
 *    reported once on stderr.
 * ====================================================================== */

/* Replaces _ark_asm_adam_step_f16 (asm/opti.s:192-360; Rust declarations
 * src/optimizer.rs:20-23 and src/ffi.rs:105-108).  AdamW with bias
 * correction and decoupled weight decay; FP16 weights updated in place,
 * FP32 grads read-only, FP32 moments in place.  t == 0 is treated as 1.
 * Bit-identical to the reference for every input (IEEE single rounding per
 * operation, the same operation order, fused m/v updates). */
ARK_API void ark_asm_adam_step_f16(uint16_t* w, const float* g, float* m, float* v, uint64_t n,
                           float lr, float beta1, float beta2, float eps, float wd,
                           uint32_t t);

/* Replaces _ark_asm_adam_step (asm/opti.s:20-177; src/ffi.rs:98-101):
 * the same update with FP32 weights. */
ARK_API void ark_asm_adam_step(float* w, const float* g, float* m, float* v, uint64_t n, float lr,
                       float beta1, float beta2, float eps, float wd, uint32_t t);

/* Replaces _ark_asm_grad_clip (asm/opti.s:369-432; src/ffi.rs:111-115).
 * Returns the pre-clip L2 norm; scales grads in place by threshold/norm iff
 * norm > threshold (a NaN norm or threshold never scales).  The norm is
 * float(sqrt(sum in double of x*x)) -- accurate to ~1e-13 relative -- where
 * the reference's four-lane f32 fold loses up to several percent at LLM
 * tensor sizes.  ark_cuda_set_compat(ARK_COMPAT_CLIP_NEON_FOLD) reproduces
 * the reference's fold bit for bit instead (serial; slow for large n). */
ARK_API float ark_asm_grad_clip(float* grads, uint64_t n, float threshold);

/* Replaces _ark_quant_f32_to_f16 (asm/kern.s:879-913; src/ffi.rs:88):
 * round-to-nearest-even, subnormals kept, overflow to +-inf, NaN to NaN. */
ARK_API void ark_quant_f32_to_f16(const float* src, uint16_t* dst, uint64_t n);

/* Replaces _ark_dequant_f16_to_f32 (asm/kern.s:835-869; src/ffi.rs:92):
 * exact widening. */
ARK_API void ark_dequant_f16_to_f32(const uint16_t* src, float* dst, uint64_t n);

/* No counterpart in the reference.  The same clip as ark_asm_grad_clip
 * (same kernels, same grid, the ARK_COMPAT_CLIP_NEON_FOLD setting honoured:
 * the same norm and grads bit for bit), for callers that cannot allocate
 * device memory: a process whose HBM is taken up front by its own pool
 * allocator, where a cudaMalloc of even a few KiB fails, and code paths
 * that must not stall other work on the device, which cudaFree does.
 * ark_asm_grad_clip allocates its scratch on first use; this entry point
 * calls no cudaMalloc, cudaFree or allocating routine.  Its scratch is a
 * static 16.5 KiB array in the library's device image (one per GPU that
 * loads the library, held until exit) with room for 2048 thread-block
 * partial sums (a B200 launches at most 1184); a launch that needs more is
 * rejected with ARK_E_UNSUPPORTED.  grads: device, scaled in place;
 * norm_out: a device float that receives the pre-clip norm; enqueued on
 * cuda_stream (NULL: the default stream), nothing is waited for.  The first
 * call on a device looks up the array's device address
 * (cudaGetSymbolAddress) and, under CUDA's default lazy module loading,
 * loads the library's device code, which takes device memory: make that
 * first call (or set CUDA_MODULE_LOADING=EAGER) before the caller's pool
 * reserves the HBM, and before any stream capture.  The address is kept for
 * the life of the process: a cudaDeviceReset after the first call is not
 * supported.  All calls share the array: calls that overlap on the GPU
 * (other streams, other threads) race. */
ARK_API int ark_cuda_grad_clip_noalloc(float* grads, uint64_t n, float threshold,
                                       float* norm_out, void* cuda_stream);

/* ---- controls for the legacy entry points (no reference counterpart;
 *      the reference has no error channel and no streams) ------------- */
#define ARK_COMPAT_CLIP_NEON_FOLD  0x1u  /* ark_asm_grad_clip: reference f32 fold */

ARK_API int         ark_cuda_last_error(void);          /* last legacy status on this thread */
ARK_API const char* ark_cuda_strerror(int status);
ARK_API int         ark_cuda_set_compat(uint32_t flags);
ARK_API int         ark_cuda_legacy_set_stream(void* cuda_stream);  /* NULL: default stream */
ARK_API int         ark_cuda_legacy_set_async(int async);           /* 1: do not wait per call */
ARK_API int         ark_cuda_legacy_sync(void);                     /* wait for queued legacy calls */
ARK_API uint32_t    ark_cuda_abi_version(void);

/* ======================================================================
 * 2. Fused whole-step API.
 *
 * Replaces, in one asynchronous call with no host synchronisation:
 *   src/training.rs:289-305  finite check over all grads + overflow backoff,
 *   src/training.rs:307-308  unscale by 1/loss_scale (:133-146),
 *   src/optimizer.rs:171-228 step_all: step += 1, lr, global L2 clip
 *                            (clip_all_grads :126-168), AdamW per tensor
 *                            with per-tensor weight decay,
 *   src/training.rs:316-326  clean-step counting and scale growth.
 * over one contiguous FLAT shard of FP16 weights / FP16 scaled grads /
 * FP32 moments.  Flat order: the weight-decayed tensors first, so that
 * decay applies to global indices [0, n_decay).
 *
 * Multi-GPU (ZeRO-1): rank r owns a contiguous shard; the only exchange is
 * a 16-byte {sum of squares, non-finite count} per rank, stored straight
 * into the peers' memory over NVLink (by pass 1's last block for shards of
 * 100M params and more, else by the update kernel) and read, with a bounded
 * wait, by the update kernel (or an NCCL all-gather between the kernels,
 * see ARK_OPT_NCCL_EXCHANGE).
 * ====================================================================== */

/* Reproduce the reference's unscale omission for the final RMSNorm gain
 * (training.rs:133-146 skips gamma_final_grad): grads with global index in
 * [keep_scaled_lo, keep_scaled_hi) are NOT divided by the loss scale. */
#define ARK_OPT_COMPAT_GAMMA_FINAL_UNSCALED 0x1u
/* Capture the step (pass 1, exchange, pass 2) in a CUDA graph on first use
 * with a given buffer set and replay it afterwards. */
#define ARK_OPT_USE_GRAPH                   0x2u
/* world_size > 1: exchange the 16-byte rank partials with an NCCL
 * all-gather between the two kernels instead of peer-to-peer stores from
 * the last block of pass 1 (chosen automatically, on every rank, when a
 * rank cannot map its peers' exchange slots). */
#define ARK_OPT_NCCL_EXCHANGE               0x4u

typedef struct ark_opt_cfg {
    uint32_t     abi_version;          /* ARK_OPT_ABI_VERSION */
    int32_t      device;               /* CUDA device of this rank */
    uint64_t     n;                    /* elements in this rank's shard */
    uint64_t     shard_offset;         /* global flat index of shard element 0 */
    uint64_t     n_decay;              /* global indices [0, n_decay) use weight_decay */
    uint64_t     keep_scaled_lo;       /* see ARK_OPT_COMPAT_GAMMA_FINAL_UNSCALED */
    uint64_t     keep_scaled_hi;
    const float* lr_table;             /* HOST array, copied at init: the lr of optimizer
                                          step t is lr_table[min(t, lr_table_len - 1)]
                                          (optimizer.rs:172-173, lr_now :80-92) */
    uint32_t     lr_table_len;         /* >= 1 */
    float        beta1, beta2, eps, weight_decay, grad_clip;
    float        scale_init;           /* training.rs:10 LOSS_SCALE_INIT (256) */
    float        scale_backoff;        /* training.rs:294 (0.5) */
    float        scale_growth;         /* training.rs:320 (2.0) */
    float        scale_min;            /* training.rs:12 LOSS_SCALE_MIN (1) */
    float        scale_max;            /* config.rs:69 loss_scale_max (8192) */
    uint32_t     scale_every;          /* training.rs:13 SCALE_UP_EVERY (2000) */
    uint32_t     max_consecutive_nans; /* training.rs:298 (200) */
    uint32_t     initial_step;         /* Optimizer.step before the first call (resume) */
    uint32_t     flags;                /* ARK_OPT_* */
    int32_t      rank, world_size;
    void*        nccl_comm;            /* ncclComm_t, required when world_size > 1 */
    void*        stream;               /* cudaStream_t every step runs on (NULL: the
                                          legacy default stream) */
    uint32_t     wait_timeout_ms;      /* limit of a device-side wait for a peer's partial
                                          (0: 5000); past it the step is skipped and the
                                          state reports ARK_E_TIMEOUT */
    uint32_t     reserved;
} ark_opt_cfg;

/* Device-resident state, read back by ark_cuda_opt_read_status. */
typedef struct ark_opt_status {
    double   last_sumsq;        /* global sum of squared unscaled grads, last clean step */
    uint64_t skipped_steps;     /* training.rs:57 */
    uint64_t steps_called;      /* steps executed on the device */
    float    loss_scale;        /* scale the NEXT backward must multiply the loss by */
    float    last_norm;         /* pre-clip global L2 norm, last clean step */
    float    last_clip_coef;    /* grad_clip/norm when clipped, else 1 */
    float    last_lr;           /* lr used by the last clean step */
    uint32_t opt_step;          /* Optimizer.step (optimizer.rs:70) */
    uint32_t clean_steps;       /* training.rs:55 */
    uint32_t consecutive_nans;  /* training.rs:57 */
    uint32_t last_overflow;     /* 1 if the last step was skipped */
    uint32_t early_stop;        /* consecutive_nans exceeded the limit */
    int32_t  error;             /* device-side error code (0 = none) */
} ark_opt_status;

typedef struct ark_opt_state ark_opt_state;

/* Allocate the device state and scratch for one shard.  No step runs. */
ARK_API int ark_cuda_opt_init(const ark_opt_cfg* cfg, ark_opt_state** out);

/* Enqueue one optimizer step on the state's stream and return without
 * waiting.  w16, g16, m, v: this rank's shard (cfg.n elements each),
 * 16-byte aligned.  g16 holds the loss-scaled FP16 gradients. */
ARK_API int ark_cuda_opt_step(ark_opt_state* st, uint16_t* w16, const uint16_t* g16, float* m,
                      float* v);

/* The gradient hand-off, for data-parallel ranks: allocate this rank's
 * FULL gradient buffer (n_full FP16 loss-scaled elements, all global
 * indices, zeroed), map every rank's buffer into every other rank
 * (collective: every rank calls it; needs the peer-to-peer exchange slots
 * when world_size > 1).  The backward writes each rank's own gradients
 * there; the library owns the buffer until ark_cuda_opt_destroy. */
ARK_API int ark_cuda_opt_grad_buffer(ark_opt_state* st, uint64_t n_full, uint16_t** g16_full);

/* One optimizer step on the SUM over ranks of every rank's full gradient
 * buffer: replaces the reference's zero-then-accumulate of the backward's
 * gradients (src/memory.rs:338-342, objc/bridge.m:907-949) followed by the
 * optimizer block.  Pass 1 reads this rank's shard range from every rank's
 * buffer over NVLink, sums the FP16 values in FP32 in rank order, rounds
 * once to FP16 into g16_shard (cfg.n elements, this device) and checks /
 * squares the result; pass 2 is the ordinary update.  Each rank's buffer
 * may be overwritten once this step has completed on its stream.
 * cfg.shard_offset must be a multiple of 8. */
ARK_API int ark_cuda_opt_step_reduce(ark_opt_state* st, uint16_t* w16, uint16_t* g16_shard,
                                     float* m, float* v);

/* ark_cuda_opt_step / ark_cuda_opt_step_reduce with options:
 *  - options & ARK_STEP_REDUCE: the reduce-scatter step (g16 receives the
 *    reduced shard), else g16 holds this rank's scaled FP16 grads;
 *  - w32_out (NULL: none; else cfg.n FP32, 16-byte aligned): every step
 *    that updates the weights also writes them widened to FP32, the copy
 *    the forward reads -- replacing the per-step ark_dequant_f16_to_f32 of
 *    every weight tensor (src/training.rs:165-186) by 4 extra bytes per
 *    parameter in pass 2.  A skipped step leaves w16 and w32_out as they
 *    are, so w32_out must be initialised once (dequant) before the first
 *    step. */
#define ARK_STEP_REDUCE 0x1u
/* ARK_STEP_GATHER_WEIGHTS: the ZeRO-1 weight all-gather fused with the
 * update.  Every step that updates the weights also stores the updated
 * shard into every rank's full weight buffer (ark_cuda_opt_weight_buffer)
 * at its global offset, with plain stores over NVLink from the update
 * kernel itself; w16 may be this rank's slice of its own full buffer.  Not
 * combined with w32_out (ARK_E_UNSUPPORTED).  cfg.shard_offset must be a
 * multiple of 8.  Before a rank reads its full buffer (the forward), it
 * calls ark_cuda_opt_weights_wait. */
#define ARK_STEP_GATHER_WEIGHTS 0x2u
ARK_API int ark_cuda_opt_step_ex(ark_opt_state* st, uint16_t* w16, uint16_t* g16, float* m,
                                 float* v, float* w32_out, uint32_t options);

/* The full FP16 weight buffer of this rank for ARK_STEP_GATHER_WEIGHTS
 * (n_full elements, all global indices, zeroed), with every rank's buffer
 * mapped into every other rank (collective: every rank calls it; needs the
 * peer-to-peer exchange slots when world_size > 1).  The consumer is the
 * forward, which reads every weight tensor (objc/bridge.m:630-737 over the
 * shared weight buffers of src/memory.rs:207-236).  The library owns the
 * buffer until ark_cuda_opt_destroy. */
ARK_API int ark_cuda_opt_weight_buffer(ark_opt_state* st, uint64_t n_full, uint16_t** w16_full);

/* Enqueue on the state's stream a bounded wait until every rank's step of
 * the same number has stored its shard into this rank's full weight buffer;
 * work enqueued after it on the stream reads the complete updated weights.
 * Call it after a step made with ARK_STEP_GATHER_WEIGHTS (on every rank):
 * after any other step nothing is published and the wait runs out.  A wait
 * that runs out leaves ARK_E_TIMEOUT in the state.  No-op with world_size 1. */
ARK_API int ark_cuda_opt_weights_wait(ark_opt_state* st);

/* Replaces the logits-gradient block of train_step (src/training.rs:228-245):
 * counts non-finite values of the unscaled FP32 logits gradients
 * (bs x vocab, device, any alignment) and multiplies every element in place
 * by the current device loss scale (x *= loss_scale).  Enqueued on the
 * state's stream, nothing is waited for.  A non-finite value makes the next
 * optimizer step on this state (on every rank) a skipped overflow step:
 * backoff, skipped and consecutive-overflow counts and the early-stop
 * check, no optimizer step -- the same transitions as the reference's
 * early return at :231-237.  Call it once per iteration, before the
 * backward and the step; on a rejected iteration the buffer's contents are
 * unspecified (the reference discards them). */
ARK_API int ark_cuda_opt_logits_check(ark_opt_state* st, float* logits_grad, uint64_t n);

/* Zero this rank's full gradient buffer (ark_cuda_opt_grad_buffer) on the
 * state's stream: ModelWeights::zero_all_grads (src/memory.rs:338-342),
 * called before every backward (src/training.rs:248) for a backward that
 * accumulates with +=.  Safe once the previous step was enqueued: no peer
 * reads this rank's buffer after that step has completed. */
ARK_API int ark_cuda_opt_zero_grads(ark_opt_state* st);

/* Wait for the state's stream and copy the device state out.  Returns
 * ARK_E_EARLY_STOP once the early-stop condition holds (training.rs:298),
 * a device error code if one was raised, else ARK_OK. */
ARK_API int ark_cuda_opt_read_status(ark_opt_state* st, ark_opt_status* out);

/* Overwrite the device state (resume: optimizer.rs:237-313 restores the
 * step count; the loss-scale fields may be restored too). */
ARK_API int ark_cuda_opt_set_status(ark_opt_state* st, const ark_opt_status* in);

/* Asynchronous host->device copy of this rank's scaled FP16 grads on the
 * state's stream (pinned host memory for full speed). */
ARK_API int ark_cuda_opt_upload_grads(ark_opt_state* st, uint16_t* g16_dev, const uint16_t* g16_host,
                              uint64_t n);

/* ZeRO-1 weight all-gather: every rank's updated shard into w16_full
 * (world_size * shard_stride elements, rank r at r * shard_stride).
 * shard_stride >= cfg.n of every rank. */
ARK_API int ark_cuda_allgather_weights(ark_opt_state* st, const uint16_t* w16_shard, uint16_t* w16_full,
                               uint64_t shard_stride);

/* Per-kernel timing with CUDA events on the state's stream for the next
 * max_steps steps (disables graph replay while active); read gives, per
 * step, {pass-1 ms, exchange ms, pass-2 ms}. */
ARK_API int ark_cuda_opt_profile_begin(ark_opt_state* st, uint32_t max_steps);
ARK_API int ark_cuda_opt_profile_read(ark_opt_state* st, float* out_ms, uint32_t capacity,
                              uint32_t* out_steps);

/* Launch geometry actually used (for reporting). */
ARK_API int ark_cuda_opt_geometry(ark_opt_state* st, uint32_t* pass1_blocks, uint32_t* pass2_blocks,
                          uint32_t* threads);

ARK_API int ark_cuda_opt_destroy(ark_opt_state* st);

/* ---- ARK4 checkpoints from device shards (src/io.rs:12-24, 410-671;
 *      rotation and call site src/training.rs:536-604) ------------------
 * tensors: the model tensors in ARK4 file order -- embed, then per layer
 * wq wk wv wo w1 w2 w3 g1 g2, then gamma_final (2 + 9 L entries) -- each
 * with its element count and its offset in the flat index space of the
 * optimizer state.  Every rank calls with its own shard (w16 / m / v, cfg.n
 * elements) and writes or reads only that shard's bytes of the one file;
 * rank 0 also writes the header and a trailer with the loss-scale state
 * (ignored by the reference's reader).  A reader must not start before
 * every writer has returned. */
typedef struct ark_ckpt_tensor {
    uint64_t numel;
    uint64_t flat_offset;
} ark_ckpt_tensor;

/* adam_step is the device optimizer step (optimizer.rs:70). */
ARK_API int ark_cuda_ckpt_save(ark_opt_state* st, const char* path,
                               const ark_ckpt_tensor* tensors, uint32_t n_tensors,
                               uint64_t global_step, const uint16_t* w16, const float* m,
                               const float* v);

/* Reads ARK4 (and ARK3: FP32 weights rounded to FP16, memory.rs:347-377)
 * into this rank's shard and sets the device step to the file's adam_step
 * (optimizer.rs:308).  The loss-scale state is restored from the trailer
 * with ARK_CKPT_RESTORE_SCALE, else reset to cfg.scale_init as the reference
 * does on resume (training.rs:120).  Record headers that do not match the
 * layout are an error (ARK_E_INVALID_ARG), not a silent cold start. */
#define ARK_CKPT_RESTORE_SCALE 0x1u
ARK_API int ark_cuda_ckpt_load(ark_opt_state* st, const char* path,
                               const ark_ckpt_tensor* tensors, uint32_t n_tensors,
                               uint64_t* global_step, uint16_t* w16, float* m, float* v,
                               uint32_t flags);

/* Build the reference lr schedule (optimizer.rs:80-92: linear warmup, then
 * cosine to lr/10 over 800k steps, all in f32) into a host table of
 * len entries, entry t = lr for optimizer step t. */
ARK_API int ark_cuda_lr_schedule(float* table_host, uint32_t len, float lr, uint32_t warmup_steps);

/* ---- NCCL helpers (communicator for ark_opt_cfg.nccl_comm) ------------ */
ARK_API int ark_cuda_nccl_unique_id(void* id_out /* 128 bytes */);
ARK_API int ark_cuda_nccl_comm_init(int world_size, int rank, const void* id /* 128 bytes */,
                            int device, void** comm_out);
ARK_API int ark_cuda_nccl_comm_destroy(void* comm);

/* ======================================================================
 * 3. Seeded synthetic inputs (benchmarks and tests): splitmix64 counter
 *    RNG keyed by (seed, stream, global index) + Irwin-Hall(12) normal.
 *    kind 0: fp16(sigma*z*mult), heavy_every>0 multiplies one element in
 *    heavy_every (by hash) by heavy_mult before rounding.
 * ====================================================================== */
ARK_API int ark_synth_f16(uint16_t* out, uint64_t n, uint64_t offset, uint64_t seed, uint64_t stream,
                  float sigma, float mult, uint32_t heavy_every, float heavy_mult,
                  void* cuda_stream);
/* fp32 sigma*z, or (sigma*z)^2 when square != 0. */
ARK_API int ark_synth_f32(float* out, uint64_t n, uint64_t offset, uint64_t seed, uint64_t stream,
                  float sigma, int square, void* cuda_stream);

#ifdef __cplusplus
}
#endif
#endif /* ARK_OPT_H */
