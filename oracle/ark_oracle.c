/*
 * ark_oracle.c -- CPU restatement of ARK's optimizer hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * library in ark_b200/csrc.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / --impl reference legs of bench.py load it.  Nothing in the
 * product path calls it, and the product never falls back to it.
 *
 * Pinning: the element-wise kernels (AdamW f16/f32, grad clip, quant/dequant)
 * are checked bit-for-bit against golden vectors produced by executing the
 * reference's own assembly text (proyecto_ark/ark01/asm/opti.s and
 * asm/kern.s) in an instruction-level AArch64 emulator
 * (tests/golden/a64emu.py, fixtures in tests/golden/).  The loss-scale state
 * machine (Rust, training.rs) cannot be executed here (no Rust toolchain); it
 * is pinned by the scale progression the reference published from its own
 * training logs (CHANGELOG.md:120-130) and otherwise restated line by line.
 *
 * Build: oracle/Makefile (gcc -O2 -ffp-contract=off -fno-fast-math, SSE
 * scalar math, so every f32 operation below rounds exactly once, as on the
 * reference's NEON/FP units with the default FPCR: RNE, no flush-to-zero).
 *
 * Reference files cited as path:line relative to proyecto_ark/ark01/.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define ORK_API __attribute__((visibility("default")))

/* ------------------------------------------------------------------------ */
/* FP16 <-> FP32 (kern.s:835-913 fcvtl / fcvtn, opti.s:279,307,318,345)      */
/* ------------------------------------------------------------------------ */

static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* Exact widening of an IEEE binary16 value (fcvtl / fcvt s,h). */
ORK_API float ork_h2f(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1Fu;
    uint32_t man = h & 0x3FFu;
    if (exp == 0x1Fu) {                       /* inf / NaN: payload kept, quiet bit forced */
        if (man == 0) return u2f(sign | 0x7F800000u);
        return u2f(sign | 0x7FC00000u | (man << 13));
    }
    if (exp == 0) {
        if (man == 0) return u2f(sign);
        /* subnormal: man * 2^-24, exact in binary32 */
        float f = (float)man * 0x1p-24f;
        return sign ? -f : f;
    }
    return u2f(sign | ((exp + 112u) << 23) | (man << 13));
}

/* Round-to-nearest-even narrowing to binary16 (fcvtn / fcvt h,s with the
 * default FPCR): subnormal results kept, overflow to +-inf, NaN stays NaN
 * (quiet bit set, top payload bits kept). */
ORK_API uint16_t ork_f2h(float f) {
    uint32_t u = f2u(f);
    uint16_t sign = (uint16_t)((u >> 16) & 0x8000u);
    uint32_t exp = (u >> 23) & 0xFFu;
    uint32_t man = u & 0x7FFFFFu;
    if (exp == 0xFFu) {
        if (man == 0) return (uint16_t)(sign | 0x7C00u);
        return (uint16_t)(sign | 0x7E00u | (man >> 13));
    }
    /* value = 1.man * 2^(exp-127); binary16 normal range exp16 = exp-112 in [1,30] */
    int32_t e = (int32_t)exp - 127;
    if (e > 15) return (uint16_t)(sign | 0x7C00u);
    uint32_t mant24 = (exp == 0) ? man : (man | 0x800000u);   /* 24-bit significand */
    int32_t e_eff = (exp == 0) ? -126 : e;
    /* target: integer q = round(|f| / 2^-24) if subnormal range, else normal */
    if (e_eff < -14) {
        /* binary16 subnormal (or zero): quantum 2^-24.  |f| = mant24 * 2^(e_eff-23) */
        int32_t shift = -24 - (e_eff - 23);     /* bits to drop, >= 1 */
        if (shift > 25) return sign;           /* below half the smallest subnormal */
        uint32_t q = mant24 >> shift;
        uint32_t rem = mant24 & ((1u << shift) - 1u);
        uint32_t half = 1u << (shift - 1);
        if (rem > half || (rem == half && (q & 1u))) q++;
        return (uint16_t)(sign | q);           /* q may carry into the normal range: correct encoding */
    }
    /* normal: keep 11 bits of mant24, drop 13 */
    uint32_t q = mant24 >> 13;
    uint32_t rem = mant24 & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) q++;
    uint32_t e16 = (uint32_t)(e_eff + 15);
    if (q == 0x800u) { q = 0x400u; e16++; }
    if (e16 >= 31u) return (uint16_t)(sign | 0x7C00u);
    return (uint16_t)(sign | (e16 << 10) | (q & 0x3FFu));
}

/* _ark_dequant_f16_to_f32 (kern.s:835-869) */
ORK_API void ork_dequant_f16_to_f32(const uint16_t* src, float* dst, uint64_t n) {
    for (uint64_t i = 0; i < n; ++i) dst[i] = ork_h2f(src[i]);
}

/* _ark_quant_f32_to_f16 (kern.s:879-913) */
ORK_API void ork_quant_f32_to_f16(const float* src, uint16_t* dst, uint64_t n) {
    for (uint64_t i = 0; i < n; ++i) dst[i] = ork_f2h(src[i]);
}

/* ------------------------------------------------------------------------ */
/* AdamW (opti.s:20-177 FP32 weights, opti.s:192-360 FP16 weights)           */
/* ------------------------------------------------------------------------ */

typedef struct {
    float b1, b2, omb1, omb2, eps, lr_eff, decay;
} ork_adam_k;

/* Per-call scalars, opti.s:210-271 (identical to :38-103). */
ORK_API void ork_adam_scalars(float lr, float b1, float b2, float eps, float wd,
                              uint32_t t, ork_adam_k* k) {
    if (t == 0) t = 1;                                  /* :211-212 cinc */
    float decay = 1.0f - lr * wd;                       /* :219-221 fmul, fsub */
    float p = 1.0f, base = b1;                          /* :223-237 binary exponentiation */
    for (uint32_t e = t; e; e >>= 1) { if (e & 1u) p = p * base; base = base * base; }
    float bc1 = 1.0f - p;
    p = 1.0f; base = b2;                                /* :239-253 */
    for (uint32_t e = t; e; e >>= 1) { if (e & 1u) p = p * base; base = base * base; }
    float bc2 = 1.0f - p;
    float lr_eff = sqrtf(bc2);                          /* :256-258 fsqrt, fdiv, fmul */
    lr_eff = lr_eff / bc1;
    lr_eff = lr_eff * lr;
    k->b1 = b1; k->b2 = b2;
    k->omb1 = 1.0f - b1;                                /* :263-265 */
    k->omb2 = 1.0f - b2;                                /* :266-268 */
    k->eps = eps; k->lr_eff = lr_eff; k->decay = decay;
}

/* One element, opti.s:285-304 (vector) == :324-343 (tail). */
static inline float ork_adam_elem(float w32, float g, float* m, float* v, const ork_adam_k* k) {
    float mm = *m * k->b1;                              /* fmul */
    mm = fmaf(k->omb1, g, mm);                          /* fmla (fused) */
    float vv = *v * k->b2;                              /* fmul */
    float gg = g * g;                                   /* fmul */
    vv = fmaf(k->omb2, gg, vv);                         /* fmla (fused) */
    float den = sqrtf(vv);                              /* fsqrt */
    den = den + k->eps;                                 /* fadd */
    float upd = mm / den;                               /* fdiv */
    upd = upd * k->lr_eff;                              /* fmul */
    float w = w32 * k->decay;                           /* fmul */
    w = w - upd;                                        /* fsub (not fused) */
    *m = mm; *v = vv;
    return w;
}

/* _ark_asm_adam_step_f16 (opti.s:192-360) */
ORK_API void ork_adam_step_f16(uint16_t* w, const float* g, float* m, float* v, uint64_t n,
                               float lr, float b1, float b2, float eps, float wd, uint32_t t) {
    ork_adam_k k; ork_adam_scalars(lr, b1, b2, eps, wd, t, &k);
    for (uint64_t i = 0; i < n; ++i)
        w[i] = ork_f2h(ork_adam_elem(ork_h2f(w[i]), g[i], &m[i], &v[i], &k));
}

/* _ark_asm_adam_step (opti.s:20-177) */
ORK_API void ork_adam_step_f32(float* w, const float* g, float* m, float* v, uint64_t n,
                               float lr, float b1, float b2, float eps, float wd, uint32_t t) {
    ork_adam_k k; ork_adam_scalars(lr, b1, b2, eps, wd, t, &k);
    for (uint64_t i = 0; i < n; ++i) w[i] = ork_adam_elem(w[i], g[i], &m[i], &v[i], &k);
}

/* ------------------------------------------------------------------------ */
/* Sums of squares                                                          */
/* ------------------------------------------------------------------------ */

/* Neumaier (compensated) accumulation of exact double squares: the result is
 * the exact sum to ~2^-100 relative, i.e. the correctly rounded double for
 * every input the tests use.  This is the "exact f64 norm" the parity
 * tolerance (1e-5 relative) is stated against. */
typedef struct { double s, c; } ork_acc;
static inline void acc_add(ork_acc* a, double x) {
    double t = a->s + x;
    if (!isfinite(t)) { a->s = t; return; }      /* inf/NaN: the plain sum is the answer */
    if (fabs(a->s) >= fabs(x)) a->c += (a->s - t) + x; else a->c += (x - t) + a->s;
    a->s = t;
}
static inline double acc_value(const ork_acc* a) { return isfinite(a->s) ? a->s + a->c : a->s; }

ORK_API double ork_sumsq_f32_exact(const float* g, uint64_t n) {
    ork_acc a = {0.0, 0.0};
    for (uint64_t i = 0; i < n; ++i) { double x = (double)g[i]; acc_add(&a, x * x); }
    return acc_value(&a);
}

/* The norm expression used by every accurate path: round the exact sum to
 * double, take a double sqrt, round to float. */
ORK_API float ork_norm_from_sumsq(double s) { return (float)sqrt(s); }

/* _ark_asm_grad_clip (opti.s:369-432), literal order: four f32 lanes each
 * accumulating fma(x,x,acc) over i = 4k+lane (:383-389), pairwise faddp
 * reduce (a0+a1)+(a2+a3) (:391-392), sequential fmadd tail (:393-398),
 * fsqrt (:400); scale iff norm > threshold as an ordered compare (b.le is
 * taken on unordered, :402-403), s = thr/norm (:405), x *= s (:410-424). */
ORK_API float ork_grad_clip_neon(float* g, uint64_t n, float thr) {
    float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
    uint64_t i = 0;
    for (; i + 4 <= n; i += 4) {
        a0 = fmaf(g[i + 0], g[i + 0], a0); a1 = fmaf(g[i + 1], g[i + 1], a1);
        a2 = fmaf(g[i + 2], g[i + 2], a2); a3 = fmaf(g[i + 3], g[i + 3], a3);
    }
    float s = (a0 + a1) + (a2 + a3);
    for (; i < n; ++i) s = fmaf(g[i], g[i], s);
    float norm = sqrtf(s);
    if (norm > thr) {
        float sc = thr / norm;
        for (uint64_t j = 0; j < n; ++j) g[j] = g[j] * sc;
    }
    return norm;
}

/* Same contract as _ark_asm_grad_clip, but the norm is the accurate one
 * (exact sum of squares); the B200 library's default legacy clip follows
 * this definition. */
ORK_API float ork_grad_clip_exact(float* g, uint64_t n, float thr) {
    float norm = ork_norm_from_sumsq(ork_sumsq_f32_exact(g, n));
    if (norm > thr) {
        float sc = thr / norm;
        for (uint64_t j = 0; j < n; ++j) g[j] = g[j] * sc;
    }
    return norm;
}

/* ------------------------------------------------------------------------ */
/* Fused flat-buffer step: AMP unscale + finite check + global norm/clip +  */
/* AdamW + loss-scale state machine (training.rs:289-326,                   */
/* optimizer.rs:126-228).                                                   */
/* ------------------------------------------------------------------------ */

/* Loss-scale + optimizer state (training.rs:54-59 fields, optimizer.rs:68-71). */
typedef struct {
    float loss_scale;
    uint32_t clean_steps;
    uint32_t consecutive_nans;
    uint32_t opt_step;
    uint64_t skipped_steps;
    uint32_t early_stop;
    uint32_t last_overflow;
    float last_norm;
    float last_clip_coef;
    float last_lr;
    uint32_t pad;
    double last_sumsq;
} ork_amp_state;

typedef struct {
    float beta1, beta2, eps, weight_decay, grad_clip;
    float scale_backoff, scale_growth, scale_min, scale_max;
    uint32_t scale_every, max_consecutive_nans;
    uint32_t lr_table_len;
    const float* lr_table;
    uint64_t n_decay;          /* global flat indices [0, n_decay) take weight decay */
    uint64_t keep_lo, keep_hi; /* global range whose grads are NOT unscaled (compat) */
} ork_step_cfg;

/* Rank-local partial of pass 1: exact sum of squares of the unscaled
 * gradient and a count of non-finite scaled gradients.
 * training.rs:291 (is_finite over all grads, memory.rs:379-395 incl.
 * gamma_final), training.rs:308 + :133-146 (unscale, gamma_final omitted in
 * compat mode), optimizer.rs:126-145 (sum of squares over all tensors). */
ORK_API void ork_partial_f16(const ork_step_cfg* cfg, const ork_amp_state* st,
                             const uint16_t* g16, uint64_t n, uint64_t offset,
                             double* sumsq, uint64_t* nonfinite) {
    float inv = 1.0f / st->loss_scale;                  /* training.rs:244 */
    /* Compensated sums over fixed chunks (in parallel), combined in chunk
     * order with the same compensation: exact to ~2^-100, independent of the
     * thread count. */
    const uint64_t chunk = 1u << 20;
    const int64_t nchunks = (int64_t)((n + chunk - 1) / chunk);
    ork_acc* parts = (ork_acc*)calloc(nchunks > 0 ? (size_t)nchunks : 1, sizeof(ork_acc));
    uint64_t bad = 0;
    #pragma omp parallel for schedule(dynamic, 4) reduction(+:bad)
    for (int64_t c = 0; c < nchunks; ++c) {
        ork_acc a = {0.0, 0.0};
        uint64_t lo = (uint64_t)c * chunk, hi = lo + chunk < n ? lo + chunk : n;
        for (uint64_t i = lo; i < hi; ++i) {
            uint16_t h = g16[i];
            if ((h & 0x7C00u) == 0x7C00u) { bad++; continue; }
            uint64_t gi = offset + i;
            float u = ork_h2f(h);
            if (!(gi >= cfg->keep_lo && gi < cfg->keep_hi)) u = u * inv;
            double d = (double)u;
            acc_add(&a, d * d);
        }
        parts[c] = a;
    }
    ork_acc tot = {0.0, 0.0};
    for (int64_t c = 0; c < nchunks; ++c) {
        acc_add(&tot, parts[c].s);
        acc_add(&tot, parts[c].c);
    }
    free(parts);
    *sumsq = acc_value(&tot);
    *nonfinite = bad;
}

/* lr used for optimizer step t (optimizer.rs:172-173: step += 1, then
 * lr_now() reads the incremented step). */
static inline float ork_lr_for(const ork_step_cfg* cfg, uint32_t t) {
    uint32_t i = t < cfg->lr_table_len ? t : cfg->lr_table_len - 1u;
    return cfg->lr_table[i];
}

/* Apply one step to this rank's shard given the GLOBAL sum of squares and
 * non-finite count.  Returns 0, 1 if the step was skipped on overflow, or 2
 * if the early-stop condition was (or had already been) hit. */
ORK_API int ork_apply_f16(const ork_step_cfg* cfg, ork_amp_state* st,
                          uint16_t* w16, const uint16_t* g16, float* m, float* v,
                          uint64_t n, uint64_t offset, double sumsq, uint64_t nonfinite) {
    if (st->early_stop) return 2;
    if (nonfinite) {                                    /* training.rs:293-305 */
        st->loss_scale = fmaxf(st->loss_scale * cfg->scale_backoff, cfg->scale_min);
        st->clean_steps = 0;
        st->skipped_steps += 1;
        st->consecutive_nans += 1;
        st->last_overflow = 1;
        if (st->consecutive_nans > cfg->max_consecutive_nans) { st->early_stop = 1; return 2; }
        return 1;
    }
    float inv = 1.0f / st->loss_scale;                  /* training.rs:244 */
    st->opt_step += 1;                                  /* optimizer.rs:172 */
    uint32_t t = st->opt_step;
    float lr = ork_lr_for(cfg, t);                      /* optimizer.rs:173 */
    float norm = ork_norm_from_sumsq(sumsq);            /* optimizer.rs:145 (accurate sum) */
    int clip = (norm > cfg->grad_clip && norm > 0.0f);  /* optimizer.rs:148 */
    float s = clip ? cfg->grad_clip / norm : 1.0f;      /* optimizer.rs:149 */
    ork_adam_k kd, k0;
    ork_adam_scalars(lr, cfg->beta1, cfg->beta2, cfg->eps, cfg->weight_decay, t, &kd);
    ork_adam_scalars(lr, cfg->beta1, cfg->beta2, cfg->eps, 0.0f, t, &k0);  /* optimizer.rs:199,225-226 */
    #pragma omp parallel for schedule(static)
    for (int64_t ii = 0; ii < (int64_t)n; ++ii) {
        uint64_t i = (uint64_t)ii, gi = offset + i;
        float g = ork_h2f(g16[i]);
        if (!(gi >= cfg->keep_lo && gi < cfg->keep_hi)) g = g * inv;     /* training.rs:308 */
        if (clip) g = g * s;                                              /* optimizer.rs:151-166 */
        const ork_adam_k* k = gi < cfg->n_decay ? &kd : &k0;
        w16[i] = ork_f2h(ork_adam_elem(ork_h2f(w16[i]), g, &m[i], &v[i], k));
    }
    st->clean_steps += 1;                               /* training.rs:317-326 */
    st->consecutive_nans = 0;
    if (st->clean_steps >= cfg->scale_every) {
        float nueva = fminf(st->loss_scale * cfg->scale_growth, cfg->scale_max);
        if (nueva > st->loss_scale) st->loss_scale = nueva;
        st->clean_steps = 0;
    }
    st->last_overflow = 0;
    st->last_norm = norm;
    st->last_sumsq = sumsq;
    st->last_clip_coef = s;
    st->last_lr = lr;
    return 0;
}

ORK_API int ork_step_flat_f16(const ork_step_cfg* cfg, ork_amp_state* st,
                              uint16_t* w16, const uint16_t* g16, float* m, float* v,
                              uint64_t n) {
    double s; uint64_t bad;
    ork_partial_f16(cfg, st, g16, n, 0, &s, &bad);
    return ork_apply_f16(cfg, st, w16, g16, m, v, n, 0, s, bad);
}

/* Gradient hand-off for data-parallel ranks: this rank's shard of the sum
 * over ranks of every rank's full FP16 gradients, accumulated in f32 in rank
 * order from 0 (the reference's zero-then-+= accumulation, memory.rs:338-342,
 * bridge.m:907-949, applied once per rank) and rounded once to FP16. */
ORK_API void ork_reduce_f16(const uint16_t* const* srcs, int nranks, uint64_t n,
                            uint64_t offset, uint16_t* out) {
    #pragma omp parallel for schedule(static)
    for (int64_t ii = 0; ii < (int64_t)n; ++ii) {
        float acc = 0.0f;
        for (int r = 0; r < nranks; ++r) acc = acc + ork_h2f(srcs[r][offset + (uint64_t)ii]);
        out[ii] = ork_f2h(acc);
    }
}

/* The logits-gradient block of train_step (training.rs:228-245): the finite
 * check over the unscaled logits gradients (:229-230); if any value is
 * non-finite the step is rejected before scaling (:231-237: the caller
 * applies the overflow transitions, the same as ork_apply_f16's overflow
 * branch), else every value is multiplied by the loss scale (:244-245,
 * `*x *= self.loss_scale`, one f32 multiply).  Returns the number of
 * non-finite values. */
ORK_API uint64_t ork_logits_check_scale(float* x, uint64_t n, float loss_scale) {
    uint64_t bad = 0;
    for (uint64_t i = 0; i < n; ++i) bad += !isfinite(x[i]);
    if (bad) return bad;
    for (uint64_t i = 0; i < n; ++i) x[i] = x[i] * loss_scale;
    return 0;
}

/* Warmup + cosine schedule, optimizer.rs:80-92, in f32 (cosf from libm). */
ORK_API float ork_lr_now(float lr, uint32_t warmup, uint32_t step) {
    if (step < warmup) return lr * ((float)step + 1.0f) / (float)warmup;
    float decay_steps = (float)(step - warmup);
    float progress = fminf(decay_steps / 800000.0f, 1.0f);
    float cosine = 0.5f * (1.0f + cosf(3.14159274101257324f * progress));
    float lr_min = lr * 0.1f;
    return lr_min + (lr - lr_min) * cosine;
}

/* ------------------------------------------------------------------------ */
/* The reference's own CPU path, literal and per tensor (training.rs:289-314 */
/* + optimizer.rs:126-228), used as the timed CPU baseline.  Grads are FP32  */
/* as in the reference (memory.rs:238-243).  Parallelised across host cores  */
/* without changing a single rounding: element-wise loops are split, each    */
/* tensor's f32 fold stays sequential, and the per-tensor sums are added in  */
/* the reference order.                                                     */
/* ------------------------------------------------------------------------ */

typedef struct {
    uint16_t* w; float* g; float* m; float* v; uint64_t n; float wd;
    uint32_t unscaled;   /* 1 = training.rs:133-146 unscales this tensor */
} ork_tensor;

/* Returns 0 = stepped, 1 = skipped on overflow. */
ORK_API int ork_ref_step_tensors(ork_tensor* ts, int nt, ork_amp_state* st,
                                 float lr, float b1, float b2, float eps, float clip,
                                 float scale_max, uint32_t every, int threads) {
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
#else
    (void)threads;
#endif
    /* training.rs:291 finite check over all grads */
    int bad = 0;
    for (int k = 0; k < nt && !bad; ++k) {
        const float* g = ts[k].g; int64_t n = (int64_t)ts[k].n; int b = 0;
        #pragma omp parallel for reduction(|:b) schedule(static)
        for (int64_t i = 0; i < n; ++i) b |= !isfinite(g[i]);
        bad |= b;
    }
    if (bad) {
        st->loss_scale = fmaxf(st->loss_scale * 0.5f, 1.0f);
        st->clean_steps = 0; st->skipped_steps++; st->consecutive_nans++;
        st->last_overflow = 1;
        if (st->consecutive_nans > 200) st->early_stop = 1;   /* training.rs:298 */
        return 1;
    }
    float inv = 1.0f / st->loss_scale;
    /* training.rs:308 unscale (vDSP_vsmul = one f32 multiply per element) */
    for (int k = 0; k < nt; ++k) {
        if (!ts[k].unscaled) continue;
        float* g = ts[k].g; int64_t n = (int64_t)ts[k].n;
        #pragma omp parallel for schedule(static)
        for (int64_t i = 0; i < n; ++i) g[i] = g[i] * inv;
    }
    st->opt_step += 1;
    uint32_t t = st->opt_step;
    /* optimizer.rs:127-145: per-tensor sequential f32 fold, summed in order */
    float* part = (float*)malloc(sizeof(float) * (size_t)nt);
    #pragma omp parallel for schedule(dynamic, 1)
    for (int k = 0; k < nt; ++k) {
        const float* g = ts[k].g; float s = 0.0f;
        for (uint64_t i = 0; i < ts[k].n; ++i) { float x = g[i] * g[i]; s = s + x; }
        part[k] = s;
    }
    float sum_sq = 0.0f;
    for (int k = 0; k < nt; ++k) sum_sq = sum_sq + part[k];
    free(part);
    float norm = sqrtf(sum_sq);
    if (norm > clip && norm > 0.0f) {
        float sc = clip / norm;
        for (int k = 0; k < nt; ++k) {
            float* g = ts[k].g; int64_t n = (int64_t)ts[k].n;
            #pragma omp parallel for schedule(static)
            for (int64_t i = 0; i < n; ++i) g[i] = g[i] * sc;
        }
    }
    /* optimizer.rs:185-227: one AdamW-f16 call per tensor */
    for (int k = 0; k < nt; ++k) {
        ork_adam_k kk; ork_adam_scalars(lr, b1, b2, eps, ts[k].wd, t, &kk);
        uint16_t* w = ts[k].w; float* g = ts[k].g; float* m = ts[k].m; float* v = ts[k].v;
        int64_t n = (int64_t)ts[k].n;
        #pragma omp parallel for schedule(static)
        for (int64_t i = 0; i < n; ++i) w[i] = ork_f2h(ork_adam_elem(ork_h2f(w[i]), g[i], &m[i], &v[i], &kk));
    }
    st->clean_steps++; st->consecutive_nans = 0;
    if (st->clean_steps >= every) {
        float nueva = fminf(st->loss_scale * 2.0f, scale_max);
        if (nueva > st->loss_scale) st->loss_scale = nueva;
        st->clean_steps = 0;
    }
    st->last_overflow = 0; st->last_norm = norm;
    return 0;
}

/* Host threads of the oracle's parallel loops from now on (checker legs
 * running in several processes at once split the cores between them). */
ORK_API void ork_set_threads(int threads) {
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
#else
    (void)threads;
#endif
}

ORK_API int ork_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* ------------------------------------------------------------------------ */
/* Seeded synthetic inputs: splitmix64 counter RNG + Irwin-Hall(12) normal.  */
/* Keyed by (seed, stream, global flat index) so any shard regenerates       */
/* identically; the CUDA generator in ark_b200/csrc/ark_synth.cu computes    */
/* the same integers and the same two float roundings.                      */
/* ------------------------------------------------------------------------ */

static inline uint64_t splitmix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

ORK_API uint64_t ork_splitmix64(uint64_t x) { return splitmix64(x); }

/* Approximately N(0,1): (sum of twelve 24-bit uniforms - 6), formed as an
 * exact integer and converted to float once (RNE), times 2^-24 (exact). */
ORK_API float ork_normal(uint64_t seed, uint64_t stream, uint64_t idx) {
    uint64_t key = splitmix64(seed ^ splitmix64(stream));
    int32_t s = 0;
    for (uint64_t j = 0; j < 6; ++j) {
        uint64_t r = splitmix64(key + idx * 6u + j);
        s += (int32_t)(r >> 40);
        s += (int32_t)((r >> 16) & 0xFFFFFFu);
    }
    return (float)(s - 6 * (1 << 24)) * 0x1p-24f;
}

/* kind: 0 = half(sigma*z*mult), 1 = float sigma*z, 2 = float (sigma*z)^2.
 * heavy_every > 0: indices with splitmix64(seed^idx^0xA5A5..) % heavy_every
 * == 0 are multiplied by heavy_mult before the final rounding. */
ORK_API void ork_synth_f16(uint16_t* out, uint64_t n, uint64_t offset, uint64_t seed,
                           uint64_t stream, float sigma, float mult,
                           uint32_t heavy_every, float heavy_mult) {
    #pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)n; ++i) {
        uint64_t gi = offset + (uint64_t)i;
        float x = ork_normal(seed, stream, gi) * sigma;
        if (heavy_every && splitmix64(seed ^ gi ^ 0xA5A5A5A5A5A5A5A5ull) % heavy_every == 0)
            x = x * heavy_mult;
        x = x * mult;
        out[i] = ork_f2h(x);
    }
}

ORK_API void ork_synth_f32(float* out, uint64_t n, uint64_t offset, uint64_t seed,
                           uint64_t stream, float sigma, int square) {
    #pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)n; ++i) {
        float x = ork_normal(seed, stream, offset + (uint64_t)i) * sigma;
        out[i] = square ? x * x : x;
    }
}

/* Element index that the trajectory config poisons at a given step. */
ORK_API uint64_t ork_inject_index(uint64_t seed, uint32_t step, uint64_t n) {
    return splitmix64(seed ^ (0xC0FFEEull + step)) % n;
}
