/* step_from_c.c -- a plain C caller of libark_cuda: the legacy per-tensor
 * AdamW entry point (as ARK's Rust code calls it, src/optimizer.rs:28-40)
 * and the fused step, on device buffers it allocates with the CUDA runtime.
 * Prints one line per check and exits non-zero on a mismatch.
 *
 *   gcc -std=c11 -I include step_from_c.c -L ark_b200/lib -lark_cuda \
 *       -L /usr/local/cuda/lib64 -lcudart -Wl,-rpath,ark_b200/lib -o step_from_c
 */
#include <cuda_runtime_api.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "ark_opt.h"

#define N 4099u

static int fail(const char* what, int code) {
    fprintf(stderr, "step_from_c: %s failed (%d: %s)\n", what, code, ark_cuda_strerror(code));
    return 1;
}

int main(void) {
    uint16_t* w = NULL;
    float *g = NULL, *m = NULL, *v = NULL;
    uint16_t* g16 = NULL;
    if (cudaMalloc((void**)&w, N * 2) || cudaMalloc((void**)&g, N * 4) ||
        cudaMalloc((void**)&m, N * 4) || cudaMalloc((void**)&v, N * 4) ||
        cudaMalloc((void**)&g16, N * 2))
        return fail("cudaMalloc", ARK_E_CUDA);
    float* hf = (float*)malloc(N * 4);
    uint16_t* hw = (uint16_t*)malloc(N * 2);
    for (unsigned i = 0; i < N; ++i) hf[i] = 0.01f * (float)((int)(i % 41) - 20);
    cudaMemcpy(g, hf, N * 4, cudaMemcpyHostToDevice);
    ark_quant_f32_to_f16(g, w, N);                  /* weights = fp16(g) */
    if (ark_cuda_last_error()) return fail("ark_quant_f32_to_f16", ark_cuda_last_error());
    cudaMemset(m, 0, N * 4);
    cudaMemset(v, 0, N * 4);

    /* legacy: one AdamW step, t = 1 (bias-corrected first step moves every
     * weight with a nonzero gradient by about lr) */
    ark_asm_adam_step_f16(w, g, m, v, N, 1e-2f, 0.9f, 0.999f, 1e-8f, 0.0f, 1);
    if (ark_cuda_last_error()) return fail("ark_asm_adam_step_f16", ark_cuda_last_error());
    cudaMemcpy(hw, w, N * 2, cudaMemcpyDeviceToHost);
    printf("legacy adam: w[0]=0x%04x w[20]=0x%04x\n", hw[0], hw[20]);

    /* fused step: scale 1024, grads = fp16(g * 1024) */
    for (unsigned i = 0; i < N; ++i) hf[i] *= 1024.0f;
    cudaMemcpy(g, hf, N * 4, cudaMemcpyHostToDevice);
    ark_quant_f32_to_f16(g, g16, N);
    const float lr = 1e-3f;
    ark_opt_cfg cfg;
    memset(&cfg, 0, sizeof(cfg));
    cfg.abi_version = ARK_OPT_ABI_VERSION;
    cfg.n = N;
    cfg.n_decay = N;
    cfg.lr_table = &lr;
    cfg.lr_table_len = 1;
    cfg.beta1 = 0.9f;
    cfg.beta2 = 0.95f;
    cfg.eps = 1e-8f;
    cfg.weight_decay = 0.1f;
    cfg.grad_clip = 1.0f;
    cfg.scale_init = 1024.0f;
    cfg.scale_backoff = 0.5f;
    cfg.scale_growth = 2.0f;
    cfg.scale_min = 1.0f;
    cfg.scale_max = 65536.0f;
    cfg.scale_every = 2000;
    cfg.max_consecutive_nans = 200;
    cfg.world_size = 1;
    ark_opt_state* st = NULL;
    int rc = ark_cuda_opt_init(&cfg, &st);
    if (rc) return fail("ark_cuda_opt_init", rc);
    for (int k = 0; k < 3; ++k) {
        rc = ark_cuda_opt_step(st, w, g16, m, v);
        if (rc) return fail("ark_cuda_opt_step", rc);
    }
    ark_opt_status s;
    rc = ark_cuda_opt_read_status(st, &s);
    if (rc) return fail("ark_cuda_opt_read_status", rc);
    printf("fused step: opt_step=%u loss_scale=%g norm=%.6g clip=%.6g overflow=%u\n", s.opt_step,
           s.loss_scale, s.last_norm, s.last_clip_coef, s.last_overflow);
    ark_cuda_opt_destroy(st);
    free(hf);
    free(hw);
    cudaFree(w);
    cudaFree(g);
    cudaFree(m);
    cudaFree(v);
    cudaFree(g16);
    return (s.opt_step == 3 && !s.last_overflow && s.last_clip_coef < 1.0f) ? 0 : 1;
}
