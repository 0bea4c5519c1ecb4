// ark_internal.h -- host-side plumbing shared by the library's translation
// units: error reporting and CUDA call checking.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>

#include "../../include/ark_opt.h"

namespace ark {

// Records and reports (once per distinct code) a failure of a void legacy
// entry point; the reference has no error channel, so stderr is the loud
// path and ark_cuda_last_error() the programmatic one.
void legacy_fail(const char* fn, int code, const char* detail);
void set_last_error(int code);

const char* status_string(int status);

#define ARK_CUDA_TRY(expr)                                                                \
    do {                                                                                  \
        cudaError_t _e = (expr);                                                          \
        if (_e != cudaSuccess) {                                                          \
            fprintf(stderr, "[ark_cuda] %s failed: %s (%s:%d)\n", #expr,                 \
                    cudaGetErrorString(_e), __FILE__, __LINE__);                          \
            return ARK_E_CUDA;                                                            \
        }                                                                                 \
    } while (0)

__host__ __device__ inline bool aligned16(const void* p) {
    return (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
}

// Blocks to launch for a grid-stride streaming kernel: every SM filled
// with as many resident blocks as the kernel's occupancy allows.
int streaming_grid(const void* kernel, int threads, size_t dyn_smem, uint64_t work_items);

// What the checkpoint code needs of an optimizer state (ark_step.cu).
struct OptView {
    int device, rank, world;
    uint64_t n, shard_offset;
    float scale_init;
};
int opt_view(const ark_opt_state* st, OptView* out);

}  // namespace ark
