"""ctypes binding of libark_cuda.so (the C ABI declared in include/ark_opt.h).

The library is built in-tree by ark_b200/csrc/Makefile.  Loading fails with
an exception when it is missing: there is no fallback implementation.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
LIB_PATH = os.path.join(PKG, "lib", "libark_cuda.so")

ARK_OPT_ABI_VERSION = 2
ARK_OK = 0
STATUS_NAMES = {
    0: "ARK_OK", -1: "ARK_E_INVALID_ARG", -2: "ARK_E_MISALIGNED", -3: "ARK_E_CUDA",
    -4: "ARK_E_NCCL", -5: "ARK_E_TIMEOUT", -6: "ARK_E_EARLY_STOP", -7: "ARK_E_NO_DEVICE",
    -8: "ARK_E_UNSUPPORTED",
}
ARK_E_EARLY_STOP = -6
ARK_COMPAT_CLIP_NEON_FOLD = 0x1
ARK_OPT_COMPAT_GAMMA_FINAL_UNSCALED = 0x1
ARK_OPT_USE_GRAPH = 0x2
ARK_OPT_NCCL_EXCHANGE = 0x4
ARK_STEP_REDUCE = 0x1
ARK_STEP_GATHER_WEIGHTS = 0x2
ARK_CKPT_RESTORE_SCALE = 0x1

c_f, c_u32, c_u64, c_i, c_i32, c_d, c_p = (ctypes.c_float, ctypes.c_uint32, ctypes.c_uint64,
                                           ctypes.c_int, ctypes.c_int32, ctypes.c_double,
                                           ctypes.c_void_p)


class OptCfg(ctypes.Structure):
    """ark_opt_cfg."""
    _fields_ = [
        ("abi_version", c_u32), ("device", c_i32), ("n", c_u64), ("shard_offset", c_u64),
        ("n_decay", c_u64), ("keep_scaled_lo", c_u64), ("keep_scaled_hi", c_u64),
        ("lr_table", ctypes.POINTER(c_f)), ("lr_table_len", c_u32),
        ("beta1", c_f), ("beta2", c_f), ("eps", c_f), ("weight_decay", c_f), ("grad_clip", c_f),
        ("scale_init", c_f), ("scale_backoff", c_f), ("scale_growth", c_f), ("scale_min", c_f),
        ("scale_max", c_f), ("scale_every", c_u32), ("max_consecutive_nans", c_u32),
        ("initial_step", c_u32), ("flags", c_u32), ("rank", c_i32), ("world_size", c_i32),
        ("nccl_comm", c_p), ("stream", c_p), ("wait_timeout_ms", c_u32), ("reserved", c_u32),
    ]


class CkptTensor(ctypes.Structure):
    """ark_ckpt_tensor."""
    _fields_ = [("numel", c_u64), ("flat_offset", c_u64)]


class OptStatus(ctypes.Structure):
    """ark_opt_status."""
    _fields_ = [
        ("last_sumsq", c_d), ("skipped_steps", c_u64), ("steps_called", c_u64),
        ("loss_scale", c_f), ("last_norm", c_f), ("last_clip_coef", c_f), ("last_lr", c_f),
        ("opt_step", c_u32), ("clean_steps", c_u32), ("consecutive_nans", c_u32),
        ("last_overflow", c_u32), ("early_stop", c_u32), ("error", c_i32),
    ]

    def as_dict(self):
        return {k: getattr(self, k) for k, _ in self._fields_}


# every symbol include/ark_opt.h declares, with its ctypes signature
SIGNATURES = {
    "ark_asm_adam_step_f16": (None, [c_p, c_p, c_p, c_p, c_u64, c_f, c_f, c_f, c_f, c_f, c_u32]),
    "ark_asm_adam_step": (None, [c_p, c_p, c_p, c_p, c_u64, c_f, c_f, c_f, c_f, c_f, c_u32]),
    "ark_asm_grad_clip": (c_f, [c_p, c_u64, c_f]),
    "ark_quant_f32_to_f16": (None, [c_p, c_p, c_u64]),
    "ark_dequant_f16_to_f32": (None, [c_p, c_p, c_u64]),
    "ark_cuda_grad_clip_noalloc": (c_i, [c_p, c_u64, c_f, c_p, c_p]),
    "ark_cuda_last_error": (c_i, []),
    "ark_cuda_strerror": (ctypes.c_char_p, [c_i]),
    "ark_cuda_set_compat": (c_i, [c_u32]),
    "ark_cuda_legacy_set_stream": (c_i, [c_p]),
    "ark_cuda_legacy_set_async": (c_i, [c_i]),
    "ark_cuda_legacy_sync": (c_i, []),
    "ark_cuda_abi_version": (c_u32, []),
    "ark_cuda_opt_init": (c_i, [ctypes.POINTER(OptCfg), ctypes.POINTER(c_p)]),
    "ark_cuda_opt_step": (c_i, [c_p, c_p, c_p, c_p, c_p]),
    "ark_cuda_opt_grad_buffer": (c_i, [c_p, c_u64, ctypes.POINTER(c_p)]),
    "ark_cuda_opt_step_reduce": (c_i, [c_p, c_p, c_p, c_p, c_p]),
    "ark_cuda_opt_step_ex": (c_i, [c_p, c_p, c_p, c_p, c_p, c_p, c_u32]),
    "ark_cuda_opt_weight_buffer": (c_i, [c_p, c_u64, ctypes.POINTER(c_p)]),
    "ark_cuda_opt_weights_wait": (c_i, [c_p]),
    "ark_cuda_opt_logits_check": (c_i, [c_p, c_p, c_u64]),
    "ark_cuda_opt_zero_grads": (c_i, [c_p]),
    "ark_cuda_opt_read_status": (c_i, [c_p, ctypes.POINTER(OptStatus)]),
    "ark_cuda_opt_set_status": (c_i, [c_p, ctypes.POINTER(OptStatus)]),
    "ark_cuda_opt_upload_grads": (c_i, [c_p, c_p, c_p, c_u64]),
    "ark_cuda_allgather_weights": (c_i, [c_p, c_p, c_p, c_u64]),
    "ark_cuda_opt_profile_begin": (c_i, [c_p, c_u32]),
    "ark_cuda_opt_profile_read": (c_i, [c_p, ctypes.POINTER(c_f), c_u32, ctypes.POINTER(c_u32)]),
    "ark_cuda_opt_geometry": (c_i, [c_p, ctypes.POINTER(c_u32), ctypes.POINTER(c_u32),
                                    ctypes.POINTER(c_u32)]),
    "ark_cuda_opt_destroy": (c_i, [c_p]),
    "ark_cuda_lr_schedule": (c_i, [ctypes.POINTER(c_f), c_u32, c_f, c_u32]),
    "ark_cuda_ckpt_save": (c_i, [c_p, ctypes.c_char_p, ctypes.POINTER(CkptTensor), c_u32, c_u64,
                                 c_p, c_p, c_p]),
    "ark_cuda_ckpt_load": (c_i, [c_p, ctypes.c_char_p, ctypes.POINTER(CkptTensor), c_u32,
                                 ctypes.POINTER(c_u64), c_p, c_p, c_p, c_u32]),
    "ark_cuda_nccl_unique_id": (c_i, [c_p]),
    "ark_cuda_nccl_comm_init": (c_i, [c_i, c_i, c_p, c_i, ctypes.POINTER(c_p)]),
    "ark_cuda_nccl_comm_destroy": (c_i, [c_p]),
    "ark_synth_f16": (c_i, [c_p, c_u64, c_u64, c_u64, c_u64, c_f, c_f, c_u32, c_f, c_p]),
    "ark_synth_f32": (c_i, [c_p, c_u64, c_u64, c_u64, c_u64, c_f, c_i, c_p]),
}


class ArkError(RuntimeError):
    def __init__(self, fn, code):
        self.code = code
        super().__init__(f"{fn} returned {code} ({STATUS_NAMES.get(code, 'unknown')})")


def build(quiet=True):
    """Compile libark_cuda.so/.a for sm_100a (nvcc cross-compiles without a GPU)."""
    cmd = ["make", "-C", os.path.join(PKG, "csrc")]
    if quiet:
        cmd.insert(1, "-s")
    subprocess.run(cmd, check=True)


_LIB = None


def lib():
    """The loaded library; raises if it has not been built."""
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `make -C ark_b200/csrc` "
                "(or __graft_entry__.build()); ark_b200 has no CPU fallback")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        if L.ark_cuda_abi_version() != ARK_OPT_ABI_VERSION:
            raise RuntimeError("libark_cuda.so ABI version mismatch: rebuild it")
        _LIB = L
    return _LIB


def check(fn, code):
    if code != ARK_OK:
        raise ArkError(fn, code)
    return code
