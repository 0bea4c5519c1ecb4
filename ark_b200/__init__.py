"""ark_b200 -- B200-native optimizer hot path of the ARK LLM trainer.

AMP unscale + inf/NaN detection, global L2 grad norm and clip, AdamW with
FP16 in-place weights over FP32 moments, the dynamic loss-scale state
machine and the FP16<->FP32 conversions, as hand-written sm_100a CUDA
behind the C ABI of include/ark_opt.h (libark_cuda.so / libark_cuda.a).
"""
from . import layout
from ._lib import ArkError, build, lib
from .optimizer import (AdamConfig, LossScaleConfig, Optimizer, adam_step, adam_step_f16,
                        dequant_f16_to_f32, grad_clip, legacy_set_async, legacy_sync, lr_schedule,
                        quant_f32_to_f16, set_compat)

__all__ = [
    "AdamConfig", "LossScaleConfig", "Optimizer", "ArkError", "adam_step", "adam_step_f16",
    "grad_clip", "quant_f32_to_f16", "dequant_f16_to_f32", "set_compat", "legacy_set_async",
    "legacy_sync", "lr_schedule", "layout", "build", "lib",
]
