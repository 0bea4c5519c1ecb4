"""Run each legacy entry point of libark_cuda once over n elements of
device memory and print its time and bandwidth (CUDA events, one warm-up
call each).  These are the five symbols ARK's Rust code binds today
(proyecto_ark/ark01/src/optimizer.rs:20-23, src/ffi.rs:88-115), plus the
allocation-free clip, which runs the same clip kernels.

  python -m ark_b200.examples.legacy_kernels [--n 134217728] [--only NAME]

Bytes per element (algorithmic): AdamW-f16 24 (w 2+2, g 4, m 4+4, v 4+4),
AdamW-f32 32, clip 12 (norm pass 4, scale pass 4+4), quant 6, dequant 6.
"""
from __future__ import annotations

import argparse
import json

import torch

import ark_b200 as ab
from ark_b200 import synth


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--n", type=int, default=1 << 27)
    ap.add_argument("--only", default="", help="run only the entry point with this name")
    ap.add_argument("--reps", type=int, default=5)
    args = ap.parse_args()
    n = args.n
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    lib = ab.lib()
    a32 = torch.empty(n, dtype=torch.float32, device=dev)
    b32 = torch.empty(n, dtype=torch.float32, device=dev)
    c32 = torch.empty(n, dtype=torch.float32, device=dev)
    d32 = torch.empty(n, dtype=torch.float32, device=dev)
    h16 = torch.empty(n, dtype=torch.float16, device=dev)
    synth.fill_f32(a32, 0, 1, 5, 0.02)
    synth.fill_f32(b32, 0, 1, 9, 1e-3)
    synth.fill_f32(c32, 0, 1, 3, 1e-4)
    synth.fill_f32(d32, 0, 1, 4, 1e-3, square=True)
    synth.fill_f16(h16, 0, 1, 1, 0.02)
    norm = torch.zeros(1, dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)
    calls = [0]

    def clip():
        # every call clips: the threshold halves each time (the norm starts near 11.6)
        thr = 8.0 * 0.5 ** calls[0]
        calls[0] += 1
        lib.ark_cuda_grad_clip_noalloc(b32.data_ptr(), n, thr, norm.data_ptr(),
                                       stream.cuda_stream)

    runs = {
        "ark_asm_adam_step_f16": (24, lambda: lib.ark_asm_adam_step_f16(
            h16.data_ptr(), b32.data_ptr(), c32.data_ptr(), d32.data_ptr(), n, 3e-4, 0.9, 0.95,
            1e-8, 0.1, 1000)),
        "ark_asm_adam_step": (32, lambda: lib.ark_asm_adam_step(
            a32.data_ptr(), b32.data_ptr(), c32.data_ptr(), d32.data_ptr(), n, 3e-4, 0.9, 0.95,
            1e-8, 0.1, 1000)),
        "ark_cuda_grad_clip_noalloc": (12, clip),
        "ark_quant_f32_to_f16": (6, lambda: lib.ark_quant_f32_to_f16(a32.data_ptr(),
                                                                       h16.data_ptr(), n)),
        "ark_dequant_f16_to_f32": (6, lambda: lib.ark_dequant_f16_to_f32(h16.data_ptr(),
                                                                         a32.data_ptr(), n)),
    }
    ab.legacy_set_async(True)
    out = {}
    try:
        for name, (bpe, fn) in runs.items():
            if args.only and name != args.only:
                continue
            fn()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(args.reps):
                fn()
            e1.record(stream)
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1) / args.reps
            out[name] = {"ms": round(ms, 4), "gbs": round(bpe * n / (ms * 1e-3) / 1e9, 1)}
        if lib.ark_cuda_last_error() != 0:
            raise ab.ArkError("legacy entry point", lib.ark_cuda_last_error())
    finally:
        ab.legacy_set_async(False)
    print(json.dumps({"n": n, "kernels": out}))


if __name__ == "__main__":
    main()
