"""Seeded synthetic optimizer inputs, generated on the device by
libark_cuda.so (ark_synth_f16 / ark_synth_f32).

Distributions of the benchmark configurations: w = fp16(N(0, 0.02)),
g = fp16(N(0, 1e-3) * loss_scale), m = N(0, 1e-4), v = N(0, 1e-3)^2, each
keyed by (seed, stream, global flat index) so every shard regenerates the
same values, bit-identical to the CPU generator the tests use.
"""
from __future__ import annotations

from . import _lib

STREAM_W, STREAM_G, STREAM_M, STREAM_V = 1, 2, 3, 4
GRAD_STEP_STREAM_BASE = 0x100     # per-step fresh gradients: stream base + step
HEAVY_EVERY, HEAVY_MULT = 100, 100.0


def _stream_handle(stream):
    if stream is None:
        return None
    return getattr(stream, "cuda_stream", stream)


def fill_f16(t, offset, seed, stream_id, sigma, mult=1.0, heavy_every=0, heavy_mult=1.0,
             cuda_stream=None):
    rc = _lib.lib().ark_synth_f16(t.data_ptr(), t.numel(), offset, seed, stream_id, sigma, mult,
                                  heavy_every, heavy_mult, _stream_handle(cuda_stream))
    _lib.check("ark_synth_f16", rc)


def fill_f32(t, offset, seed, stream_id, sigma, square=False, cuda_stream=None):
    rc = _lib.lib().ark_synth_f32(t.data_ptr(), t.numel(), offset, seed, stream_id, sigma,
                                  1 if square else 0, _stream_handle(cuda_stream))
    _lib.check("ark_synth_f32", rc)


def make_state(n, offset, seed, device, loss_scale=65536.0, heavy=False, grad_stream=STREAM_G,
               cuda_stream=None):
    """Allocate and fill (w16, g16, m, v) for global range [offset, offset+n)."""
    import torch
    w16 = torch.empty(n, dtype=torch.float16, device=device)
    g16 = torch.empty(n, dtype=torch.float16, device=device)
    m = torch.empty(n, dtype=torch.float32, device=device)
    v = torch.empty(n, dtype=torch.float32, device=device)
    fill_f16(w16, offset, seed, STREAM_W, 0.02, cuda_stream=cuda_stream)
    fill_grads(g16, offset, seed, loss_scale, heavy, grad_stream, cuda_stream)
    fill_f32(m, offset, seed, STREAM_M, 1e-4, cuda_stream=cuda_stream)
    fill_f32(v, offset, seed, STREAM_V, 1e-3, square=True, cuda_stream=cuda_stream)
    return w16, g16, m, v


def fill_grads(g16, offset, seed, loss_scale, heavy=False, grad_stream=STREAM_G, cuda_stream=None):
    fill_f16(g16, offset, seed, grad_stream, 1e-3, mult=loss_scale,
             heavy_every=HEAVY_EVERY if heavy else 0, heavy_mult=HEAVY_MULT if heavy else 1.0,
             cuda_stream=cuda_stream)
