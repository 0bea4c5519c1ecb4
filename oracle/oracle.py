"""ctypes binding of the CPU oracle (oracle/liboracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU-baseline legs of bench.py, never by the ark_b200 package.  See the header
of ark_oracle.c for what each function restates and how it is pinned.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")

c_f, c_u32, c_u64, c_i, c_d, c_p = (ctypes.c_float, ctypes.c_uint32, ctypes.c_uint64,
                                    ctypes.c_int, ctypes.c_double, ctypes.c_void_p)


class AmpState(ctypes.Structure):
    """Mirror of ork_amp_state."""
    _fields_ = [("loss_scale", c_f), ("clean_steps", c_u32), ("consecutive_nans", c_u32),
                ("opt_step", c_u32), ("skipped_steps", c_u64), ("early_stop", c_u32),
                ("last_overflow", c_u32), ("last_norm", c_f), ("last_clip_coef", c_f),
                ("last_lr", c_f), ("pad", c_u32), ("last_sumsq", c_d)]


class StepCfg(ctypes.Structure):
    """Mirror of ork_step_cfg."""
    _fields_ = [("beta1", c_f), ("beta2", c_f), ("eps", c_f), ("weight_decay", c_f),
                ("grad_clip", c_f), ("scale_backoff", c_f), ("scale_growth", c_f),
                ("scale_min", c_f), ("scale_max", c_f), ("scale_every", c_u32),
                ("max_consecutive_nans", c_u32), ("lr_table_len", c_u32),
                ("lr_table", ctypes.POINTER(c_f)), ("n_decay", c_u64),
                ("keep_lo", c_u64), ("keep_hi", c_u64)]


class Tensor(ctypes.Structure):
    """Mirror of ork_tensor."""
    _fields_ = [("w", c_p), ("g", c_p), ("m", c_p), ("v", c_p), ("n", c_u64), ("wd", c_f),
                ("unscaled", c_u32)]


def build():
    subprocess.run(["make", "-s", "-C", HERE], check=True)


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        sig = {
            "ork_h2f": (c_f, [ctypes.c_uint16]),
            "ork_f2h": (ctypes.c_uint16, [c_f]),
            "ork_dequant_f16_to_f32": (None, [c_p, c_p, c_u64]),
            "ork_quant_f32_to_f16": (None, [c_p, c_p, c_u64]),
            "ork_adam_step_f16": (None, [c_p, c_p, c_p, c_p, c_u64, c_f, c_f, c_f, c_f, c_f, c_u32]),
            "ork_adam_step_f32": (None, [c_p, c_p, c_p, c_p, c_u64, c_f, c_f, c_f, c_f, c_f, c_u32]),
            "ork_sumsq_f32_exact": (c_d, [c_p, c_u64]),
            "ork_norm_from_sumsq": (c_f, [c_d]),
            "ork_grad_clip_neon": (c_f, [c_p, c_u64, c_f]),
            "ork_grad_clip_exact": (c_f, [c_p, c_u64, c_f]),
            "ork_partial_f16": (None, [ctypes.POINTER(StepCfg), ctypes.POINTER(AmpState), c_p, c_u64,
                                       c_u64, ctypes.POINTER(c_d), ctypes.POINTER(c_u64)]),
            "ork_apply_f16": (c_i, [ctypes.POINTER(StepCfg), ctypes.POINTER(AmpState), c_p, c_p, c_p,
                                    c_p, c_u64, c_u64, c_d, c_u64]),
            "ork_step_flat_f16": (c_i, [ctypes.POINTER(StepCfg), ctypes.POINTER(AmpState), c_p, c_p,
                                        c_p, c_p, c_u64]),
            "ork_lr_now": (c_f, [c_f, c_u32, c_u32]),
            "ork_reduce_f16": (None, [ctypes.POINTER(c_p), c_i, c_u64, c_u64, c_p]),
            "ork_ref_step_tensors": (c_i, [ctypes.POINTER(Tensor), c_i, ctypes.POINTER(AmpState), c_f,
                                           c_f, c_f, c_f, c_f, c_f, c_u32, c_i]),
            "ork_max_threads": (c_i, []),
            "ork_set_threads": (None, [c_i]),
            "ork_splitmix64": (c_u64, [c_u64]),
            "ork_normal": (c_f, [c_u64, c_u64, c_u64]),
            "ork_synth_f16": (None, [c_p, c_u64, c_u64, c_u64, c_u64, c_f, c_f, c_u32, c_f]),
            "ork_synth_f32": (None, [c_p, c_u64, c_u64, c_u64, c_u64, c_f, c_i]),
            "ork_inject_index": (c_u64, [c_u64, c_u32, c_u64]),
            "ork_logits_check_scale": (c_u64, [c_p, c_u64, c_f]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def ptr(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(c_p)


# ------------------------------------------------------------------ wrappers
def adam_step_f16(w16, g, m, v, lr, b1, b2, eps, wd, t):
    w16, g, m, v = (np.array(a, copy=True) for a in (w16, g, m, v))
    lib().ork_adam_step_f16(ptr(w16), ptr(g), ptr(m), ptr(v), len(g), lr, b1, b2, eps, wd, t)
    return w16, m, v


def adam_step_f32(w, g, m, v, lr, b1, b2, eps, wd, t):
    w, g, m, v = (np.array(a, copy=True) for a in (w, g, m, v))
    lib().ork_adam_step_f32(ptr(w), ptr(g), ptr(m), ptr(v), len(g), lr, b1, b2, eps, wd, t)
    return w, m, v


def grad_clip_neon(g, thr):
    g = np.array(g, np.float32, copy=True)
    norm = lib().ork_grad_clip_neon(ptr(g), len(g), thr)
    return np.float32(norm), g


def grad_clip_exact(g, thr):
    g = np.array(g, np.float32, copy=True)
    norm = lib().ork_grad_clip_exact(ptr(g), len(g), thr)
    return np.float32(norm), g


def sumsq_f32_exact(g):
    g = np.ascontiguousarray(g, np.float32)
    return lib().ork_sumsq_f32_exact(ptr(g), len(g))


def quant(x):
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty(len(x), np.uint16)
    lib().ork_quant_f32_to_f16(ptr(x), ptr(out), len(x))
    return out


def dequant(h):
    h = np.ascontiguousarray(h, np.uint16)
    out = np.empty(len(h), np.float32)
    lib().ork_dequant_f16_to_f32(ptr(h), ptr(out), len(h))
    return out


def make_cfg(beta1=0.9, beta2=0.95, eps=1e-8, weight_decay=0.1, grad_clip=1.0,
             scale_backoff=0.5, scale_growth=2.0, scale_min=1.0, scale_max=8192.0,
             scale_every=2000, max_consecutive_nans=200, lr_table=(3e-4,),
             n_decay=0, keep_lo=0, keep_hi=0):
    table = np.ascontiguousarray(np.asarray(lr_table, np.float32))
    cfg = StepCfg(beta1, beta2, eps, weight_decay, grad_clip, scale_backoff, scale_growth,
                  scale_min, scale_max, scale_every, max_consecutive_nans, len(table),
                  table.ctypes.data_as(ctypes.POINTER(c_f)), n_decay, keep_lo, keep_hi)
    cfg._table = table  # keep alive
    return cfg


def make_state(loss_scale=256.0, opt_step=0):
    st = AmpState()
    st.loss_scale = loss_scale
    st.opt_step = opt_step
    return st


def partial_f16(cfg, st, g16, offset=0):
    g16 = np.ascontiguousarray(g16, np.uint16)
    s, bad = c_d(), c_u64()
    lib().ork_partial_f16(ctypes.byref(cfg), ctypes.byref(st), ptr(g16), len(g16), offset,
                          ctypes.byref(s), ctypes.byref(bad))
    return s.value, bad.value


def apply_f16(cfg, st, w16, g16, m, v, offset, sumsq, nonfinite):
    """In place on w16, m, v (numpy arrays).  Returns the oracle's code."""
    return lib().ork_apply_f16(ctypes.byref(cfg), ctypes.byref(st), ptr(w16), ptr(g16), ptr(m),
                               ptr(v), len(g16), offset, sumsq, nonfinite)


def step_flat_f16(cfg, st, w16, g16, m, v):
    return lib().ork_step_flat_f16(ctypes.byref(cfg), ctypes.byref(st), ptr(w16), ptr(g16),
                                   ptr(m), ptr(v), len(g16))


def reduce_f16(srcs, n, offset):
    """Shard [offset, offset+n) of the rank-ordered f32 sum of FP16 buffers."""
    srcs = [np.ascontiguousarray(x, np.uint16) for x in srcs]
    arr = (c_p * len(srcs))(*[x.ctypes.data for x in srcs])
    out = np.empty(n, np.uint16)
    lib().ork_reduce_f16(arr, len(srcs), n, offset, ptr(out))
    return out


def logits_check_scale(x, loss_scale):
    """training.rs:228-245 on a copy: (non-finite count, logits after the
    block -- scaled when every value is finite, else unchanged)."""
    x = np.array(x, np.float32, copy=True)
    bad = lib().ork_logits_check_scale(ptr(x), len(x), loss_scale)
    return int(bad), x


def synth_f16(n, offset, seed, stream, sigma, mult=1.0, heavy_every=0, heavy_mult=1.0):
    out = np.empty(n, np.uint16)
    lib().ork_synth_f16(ptr(out), n, offset, seed, stream, sigma, mult, heavy_every, heavy_mult)
    return out


def synth_f32(n, offset, seed, stream, sigma, square=False):
    out = np.empty(n, np.float32)
    lib().ork_synth_f32(ptr(out), n, offset, seed, stream, sigma, int(square))
    return out


def load_golden(path=None):
    """Load tests/golden/golden_asm.npz -> (meta dict, arrays)."""
    import json
    if path is None:
        path = os.path.join(os.path.dirname(HERE), "tests", "golden", "golden_asm.npz")
    z = np.load(path)
    meta = json.loads(bytes(z["meta"]).decode())
    return meta, z
