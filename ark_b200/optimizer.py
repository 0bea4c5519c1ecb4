"""Host-side mirror of ARK's optimizer interface over the B200 library.

Reference interface (proyecto_ark/ark01):
  * AdamConfig, Optimizer.step_all, lr_now       src/optimizer.rs:44-228
  * the AMP loss-scale block of Trainer          src/training.rs:8-13, 54-59,
                                                 228-245, 289-326
  * the native kernels bound over FFI            src/ffi.rs:88-115,
                                                 src/optimizer.rs:20-23

`Optimizer.step_all` runs the whole optimizer block of train_step (finite
check, unscale, global clip, AdamW on every tensor, loss-scale update) as one
asynchronous device step over a flat shard; `status()` is the only call that
waits.  The module-level functions are the legacy per-tensor kernels with the
reference's signatures.  Buffers are CUDA tensors (torch is used only for
device memory and streams); every call goes through libark_cuda.so.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

from . import _lib
from .layout import Layout, flat_layout


# ----------------------------------------------------------------- configs
@dataclass
class AdamConfig:
    """optimizer.rs:44-66 (defaults as in AdamConfig::default)."""
    lr: float = 3e-4
    beta1: float = 0.9
    beta2: float = 0.999
    eps: float = 1e-8
    weight_decay: float = 0.01
    grad_clip: float = 1.0
    warmup_steps: int = 100


@dataclass
class LossScaleConfig:
    """training.rs:8-13 (init 256, min 1, growth every 2000 clean steps),
    the x0.5 backoff and x2 growth of :294/:320, config.rs:69 (max 8192) and
    the early stop after more than 200 consecutive overflows (:298)."""
    init: float = 256.0
    backoff: float = 0.5
    growth: float = 2.0
    min: float = 1.0
    max: float = 8192.0
    every: int = 2000
    max_consecutive_nans: int = 200


def lr_schedule(cfg: AdamConfig, length: int) -> np.ndarray:
    """Table of lr_now() (optimizer.rs:80-92) for optimizer steps 0..length-1."""
    out = np.empty(length, np.float32)
    _lib.check("ark_cuda_lr_schedule", _lib.lib().ark_cuda_lr_schedule(
        out.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), length, cfg.lr, cfg.warmup_steps))
    return out


def _ptr(t, dtype_name, numel=None):
    import torch
    if t is None:
        return None
    if isinstance(t, int):
        return t
    if not isinstance(t, torch.Tensor):
        raise TypeError("expected a CUDA torch.Tensor or a raw device pointer")
    if not t.is_cuda:
        raise ValueError("buffers must be CUDA tensors (device memory)")
    if not t.is_contiguous():
        raise ValueError("buffers must be contiguous")
    want = {"f16": (torch.float16, torch.uint16, torch.int16, torch.bfloat16),
            "f32": (torch.float32,)}[dtype_name]
    if t.dtype not in want:
        raise TypeError(f"expected {dtype_name} storage, got {t.dtype}")
    if dtype_name == "f16" and t.dtype == torch.bfloat16:
        raise TypeError("FP16 buffers must hold IEEE binary16 bits, not bfloat16")
    if numel is not None and t.numel() < numel:
        raise ValueError(f"buffer has {t.numel()} elements, need {numel}")
    return t.data_ptr()


# ----------------------------------------------------------------- fused step
class Optimizer:
    """Optimizer.step_all + the AMP loss scaler, on one flat ZeRO-1 shard.

    layout:  a Layout (flat order: decayed tensors first) or an int (one
             decayed flat buffer of that many elements).
    rank/world/comm: the shard of this process; comm is an NCCL communicator
             handle (see ark_b200.dist) when world > 1.
    lr_table: lr per optimizer step (index t); default: the reference
             schedule lr_now() (warmup, then cosine over 800k steps), or the
             constant adam.lr when constant_lr is set.
    shard:   explicit global [lo, hi) instead of the ZeRO-1 shard of rank.
    stream:  CUDA stream (torch.cuda.Stream or raw handle) every step runs on;
             default: torch's current stream, so the step is ordered after the
             torch work that produced the gradients.
    nccl_exchange: world > 1: exchange the partials with an NCCL all-gather
             instead of peer-to-peer stores from pass 1.
    wait_timeout_ms: limit of the device-side wait for peers' partials.
    """

    def __init__(self, layout, adam: AdamConfig | None = None,
                 scale: LossScaleConfig | None = None, *, device: int = 0, rank: int = 0,
                 world: int = 1, comm=None, stream=None, lr_table=None, constant_lr: bool = False,
                 initial_step: int = 0, compat_gamma_final_unscaled: bool = False,
                 use_graph: bool = False, shard=None, nccl_exchange: bool = False,
                 wait_timeout_ms: int = 0):
        self.layout = layout if isinstance(layout, Layout) else flat_layout(int(layout))
        self.adam = adam or AdamConfig()
        self.scale_cfg = scale or LossScaleConfig()
        self.rank, self.world = rank, world
        self.lo, self.hi = self.layout.shard(rank, world) if shard is None else shard
        if not (0 <= self.lo <= self.hi <= self.layout.n):
            raise ValueError("shard outside the layout")
        self.n = self.hi - self.lo
        if lr_table is None:
            if constant_lr:
                lr_table = np.array([self.adam.lr], np.float32)
            else:
                # warmup then cosine over 800k steps; entries past the end reuse the last one
                lr_table = lr_schedule(self.adam, max(self.adam.warmup_steps, 1) + 800_001)
        self.lr_table = np.ascontiguousarray(np.asarray(lr_table, np.float32))
        gf_lo, gf_hi = self.layout.gamma_final_range()
        flags = 0
        if compat_gamma_final_unscaled:
            flags |= _lib.ARK_OPT_COMPAT_GAMMA_FINAL_UNSCALED
        if use_graph:
            flags |= _lib.ARK_OPT_USE_GRAPH
        if nccl_exchange:
            flags |= _lib.ARK_OPT_NCCL_EXCHANGE
        cfg = _lib.OptCfg()
        cfg.abi_version = _lib.ARK_OPT_ABI_VERSION
        cfg.device = device
        cfg.n = self.n
        cfg.shard_offset = self.lo
        cfg.n_decay = self.layout.n_decay
        cfg.keep_scaled_lo, cfg.keep_scaled_hi = gf_lo, gf_hi
        cfg.lr_table = self.lr_table.ctypes.data_as(ctypes.POINTER(ctypes.c_float))
        cfg.lr_table_len = len(self.lr_table)
        a, s = self.adam, self.scale_cfg
        cfg.beta1, cfg.beta2, cfg.eps = a.beta1, a.beta2, a.eps
        cfg.weight_decay, cfg.grad_clip = a.weight_decay, a.grad_clip
        cfg.scale_init, cfg.scale_backoff, cfg.scale_growth = s.init, s.backoff, s.growth
        cfg.scale_min, cfg.scale_max = s.min, s.max
        cfg.scale_every, cfg.max_consecutive_nans = s.every, s.max_consecutive_nans
        cfg.initial_step = initial_step
        cfg.flags = flags
        cfg.rank, cfg.world_size = rank, world
        cfg.nccl_comm = comm
        if stream is None:
            import torch
            stream = torch.cuda.current_stream(device).cuda_stream
        cfg.stream = getattr(stream, "cuda_stream", stream)
        self.stream_handle = cfg.stream
        cfg.wait_timeout_ms = wait_timeout_ms
        self._cfg = cfg
        h = ctypes.c_void_p()
        _lib.check("ark_cuda_opt_init", _lib.lib().ark_cuda_opt_init(ctypes.byref(cfg),
                                                                      ctypes.byref(h)))
        self._h = h

    # -- the step ---------------------------------------------------------
    def step_all(self, w16, g16, m, v):
        """Enqueue one optimizer step (training.rs:289-326 + optimizer.rs:171-228)
        on this shard.  Asynchronous: nothing is waited for."""
        L = _lib.lib()
        rc = L.ark_cuda_opt_step(self._h, _ptr(w16, "f16", self.n), _ptr(g16, "f16", self.n),
                                 _ptr(m, "f32", self.n), _ptr(v, "f32", self.n))
        _lib.check("ark_cuda_opt_step", rc)

    def grad_buffer(self, n_full: int | None = None):
        """This rank's full gradient buffer for step_reduce (FP16, all
        n_full global elements, zeroed), as a CUDA tensor over library
        memory.  Collective: every rank calls it."""
        n_full = self.layout.n if n_full is None else int(n_full)
        p = ctypes.c_void_p()
        _lib.check("ark_cuda_opt_grad_buffer",
                   _lib.lib().ark_cuda_opt_grad_buffer(self._h, n_full, ctypes.byref(p)))
        self._gbuf = self._device_view(p.value, n_full, "<f2")
        return self._gbuf

    def _device_view(self, ptr, n, typestr):
        import torch

        class _View:
            __cuda_array_interface__ = {"shape": (n,), "typestr": typestr, "data": (ptr, False),
                                        "version": 3, "strides": None}

        return torch.as_tensor(_View(), device=torch.device("cuda", self._cfg.device))

    def weight_buffer(self, n_full: int | None = None):
        """This rank's full FP16 weight buffer for step_gather (all n_full
        global elements, zeroed), as a CUDA tensor over library memory,
        mapped into every rank.  Collective: every rank calls it."""
        n_full = self.layout.n if n_full is None else int(n_full)
        p = ctypes.c_void_p()
        _lib.check("ark_cuda_opt_weight_buffer",
                   _lib.lib().ark_cuda_opt_weight_buffer(self._h, n_full, ctypes.byref(p)))
        self._wbuf = self._device_view(p.value, n_full, "<f2")
        return self._wbuf

    def step_gather(self, w16, g16, m, v, reduce: bool = False):
        """step_all (or step_reduce) fused with the ZeRO-1 weight all-gather:
        the update kernel also stores the updated shard into every rank's
        weight_buffer().  w16 may be this rank's slice of that buffer."""
        opts = _lib.ARK_STEP_GATHER_WEIGHTS | (_lib.ARK_STEP_REDUCE if reduce else 0)
        rc = _lib.lib().ark_cuda_opt_step_ex(
            self._h, _ptr(w16, "f16", self.n), _ptr(g16, "f16", self.n), _ptr(m, "f32", self.n),
            _ptr(v, "f32", self.n), None, opts)
        _lib.check("ark_cuda_opt_step_ex", rc)

    def weights_wait(self):
        """Order this stream's next work after every rank's stores of the
        last step_gather into this rank's weight_buffer() (bounded wait)."""
        _lib.check("ark_cuda_opt_weights_wait", _lib.lib().ark_cuda_opt_weights_wait(self._h))

    def logits_check(self, logits_grad):
        """training.rs:228-245 on the device: count non-finite logits
        gradients (FP32 CUDA tensor) and multiply them in place by the
        current loss scale; a non-finite value makes the next step a skipped
        overflow step.  Asynchronous."""
        n = logits_grad.numel()
        _lib.check("ark_cuda_opt_logits_check", _lib.lib().ark_cuda_opt_logits_check(
            self._h, _ptr(logits_grad, "f32", n), n))

    def zero_grads(self):
        """Zero this rank's grad_buffer() on the step's stream
        (memory.rs:338-342), for a backward that accumulates with +=."""
        _lib.check("ark_cuda_opt_zero_grads", _lib.lib().ark_cuda_opt_zero_grads(self._h))

    def step_reduce(self, w16, g16_shard, m, v):
        """One step on the sum over ranks of every rank's grad_buffer():
        the gradient hand-off fused with pass 1 (peer reads over NVLink);
        the reduced FP16 shard is written to g16_shard."""
        rc = _lib.lib().ark_cuda_opt_step_reduce(
            self._h, _ptr(w16, "f16", self.n), _ptr(g16_shard, "f16", self.n),
            _ptr(m, "f32", self.n), _ptr(v, "f32", self.n))
        _lib.check("ark_cuda_opt_step_reduce", rc)

    def step_all_w32(self, w16, g16, m, v, w32, reduce: bool = False):
        """step_all (or step_reduce) that also writes the updated weights
        widened to FP32 into w32 -- the forward's copy, in place of a
        separate dequant of every weight tensor each step."""
        rc = _lib.lib().ark_cuda_opt_step_ex(
            self._h, _ptr(w16, "f16", self.n), _ptr(g16, "f16", self.n), _ptr(m, "f32", self.n),
            _ptr(v, "f32", self.n), _ptr(w32, "f32", self.n),
            _lib.ARK_STEP_REDUCE if reduce else 0)
        _lib.check("ark_cuda_opt_step_ex", rc)

    def upload_grads(self, g16_dev, g16_host):
        """Asynchronous H2D copy of this shard's scaled grads (host tensor or
        numpy array; pinned memory for full speed)."""
        if hasattr(g16_host, "data_ptr"):
            hp = g16_host.data_ptr()
        else:
            hp = np.ascontiguousarray(g16_host).ctypes.data
        rc = _lib.lib().ark_cuda_opt_upload_grads(self._h, _ptr(g16_dev, "f16", self.n), hp,
                                                  self.n)
        _lib.check("ark_cuda_opt_upload_grads", rc)

    def read_status(self):
        """Wait for the stream; returns (status code, ark_opt_status dict)."""
        st = _lib.OptStatus()
        rc = _lib.lib().ark_cuda_opt_read_status(self._h, ctypes.byref(st))
        return rc, st.as_dict()

    def status(self):
        rc, st = self.read_status()
        if rc not in (_lib.ARK_OK, _lib.ARK_E_EARLY_STOP):
            raise _lib.ArkError("ark_cuda_opt_read_status", rc)
        return st

    def set_status(self, **fields):
        """Overwrite state fields (resume: optimizer.rs:308 sets step)."""
        _, cur = self.read_status()
        cur.update(fields)
        st = _lib.OptStatus(**cur)
        _lib.check("ark_cuda_opt_set_status",
                   _lib.lib().ark_cuda_opt_set_status(self._h, ctypes.byref(st)))

    @property
    def step(self) -> int:
        """Optimizer.step (optimizer.rs:70); waits for the device."""
        return self.status()["opt_step"]

    @property
    def loss_scale(self) -> float:
        return self.status()["loss_scale"]

    def lr_now(self, step: int) -> float:
        return float(self.lr_table[min(step, len(self.lr_table) - 1)])

    def allgather_weights(self, w16_shard, w16_full, shard_stride: int):
        rc = _lib.lib().ark_cuda_allgather_weights(self._h, _ptr(w16_shard, "f16", self.n),
                                                   _ptr(w16_full, "f16"), shard_stride)
        _lib.check("ark_cuda_allgather_weights", rc)

    def profile_begin(self, max_steps: int):
        _lib.check("ark_cuda_opt_profile_begin",
                   _lib.lib().ark_cuda_opt_profile_begin(self._h, max_steps))

    def profile_read(self, capacity: int):
        """Per step [pass-1 ms, exchange ms, pass-2 ms] from CUDA events."""
        buf = (ctypes.c_float * (3 * capacity))()
        k = ctypes.c_uint32()
        _lib.check("ark_cuda_opt_profile_read",
                   _lib.lib().ark_cuda_opt_profile_read(self._h, buf, capacity, ctypes.byref(k)))
        return np.frombuffer(buf, np.float32)[: 3 * k.value].reshape(k.value, 3).copy()

    def geometry(self):
        b1, b2, t = ctypes.c_uint32(), ctypes.c_uint32(), ctypes.c_uint32()
        _lib.check("ark_cuda_opt_geometry", _lib.lib().ark_cuda_opt_geometry(
            self._h, ctypes.byref(b1), ctypes.byref(b2), ctypes.byref(t)))
        return {"pass1_blocks": b1.value, "pass2_blocks": b2.value, "threads": t.value}

    def close(self):
        if getattr(self, "_h", None):
            _lib.lib().ark_cuda_opt_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ----------------------------------------------------------------- legacy kernels
def _legacy_check(fn):
    rc = _lib.lib().ark_cuda_last_error()
    if rc != _lib.ARK_OK:
        raise _lib.ArkError(fn, rc)


def adam_step_f16(w, g, m, v, lr, beta1, beta2, eps, wd, t):
    """ark_asm_adam_step_f16 (opti.s:192-360) on device tensors."""
    n = g.numel()
    _lib.lib().ark_asm_adam_step_f16(_ptr(w, "f16", n), _ptr(g, "f32", n), _ptr(m, "f32", n),
                                     _ptr(v, "f32", n), n, lr, beta1, beta2, eps, wd, t)
    _legacy_check("ark_asm_adam_step_f16")


def adam_step(w, g, m, v, lr, beta1, beta2, eps, wd, t):
    """ark_asm_adam_step (opti.s:20-177) on device tensors."""
    n = g.numel()
    _lib.lib().ark_asm_adam_step(_ptr(w, "f32", n), _ptr(g, "f32", n), _ptr(m, "f32", n),
                                 _ptr(v, "f32", n), n, lr, beta1, beta2, eps, wd, t)
    _legacy_check("ark_asm_adam_step")


def grad_clip(g, threshold) -> float:
    """ark_asm_grad_clip (opti.s:369-432): returns the pre-clip norm."""
    n = g.numel()
    norm = _lib.lib().ark_asm_grad_clip(_ptr(g, "f32", n), n, threshold)
    _legacy_check("ark_asm_grad_clip")
    return norm


def quant_f32_to_f16(src, dst):
    n = src.numel()
    _lib.lib().ark_quant_f32_to_f16(_ptr(src, "f32", n), _ptr(dst, "f16", n), n)
    _legacy_check("ark_quant_f32_to_f16")


def dequant_f16_to_f32(src, dst):
    n = src.numel()
    _lib.lib().ark_dequant_f16_to_f32(_ptr(src, "f16", n), _ptr(dst, "f32", n), n)
    _legacy_check("ark_dequant_f16_to_f32")


def set_compat(flags: int):
    _lib.check("ark_cuda_set_compat", _lib.lib().ark_cuda_set_compat(flags))


def legacy_set_async(flag: bool):
    _lib.lib().ark_cuda_legacy_set_async(1 if flag else 0)


def legacy_sync():
    _lib.check("ark_cuda_legacy_sync", _lib.lib().ark_cuda_legacy_sync())
