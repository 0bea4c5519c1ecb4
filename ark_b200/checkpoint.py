"""ARK4 checkpoints of a (sharded) optimizer state, through libark_cuda.

File format and order: proyecto_ark/ark01/src/io.rs:12-24, 432-500; the
rotating file name of training.rs:583-586.  Each rank saves / loads only its
own shard of the one file (see ark_cuda_ckpt_save in include/ark_opt.h).
"""
from __future__ import annotations

import ctypes

from . import _lib
from .layout import Layout
from .optimizer import Optimizer, _ptr


def ckpt_tensors(layout: Layout):
    """The model tensors in ARK4 file order (embed, the 9 tensors of every
    layer, gamma_final) with their offsets in the flat index space."""
    names = [t.name for t in layout.tensors]
    if names[:2] != ["embed", "gamma_final"] or (len(names) - 2) % 9:
        raise ValueError("not an ARK decoder layout")
    order = [layout.tensors[0]] + layout.tensors[2:] + [layout.tensors[1]]
    arr = (_lib.CkptTensor * len(order))()
    for i, t in enumerate(order):
        arr[i].numel = t.numel
        arr[i].flat_offset = layout.offsets[t.name]
    return arr


def rotating_path(ckpt_path: str, step: int, every: int = 500) -> str:
    """training.rs:583-586: <base>_rot<slot>.bin with slot = (step / every) % 3."""
    base = ckpt_path[:-4] if ckpt_path.endswith(".bin") else ckpt_path
    pos = base.rfind("_rot")
    if pos >= 0:
        base = base[:pos]
    return f"{base}_rot{(step // every) % 3}.bin"


def save(opt: Optimizer, path: str, w16, m, v, global_step: int):
    t = ckpt_tensors(opt.layout)
    rc = _lib.lib().ark_cuda_ckpt_save(opt._h, path.encode(), t, len(t), global_step,
                                       _ptr(w16, "f16", opt.n), _ptr(m, "f32", opt.n),
                                       _ptr(v, "f32", opt.n))
    _lib.check("ark_cuda_ckpt_save", rc)


def load(opt: Optimizer, path: str, w16, m, v, restore_scale: bool = True) -> int:
    """Returns the file's global_step; sets the device optimizer step."""
    t = ckpt_tensors(opt.layout)
    gs = ctypes.c_uint64()
    rc = _lib.lib().ark_cuda_ckpt_load(opt._h, path.encode(), t, len(t), ctypes.byref(gs),
                                       _ptr(w16, "f16", opt.n), _ptr(m, "f32", opt.n),
                                       _ptr(v, "f32", opt.n),
                                       _lib.ARK_CKPT_RESTORE_SCALE if restore_scale else 0)
    _lib.check("ark_cuda_ckpt_load", rc)
    return gs.value
