"""CPU restatement of ARK's checkpoint writer and reader (TEST
INFRASTRUCTURE ONLY: the checker for ark_cuda_ckpt_save / _load).

proyecto_ark/ark01/src/io.rs:432-500 (CheckpointV3::save_fp16, format V4)
and :504-636 (load of V4 and V3); tensor order from training.rs:536-604.
"""
from __future__ import annotations

import struct

import numpy as np

MAGIC_V4 = 0x4B345241
MAGIC_V3 = 0x4B335241


def file_order(layout):
    """Model tensors in ARK4 order: embed, layers (9 each), gamma_final."""
    return [layout.tensors[0]] + layout.tensors[2:] + [layout.tensors[1]]


def records(layout):
    """[(tensor, kind)] in file order; kind 0 = w, 1 = m, 2 = v."""
    ts = file_order(layout)
    L = (len(ts) - 2) // 9
    out = [(ts[0], k) for k in range(3)]
    for l in range(L):
        for k in range(3):
            out += [(ts[1 + 9 * l + i], k) for i in range(9)]
    out += [(ts[-1], k) for k in range(3)]
    return out


def save_v4(path, layout, global_step, adam_step, w16, m, v):
    """io.rs:432-500 from flat arrays (indices per layout.offsets)."""
    recs = records(layout)
    with open(path, "wb") as f:
        f.write(struct.pack("<IQQQ", MAGIC_V4, global_step, adam_step, len(recs)))
        for t, k in recs:
            o = layout.offsets[t.name]
            src = (w16, m, v)[k][o:o + t.numel]
            f.write(struct.pack("<QQ", t.numel, 0 if k == 0 else 1))
            f.write(np.ascontiguousarray(src, np.uint16 if k == 0 else np.float32).tobytes())


def save_v3(path, layout, global_step, adam_step, w32, m, v):
    """ARK3: FP32 weights and moments, no type field, no gamma_final
    (io.rs:597-636 reads it back)."""
    recs = records(layout)[:-3]
    with open(path, "wb") as f:
        f.write(struct.pack("<IQQQ", MAGIC_V3, global_step, adam_step, len(recs)))
        for t, k in recs:
            o = layout.offsets[t.name]
            src = (w32, m, v)[k][o:o + t.numel]
            f.write(struct.pack("<Q", t.numel))
            f.write(np.ascontiguousarray(src, np.float32).tobytes())


def load_v4(path, layout):
    """io.rs:541-595: returns (global_step, adam_step, w16, m, v, trailer)
    with flat arrays (trailer = bytes after the last tensor, if any)."""
    data = open(path, "rb").read()
    magic, gs, adam, nt = struct.unpack_from("<IQQQ", data, 0)
    assert magic == MAGIC_V4
    recs = records(layout)
    assert nt == len(recs)
    w16 = np.zeros(layout.n, np.uint16)
    m = np.zeros(layout.n, np.float32)
    v = np.zeros(layout.n, np.float32)
    off = 28
    for t, k in recs:
        n, typ = struct.unpack_from("<QQ", data, off)
        off += 16
        assert n == t.numel and typ == (0 if k == 0 else 1)
        dt = np.uint16 if typ == 0 else np.float32
        arr = np.frombuffer(data, dt, n, off)
        off += n * np.dtype(dt).itemsize
        o = layout.offsets[t.name]
        (w16, m, v)[k][o:o + n] = arr
    return gs, adam, w16, m, v, data[off:]
