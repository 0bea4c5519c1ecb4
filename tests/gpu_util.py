"""Helpers shared by the GPU parity tests (host<->device with exact bits)."""
import numpy as np


def dev(a):
    import torch
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.float16).copy()).cuda()
    return torch.from_numpy(a.copy()).cuda()


def host(t):
    import torch
    a = t.detach().cpu()
    if a.dtype == torch.float16:
        return a.numpy().view(np.uint16)
    return a.numpy()


def same_f32(a, b):
    """float32 arrays bit-equal, any NaN equal to any NaN."""
    a, b = np.asarray(a, np.float32), np.asarray(b, np.float32)
    if a.shape != b.shape:
        return False
    na, nb = np.isnan(a), np.isnan(b)
    return bool(np.array_equal(na, nb) and np.array_equal(a[~na].view(np.uint32),
                                                          b[~nb].view(np.uint32)))


def f16_isnan(h):
    h = np.asarray(h, np.uint16)
    return ((h & 0x7C00) == 0x7C00) & ((h & 0x3FF) != 0)


def same_f16(a, b):
    a, b = np.asarray(a, np.uint16), np.asarray(b, np.uint16)
    if a.shape != b.shape:
        return False
    na, nb = f16_isnan(a), f16_isnan(b)
    return bool(np.array_equal(na, nb) and np.array_equal(a[~na], b[~nb]))


def first_diff(a, b):
    idx = np.nonzero(np.asarray(a) != np.asarray(b))[0]
    return int(idx[0]) if len(idx) else None
