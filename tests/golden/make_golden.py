"""Generate the golden vectors under tests/golden/ by executing ARK's own
assembly (proyecto_ark/ark01/asm/opti.s, asm/kern.s) in the AArch64 emulator
of a64emu.py.

Run in a checkout that has the reference tree next to it:

    python tests/golden/make_golden.py --reference <path to the ARK tree>

The output (golden_asm.npz) is committed; the reference tree is only needed
to regenerate it.  Inputs are drawn from numpy's PCG64 with fixed seeds, and
include the edge cases the kernels branch on: lengths that exercise the
8-/4-wide loops and every tail length, t = 0 (coerced to 1 by the kernel) and
large t, wd = 0, zero moments, FP16 overflow/subnormal weights, and the
special values of the FP16 conversions.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import sys

import numpy as np

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
import a64emu  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
EKO = dict(lr=3e-4, b1=0.9, b2=0.95, eps=1e-8, wd=0.1, t=1000)


def _adam_inputs(rng, n, kind="eko"):
    w = rng.normal(0, 0.02, n).astype(np.float32)
    g = rng.normal(0, 1e-3, n).astype(np.float32)
    m = rng.normal(0, 1e-4, n).astype(np.float32)
    v = (rng.normal(0, 1e-3, n) ** 2).astype(np.float32)
    if kind == "zero_moments":
        m[:] = 0
        v[:] = 0
    elif kind == "extreme":
        # weights at the FP16 limits and in the subnormal range, large grads
        w[0::5] = 65504.0
        w[1::5] = -65504.0
        w[2::5] = 3e-6
        w[3::5] = -6.0e-8
        g = (g * 1e4).astype(np.float32)
        g[4::7] = 0.0
        m[::3] = 0.0
        v[::2] = 0.0
    elif kind == "subnormal_state":
        m = (m * 1e-34).astype(np.float32)
        v = (v * 1e-33).astype(np.float32)
        g = (g * 1e-36).astype(np.float32)
    return w, g, m, v


def adam_cases():
    cases = []
    for n in (0, 1, 3, 4, 5, 7, 8, 9, 768, 4097):
        cases.append(dict(n=n, kind="eko", **EKO))
    for t in (0, 1, 2, 7, 360000, 0xFFFFFFFF):
        cases.append(dict(n=9, kind="eko", **{**EKO, "t": t}))
    cases.append(dict(n=768, kind="eko", **{**EKO, "wd": 0.0}))
    cases.append(dict(n=64, kind="eko", lr=3e-4, b1=0.9, b2=0.999, eps=1e-8, wd=0.01, t=5))
    cases.append(dict(n=61, kind="zero_moments", **{**EKO, "t": 1}))
    cases.append(dict(n=103, kind="extreme", lr=1.0, b1=0.9, b2=0.95, eps=1e-8, wd=0.1, t=3))
    cases.append(dict(n=33, kind="subnormal_state", **{**EKO, "eps": 1e-30}))
    cases.append(dict(n=257, kind="eko", lr=5e-2, b1=0.5, b2=0.75, eps=1e-3, wd=0.5, t=11))
    return cases


def clip_cases(rng):
    out = []
    for n in (0, 1, 3, 4, 5, 8, 777, 4097):
        out.append((rng.normal(0, 1, n).astype(np.float32), 1.0))
    out.append((rng.normal(0, 1e-3, 300).astype(np.float32), 1.0))        # no clip
    out.append((rng.normal(0, 1, 64).astype(np.float32), 0.5))
    z = np.zeros(16, np.float32)
    out.append((z, 1.0))                                                  # norm 0
    g = rng.normal(0, 1, 21).astype(np.float32)
    g[7] = np.nan
    out.append((g, 1.0))                                                  # NaN norm: no scale
    g = rng.normal(0, 1, 12).astype(np.float32)
    g[3] = np.inf
    out.append((g, 1.0))                                                  # inf norm: scale by 0
    out.append((rng.normal(0, 1, 40).astype(np.float32), float("nan")))   # NaN threshold
    return out


def quant_input(rng):
    specials = np.array([
        0.0, -0.0, 1.0, -1.0, 0.5, 65504.0, -65504.0, 65519.0, 65519.996, 65520.0, -65520.0,
        1e5, -1e5, 3.4e38, np.inf, -np.inf, 6.1035156e-05, 6.097555e-05, 5.9604645e-08,
        2.9802322e-08, 2.9802326e-08, 8.940697e-08, 1e-10, -1e-10, 1.4e-45, 1.17549435e-38,
        1.0009765625, 1.00048828125, 1.00146484375, 2049.0, 2051.0, -2051.0, 4097.0,
    ], dtype=np.float32)
    nan_bits = np.array([0x7FC00000, 0xFFC00001, 0x7F800001, 0x7FBFFFFF, 0x7FC12345],
                        dtype=np.uint32).view(np.float32)
    rnd = np.concatenate([
        rng.normal(0, 1, 1000), rng.normal(0, 1e-5, 1000), rng.normal(0, 3e4, 1000),
        rng.uniform(-1e-7, 1e-7, 1000),
    ]).astype(np.float32)
    x = np.concatenate([specials, nan_bits, rnd]).astype(np.float32)
    # every f16 value and both neighbouring midpoints (ties) of a sample of them
    h = rng.integers(0, 0x7C00, 300).astype(np.uint16)
    hv = h.view(np.float16).astype(np.float32)
    nxt = (h + 1).view(np.float16).astype(np.float32)
    mids = ((hv.astype(np.float64) + nxt.astype(np.float64)) / 2).astype(np.float32)
    return np.concatenate([x, mids, -mids]).astype(np.float32)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path to the ARK repository root")
    ap.add_argument("--out", default=os.path.join(HERE, "golden_asm.npz"))
    args = ap.parse_args()
    asm_dir = os.path.join(args.reference, "proyecto_ark", "ark01", "asm")
    opti_path, kern_path = os.path.join(asm_dir, "opti.s"), os.path.join(asm_dir, "kern.s")
    opti, kern = a64emu.AsmModule(opti_path), a64emu.AsmModule(kern_path)
    arrays, meta = {}, {"source": {}, "adam_f16": [], "adam_f32": [], "clip": [], "quant": [], "dequant": []}
    for p in (opti_path, kern_path):
        with open(p, "rb") as f:
            meta["source"][os.path.basename(p)] = hashlib.sha256(f.read()).hexdigest()

    rng = np.random.default_rng(20261201)
    for i, c in enumerate(adam_cases()):
        w, g, m, v = _adam_inputs(rng, c["n"], c["kind"])
        w16 = w.astype(np.float16).view(np.uint16)
        W, M, V = opti.adam_step_f16(w16, g, m, v, c["lr"], c["b1"], c["b2"], c["eps"], c["wd"], c["t"])
        k = f"adam16_{i}"
        arrays.update({k + "_w": w16, k + "_g": g, k + "_m": m, k + "_v": v,
                       k + "_W": W, k + "_M": M, k + "_V": V})
        meta["adam_f16"].append({"key": k, **c})
    for i, c in enumerate([dict(n=n, kind="eko", **EKO) for n in (0, 5, 8, 13, 256)]
                          + [dict(n=50, kind="extreme", lr=1.0, b1=0.9, b2=0.95, eps=1e-8, wd=0.1, t=2)]):
        w, g, m, v = _adam_inputs(rng, c["n"], c["kind"])
        W, M, V = opti.adam_step_f32(w, g, m, v, c["lr"], c["b1"], c["b2"], c["eps"], c["wd"], c["t"])
        k = f"adam32_{i}"
        arrays.update({k + "_w": w, k + "_g": g, k + "_m": m, k + "_v": v,
                       k + "_W": W, k + "_M": M, k + "_V": V})
        meta["adam_f32"].append({"key": k, **c})
    for i, (g, thr) in enumerate(clip_cases(rng)):
        norm, G = opti.grad_clip(g, thr)
        k = f"clip_{i}"
        arrays.update({k + "_g": g, k + "_G": G, k + "_norm": np.array([norm], np.float32)})
        meta["clip"].append({"key": k, "n": int(len(g)), "thr": float(thr)})
    x = quant_input(rng)
    for i, n in enumerate((len(x), 7, 12, 0)):
        src = x[:n]
        arrays[f"quant_{i}_x"] = src
        arrays[f"quant_{i}_h"] = kern.quant_f32_to_f16(src)
        meta["quant"].append({"key": f"quant_{i}", "n": int(n)})
    allh = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    for i, src in enumerate((np.concatenate([allh, allh[:7]]), allh[:13], allh[:0])):
        arrays[f"dequant_{i}_h"] = src
        arrays[f"dequant_{i}_f"] = kern.dequant_f16_to_f32(src)
        meta["dequant"].append({"key": f"dequant_{i}", "n": int(len(src))})

    arrays["meta"] = np.frombuffer(json.dumps(meta, sort_keys=True).encode(), dtype=np.uint8)
    np.savez_compressed(args.out, **arrays)
    print(f"wrote {args.out}: {len(meta['adam_f16'])} adam_f16, {len(meta['adam_f32'])} adam_f32, "
          f"{len(meta['clip'])} clip, {len(meta['quant'])} quant, {len(meta['dequant'])} dequant cases")


if __name__ == "__main__":
    main()
