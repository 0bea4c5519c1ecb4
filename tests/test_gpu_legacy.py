"""The five legacy entry points (same names and signatures as ARK's
libark_asm.a) on a B200, through the C ABI, against golden vectors produced
by the reference's own assembly and against the CPU oracle."""
import numpy as np
import pytest

import ark_b200 as ab
from gpu_util import dev, host, same_f16, same_f32

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def golden(oracle):
    return oracle.load_golden()


def test_adam_f16_golden_bit_exact(golden):
    meta, z = golden
    for c in meta["adam_f16"]:
        k = c["key"]
        if c["n"] == 0:
            continue
        w, g, m, v = dev(z[k + "_w"]), dev(z[k + "_g"]), dev(z[k + "_m"]), dev(z[k + "_v"])
        ab.adam_step_f16(w, g, m, v, c["lr"], c["b1"], c["b2"], c["eps"], c["wd"], c["t"])
        assert same_f16(host(w), z[k + "_W"]), k
        assert same_f32(host(m), z[k + "_M"]), k
        assert same_f32(host(v), z[k + "_V"]), k


def test_adam_f32_golden_bit_exact(golden):
    meta, z = golden
    for c in meta["adam_f32"]:
        k = c["key"]
        if c["n"] == 0:
            continue
        w, g, m, v = dev(z[k + "_w"]), dev(z[k + "_g"]), dev(z[k + "_m"]), dev(z[k + "_v"])
        ab.adam_step(w, g, m, v, c["lr"], c["b1"], c["b2"], c["eps"], c["wd"], c["t"])
        for t, key in ((w, "_W"), (m, "_M"), (v, "_V")):
            assert same_f32(host(t), z[k + key]), k + key


@pytest.mark.parametrize("n,shift", [(1_000_003, 0), (1_000_003, 1), (4099, 3), (17, 2)])
def test_adam_f16_random_vs_oracle(oracle, n, shift):
    """Large and misaligned (views starting `shift` elements in) buffers."""
    w = oracle.synth_f16(n + shift, 0, 21, 1, 0.02)
    g = oracle.synth_f32(n + shift, 0, 21, 2, 1e-3)
    m = oracle.synth_f32(n + shift, 0, 21, 3, 1e-4)
    v = oracle.synth_f32(n + shift, 0, 21, 4, 1e-3, square=True)
    W, M, V = oracle.adam_step_f16(w[shift:], g[shift:], m[shift:], v[shift:],
                                   3e-4, 0.9, 0.95, 1e-8, 0.1, 1000)
    dw, dg, dm, dv = dev(w), dev(g), dev(m), dev(v)
    ab.adam_step_f16(dw[shift:], dg[shift:], dm[shift:], dv[shift:], 3e-4, 0.9, 0.95, 1e-8, 0.1,
                     1000)
    assert same_f16(host(dw)[shift:], W)
    assert same_f32(host(dm)[shift:], M) and same_f32(host(dv)[shift:], V)
    assert np.array_equal(host(dw)[:shift], w[:shift])           # untouched prefix


def test_grad_clip_accurate_norm(oracle, golden):
    meta, z = golden
    cases = [(z[c["key"] + "_g"], c["thr"]) for c in meta["clip"]]
    cases.append((oracle.synth_f32(3_000_001, 0, 4, 9, 1e-3), 1.0))
    cases.append((oracle.synth_f32(24_576_000, 0, 4, 9, 1e-3), 1.0))   # EKO embedding size
    for g, thr in cases:
        ref_norm, ref_g = oracle.grad_clip_exact(g, thr)
        d = dev(g)
        norm = np.float32(ab.grad_clip(d, thr))
        if not np.isfinite(ref_norm):
            assert (np.isnan(norm) and np.isnan(ref_norm)) or norm == ref_norm
            assert same_f32(host(d), ref_g)
            continue
        assert abs(float(norm) - float(ref_norm)) <= 1e-5 * max(float(ref_norm), 1e-30)
        if norm == ref_norm:
            assert same_f32(host(d), ref_g)


def test_grad_clip_reference_fold_compat(golden):
    meta, z = golden
    ab.set_compat(ab._lib.ARK_COMPAT_CLIP_NEON_FOLD)
    try:
        for c in meta["clip"]:
            k = c["key"]
            d = dev(z[k + "_g"])
            norm = np.float32(ab.grad_clip(d, c["thr"]))
            assert same_f32([norm], z[k + "_norm"]), k
            assert same_f32(host(d), z[k + "_G"]), k
    finally:
        ab.set_compat(0)


def test_quant_dequant_golden(golden):
    import torch
    meta, z = golden
    for c in meta["quant"]:
        k = c["key"]
        if c["n"] == 0:
            continue
        src = dev(z[k + "_x"])
        dst = torch.empty(c["n"], dtype=torch.float16, device="cuda")
        ab.quant_f32_to_f16(src, dst)
        assert same_f16(host(dst), z[k + "_h"]), k
    for c in meta["dequant"]:
        k = c["key"]
        if c["n"] == 0:
            continue
        src = dev(z[k + "_h"])
        dst = torch.empty(c["n"], dtype=torch.float32, device="cuda")
        ab.dequant_f16_to_f32(src, dst)
        assert same_f32(host(dst), z[k + "_f"]), k


@pytest.mark.parametrize("shift", [0, 1, 5])
def test_conversions_misaligned_vs_oracle(oracle, shift):
    import torch
    n = 100_003
    x = oracle.synth_f32(n + shift, 0, 8, 5, 300.0)
    src = dev(x)
    dst = torch.zeros(n + shift, dtype=torch.float16, device="cuda")
    ab.quant_f32_to_f16(src[shift:], dst[shift:])
    assert np.array_equal(host(dst)[shift:], oracle.quant(x[shift:]))
    back = torch.zeros(n + shift, dtype=torch.float32, device="cuda")
    ab.dequant_f16_to_f32(dst[shift:], back[shift:])
    assert same_f32(host(back)[shift:], oracle.dequant(host(dst)[shift:]))


def test_n_zero_is_a_no_op():
    L = ab.lib()
    L.ark_asm_adam_step_f16(None, None, None, None, 0, 1e-3, 0.9, 0.95, 1e-8, 0.1, 1)
    assert L.ark_cuda_last_error() == 0
    assert L.ark_asm_grad_clip(None, 0, 1.0) == 0.0
    L.ark_quant_f32_to_f16(None, None, 0)
    L.ark_dequant_f16_to_f32(None, None, 0)
    assert L.ark_cuda_last_error() == 0


def test_null_pointer_is_reported_not_crashed():
    L = ab.lib()
    L.ark_asm_adam_step_f16(None, None, None, None, 8, 1e-3, 0.9, 0.95, 1e-8, 0.1, 1)
    assert L.ark_cuda_last_error() == -1
    with pytest.raises(ab.ArkError):
        ab.optimizer._legacy_check("ark_asm_adam_step_f16")
