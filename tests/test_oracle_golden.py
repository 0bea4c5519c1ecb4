"""The CPU oracle against golden vectors produced by executing the
reference's own assembly (opti.s, kern.s) in tests/golden/a64emu.py.
Bit-exact; a NaN matches any NaN (the payload of a NaN produced by an invalid
operation is architecture-specific: 0x7FC00000 on Arm, 0xFFC00000 on x86).
The FP16 conversions keep NaN payloads and are compared bit for bit."""
import numpy as np
import pytest


@pytest.fixture(scope="module")
def golden(oracle):
    return oracle.load_golden()


def _bits(a):
    return np.asarray(a).view(np.uint32 if np.asarray(a).dtype == np.float32 else np.uint16)


def same(a, b):
    """Bit-equal float32 arrays, any NaN equal to any NaN."""
    a, b = np.asarray(a, np.float32), np.asarray(b, np.float32)
    if a.shape != b.shape:
        return False
    na, nb = np.isnan(a), np.isnan(b)
    return bool(np.array_equal(na, nb) and np.array_equal(_bits(a[~na]), _bits(b[~nb])))


def test_golden_provenance(golden):
    meta, _ = golden
    assert set(meta["source"]) == {"opti.s", "kern.s"}
    assert len(meta["adam_f16"]) >= 20 and len(meta["clip"]) >= 10


def test_adam_f16_bit_exact(oracle, golden):
    meta, z = golden
    for c in meta["adam_f16"]:
        k = c["key"]
        W, M, V = oracle.adam_step_f16(z[k + "_w"], z[k + "_g"], z[k + "_m"], z[k + "_v"],
                                       c["lr"], c["b1"], c["b2"], c["eps"], c["wd"], c["t"])
        assert np.array_equal(W, z[k + "_W"]), k
        assert same(M, z[k + "_M"]), k
        assert same(V, z[k + "_V"]), k


def test_adam_f32_bit_exact(oracle, golden):
    meta, z = golden
    for c in meta["adam_f32"]:
        k = c["key"]
        W, M, V = oracle.adam_step_f32(z[k + "_w"], z[k + "_g"], z[k + "_m"], z[k + "_v"],
                                       c["lr"], c["b1"], c["b2"], c["eps"], c["wd"], c["t"])
        for a, b in ((W, "_W"), (M, "_M"), (V, "_V")):
            assert same(a, z[k + b]), k + b


def test_grad_clip_literal_fold_bit_exact(oracle, golden):
    meta, z = golden
    for c in meta["clip"]:
        k = c["key"]
        norm, G = oracle.grad_clip_neon(z[k + "_g"], c["thr"])
        assert same([norm], z[k + "_norm"]), k
        assert same(G, z[k + "_G"]), k


def test_grad_clip_exact_norm_within_tolerance(oracle, golden):
    """The accurate norm (what the B200 library returns) against the
    reference's 4-lane f32 fold: within the 1e-5 relative parity bound at
    these sizes."""
    meta, z = golden
    for c in meta["clip"]:
        k = c["key"]
        g = z[k + "_g"]
        if not np.all(np.isfinite(g)) or c["n"] == 0:
            continue
        norm, _ = oracle.grad_clip_exact(g, c["thr"])
        ref = z[k + "_norm"][0]
        if ref == 0:
            assert norm == 0
        else:
            assert abs(float(norm) - float(ref)) <= 1e-5 * float(ref), k


def test_quant_dequant_bit_exact(oracle, golden):
    meta, z = golden
    for c in meta["quant"]:
        k = c["key"]
        assert np.array_equal(oracle.quant(z[k + "_x"]), z[k + "_h"]), k
    for c in meta["dequant"]:
        k = c["key"]
        assert np.array_equal(_bits(oracle.dequant(z[k + "_h"])), _bits(z[k + "_f"])), k


def test_dequant_covers_every_half(golden):
    meta, z = golden
    h = z["dequant_0_h"]
    assert len(np.unique(h)) == 65536
