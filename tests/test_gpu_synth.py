"""The device input generator is bit-identical to the CPU one (so the
oracle can regenerate any shard the benchmark and the tests use)."""
import numpy as np
import pytest
import torch

from ark_b200 import synth
from gpu_util import host

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("offset", [0, 12345, 2**33 + 7])
def test_synth_matches_cpu(oracle, offset):
    n = 50_001
    t16 = torch.empty(n, dtype=torch.float16, device="cuda")
    synth.fill_f16(t16, offset, 99, 2, 1e-3, mult=65536.0, heavy_every=100, heavy_mult=100.0)
    ref16 = oracle.synth_f16(n, offset, 99, 2, 1e-3, 65536.0, 100, 100.0)
    assert np.array_equal(host(t16), ref16)
    t32 = torch.empty(n, dtype=torch.float32, device="cuda")
    synth.fill_f32(t32, offset, 99, 4, 1e-3, square=True)
    ref32 = oracle.synth_f32(n, offset, 99, 4, 1e-3, square=True)
    assert np.array_equal(host(t32).view(np.uint32), ref32.view(np.uint32))


def test_distribution_moments():
    n = 4_000_000
    t = torch.empty(n, dtype=torch.float32, device="cuda")
    synth.fill_f32(t, 0, 1, 3, 1.0)
    x = t.double()
    assert abs(x.mean().item()) < 2e-3 and abs(x.std().item() - 1.0) < 2e-3
