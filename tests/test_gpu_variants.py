"""Every launch-shape variant of the step (ARK_PASS1_VARIANT,
ARK_PASS2_VARIANT, ARK_PASS2W_VARIANT) and the ordinary (non-programmatic)
launch of pass 2 (ARK_PDL=0) against the CPU oracle: the knobs are read at
ark_cuda_opt_init, so each case builds its own optimizer under its own
environment.  Flags and scale exactly, w, m, v bit for bit."""
import numpy as np
import pytest
import torch

import ark_b200 as ab
from ark_b200 import layout
from gpu_util import dev, host, same_f16, same_f32
from test_gpu_step import SEED, oracle_bufs, run_steps, tiny

pytestmark = pytest.mark.gpu

N_PASS1, N_PASS2 = 10, 7

CASES = ([{"ARK_PDL": "0"}] + [{"ARK_PASS1_VARIANT": str(i)} for i in range(N_PASS1)] +
         [{"ARK_PASS2_VARIANT": str(i)} for i in range(N_PASS2)] +
         # who reduces pass 1's block partials: pass 1's last block (1) or
         # every pass-2 block (0), each with both pass-2 shapes
         [{"ARK_P1_LAST": r, "ARK_PASS2_VARIANT": v} for r in ("0", "1") for v in ("1", "4")])


def case_id(env):
    return ",".join(f"{k[4:].lower()}={v}" for k, v in env.items())


@pytest.mark.parametrize("env", CASES, ids=case_id)
def test_variant_matches_oracle(oracle, env, monkeypatch):
    for k, v in env.items():
        monkeypatch.setenv(k, v)
    st, _ = run_steps(oracle, layout.flat_layout(2048 * 296 * 2 + 8 * 11 + 5), steps=3,
                      inject={2: 0x7C00})
    assert st["skipped_steps"] == 1 and st["opt_step"] == 2


@pytest.mark.parametrize("env", [{"ARK_PASS1_VARIANT": str(i)} for i in (1, 7)] +
                         [{"ARK_PASS2_VARIANT": str(i)} for i in (1, 4, 5)], ids=case_id)
def test_variant_compat_kept_range(oracle, env, monkeypatch):
    """The kernels compiled for a non-empty kept range (compat mode)."""
    for k, v in env.items():
        monkeypatch.setenv(k, v)
    st, _ = run_steps(oracle, tiny(), steps=2, compat=True)
    assert st["opt_step"] == 2


@pytest.mark.parametrize("var,p1_last", [(v, None) for v in range(N_PASS2)] +
                         [(4, "0"), (4, "1")])
def test_fp32_copy_variant(oracle, var, p1_last, monkeypatch):
    """ARK_PASS2W_VARIANT: the step that also writes FP32 weights."""
    monkeypatch.setenv("ARK_PASS2W_VARIANT", str(var))
    if p1_last is not None:
        monkeypatch.setenv("ARK_P1_LAST", p1_last)
    L = layout.flat_layout(300_007)
    opt = ab.Optimizer(L, ab.AdamConfig(lr=3e-4, beta1=0.9, beta2=0.95, eps=1e-8,
                                        weight_decay=0.1, grad_clip=1.0),
                       ab.LossScaleConfig(init=65536.0, every=50, max=2.0 ** 24),
                       constant_lr=True, initial_step=999)
    n = opt.n
    w, g, m, v = oracle_bufs(oracle, n, 0, SEED, 65536.0)
    dw, dg, dm, dv = dev(w), dev(g), dev(m), dev(v)
    w32 = torch.full((n,), float("nan"), dtype=torch.float32, device="cuda")
    opt.step_all_w32(dw, dg, dm, dv, w32)
    cfg = oracle.make_cfg(n_decay=L.n_decay, scale_every=50, scale_max=2.0 ** 24)
    ost = oracle.make_state(65536.0, opt_step=999)
    s, bad = oracle.partial_f16(cfg, ost, g, 0)
    oracle.apply_f16(cfg, ost, w, g, m, v, 0, s, bad)
    assert same_f16(host(dw), w) and same_f32(host(dm), m) and same_f32(host(dv), v)
    assert np.array_equal(host(w32), oracle.dequant(w))
    opt.close()
