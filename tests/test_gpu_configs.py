"""Full-size BASELINE configurations on one B200: the 1.3B decoder, the 7B
decoder with heavy-tailed gradients (1 % of elements x100, clipping active)
and a flat buffer past 2^32 elements (64-bit indexing).

Checks that hold at any size: the device's global sum of squares against
the oracle's exact sum over every element, the overflow / clip decision and
the state, and w, m, v bit for bit on sampled windows (the ends, the
weight-decay boundary, tensor boundaries, and around 2^31 / 2^32)."""
import numpy as np
import pytest
import torch

import ark_b200 as ab
from ark_b200 import layout, synth
from gpu_util import same_f16, same_f32

pytestmark = pytest.mark.gpu

SEED = 4242
SCALE = 65536.0


def _fits(n):
    torch.cuda.empty_cache()
    free, _ = torch.cuda.mem_get_info()
    return free > n * 14 * 1.08 + (2 << 30)


def _windows(L, extra=()):
    n = L.n
    w = [(0, 4096), (max(0, n - 4096), n), (n // 2 - 2048, n // 2 + 2048)]
    if 0 < L.n_decay < n:
        w.append((L.n_decay - 2048, min(n, L.n_decay + 2048)))
    for t in L.flat[1:6] + L.flat[-3:]:
        o = L.offsets[t.name]
        w.append((max(0, o - 1000), min(n, o + 1000)))
    w += [e for e in extra if e[1] <= n]
    return sorted(set(w))


def _full_size_check(oracle, L, heavy, extra_windows=()):
    if not _fits(L.n):
        pytest.skip("not enough device memory for this configuration")
    adam = ab.AdamConfig(lr=3e-4, beta1=0.9, beta2=0.95, eps=1e-8, weight_decay=0.1,
                         grad_clip=1.0)
    sc = ab.LossScaleConfig(init=SCALE, every=2000, max=2.0 ** 24)
    opt = ab.Optimizer(L, adam, sc, constant_lr=True, initial_step=999)
    w16, g16, m, v = synth.make_state(L.n, 0, SEED, "cuda", loss_scale=SCALE, heavy=heavy)
    wins = _windows(L, extra_windows)
    pre = {win: (w16[win[0]:win[1]].cpu().numpy().view(np.uint16).copy(),
                 m[win[0]:win[1]].cpu().numpy().copy(), v[win[0]:win[1]].cpu().numpy().copy())
           for win in wins}
    g_host = g16.cpu().numpy().view(np.uint16)
    opt.step_all(w16, g16, m, v)
    st = opt.status()
    cfg = oracle.make_cfg(n_decay=L.n_decay, scale_every=2000, scale_max=2.0 ** 24)
    ost = oracle.make_state(SCALE, opt_step=999)
    sumsq, bad = oracle.partial_f16(cfg, ost, g_host, 0)
    assert bad == 0 and st["last_overflow"] == 0 and st["opt_step"] == 1000
    assert abs(st["last_sumsq"] - sumsq) <= 1e-12 * sumsq
    norm = np.float32(np.sqrt(sumsq))
    assert abs(st["last_norm"] - norm) <= 1e-5 * norm
    assert st["last_clip_coef"] < 1.0                      # clipping active in every config
    for (lo, hi), (w0, m0, v0) in pre.items():
        ow, om, ov = w0.copy(), m0.copy(), v0.copy()
        wst = oracle.make_state(SCALE, opt_step=999)
        # the oracle's own exact sum drives the clip coefficient of the windows
        oracle.apply_f16(cfg, wst, ow, np.ascontiguousarray(g_host[lo:hi]), om, ov, lo,
                         sumsq, 0)
        assert same_f16(w16[lo:hi].cpu().numpy().view(np.uint16), ow), (lo, hi)
        assert same_f32(m[lo:hi].cpu().numpy(), om), (lo, hi)
        assert same_f32(v[lo:hi].cpu().numpy(), ov), (lo, hi)
    opt.close()
    return st


def test_decoder_1p3b_full_size(oracle):
    st = _full_size_check(oracle, layout.decoder_1p3b_layout(), heavy=False)
    assert st["last_norm"] > 30


def test_decoder_7b_heavy_tailed_full_size(oracle):
    st = _full_size_check(oracle, layout.decoder_7b_layout(), heavy=True)
    assert st["last_clip_coef"] < 0.01


def test_flat_beyond_2_pow_32(oracle):
    n = (1 << 32) + 8 * 3 + 5
    extra = [((1 << 31) - 2048, (1 << 31) + 2048), ((1 << 32) - 2048, (1 << 32) + 29)]
    _full_size_check(oracle, layout.flat_layout(n), heavy=False, extra_windows=extra)
