"""The whole-step API (ark_cuda_opt_*) on a B200 against the CPU
oracle: finite check, unscale, global norm and clip, AdamW over the flat
decayed-first layout, and the loss-scale state machine, step by step.
Flags and scale sequences are compared exactly; the norm within 1e-5
relative (it is bit-identical in practice); w, m, v bit for bit."""
import numpy as np
import pytest
import torch

import ark_b200 as ab
from ark_b200 import layout, synth
from gpu_util import dev, first_diff, host, same_f16, same_f32

pytestmark = pytest.mark.gpu

SEED = 1234
STATE_KEYS = ("loss_scale", "opt_step", "clean_steps", "consecutive_nans", "skipped_steps",
              "last_overflow", "early_stop")


def oracle_bufs(oracle, n, lo, seed, scale, heavy=False, grad_stream=synth.STREAM_G):
    w = oracle.synth_f16(n, lo, seed, synth.STREAM_W, 0.02)
    g = oracle.synth_f16(n, lo, seed, grad_stream, 1e-3, scale,
                         synth.HEAVY_EVERY if heavy else 0, synth.HEAVY_MULT if heavy else 1.0)
    m = oracle.synth_f32(n, lo, seed, synth.STREAM_M, 1e-4)
    v = oracle.synth_f32(n, lo, seed, synth.STREAM_V, 1e-3, square=True)
    return w, g, m, v


def check_state(dev_st, ost, where=""):
    for k in STATE_KEYS:
        assert dev_st[k] == getattr(ost, k), f"{where}: {k} {dev_st[k]} vs {getattr(ost, k)}"
    if not ost.last_overflow and ost.opt_step:
        rel = abs(dev_st["last_norm"] - ost.last_norm) / max(ost.last_norm, 1e-30)
        assert rel <= 1e-5, f"{where}: norm {dev_st['last_norm']} vs {ost.last_norm}"
        assert dev_st["last_lr"] == ost.last_lr


def run_steps(oracle, L, *, steps, scale0=65536.0, initial_step=0, shard=None, compat=False,
              inject=None, lr_table=(3e-4,), use_graph=False, adam=None, scale_cfg=None,
              fresh_grads=True, max_nans=200, heavy=False):
    adam = adam or ab.AdamConfig(lr=3e-4, beta1=0.9, beta2=0.95, eps=1e-8, weight_decay=0.1,
                                 grad_clip=1.0)
    scale_cfg = scale_cfg or ab.LossScaleConfig(init=scale0, every=50, max=2.0 ** 24,
                                                max_consecutive_nans=max_nans)
    opt = ab.Optimizer(L, adam, scale_cfg, lr_table=np.asarray(lr_table, np.float32),
                       initial_step=initial_step, shard=shard, compat_gamma_final_unscaled=compat,
                       use_graph=use_graph)
    lo, n = opt.lo, opt.n
    w, g, m, v = oracle_bufs(oracle, n, lo, SEED, scale0, heavy)
    dw, dg, dm, dv = dev(w), dev(g), dev(m), dev(v)
    gf = L.gamma_final_range()
    cfg = oracle.make_cfg(beta1=adam.beta1, beta2=adam.beta2, eps=adam.eps,
                          weight_decay=adam.weight_decay, grad_clip=adam.grad_clip,
                          scale_backoff=scale_cfg.backoff, scale_growth=scale_cfg.growth,
                          scale_min=scale_cfg.min, scale_max=scale_cfg.max,
                          scale_every=scale_cfg.every,
                          max_consecutive_nans=scale_cfg.max_consecutive_nans,
                          lr_table=lr_table, n_decay=L.n_decay,
                          keep_lo=gf[0] if compat else 0, keep_hi=gf[1] if compat else 0)
    ost = oracle.make_state(scale0, opt_step=initial_step)
    for k in range(1, steps + 1):
        if fresh_grads and k > 1:
            sc = np.float32(ost.loss_scale)
            g = oracle.synth_f16(n, lo, SEED, synth.GRAD_STEP_STREAM_BASE + k, 1e-3, sc)
            synth.fill_f16(dg, lo, SEED, synth.GRAD_STEP_STREAM_BASE + k, 1e-3, mult=float(sc))
        if inject and k in inject:
            idx = oracle.lib().ork_inject_index(SEED, k, n)
            g[idx] = inject[k]
            dg.view(torch.int16)[idx] = int(np.int16(np.uint16(inject[k]).view(np.int16)))
        s, bad = oracle.partial_f16(cfg, ost, g, lo)
        oracle.apply_f16(cfg, ost, w, g, m, v, lo, s, bad)
        opt.step_all(dw, dg, dm, dv)
        check_state(opt.status(), ost, f"step {k}")
    hw, hm, hv = host(dw), host(dm), host(dv)
    assert same_f16(hw, w), f"w first diff at {first_diff(hw, w)}"
    assert same_f32(hm, m), f"m first diff at {first_diff(hm, m)}"
    assert same_f32(hv, v), f"v first diff at {first_diff(hv, v)}"
    st = opt.status()
    opt.close()
    return st, ost


def tiny():
    return layout.decoder_layout("tiny", 3, 32, 72, 97)


def test_tiny_decoder_multi_step(oracle):
    st, _ = run_steps(oracle, tiny(), steps=6, inject={3: 0x7E00})
    assert st["opt_step"] == 5 and st["skipped_steps"] == 1


def test_compat_gamma_final_unscaled(oracle):
    st, _ = run_steps(oracle, tiny(), steps=3, compat=True)
    assert st["opt_step"] == 3


@pytest.mark.parametrize("shard", [(1024, 8231), (0, 7), (128, 128 + 8 * 37), (0, 0)])
def test_shard_offsets_and_ragged_sizes(oracle, shard):
    L = tiny()
    run_steps(oracle, L, steps=2, shard=shard)


@pytest.mark.parametrize("n", [2048 * 296 * 3 + 8 * 5 + 3, 256 * 8 * 1184 * 2 + 8, 17])
def test_grid_stride_boundaries(oracle, n):
    """Flat sizes around whole grid-stride sweeps (296 / 1184 blocks of 256
    threads, 8 elements each), with a ragged tail."""
    run_steps(oracle, layout.flat_layout(n), steps=2, inject={2: 0x7C00})


def test_warmup_lr_table_and_resume_step(oracle):
    tab = ab.lr_schedule(ab.AdamConfig(lr=1e-3, warmup_steps=10), 40)
    run_steps(oracle, tiny(), steps=4, lr_table=tab, initial_step=7)


def test_no_clip_path(oracle):
    adam = ab.AdamConfig(lr=3e-4, beta1=0.9, beta2=0.95, eps=1e-8, weight_decay=0.1,
                         grad_clip=1e9)
    st, _ = run_steps(oracle, tiny(), steps=2, adam=adam)
    assert st["last_clip_coef"] == 1.0


def test_graph_replay_matches(oracle):
    run_steps(oracle, tiny(), steps=4, use_graph=True, inject={2: 0x7C00})


def test_early_stop(oracle):
    inject = {k: 0xFC00 for k in range(1, 7)}
    st, ost = run_steps(oracle, tiny(), steps=6, inject=inject, max_nans=3)
    assert st["early_stop"] == 1 and ost.early_stop == 1
    assert st["consecutive_nans"] == 4 and st["opt_step"] == 0


@pytest.mark.parametrize("scale0", [1000.0, 3.0 * 2.0 ** 10])
def test_non_power_of_two_scale(oracle, scale0):
    """A loss scale that is not a power of two takes the general unscale
    path (fp32(h) * inv rounded in f32 as the reference does, FP16 bit
    patterns checked for inf/NaN); backoff keeps it non-power-of-two."""
    st, _ = run_steps(oracle, tiny(), steps=5, scale0=scale0, inject={2: 0x7C00, 4: 0xFE00})
    assert st["skipped_steps"] == 2 and st["opt_step"] == 3


@pytest.mark.parametrize("scale0", [65536.0, 1000.0])
def test_nonfinite_positions(scale0):
    """The overflow flag for one inf/NaN (or largest finite) value at the
    first element, inside the first vector, mid-array, in the last whole
    vector and in the ragged tail; power-of-two and general scale paths."""
    n = 2048 * 296 + 8 * 3 + 5
    opt = ab.Optimizer(layout.flat_layout(n), constant_lr=True,
                       scale=ab.LossScaleConfig(init=scale0, min=2.0 ** -20, max=2.0 ** 24))
    w16, g16, m, v = synth.make_state(n, 0, 7, "cuda", loss_scale=1.0)
    gi = g16.view(torch.int16)
    clean = gi.clone()
    cases = [(0x7C00, 1), (0xFC00, 1), (0x7E01, 1), (0xFFFF, 1), (0x7BFF, 0), (0xFBFF, 0),
             (0x0001, 0)]
    skipped = 0
    for pos in (0, 7, n // 2, n - 6, n - 1):
        for val, bad in cases:
            gi.copy_(clean)
            gi[pos] = int(np.uint16(val).view(np.int16))
            opt.step_all(w16, g16, m, v)
            st = opt.status()
            assert st["last_overflow"] == bad, (pos, hex(val))
            skipped += bad
            assert st["skipped_steps"] == skipped
    opt.close()


def test_eko_full_step_bit_exact(oracle):
    """EKO-237M full optimizer step, t = 1000, scale 65536."""
    st, ost = run_steps(oracle, layout.eko_layout(), steps=1, initial_step=999, fresh_grads=False)
    assert st["opt_step"] == 1000 and st["last_clip_coef"] < 1.0
    assert st["last_norm"] == ost.last_norm


def test_trajectory_200_steps_flags_and_scale(oracle):
    """200 steps of fresh seeded grads with +inf/NaN injected at
    steps 17, 18, 90; scale init 65536, backoff 0.5, growth x2 every 50
    clean steps, max 2^24.  Every element checked at 1M params; the
    flags/scale sequence additionally at the full EKO size below."""
    inject = {17: 0x7C00, 18: 0x7E00, 90: 0x7C00}
    st, ost = run_steps(oracle, layout.flat_layout(1_000_003), steps=200, inject=inject)
    assert st["skipped_steps"] == 3 and st["opt_step"] == 197


def test_trajectory_200_steps_eko_size(oracle):
    L = layout.eko_layout()
    scale_cfg = ab.LossScaleConfig(init=65536.0, every=50, max=2.0 ** 24)
    adam = ab.AdamConfig(lr=3e-4, beta1=0.9, beta2=0.95, eps=1e-8, weight_decay=0.1,
                         grad_clip=1.0)
    opt = ab.Optimizer(L, adam, scale_cfg, constant_lr=True, initial_step=999)
    dw, dg, dm, dv = synth.make_state(L.n, 0, SEED, "cuda", loss_scale=65536.0)
    cfg = oracle.make_cfg(scale_every=50, scale_max=2.0 ** 24)
    ost = oracle.make_state(65536.0, opt_step=999)
    w, g, m, v = oracle_bufs(oracle, 8, 0, SEED, 1.0)
    seq_dev, seq_ref = [], []
    inject = {17: 0x7C00, 18: 0x7E00, 90: 0x7C00}
    for k in range(1, 201):
        sc = opt.status()["loss_scale"]
        synth.fill_grads(dg, 0, SEED, sc, grad_stream=synth.GRAD_STEP_STREAM_BASE + k)
        if k in inject:
            idx = oracle.lib().ork_inject_index(SEED, k, L.n)
            dg.view(torch.int16)[idx] = int(np.uint16(inject[k]).view(np.int16))
        opt.step_all(dw, dg, dm, dv)
        s = opt.status()
        seq_dev.append((s["last_overflow"], s["loss_scale"], s["opt_step"], s["clean_steps"]))
        oracle.apply_f16(cfg, ost, w, g, m, v, 0, 1.0, 1 if k in inject else 0)
        seq_ref.append((ost.last_overflow, ost.loss_scale, ost.opt_step, ost.clean_steps))
    assert seq_dev == seq_ref
    assert [k + 1 for k, s in enumerate(seq_dev) if s[0]] == [17, 18, 90]
    opt.close()


def test_bad_arguments():
    import ctypes
    opt = ab.Optimizer(tiny(), constant_lr=True)
    t = torch.zeros(opt.n + 8, dtype=torch.float16, device="cuda")
    f = torch.zeros(opt.n + 8, dtype=torch.float32, device="cuda")
    rc = ab.lib().ark_cuda_opt_step(opt._h, t.data_ptr() + 2, t.data_ptr(), f.data_ptr(),
                                    f.data_ptr())
    assert rc == -2
    cfg = ab._lib.OptCfg()
    h = ctypes.c_void_p()
    assert ab.lib().ark_cuda_opt_init(ctypes.byref(cfg), ctypes.byref(h)) == -1
    opt.close()


@pytest.mark.parametrize("use_graph", [False, True])
def test_profile_events(use_graph):
    """Per-kernel CUDA events, also inside graph replays (event-record nodes
    retargeted per replay)."""
    L = layout.flat_layout(10_000_000)
    opt = ab.Optimizer(L, constant_lr=True, use_graph=use_graph)
    bufs = synth.make_state(L.n, 0, 3, "cuda")
    opt.profile_begin(3)
    for _ in range(3):
        opt.step_all(*bufs)
    prof = opt.profile_read(3)
    assert prof.shape == (3, 3) and (prof[:, 0] > 0).all() and (prof[:, 2] > 0).all()
    assert len(set(prof[:, 2].tolist())) > 1          # three distinct measurements
    for _ in range(2):                                 # replays without profiling still run
        opt.step_all(*bufs)
    assert opt.status()["steps_called"] == 5
    opt.close()


@pytest.mark.parametrize("shard", [None, (1024, 8232)])
def test_reduce_step_single_rank(oracle, shard):
    """step_reduce on one rank: the shard of the (one-rank) sum of the full
    gradient buffer, then the ordinary step, against the oracle."""
    L = tiny()
    adam = ab.AdamConfig(lr=3e-4, beta1=0.9, beta2=0.95, eps=1e-8, weight_decay=0.1,
                         grad_clip=1.0)
    sc = ab.LossScaleConfig(init=65536.0, every=50, max=2.0 ** 24)
    opt = ab.Optimizer(L, adam, sc, constant_lr=True, initial_step=999, shard=shard)
    lo, n = opt.lo, opt.n
    full = opt.grad_buffer()
    assert full.numel() == L.n and int(full.view(torch.int16).abs().sum()) == 0
    w, _, m, v = oracle_bufs(oracle, n, lo, SEED, 65536.0)
    dw, dm, dv = dev(w), dev(m), dev(v)
    shard_g = torch.zeros(n, dtype=torch.float16, device="cuda")
    cfg = oracle.make_cfg(n_decay=L.n_decay, scale_every=50, scale_max=2.0 ** 24)
    ost = oracle.make_state(65536.0, opt_step=999)
    for k in range(1, 4):
        synth.fill_f16(full, 0, SEED, 0x300 + k, 1e-3, mult=65536.0)
        g_full = oracle.synth_f16(L.n, 0, SEED, 0x300 + k, 1e-3, 65536.0)
        if k == 2:
            full.view(torch.int16)[lo + 5] = 0x7C00
            g_full[lo + 5] = 0x7C00
        opt.step_reduce(dw, shard_g, dm, dv)
        g = oracle.reduce_f16([g_full], n, lo)
        assert same_f16(host(shard_g), g)
        s, bad = oracle.partial_f16(cfg, ost, g, lo)
        oracle.apply_f16(cfg, ost, w, g, m, v, lo, s, bad)
        check_state(opt.status(), ost, f"step {k}")
    assert same_f16(host(dw), w) and same_f32(host(dm), m) and same_f32(host(dv), v)
    opt.close()


@pytest.mark.parametrize("reduce", [False, True])
def test_step_writes_fp32_weight_copy(oracle, reduce):
    """ark_cuda_opt_step_ex with w32_out: the updated weights widened to FP32
    (the forward's copy, training.rs:165-186) on every updating step; a
    skipped step leaves them alone."""
    L = tiny()
    opt = ab.Optimizer(L, ab.AdamConfig(lr=3e-4, beta1=0.9, beta2=0.95, eps=1e-8,
                                        weight_decay=0.1, grad_clip=1.0),
                       ab.LossScaleConfig(init=65536.0, every=50, max=2.0 ** 24),
                       constant_lr=True, initial_step=999)
    n = opt.n
    w, g, m, v = oracle_bufs(oracle, n, 0, SEED, 65536.0)
    dw, dg, dm, dv = dev(w), dev(g), dev(m), dev(v)
    if reduce:
        full = opt.grad_buffer()
        full.copy_(dg)
    w32 = torch.from_numpy(oracle.dequant(w)).cuda()
    cfg = oracle.make_cfg(n_decay=L.n_decay, scale_every=50, scale_max=2.0 ** 24)
    ost = oracle.make_state(65536.0, opt_step=999)
    for k in range(1, 4):
        if k == 2:
            g[7] = 0x7C00
            (full if reduce else dg).view(torch.int16)[7] = 0x7C00
        if k == 3:
            g[7] = oracle.synth_f16(1, 7, SEED, synth.STREAM_G, 1e-3, 65536.0)[0]
            (full if reduce else dg).view(torch.int16)[7] = int(np.int16(np.uint16(g[7]).view(np.int16)))
        before = host(w32).copy()
        opt.step_all_w32(dw, dg, dm, dv, w32, reduce=reduce)
        s, bad = oracle.partial_f16(cfg, ost, g, 0)
        oracle.apply_f16(cfg, ost, w, g, m, v, 0, s, bad)
        check_state(opt.status(), ost, f"step {k}")
        if k == 2:
            assert np.array_equal(host(w32).view(np.uint32), before.view(np.uint32))
        else:
            assert same_f32(host(w32), oracle.dequant(w))
    assert same_f16(host(dw), w) and same_f32(host(dm), m) and same_f32(host(dv), v)
    opt.close()
