"""The logits-gradient check (training.rs:228-245) and the weight all-gather
fused with the update, on one B200, through the C ABI, against the CPU
oracle.

Logits: the scaled logits bit for bit on accepted iterations, and the
per-iteration loss-scale state (scale, optimizer step, overflow flag, clean
and consecutive-overflow counts, skipped steps) bit for bit over a
trajectory that rejects iterations at the logits check, at the gradient
check and at both, then runs into the early stop.

Gather (world 1): the full weight buffer receives exactly the weights the
plain step produces, with the shard given as a separate buffer or as a
slice of the full buffer; a skipped step leaves it unchanged."""
import numpy as np
import pytest
import torch

import ark_b200 as ab
from ark_b200 import layout, synth
from gpu_util import dev, host, same_f32

pytestmark = pytest.mark.gpu

SEED, SCALE = 515, 1024.0
HP = dict(lr=3e-4, beta1=0.9, beta2=0.95, eps=1e-8, weight_decay=0.1, grad_clip=1.0)


def _oracle_state_tuple(st):
    return (st.loss_scale, st.opt_step, st.last_overflow, st.clean_steps, st.consecutive_nans,
            st.skipped_steps, st.early_stop)


def _dev_state_tuple(s):
    return (s["loss_scale"], s["opt_step"], s["last_overflow"], s["clean_steps"],
            s["consecutive_nans"], s["skipped_steps"], s["early_stop"])


def test_logits_check_scales_and_skips_like_the_reference(oracle):
    L = layout.decoder_layout("logits", 2, 64, 160, 301)
    n = L.n
    n_logits = 3 * 1001 + 3                       # bs x vocab, not a multiple of 4
    sc = ab.LossScaleConfig(init=SCALE, every=3, max=2.0 ** 24, max_consecutive_nans=3)
    opt = ab.Optimizer(L, ab.AdamConfig(**HP), sc, constant_lr=True, initial_step=10)
    w16, g16, m, v = synth.make_state(n, 0, SEED, "cuda", loss_scale=SCALE)
    w = oracle.synth_f16(n, 0, SEED, synth.STREAM_W, 0.02)
    m_h = oracle.synth_f32(n, 0, SEED, synth.STREAM_M, 1e-4)
    v_h = oracle.synth_f32(n, 0, SEED, synth.STREAM_V, 1e-3, square=True)
    cfg = oracle.make_cfg(n_decay=L.n_decay, scale_every=3, scale_max=2.0 ** 24,
                          max_consecutive_nans=3, **{k: HP[k] for k in
                                                     ("beta1", "beta2", "eps", "weight_decay",
                                                      "grad_clip")})
    st = oracle.make_state(SCALE, opt_step=10)
    bad_logits = {3, 6, 9, 10, 11, 12}             # 9..12: four in a row -> early stop
    bad_grads = {5, 6}
    for k in range(1, 13):
        lg = oracle.synth_f32(n_logits + 1, 0, SEED, 0x700 + k, 1e-2)
        if k in bad_logits:
            lg[1 + (k * 977) % n_logits] = np.nan if k % 2 else -np.inf
        g = oracle.synth_f16(n, 0, SEED, 0x100 + k, 1e-3, st.loss_scale)
        if k in bad_grads:
            g[(k * 7919) % n] = 0x7C00
        # device: logits check on an unaligned view, then the step
        d_lg = dev(lg)
        opt.logits_check(d_lg[1:])
        g16.copy_(torch.from_numpy(g.view(np.float16).copy()))
        opt.step_all(w16, g16, m, v)
        rc, s = opt.read_status()
        # oracle: training.rs:228-245, then :289-326 when the logits pass
        nb, ref_lg = oracle.logits_check_scale(lg[1:], st.loss_scale)
        if nb:
            oracle.apply_f16(cfg, st, w, g, m_h, v_h, 0, 0.0, 1)   # same transitions
        else:
            s_sum, bad = oracle.partial_f16(cfg, st, g, 0)
            oracle.apply_f16(cfg, st, w, g, m_h, v_h, 0, s_sum, bad)
            assert same_f32(host(d_lg)[1:], ref_lg), k         # scaled bit for bit
        assert host(d_lg)[0] == lg[0], k                      # element before the view
        assert _dev_state_tuple(s) == _oracle_state_tuple(st), (k, s)
        assert rc == (ab._lib.ARK_E_EARLY_STOP if st.early_stop else 0), (k, rc)
    assert st.early_stop == 1
    assert np.array_equal(host(w16), w)
    assert same_f32(host(m), m_h) and same_f32(host(v), v_h)
    opt.close()


@pytest.mark.parametrize("p1_last", ["0", "1"])
def test_logits_check_empty_and_count_reset(p1_last, monkeypatch):
    """With either side forming the rank partial (pass 2, or pass 1's last
    block), which is also where the logits count is consumed."""
    monkeypatch.setenv("ARK_P1_LAST", p1_last)
    L = layout.flat_layout(4096)
    opt = ab.Optimizer(L, ab.AdamConfig(**HP), ab.LossScaleConfig(init=SCALE), constant_lr=True)
    bufs = synth.make_state(L.n, 0, 3, "cuda", loss_scale=SCALE)
    ab.lib().ark_cuda_opt_logits_check(opt._h, None, 0)            # n == 0: no-op
    x = torch.tensor([1.0, float("nan"), 2.0], device="cuda")
    opt.logits_check(x)
    opt.step_all(*bufs)
    assert opt.status()["last_overflow"] == 1
    opt.step_all(*bufs)                                              # the count was consumed
    s = opt.status()
    assert s["last_overflow"] == 0 and s["opt_step"] == 1
    opt.close()


@pytest.mark.parametrize("in_place", [False, True])
def test_fused_weight_gather_single_rank(oracle, in_place):
    L = layout.decoder_layout("gather", 2, 64, 160, 257)
    n = L.n
    sc = ab.LossScaleConfig(init=SCALE, every=50, max=2.0 ** 24)
    ref = ab.Optimizer(L, ab.AdamConfig(**HP), sc, constant_lr=True, initial_step=5)
    opt = ab.Optimizer(L, ab.AdamConfig(**HP), sc, constant_lr=True, initial_step=5,
                       use_graph=True)
    rw, rg, rm, rv = synth.make_state(n, 0, SEED, "cuda", loss_scale=SCALE)
    w16, g16, m, v = (t.clone() for t in (rw, rg, rm, rv))
    full = opt.weight_buffer()
    assert full.numel() == n and int(full.view(torch.int16).abs().sum()) == 0
    if in_place:
        full.copy_(w16)
        w16 = full[opt.lo:opt.hi]                  # the shard is the full buffer's slice
    for k in range(3):
        if k == 1:                                 # an overflow step: nothing is stored
            rg.view(torch.int16)[n // 3] = 0x7C00
            g16.view(torch.int16)[n // 3] = 0x7C00
        if k == 2:
            synth.fill_grads(rg, 0, SEED + 1, SCALE)
            synth.fill_grads(g16, 0, SEED + 1, SCALE)
        ref.step_all(rw, rg, rm, rv)
        opt.step_gather(w16, g16, m, v)
        opt.weights_wait()
        torch.cuda.synchronize()
        assert torch.equal(full.view(torch.int16), rw.view(torch.int16)), k
        assert torch.equal(w16.view(torch.int16), rw.view(torch.int16)), k
    assert opt.status()["last_overflow"] == 0 and opt.status()["opt_step"] == 7
    assert opt.status()["skipped_steps"] == 1
    assert torch.equal(m.view(torch.int32), rm.view(torch.int32))
    assert torch.equal(v.view(torch.int32), rv.view(torch.int32))
    # the plain step against the oracle was checked elsewhere; spot-check here
    assert ref.status()["opt_step"] == 7
    ref.close()
    opt.close()


def test_gather_option_errors():
    L = layout.flat_layout(1024)
    opt = ab.Optimizer(L, constant_lr=True)
    w16, g16, m, v = synth.make_state(L.n, 0, 1, "cuda")
    with pytest.raises(ab.ArkError):                # no weight buffer yet
        opt.step_gather(w16, g16, m, v)
    opt.weight_buffer()
    w32 = torch.empty(L.n, dtype=torch.float32, device="cuda")
    rc = ab.lib().ark_cuda_opt_step_ex(opt._h, w16.data_ptr(), g16.data_ptr(), m.data_ptr(),
                                       v.data_ptr(), w32.data_ptr(),
                                       ab._lib.ARK_STEP_GATHER_WEIGHTS)
    assert rc == -8                                 # ARK_E_UNSUPPORTED with w32_out
    opt.close()


def test_zero_grads_clears_the_handoff_buffer():
    L = layout.flat_layout(1 << 16)
    opt = ab.Optimizer(L, constant_lr=True)
    with pytest.raises(ab.ArkError):                # no gradient buffer yet
        opt.zero_grads()
    full = opt.grad_buffer()
    synth.fill_f16(full, 0, 9, 2, 1e-3, mult=SCALE)
    assert int(full.view(torch.int16).ne(0).sum()) > 0
    opt.zero_grads()
    torch.cuda.synchronize()
    assert int(full.view(torch.int16).ne(0).sum()) == 0
    opt.close()


def test_gather_with_reduce_single_rank():
    """ARK_STEP_REDUCE | ARK_STEP_GATHER_WEIGHTS: the hand-off, the update
    and the weight all-gather in one step, against the hand-off step alone."""
    L = layout.decoder_layout("gred", 2, 64, 160, 211)
    n = L.n
    sc = ab.LossScaleConfig(init=SCALE, every=50, max=2.0 ** 24)
    ref = ab.Optimizer(L, ab.AdamConfig(**HP), sc, constant_lr=True, initial_step=3)
    opt = ab.Optimizer(L, ab.AdamConfig(**HP), sc, constant_lr=True, initial_step=3)
    rw, _, rm, rv = synth.make_state(n, 0, SEED, "cuda", loss_scale=SCALE)
    w_full = opt.weight_buffer()
    w_full.copy_(rw)
    w16, m, v = w_full[opt.lo:opt.hi], rm.clone(), rv.clone()
    rg_full, g_full = ref.grad_buffer(), opt.grad_buffer()
    rshard = torch.zeros(n, dtype=torch.float16, device="cuda")
    shard = torch.zeros(n, dtype=torch.float16, device="cuda")
    for k in range(3):
        synth.fill_f16(rg_full, 0, SEED, 0x500 + k, 1e-3, mult=SCALE)
        g_full.copy_(rg_full)
        ref.step_reduce(rw, rshard, rm, rv)
        opt.step_gather(w16, shard, m, v, reduce=True)
        opt.weights_wait()
        torch.cuda.synchronize()
        assert torch.equal(shard.view(torch.int16), rshard.view(torch.int16)), k
        assert torch.equal(w_full.view(torch.int16), rw.view(torch.int16)), k
    assert torch.equal(m.view(torch.int32), rm.view(torch.int32))
    assert torch.equal(v.view(torch.int32), rv.view(torch.int32))
    assert opt.status()["opt_step"] == ref.status()["opt_step"] == 6
    ref.close()
    opt.close()
