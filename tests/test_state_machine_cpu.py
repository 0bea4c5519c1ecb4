"""The oracle's step semantics on CPU: the loss-scale state machine against
the scale progression the reference published from its own training run
(CHANGELOG.md:120-130), the overflow / early-stop rules of training.rs, and
the flat decayed-first layout against the reference's per-tensor calls."""
import numpy as np
import pytest

from ark_b200 import layout


def tiny_bufs(oracle, n, seed=7, scale=256.0):
    w = oracle.synth_f16(n, 0, seed, 1, 0.02)
    g = oracle.synth_f16(n, 0, seed, 2, 1e-3, scale)
    m = oracle.synth_f32(n, 0, seed, 3, 1e-4)
    v = oracle.synth_f32(n, 0, seed, 4, 1e-3, square=True)
    return w, g, m, v


def test_published_scale_progression(oracle):
    """CHANGELOG.md:122-128: local steps 1-1,999 at scale 256, 2,000-3,999 at
    512, 4,000-5,999 at 1,024, 6,000-7,999 at 2,048, 8,000+ 4,096 -> 8,192;
    config max 8192 (config.rs:69), growth every 2000 clean steps."""
    cfg = oracle.make_cfg(scale_every=2000, scale_max=8192.0)
    st = oracle.make_state(256.0)
    w, g, m, v = tiny_bufs(oracle, 8, scale=256.0)
    seen = {}
    for k in range(1, 12_001):
        rc = oracle.apply_f16(cfg, st, w, g, m, v, 0, 1.0, 0)  # a clean step
        assert rc == 0
        seen[k] = st.loss_scale
    assert seen[1] == seen[1999] == 256.0
    assert seen[2000] == seen[3999] == 512.0
    assert seen[4000] == seen[5999] == 1024.0
    assert seen[6000] == seen[7999] == 2048.0
    assert seen[8000] == 4096.0 and seen[10000] == 8192.0 and seen[12000] == 8192.0
    assert st.opt_step == 12000 and st.skipped_steps == 0


def test_overflow_backoff_min_and_early_stop(oracle):
    cfg = oracle.make_cfg(scale_min=1.0, max_consecutive_nans=200)
    st = oracle.make_state(4.0, opt_step=10)
    w, g, m, v = tiny_bufs(oracle, 9)
    w0, m0, v0 = w.copy(), m.copy(), v.copy()
    scales = []
    for k in range(1, 202):
        rc = oracle.apply_f16(cfg, st, w, g, m, v, 0, 1.0, 1)
        scales.append(st.loss_scale)
        assert rc == (2 if k == 201 else 1)
    assert scales[:4] == [2.0, 1.0, 1.0, 1.0]                 # training.rs:294 max(scale*0.5, 1)
    assert st.consecutive_nans == 201 and st.early_stop == 1
    assert st.skipped_steps == 201 and st.opt_step == 10      # no step on overflow
    assert np.array_equal(w, w0) and np.array_equal(m, m0) and np.array_equal(v, v0)
    assert oracle.apply_f16(cfg, st, w, g, m, v, 0, 1.0, 0) == 2   # stays stopped


def test_clean_step_resets_counters(oracle):
    cfg = oracle.make_cfg(scale_every=3, scale_max=64.0)
    st = oracle.make_state(16.0)
    w, g, m, v = tiny_bufs(oracle, 5)
    seq = [0, 0, 1, 0, 0, 0, 0, 0, 0, 1, 1, 0]
    out = []
    for bad in seq:
        oracle.apply_f16(cfg, st, w, g, m, v, 0, 1.0, bad)
        out.append((st.loss_scale, st.clean_steps, st.consecutive_nans, st.opt_step))
    assert out[2] == (8.0, 0, 1, 2)
    assert out[5] == (16.0, 0, 0, 5)      # third clean step since the overflow -> x2
    assert out[8] == (32.0, 0, 0, 8)
    assert out[10] == (8.0, 0, 2, 8)
    assert out[11] == (8.0, 1, 0, 9)


def test_growth_capped_by_max(oracle):
    cfg = oracle.make_cfg(scale_every=1, scale_max=1000.0)
    st = oracle.make_state(512.0)
    w, g, m, v = tiny_bufs(oracle, 3)
    oracle.apply_f16(cfg, st, w, g, m, v, 0, 1.0, 0)
    assert st.loss_scale == 1000.0                      # min(1024, 1000) > 512
    oracle.apply_f16(cfg, st, w, g, m, v, 0, 1.0, 0)
    assert st.loss_scale == 1000.0 and st.clean_steps == 0


def small_decoder():
    return layout.decoder_layout("tiny", 2, 16, 40, 50)


@pytest.mark.parametrize("compat", [False, True])
def test_flat_step_equals_reference_per_tensor_calls(oracle, compat):
    """optimizer.rs:171-228 calls adam_step_f16 once per tensor in reference
    order with per-tensor wd, after training.rs unscale and the global clip.
    The flat decayed-first step must produce identical bits."""
    L = small_decoder()
    n, scale = L.n, 1024.0
    w, g, m, v = tiny_bufs(oracle, n, seed=11, scale=scale)
    lo, hi = L.gamma_final_range()
    cfg = oracle.make_cfg(weight_decay=0.1, grad_clip=1e-3, lr_table=(1e-3,), n_decay=L.n_decay,
                          keep_lo=lo if compat else 0, keep_hi=hi if compat else 0)
    st = oracle.make_state(scale, opt_step=41)
    wf, mf, vf = w.copy(), m.copy(), v.copy()
    assert oracle.step_flat_f16(cfg, st, wf, g, mf, vf) == 0
    assert st.opt_step == 42 and st.last_clip_coef < 1.0
    # reference: per tensor, in reference order
    s = np.float32(st.last_clip_coef)
    inv = np.float32(1.0) / np.float32(scale)
    for t in L.tensors:
        o = L.offsets[t.name]
        sl = slice(o, o + t.numel)
        g32 = oracle.dequant(g[sl])
        if not (compat and t.name == "gamma_final"):
            g32 = (g32 * inv).astype(np.float32)
        g32 = (g32 * s).astype(np.float32)
        wd = 0.1 if t.decay else 0.0
        W, M, V = oracle.adam_step_f16(w[sl], g32, m[sl], v[sl], 1e-3, 0.9, 0.95, 1e-8, wd, 42)
        assert np.array_equal(W, wf[sl]), t.name
        assert np.array_equal(M.view(np.uint32), mf[sl].view(np.uint32)), t.name
        assert np.array_equal(V.view(np.uint32), vf[sl].view(np.uint32)), t.name


def test_norm_is_exact_and_the_reference_fold_is_not(oracle):
    """optimizer.rs:130 folds x*x sequentially in f32; at the 24.6M-element
    embedding the fold is far from the exact norm, so parity is stated
    against the exact (f64) norm."""
    n = 2_000_000
    g = oracle.synth_f32(n, 0, 3, 9, 1e-3)
    exact = np.sqrt(oracle.sumsq_f32_exact(g))
    fold = np.float32(0.0)
    acc = np.float32(0.0)
    sq = (g * g).astype(np.float32)
    # sequential f32 fold, chunked cumsum in float32 preserves the order
    acc = np.cumsum(sq, dtype=np.float32)[-1]
    fold = np.sqrt(acc)
    assert abs(fold - exact) / exact > 1e-4
    ref = np.sqrt(np.sum(g.astype(np.float64) ** 2))
    assert abs(ref - exact) / exact < 1e-12


def test_logits_block_restatement(oracle):
    """training.rs:228-245: any non-finite logits gradient rejects the step
    before scaling (the buffer is left as it was); otherwise every value is
    multiplied by the loss scale, one f32 multiply each."""
    x = np.array([1.5, -2.25, 3e-8, 65504.0, 1e30], np.float32)
    bad, y = oracle.logits_check_scale(x, 1024.0)
    assert bad == 0
    assert np.array_equal(y.view(np.uint32), (x * np.float32(1024.0)).view(np.uint32))
    assert np.isinf(oracle.logits_check_scale(np.array([1e36], np.float32), 1e4)[1][0])
    for poison in (np.nan, np.inf, -np.inf):
        z = x.copy()
        z[2] = poison
        bad, y = oracle.logits_check_scale(z, 1024.0)
        assert bad == 1 and np.array_equal(y.view(np.uint32), z.view(np.uint32))
    assert oracle.logits_check_scale(np.zeros(0, np.float32), 2.0)[0] == 0
