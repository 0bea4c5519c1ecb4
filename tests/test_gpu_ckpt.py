"""ARK4 checkpoints written and read by libark_cuda from device shards,
checked against the test-side restatement of the reference's writer and
reader (oracle/ark4.py, io.rs:432-636)."""
import numpy as np
import pytest
import torch

import ark_b200 as ab
from ark_b200 import checkpoint, layout, synth
from gpu_util import dev, host
from oracle import ark4

pytestmark = pytest.mark.gpu

SEED = 8080


def _opt(L, **kw):
    return ab.Optimizer(L, ab.AdamConfig(lr=3e-4, beta1=0.9, beta2=0.95, eps=1e-8,
                                         weight_decay=0.1, grad_clip=1.0),
                        ab.LossScaleConfig(init=4096.0, every=2, max=2.0 ** 24),
                        constant_lr=True, initial_step=41, **kw)


def _stepped(L, steps=3, shard=None):
    opt = _opt(L, shard=shard)
    bufs = synth.make_state(opt.n, opt.lo, SEED, "cuda", loss_scale=4096.0)
    for _ in range(steps):
        opt.step_all(*bufs)
    return opt, bufs


def test_save_matches_reference_reader(tmp_path):
    L = layout.decoder_layout("ck", 3, 64, 160, 211)
    opt, (w16, g16, m, v) = _stepped(L)
    st = opt.status()
    p = str(tmp_path / "a.bin")
    checkpoint.save(opt, p, w16, m, v, global_step=777)
    gs, adam, w2, m2, v2, tail = ark4.load_v4(p, L)
    assert gs == 777 and adam == st["opt_step"] == 44
    assert np.array_equal(w2, host(w16))
    assert np.array_equal(m2.view(np.uint32), host(m).view(np.uint32))
    assert np.array_equal(v2.view(np.uint32), host(v).view(np.uint32))
    assert tail[:4] == b"ARKS" and len(tail) == 8 + 64
    saved = ab._lib.OptStatus.from_buffer_copy(tail[8:])
    assert saved.loss_scale == st["loss_scale"] and saved.clean_steps == st["clean_steps"]
    opt.close()


@pytest.mark.parametrize("restore_scale", [False, True])
def test_load_reference_written_file_and_resume(tmp_path, restore_scale):
    L = layout.decoder_layout("ck", 3, 64, 160, 211)
    opt, (w16, g16, m, v) = _stepped(L, steps=5)
    st = opt.status()
    p = str(tmp_path / "b.bin")
    checkpoint.save(opt, p, w16, m, v, global_step=5)
    # resume into a fresh state: same weights, moments, step -> same next step
    opt2 = _opt(L)
    w2 = torch.zeros_like(w16)
    m2, v2 = torch.zeros_like(m), torch.zeros_like(v)
    assert checkpoint.load(opt2, p, w2, m2, v2, restore_scale=restore_scale) == 5
    st2 = opt2.status()
    assert st2["opt_step"] == st["opt_step"]
    if restore_scale:
        assert st2["loss_scale"] == st["loss_scale"] and st2["clean_steps"] == st["clean_steps"]
    else:
        assert st2["loss_scale"] == 4096.0 and st2["clean_steps"] == 0   # training.rs:120
    assert torch.equal(w2.view(torch.int16), w16.view(torch.int16))
    if restore_scale:
        opt.step_all(w16, g16, m, v)
        opt2.step_all(w2, g16, m2, v2)
        assert torch.equal(w2.view(torch.int16), w16.view(torch.int16))
        assert torch.equal(m2.view(torch.int32), m.view(torch.int32))
        assert torch.equal(v2.view(torch.int32), v.view(torch.int32))
    # a file written by the reference's writer (restated) loads as well
    q = str(tmp_path / "ref.bin")
    ark4.save_v4(q, L, 9, 123, host(w16), host(m), host(v))
    assert checkpoint.load(opt2, q, w2, m2, v2) == 9
    assert opt2.status()["opt_step"] == 123 and opt2.status()["loss_scale"] == 4096.0
    assert torch.equal(w2.view(torch.int16), w16.view(torch.int16))
    opt.close()
    opt2.close()


def test_load_v3_rounds_weights(tmp_path, oracle):
    L = layout.decoder_layout("ck", 2, 32, 96, 101)
    rng = np.random.default_rng(1)
    w32 = (rng.normal(size=L.n) * 0.02).astype(np.float32)
    m = rng.normal(size=L.n).astype(np.float32)
    v = (rng.normal(size=L.n) ** 2).astype(np.float32)
    p = str(tmp_path / "v3.bin")
    ark4.save_v3(p, L, 3, 30, w32, m, v)
    opt = _opt(L)
    w2 = torch.zeros(L.n, dtype=torch.float16, device="cuda")
    m2 = torch.zeros(L.n, dtype=torch.float32, device="cuda")
    v2 = torch.zeros_like(m2)
    assert checkpoint.load(opt, p, w2, m2, v2) == 3
    gf = slice(*L.gamma_final_range())              # not in V3 files: left as it was
    exp_w = oracle.quant(w32)
    exp_w[gf] = 0
    got = host(w2)
    assert np.array_equal(got, exp_w)
    assert np.array_equal(host(m2)[:gf.start], m[:gf.start])
    assert opt.status()["opt_step"] == 30
    opt.close()


def test_sharded_save_and_load(tmp_path):
    """Two shards saved into one file give the same tensors as the whole
    state; each shard loads back its own part."""
    L = layout.decoder_layout("ck", 3, 64, 160, 211)
    full, (fw, _, fm, fv) = _stepped(L)
    lo = (L.n // 2) // 128 * 128
    parts = [_stepped(L, shard=(0, lo)), _stepped(L, shard=(lo, L.n))]
    p = str(tmp_path / "s.bin")
    for opt, (w, g, m, v) in parts:
        checkpoint.save(opt, p, w, m, v, global_step=1)
    _, _, w2, m2, v2, _ = ark4.load_v4(p, L)
    # shards of independently stepped halves: compare each half with its own state
    for (opt, (w, g, m, v)) in parts:
        sl = slice(opt.lo, opt.hi)
        assert np.array_equal(w2[sl], host(w))
        assert np.array_equal(m2[sl].view(np.uint32), host(m).view(np.uint32))
    for opt, (w, g, m, v) in parts:
        wz, mz, vz = torch.zeros_like(w), torch.zeros_like(m), torch.zeros_like(v)
        checkpoint.load(opt, p, wz, mz, vz)
        assert torch.equal(wz.view(torch.int16), w.view(torch.int16))
        assert torch.equal(vz.view(torch.int32), v.view(torch.int32))
        opt.close()
    full.close()


def test_layout_mismatch_is_an_error(tmp_path):
    L = layout.decoder_layout("ck", 2, 32, 96, 101)
    L2 = layout.decoder_layout("ck", 2, 32, 96, 103)
    opt, (w, g, m, v) = _stepped(L, steps=1)
    p = str(tmp_path / "x.bin")
    checkpoint.save(opt, p, w, m, v, 0)
    opt2 = _opt(L2)
    z16 = torch.zeros(L2.n, dtype=torch.float16, device="cuda")
    z32 = torch.zeros(L2.n, dtype=torch.float32, device="cuda")
    with pytest.raises(ab.ArkError):
        checkpoint.load(opt2, p, z16, z32, z32.clone())
    opt.close()
    opt2.close()
