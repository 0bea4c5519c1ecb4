"""ARK4 layout logic on CPU: file order, record offsets, rotation names,
and the test-side restatement of the reference's writer/reader."""
import struct

import numpy as np

from ark_b200 import checkpoint, layout
from oracle import ark4


def test_file_order_and_counts():
    L = layout.eko_layout()
    t = checkpoint.ckpt_tensors(L)
    assert len(t) == 272 and len(ark4.records(L)) == 816          # 3 + 30*27 + 3
    assert t[0].numel == 32000 * 768 and t[0].flat_offset == 0
    assert t[271].numel == 768 and t[271].flat_offset == L.gamma_final_range()[0]
    assert [t[1 + i].numel for i in range(9)] == [768 * 768] * 4 + [768 * 2048] * 3 + [768] * 2


def test_rotating_path():
    # training.rs:583-586
    assert checkpoint.rotating_path("ckpt.bin", 0) == "ckpt_rot0.bin"
    assert checkpoint.rotating_path("ckpt_rot2.bin", 500) == "ckpt_rot1.bin"
    assert checkpoint.rotating_path("a/b.bin", 1500, 500) == "a/b_rot0.bin"


def test_reference_format_roundtrip(tmp_path):
    L = layout.decoder_layout("t", 2, 16, 40, 50)
    rng = np.random.default_rng(0)
    w = rng.integers(0, 1 << 15, L.n).astype(np.uint16)
    m = rng.normal(size=L.n).astype(np.float32)
    v = rng.normal(size=L.n).astype(np.float32)
    p = tmp_path / "c.bin"
    ark4.save_v4(str(p), L, 1234, 987, w, m, v)
    raw = p.read_bytes()
    assert raw[:4] == b"AR4K" and struct.unpack_from("<QQQ", raw, 4) == (1234, 987, 3 + 2 * 27 + 3)
    gs, adam, w2, m2, v2, tail = ark4.load_v4(str(p), L)
    assert (gs, adam, tail) == (1234, 987, b"")
    assert np.array_equal(w, w2) and np.array_equal(m, m2) and np.array_equal(v, v2)
    assert len(raw) == 28 + 60 * 16 + L.n * (2 + 4 + 4)
