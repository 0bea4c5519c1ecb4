"""Model layouts: parameter counts, tensor order and ZeRO-1 shards."""
import pytest

from ark_b200 import layout


def test_eko_param_count_and_tensors():
    L = layout.eko_layout()
    # V*d + d + L*(4d^2 + 3dh + 2d)  (memory.rs:332-336, 450-454)
    assert L.n == 236_959_488 == 32000 * 768 + 768 + 30 * (4 * 768 ** 2 + 3 * 768 * 2048 + 2 * 768)
    assert L.n_tensors == 272
    assert max(t.numel for t in L.tensors) == 24_576_000
    assert sum(1 for t in L.tensors if t.numel == 768) == 61


@pytest.mark.parametrize("fn,n", [(layout.decoder_1p3b_layout, 1_279_887_360),
                                  (layout.decoder_7b_layout, 6_607_343_616)])
def test_large_decoder_counts(fn, n):
    assert fn().n == n


def test_flat_order_decay_boundary():
    L = layout.eko_layout()
    assert all(t.decay for t in L.flat[: sum(t.decay for t in L.tensors)])
    assert L.n_decay == sum(t.numel for t in L.tensors if t.decay)
    lo, hi = L.gamma_final_range()
    assert (lo, hi) == (L.n_decay, L.n_decay + 768)
    # reference order is preserved inside each group
    names = [t.name for t in L.flat]
    assert names[0] == "embed" and names[1] == "l0.wq" and names[L.flat.index(L.flat[-1])] == "l29.g2"


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_shards_partition_and_align(world):
    L = layout.eko_layout()
    prev = 0
    for r in range(world):
        lo, hi = L.shard(r, world)
        assert lo == prev and hi >= lo
        assert lo % layout.SHARD_ALIGN == 0
        prev = hi
    assert prev == L.n


def test_shard_small_buffers():
    assert layout.shard_bounds(100, 0, 4) == (0, 0)
    assert layout.shard_bounds(100, 3, 4) == (0, 100)
    with pytest.raises(ValueError):
        layout.shard_bounds(100, 4, 4)
