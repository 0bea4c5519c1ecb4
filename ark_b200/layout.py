"""Parameter layouts of the models the optimizer path is benchmarked on, and
their flat, ZeRO-1-sharded form.

Reference tensor set and order (proyecto_ark/ark01/src/memory.rs:202-255,
379-395; optimizer.rs:185-227): embed [V x d], gamma_final [d], then per
layer wq wk wv wo [d x d], w1 [d x h], w2 [h x d], w3 [d x h], g1 g2 [d].
Weight decay applies to embed and the seven matrices of each layer; the
RMSNorm gains (gamma_final, g1, g2) use wd = 0 (optimizer.rs:199, 225-226).

Flat order used on the device: every decayed tensor first (reference
order), then every non-decayed tensor (reference order), so that decay is a
single boundary, n_decay.  gamma_final is the first non-decayed tensor, at
[n_decay, n_decay + d), which is the range the
ARK_OPT_COMPAT_GAMMA_FINAL_UNSCALED mode leaves scaled (training.rs:133-146).
"""
from __future__ import annotations

from dataclasses import dataclass, field

SHARD_ALIGN = 128  # shard boundaries in elements (16-byte aligned for every dtype)


@dataclass(frozen=True)
class TensorSpec:
    name: str
    numel: int
    decay: bool


@dataclass
class Layout:
    name: str
    tensors: list                        # reference order
    flat: list = field(default_factory=list)     # device flat order
    offsets: dict = field(default_factory=dict)  # name -> flat offset

    def __post_init__(self):
        dec = [t for t in self.tensors if t.decay]
        nodec = [t for t in self.tensors if not t.decay]
        self.flat = dec + nodec
        off = 0
        for t in self.flat:
            self.offsets[t.name] = off
            off += t.numel
        self.n = off
        self.n_decay = sum(t.numel for t in dec)

    @property
    def n_tensors(self):
        return len(self.tensors)

    def gamma_final_range(self):
        if "gamma_final" not in self.offsets:
            return (0, 0)
        o = self.offsets["gamma_final"]
        t = next(t for t in self.tensors if t.name == "gamma_final")
        return (o, o + t.numel)

    def shard(self, rank: int, world: int):
        """Contiguous ZeRO-1 shard [lo, hi) of rank, boundaries rounded down
        to SHARD_ALIGN elements; the last rank takes the remainder."""
        return shard_bounds(self.n, rank, world)


def shard_bounds(n: int, rank: int, world: int):
    if not (0 <= rank < world):
        raise ValueError("rank out of range")

    def b(r):
        if r >= world:
            return n
        return (r * n // world) // SHARD_ALIGN * SHARD_ALIGN

    return b(rank), b(rank + 1)


def decoder_layout(name, n_layers, d, h, vocab):
    """ARK's decoder (memory.rs:202-255): tied embedding, RMSNorm gains,
    SwiGLU FFN with hidden size h."""
    ts = [TensorSpec("embed", vocab * d, True), TensorSpec("gamma_final", d, False)]
    for l in range(n_layers):
        ts += [
            TensorSpec(f"l{l}.wq", d * d, True), TensorSpec(f"l{l}.wk", d * d, True),
            TensorSpec(f"l{l}.wv", d * d, True), TensorSpec(f"l{l}.wo", d * d, True),
            TensorSpec(f"l{l}.w1", d * h, True), TensorSpec(f"l{l}.w2", h * d, True),
            TensorSpec(f"l{l}.w3", d * h, True),
            TensorSpec(f"l{l}.g1", d, False), TensorSpec(f"l{l}.g2", d, False),
        ]
    return Layout(name, ts)


def eko_layout():
    """EKO-237M: 30 layers, d 768, 12 heads, SwiGLU 2048, vocab 32000."""
    return decoder_layout("EKO-237M", 30, 768, 2048, 32000)


def decoder_1p3b_layout():
    return decoder_layout("decoder-1.3B", 24, 2048, 5504, 32000)


def decoder_7b_layout():
    return decoder_layout("decoder-7B", 32, 4096, 11008, 32000)


def flat_layout(n: int):
    """A single contiguous decayed buffer (the flat bandwidth sweep)."""
    return Layout(f"flat-{n}", [TensorSpec("flat", n, True)])


LAYOUTS = {
    "eko": eko_layout,
    "1.3b": decoder_1p3b_layout,
    "7b": decoder_7b_layout,
}
