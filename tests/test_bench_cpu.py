"""Host logic of bench.py that needs no GPU: the L2-flush decision and the
reference arm's CPU step (the oracle port of the reference's per-tensor
path) on a small decoder layout, full and as a bounded prefix."""
import bench
from ark_b200 import layout


def test_flush_decision_eko():
    n = layout.eko_layout().n
    assert not bench.needs_flush(n, 1)
    assert not bench.needs_flush(n, 4)          # 711 MB per GPU >= 4 x 126 MiB
    assert bench.needs_flush(n, 8)              # 355 MB per GPU
    assert bench.needs_flush(1 << 22, 1) and not bench.needs_flush(1 << 26, 1)


def test_reference_step_runs_on_the_host(oracle):
    L = layout.decoder_layout("tiny", 3, 32, 72, 97)
    step = bench.cpu_reference_step_setup(L, threads=2)
    assert step.n_params == L.n and step.n_tensors == L.n_tensors
    assert step() > 0 and step() > 0


def test_bounded_reference_step_takes_a_prefix(oracle):
    L = layout.decoder_layout("tiny", 3, 32, 72, 97)
    step, t_full = bench.bounded_reference_step(L, 2, 10, budget_s=1e-9)
    assert t_full > 0
    assert step.n_tensors == 1 and step.n_params == L.tensors[0].numel
    full, _ = bench.bounded_reference_step(L, 2, 1, budget_s=60.0)
    assert full.n_tensors == L.n_tensors


def test_parity_windows_cover_each_shard_boundary():
    """The parity leg's windows lie inside the rank's shard and include its
    two ends and every weight-decay / tensor boundary inside it."""
    L = layout.eko_layout()
    for world in (1, 2, 8):
        for r in range(world):
            lo, hi = L.shard(r, world)
            wins = bench._windows_of_shard(L, lo, hi)
            assert wins and all(lo <= a < b <= hi for a, b in wins)
            assert any(a == lo for a, _ in wins) and any(b == hi for _, b in wins)
            bounds = [L.n_decay] + [L.offsets[t.name] for t in L.flat]
            for x in bounds:
                if lo + 1024 <= x <= hi - 1024:
                    assert any(a < x < b for a, b in wins), (world, r, x)


def test_numa_lookup_tolerates_missing_sysfs():
    assert bench.numa_local_cpus(0) is None or isinstance(bench.numa_local_cpus(0), set)
