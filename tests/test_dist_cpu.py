"""World-size-2 sharding on CPU over gloo: each rank owns a ZeRO-1 shard,
computes its pass-1 partial, the partials are all-gathered and combined in
rank order (as the device step does), and each rank applies the step to its
shard.  The gathered result must equal the single-rank step bit for bit.
Also exercises the NCCL unique-id broadcast used by ark_b200.dist."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from ark_b200 import layout


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    import torch
    import torch.distributed as dist

    from ark_b200 import dist as adist
    from oracle import oracle

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        L = layout.decoder_layout("tiny", 3, 32, 72, 97)
        lo, hi = L.shard(rank, world)
        n = hi - lo
        scale = 4096.0
        w = oracle.synth_f16(n, lo, 5, 1, 0.02)
        g = oracle.synth_f16(n, lo, 5, 2, 1e-3, scale)
        m = oracle.synth_f32(n, lo, 5, 3, 1e-4)
        v = oracle.synth_f32(n, lo, 5, 4, 1e-3, square=True)
        cfg = oracle.make_cfg(weight_decay=0.1, grad_clip=0.05, n_decay=L.n_decay)
        st = oracle.make_state(scale, opt_step=999)
        s, bad = oracle.partial_f16(cfg, st, g, lo)
        part = torch.tensor([s, float(bad)], dtype=torch.float64)
        parts = [torch.zeros(2, dtype=torch.float64) for _ in range(world)]
        dist.all_gather(parts, part)
        total = 0.0
        nbad = 0
        for p in parts:                      # rank order
            total += float(p[0])
            nbad += int(p[1])
        rc = oracle.apply_f16(cfg, st, w, g, m, v, lo, total, nbad)
        # NCCL unique-id broadcast path (bytes only; no GPU needed)
        uid = adist.share_unique_id(bytes(range(128)) if rank == 0 else None, rank)
        q.put((rank, lo, hi, rc, w, m, v, st.last_norm, st.loss_scale, uid))
    finally:
        dist.destroy_process_group()


def test_two_rank_shards_match_single_rank(oracle):
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=120) for _ in range(world)], key=lambda r: r[0])
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    L = layout.decoder_layout("tiny", 3, 32, 72, 97)
    n, scale = L.n, 4096.0
    w = oracle.synth_f16(n, 0, 5, 1, 0.02)
    g = oracle.synth_f16(n, 0, 5, 2, 1e-3, scale)
    m = oracle.synth_f32(n, 0, 5, 3, 1e-4)
    v = oracle.synth_f32(n, 0, 5, 4, 1e-3, square=True)
    cfg = oracle.make_cfg(weight_decay=0.1, grad_clip=0.05, n_decay=L.n_decay)
    st = oracle.make_state(scale, opt_step=999)
    assert oracle.step_flat_f16(cfg, st, w, g, m, v) == 0
    for rank, lo, hi, rc, ws, ms, vs, norm, ls, uid in res:
        assert rc == 0
        assert np.array_equal(ws, w[lo:hi])
        assert np.array_equal(ms.view(np.uint32), m[lo:hi].view(np.uint32))
        assert np.array_equal(vs.view(np.uint32), v[lo:hi].view(np.uint32))
        assert norm == st.last_norm and ls == st.loss_scale
        assert uid == bytes(range(128))
    assert res[0][2] == res[1][1] and res[1][2] == n
