"""The ZeRO-1 sharded step on 2 GPUs (one process per GPU, the library's
peer-to-peer exchange of the 16-byte partials, or NCCL) against the CPU oracle run on
the whole buffer: every rank's shard bit for bit, the replicated loss-scale
state identical on every rank, and the FP16 weight all-gather.  Skipped
when fewer than 2 GPUs are visible."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp
from gpu_util import same_f16

pytestmark = pytest.mark.gpu

WORLD = 2
# world sizes of the parity test: 2, and 4 / 8 where that many GPUs are visible
WORLDS = [w for w in (2, 4, 8) if w <= max(torch.cuda.device_count(), 2)]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank_main(rank, world, port, q, nccl_exchange, p1_last=None):
    import datetime

    if p1_last is not None:   # who forms the rank partial: pass 1's last block or pass 2
        os.environ["ARK_P1_LAST"] = p1_last

    import torch.distributed as dist

    import ark_b200 as ab
    from ark_b200 import dist as adist
    from ark_b200 import layout, synth
    from oracle import oracle

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    comm = None
    try:
        comm = adist.nccl_comm(rank, world, rank)
        L = layout.decoder_layout("multi", 4, 96, 256, 1000)
        seed, scale = 77, 65536.0
        adam = ab.AdamConfig(lr=3e-4, beta1=0.9, beta2=0.95, eps=1e-8, weight_decay=0.1,
                             grad_clip=1.0)
        sc = ab.LossScaleConfig(init=scale, every=3, max=2.0 ** 24)
        opt = ab.Optimizer(L, adam, sc, device=rank, rank=rank, world=world, comm=comm,
                           constant_lr=True, initial_step=999, nccl_exchange=nccl_exchange)
        lo, hi, n = opt.lo, opt.hi, opt.n
        w16, g16, m, v = synth.make_state(n, lo, seed, "cuda", loss_scale=scale)
        inject_step = 3
        statuses = []
        for k in range(1, 6):
            if k == inject_step:
                idx = int(oracle.lib().ork_inject_index(seed, k, L.n))
                if lo <= idx < hi:
                    g16.view(torch.int16)[idx - lo] = 0x7C00
            if k == inject_step + 1:
                synth.fill_grads(g16, lo, seed, scale)        # clean grads again
            opt.step_all(w16, g16, m, v)
            statuses.append(opt.status())
        stride = -(-L.n // world) + 128
        full = torch.zeros(stride * world, dtype=torch.float16, device="cuda")
        shard = torch.zeros(stride, dtype=torch.float16, device="cuda")
        shard[:n] = w16
        opt.allgather_weights(shard, full, stride)
        torch.cuda.synchronize()
        q.put((rank, lo, hi, w16.cpu().numpy().view(np.uint16), m.cpu().numpy(),
               v.cpu().numpy(), statuses, full.cpu().numpy().view(np.uint16), stride))
        opt.close()
    finally:
        if comm:
            adist.nccl_comm_destroy(comm)
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < WORLD, reason="needs 2 GPUs")
@pytest.mark.parametrize("world", WORLDS)
@pytest.mark.parametrize("nccl_exchange,p1_last", [(False, None), (True, None), (False, "1")],
                         ids=["p2p", "nccl", "p2p-p1last"])
def test_multi_gpu_zero1_step_matches_oracle(oracle, nccl_exchange, p1_last, world):
    from ark_b200 import layout, synth
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q, nccl_exchange, p1_last))
             for r in range(world)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=300) for _ in range(world)], key=lambda r: r[0])
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    # oracle on the whole buffer, same schedule
    L = layout.decoder_layout("multi", 4, 96, 256, 1000)
    seed, scale, n = 77, 65536.0, L.n
    w = oracle.synth_f16(n, 0, seed, synth.STREAM_W, 0.02)
    g = oracle.synth_f16(n, 0, seed, synth.STREAM_G, 1e-3, scale)
    g_clean = g.copy()
    m = oracle.synth_f32(n, 0, seed, synth.STREAM_M, 1e-4)
    v = oracle.synth_f32(n, 0, seed, synth.STREAM_V, 1e-3, square=True)
    cfg = oracle.make_cfg(n_decay=L.n_decay, scale_every=3, scale_max=2.0 ** 24)
    st = oracle.make_state(scale, opt_step=999)
    ref_states = []
    for k in range(1, 6):
        if k == 3:
            g[oracle.lib().ork_inject_index(seed, k, n)] = 0x7C00
        if k == 4:
            g = g_clean.copy()
        s, bad = oracle.partial_f16(cfg, st, g, 0)
        oracle.apply_f16(cfg, st, w, g, m, v, 0, s, bad)
        ref_states.append((st.loss_scale, st.opt_step, st.last_overflow, st.clean_steps,
                           st.last_norm))
    for rank, lo, hi, ws, ms, vs, sts, full, stride in res:
        assert np.array_equal(ws, w[lo:hi]), rank
        assert np.array_equal(ms.view(np.uint32), m[lo:hi].view(np.uint32)), rank
        assert np.array_equal(vs.view(np.uint32), v[lo:hi].view(np.uint32)), rank
        got = [(s["loss_scale"], s["opt_step"], s["last_overflow"], s["clean_steps"],
                s["last_norm"]) for s in sts]
        for a, b in zip(got, ref_states):
            assert a[:4] == b[:4]
            assert abs(a[4] - b[4]) <= 1e-5 * max(b[4], 1e-30)
        for r2, lo2, hi2, *_ in res:                      # all-gathered weights
            assert np.array_equal(full[r2 * stride: r2 * stride + (hi2 - lo2)], w[lo2:hi2])
    assert all(r[6][-1] == res[0][6][-1] for r in res)    # replicated state identical


def _timeout_rank_main(rank, world, port, q, go):
    import datetime

    import torch.distributed as dist

    import ark_b200 as ab
    from ark_b200 import dist as adist
    from ark_b200 import layout, synth

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    comm = adist.nccl_comm(rank, world, rank)
    L = layout.flat_layout(1 << 20)
    opt = ab.Optimizer(L, rank=rank, world=world, comm=comm, device=rank, constant_lr=True,
                       wait_timeout_ms=500)
    bufs = synth.make_state(opt.n, opt.lo, 5, "cuda")
    opt.step_all(*bufs)                       # one step together
    rc0, st0 = opt.read_status()
    dist.barrier()
    result = None
    if rank == 0:
        opt.step_all(*bufs)                   # rank 1 has left: the wait must run out
        rc1, st1 = opt.read_status()
        # the context is still usable after the timeout
        x = torch.ones(1024, device="cuda").sum().item()
        result = (rc0, st0["opt_step"], rc1, st1["error"], st1["opt_step"], x)
        go.set()
    else:
        go.wait(120)                          # stay alive (slots mapped) until rank 0 is done
        result = (rc0, st0["opt_step"])
    q.put((rank, result))
    opt.close()
    adist.nccl_comm_destroy(comm)
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < WORLD, reason="needs 2 GPUs")
def test_peer_wait_times_out_when_a_rank_leaves():
    port = _free_port()
    ctx = mp.get_context("spawn")
    q, go = ctx.Queue(), ctx.Event()
    procs = [ctx.Process(target=_timeout_rank_main, args=(r, WORLD, port, q, go))
             for r in range(WORLD)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in range(WORLD))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    rc0, step0, rc1, err, step_after, x = res[0]
    assert rc0 == 0 and step0 == 1 and res[1] == (0, 1)
    assert rc1 == -5 and err == -5           # ARK_E_TIMEOUT, step skipped
    assert step_after == 1 and x == 1024.0


def _reduce_rank_main(rank, world, port, q):
    import datetime

    import torch.distributed as dist

    import ark_b200 as ab
    from ark_b200 import dist as adist
    from ark_b200 import layout, synth

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    comm = adist.nccl_comm(rank, world, rank)
    try:
        L = layout.decoder_layout("multi", 4, 96, 256, 1000)
        adam = ab.AdamConfig(lr=3e-4, beta1=0.9, beta2=0.95, eps=1e-8, weight_decay=0.1,
                             grad_clip=1.0)
        sc = ab.LossScaleConfig(init=4096.0, every=2, max=2.0 ** 24)
        opt = ab.Optimizer(L, adam, sc, device=rank, rank=rank, world=world, comm=comm,
                           constant_lr=True, initial_step=999)
        lo, hi, n = opt.lo, opt.hi, opt.n
        w16, _, m, v = synth.make_state(n, lo, 91, "cuda", loss_scale=4096.0)
        full = opt.grad_buffer()
        shard_g = torch.zeros(n, dtype=torch.float16, device="cuda")
        statuses, shards = [], []
        for k in range(1, 5):
            # this rank's backward output for step k (stream 0x400 + 16 k + rank)
            synth.fill_f16(full, 0, 91, 0x400 + 16 * k + rank, 1e-3, mult=4096.0)
            if k == 2 and rank == world - 1:
                full.view(torch.int16)[L.n // 2] = 0x7E00
            opt.step_reduce(w16, shard_g, m, v)
            statuses.append(opt.status())
            shards.append(shard_g.cpu().numpy().view(np.uint16).copy())
        q.put((rank, lo, hi, w16.cpu().numpy().view(np.uint16), m.cpu().numpy(),
               v.cpu().numpy(), statuses, shards))
        opt.close()
    finally:
        adist.nccl_comm_destroy(comm)
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < WORLD, reason="needs 2 GPUs")
@pytest.mark.parametrize("world", WORLDS)
def test_reduce_scatter_step_matches_oracle(oracle, world):
    """The gradient hand-off fused with pass 1: every rank reads its shard of
    every rank's full gradient buffer over NVLink and sums in rank order."""
    from ark_b200 import layout, synth
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_reduce_rank_main, args=(r, world, port, q))
             for r in range(world)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=300) for _ in range(world)], key=lambda r: r[0])
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    L = layout.decoder_layout("multi", 4, 96, 256, 1000)
    n = L.n
    w = oracle.synth_f16(n, 0, 91, synth.STREAM_W, 0.02)
    m = oracle.synth_f32(n, 0, 91, synth.STREAM_M, 1e-4)
    v = oracle.synth_f32(n, 0, 91, synth.STREAM_V, 1e-3, square=True)
    cfg = oracle.make_cfg(n_decay=L.n_decay, scale_every=2, scale_max=2.0 ** 24)
    st = oracle.make_state(4096.0, opt_step=999)
    ref_states, ref_shards = [], []
    for k in range(1, 5):
        fulls = [oracle.synth_f16(n, 0, 91, 0x400 + 16 * k + r, 1e-3, 4096.0)
                 for r in range(world)]
        if k == 2:
            fulls[world - 1][n // 2] = 0x7E00
        g = oracle.reduce_f16(fulls, n, 0)
        ref_shards.append(g)
        s, bad = oracle.partial_f16(cfg, st, g, 0)
        oracle.apply_f16(cfg, st, w, g, m, v, 0, s, bad)
        ref_states.append((st.loss_scale, st.opt_step, st.last_overflow, st.clean_steps))
    for rank, lo, hi, ws, ms, vs, sts, shards in res:
        for k in range(4):
            # NaN payloads differ (CUDA returns a canonical NaN); any NaN matches
            assert same_f16(shards[k], ref_shards[k][lo:hi]), (rank, k)
            s = sts[k]
            assert (s["loss_scale"], s["opt_step"], s["last_overflow"], s["clean_steps"]) == \
                ref_states[k], (rank, k)
        assert np.array_equal(ws, w[lo:hi]), rank
        assert np.array_equal(ms.view(np.uint32), m[lo:hi].view(np.uint32)), rank
        assert np.array_equal(vs.view(np.uint32), v[lo:hi].view(np.uint32)), rank


def _gather_rank_main(rank, world, port, q):
    import datetime

    import torch.distributed as dist

    import ark_b200 as ab
    from ark_b200 import dist as adist
    from ark_b200 import layout, synth

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    comm = adist.nccl_comm(rank, world, rank)
    try:
        L = layout.decoder_layout("multi", 4, 96, 256, 1000)
        adam = ab.AdamConfig(lr=3e-4, beta1=0.9, beta2=0.95, eps=1e-8, weight_decay=0.1,
                             grad_clip=1.0)
        sc = ab.LossScaleConfig(init=2048.0, every=2, max=2.0 ** 24)
        opt = ab.Optimizer(L, adam, sc, device=rank, rank=rank, world=world, comm=comm,
                           constant_lr=True, initial_step=99, use_graph=True)
        lo, hi, n = opt.lo, opt.hi, opt.n
        full = opt.weight_buffer()
        _, g16, m, v = synth.make_state(n, lo, 33, "cuda", loss_scale=2048.0)
        w16 = full[lo:hi]                              # the shard lives in the full buffer
        synth.fill_f16(w16, lo, 33, synth.STREAM_W, 0.02)
        logits = torch.empty(4099, dtype=torch.float32, device="cuda")
        statuses, fulls = [], []
        for k in range(1, 6):
            synth.fill_f32(logits, 0, 33, 0x900 + 16 * k + rank, 1e-2)
            if k == 2 and rank == world - 1:
                logits[17] = float("nan")              # one rank's logits are bad
            opt.logits_check(logits)
            synth.fill_grads(g16, lo, 33 + k, opt.status()["loss_scale"])
            opt.step_gather(w16, g16, m, v)
            opt.weights_wait()
            statuses.append(opt.status())
            fulls.append(full.cpu().numpy().view(np.uint16).copy())
        q.put((rank, lo, hi, statuses, fulls, m.cpu().numpy(), v.cpu().numpy()))
        opt.close()
    finally:
        adist.nccl_comm_destroy(comm)
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < WORLD, reason="needs 2 GPUs")
@pytest.mark.parametrize("world", WORLDS)
def test_fused_weight_gather_and_logits_check_match_oracle(oracle, world):
    """Every rank's full weight buffer equals the oracle's whole-buffer
    weights after every step (the shard stored by the update kernel into
    every peer over NVLink); one rank's non-finite logits skip the step on
    every rank."""
    from ark_b200 import layout, synth
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_gather_rank_main, args=(r, world, port, q))
             for r in range(world)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=300) for _ in range(world)], key=lambda r: r[0])
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    L = layout.decoder_layout("multi", 4, 96, 256, 1000)
    n = L.n
    w = oracle.synth_f16(n, 0, 33, synth.STREAM_W, 0.02)
    m = oracle.synth_f32(n, 0, 33, synth.STREAM_M, 1e-4)
    v = oracle.synth_f32(n, 0, 33, synth.STREAM_V, 1e-3, square=True)
    cfg = oracle.make_cfg(n_decay=L.n_decay, scale_every=2, scale_max=2.0 ** 24)
    st = oracle.make_state(2048.0, opt_step=99)
    ref_w, ref_st = [], []
    for k in range(1, 6):
        g = oracle.synth_f16(n, 0, 33 + k, synth.STREAM_G, 1e-3, st.loss_scale)
        if k == 2:
            oracle.apply_f16(cfg, st, w, g, m, v, 0, 0.0, 1)    # rejected at the logits check
        else:
            s, bad = oracle.partial_f16(cfg, st, g, 0)
            oracle.apply_f16(cfg, st, w, g, m, v, 0, s, bad)
        ref_w.append(w.copy())
        ref_st.append((st.loss_scale, st.opt_step, st.last_overflow, st.clean_steps))
    for rank, lo, hi, sts, fulls, ms, vs in res:
        for k in range(5):
            assert np.array_equal(fulls[k], ref_w[k]), (rank, k)
            s = sts[k]
            assert (s["loss_scale"], s["opt_step"], s["last_overflow"], s["clean_steps"]) == \
                ref_st[k], (rank, k, s)
        assert np.array_equal(ms.view(np.uint32), m[lo:hi].view(np.uint32)), rank
        assert np.array_equal(vs.view(np.uint32), v[lo:hi].view(np.uint32)), rank


def _windows_of_shard(L, lo, hi, span=2048):
    """Windows of [lo, hi): the shard ends, the weight-decay boundary and
    tensor boundaries that fall inside it."""
    cand = [lo, hi - span, (lo + hi) // 2, L.n_decay - span // 2]
    cand += [L.offsets[t.name] - span // 2 for t in L.flat]
    out = set()
    for a in cand:
        a = max(lo, min(a, hi - span))
        if lo <= a < hi:
            out.add((a, min(a + span, hi)))
    return sorted(out)


def _big_rank_main(rank, world, port, q, workload):
    import datetime

    os.environ["OMP_NUM_THREADS"] = str(max(1, (os.cpu_count() or 8) // world))
    import torch.distributed as dist

    import ark_b200 as ab
    from ark_b200 import dist as adist
    from ark_b200 import layout, synth
    from oracle import oracle

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=300))
    comm = adist.nccl_comm(rank, world, rank)
    try:
        L = layout.LAYOUTS[workload]()
        heavy = workload == "7b"
        adam = ab.AdamConfig(lr=3e-4, beta1=0.9, beta2=0.95, eps=1e-8, weight_decay=0.1,
                             grad_clip=1.0)
        sc = ab.LossScaleConfig(init=65536.0, every=2000, max=2.0 ** 24)
        opt = ab.Optimizer(L, adam, sc, device=rank, rank=rank, world=world, comm=comm,
                           constant_lr=True, initial_step=999)
        lo, hi, n = opt.lo, opt.hi, opt.n
        w16, g16, m, v = synth.make_state(n, lo, 4242, "cuda", loss_scale=65536.0, heavy=heavy)
        opt.step_all(w16, g16, m, v)
        st = opt.status()
        wins = _windows_of_shard(L, lo, hi)
        got = [(a, b, w16[a - lo:b - lo].cpu().numpy().view(np.uint16).copy(),
                m[a - lo:b - lo].cpu().numpy().copy(), v[a - lo:b - lo].cpu().numpy().copy())
               for a, b in wins]
        g_host = oracle.synth_f16(n, lo, 4242, synth.STREAM_G, 1e-3, 65536.0,
                                  synth.HEAVY_EVERY if heavy else 0,
                                  synth.HEAVY_MULT if heavy else 1.0)
        cfg = oracle.make_cfg(n_decay=L.n_decay, scale_every=2000, scale_max=2.0 ** 24)
        sumsq, bad = oracle.partial_f16(cfg, oracle.make_state(65536.0, 999), g_host, lo)
        gwin = [np.ascontiguousarray(g_host[a - lo:b - lo]) for a, b in wins]
        q.put((rank, lo, hi, sumsq, bad, st, got, gwin))
        opt.close()
    finally:
        adist.nccl_comm_destroy(comm)
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 8, reason="needs 8 GPUs")
def test_7b_sharded_over_8_windows_match_oracle(oracle):
    """BASELINE's 7B configuration (heavy-tailed gradients, clipping active)
    ZeRO-1 sharded over 8 B200: every rank's windows (shard ends, the
    weight-decay boundary, tensor boundaries) bit for bit against the
    oracle driven by the oracle's own global sum of squares, and the
    replicated state identical on every rank."""
    from ark_b200 import layout, synth
    world = 8
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_big_rank_main, args=(r, world, port, q, "7b"))
             for r in range(world)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=900) for _ in range(world)], key=lambda r: r[0])
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    L = layout.LAYOUTS["7b"]()
    sumsq = 0.0
    for r in res:                                     # rank order
        sumsq += r[3]
        assert r[4] == 0
    cfg = oracle.make_cfg(n_decay=L.n_decay, scale_every=2000, scale_max=2.0 ** 24)
    norm = np.float32(np.sqrt(sumsq))
    sts = [r[5] for r in res]
    assert all(s == sts[0] for s in sts)              # replicated state identical
    assert abs(sts[0]["last_sumsq"] - sumsq) <= 1e-12 * sumsq
    assert abs(sts[0]["last_norm"] - norm) <= 1e-5 * norm
    assert sts[0]["last_clip_coef"] < 0.01 and sts[0]["opt_step"] == 1000
    for rank, lo, hi, _, _, _, got, gwin in res:
        for (a, b, dw, dm, dv), g in zip(got, gwin):
            w = oracle.synth_f16(b - a, a, 4242, synth.STREAM_W, 0.02)
            m = oracle.synth_f32(b - a, a, 4242, synth.STREAM_M, 1e-4)
            v = oracle.synth_f32(b - a, a, 4242, synth.STREAM_V, 1e-3, square=True)
            ost = oracle.make_state(65536.0, opt_step=999)
            oracle.apply_f16(cfg, ost, w, g, m, v, a, sumsq, 0)
            assert np.array_equal(dw, w), (rank, a)
            assert np.array_equal(dm.view(np.uint32), m.view(np.uint32)), (rank, a)
            assert np.array_equal(dv.view(np.uint32), v.view(np.uint32)), (rank, a)
