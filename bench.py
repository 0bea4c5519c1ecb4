"""Benchmark of the ARK optimizer hot path on B200.

Workload: the EKO-237M full optimizer step --
finite check + unscale + global L2 norm and clip + AdamW (FP16 weights in
place, FP32 m/v) + loss-scale update -- over all 236,959,488 parameters,
ZeRO-1-sharded over the N GPUs of one node (one process per GPU).  Inputs
are seeded synthetic tensors with the BASELINE distributions, generated on
the device.  The optimizer state (2.8 GB of w, g, m, v at N=1) is far larger
than the 126 MB L2, so no flush is needed between steps; states below four
times the L2 (small --params sizes) are timed step by step with a 256 MiB
write between steps that evicts the L2.

Metric: step time and achieved HBM bandwidth, counted as 24 algorithmic
bytes per parameter per step (pass 1 reads the 2-byte gradient; pass 2
reads g, w, m, v and writes w, m, v: 22 bytes); value = 24 * N_params /
step time, whole job (all GPUs).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
  (N > 1: python -m torch.distributed.run --nproc-per-node N bench.py --gpus N ...)
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "AdamW+clip step time & achieved HBM GB/s, EKO-237M fp16, 1/2/4/8 B200"
BYTES_PER_PARAM = 24          # algorithmic bytes per parameter per step
PASS2_BYTES_PER_PARAM = 22    # dominant kernel: pass 2
PASS1_BYTES_PER_PARAM = 2
SEED = 20261201
EKO_HPARAMS = dict(lr=3e-4, beta1=0.9, beta2=0.95, eps=1e-8, weight_decay=0.1, grad_clip=1.0)
START_STEP = 1000             # configs[0]: "step 1000"
LOSS_SCALE = 65536.0
L2_BYTES = 126 * 2 ** 20
STATE_BYTES_PER_PARAM = 12    # resident w16 + g16 + m + v
FLUSH_BYTES = 256 * 2 ** 20


def measured_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs)"
    except Exception:
        return 6650.0, "fallback 6.65 TB/s (MEASURED_PEAKS.json absent)"


# DRAM bytes (read + write) per parameter of one pass-2 launch, from one ncu
# capture of the default pass-2 kernel on a 128 Mi-param flat case (state
# above the L2), scaled by the shard's parameters for roofline.traffic:
#   ncu --metrics dram__bytes_read.sum,dram__bytes_write.sum,gpu__time_duration.sum \
#       --clock-control none -k regex:pass2_kernel -s 6 -c 1 \
#       python bench.py --params 134217728 --steps 3 --warmup 3 --no-graph (+ no extra legs)
# Refresh it whenever pass 2 changes.
PASS2_DRAM_BYTES_PER_PARAM = 21.58
NVLINK_PEER_COPY_GBS = 770.0  # measured peer copy per direction per GPU on this pool


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 50 ms; summary()
    keeps the samples taken inside the timed window [t0, t1]."""
    Q = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_ids):
        self.gpu = ",".join(gpu_ids)
        self.proc = None
        self.path = None
        self.t0 = self.t1 = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(prefix="ark_clocks_", suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
            time.sleep(1.0)           # let the sampler start before the timed region
        except OSError:
            self.proc = None
        return self

    def mark(self, which):
        setattr(self, which, time.time())

    def __exit__(self, *a):
        if self.proc:
            time.sleep(0.2)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        import datetime
        if not self.proc or not self.path:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = []
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 10:
                continue
            try:
                ts = datetime.datetime.strptime(parts[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                rows.append((ts, float(parts[2]), float(parts[3]), parts[6:10], parts[4]))
            except ValueError:
                continue
        os.unlink(self.path)
        inside = [r for r in rows if self.t0 and self.t0 <= r[0] <= self.t1]
        widened = False
        if not inside and rows and self.t0:
            # window shorter than the sampling period: nearest samples around it
            inside = [r for r in rows if self.t0 - 0.25 <= r[0] <= self.t1 + 0.25]
            widened = True
        if not inside:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"],
                    "samples": 0}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in inside for i in range(4) if r[3][i] == "Active"})
        out = {"sm_mhz": statistics.median(r[1] for r in inside),
               "sm_max_mhz": max(r[2] for r in inside), "reasons": reasons,
               "samples": len(inside)}
        if widened:
            out["window"] = "timed region shorter than the 50 ms sampling period; +-250 ms"
        return out


def nvidia_smi_ids(devices):
    """nvidia-smi ids (UUIDs) of CUDA devices: nvidia-smi numbers GPUs
    physically and ignores CUDA_VISIBLE_DEVICES."""
    import torch
    out = []
    for d in devices:
        try:
            out.append("GPU-" + str(torch.cuda.get_device_properties(d).uuid))
        except Exception:
            out.append(str(d))
    return out


def cpu_reference_step_setup(L, threads, n_tensors=None):
    """The reference's own CPU path (per tensor, FP32 grads) on this host,
    over the first n_tensors tensors of the reference order (all by
    default)."""
    from oracle import oracle
    k = L.n_tensors if n_tensors is None else n_tensors
    tensors = L.tensors[:k]
    n = sum(t.numel for t in tensors)
    w16 = oracle.synth_f16(n, 0, SEED, 1, 0.02)
    g32 = oracle.dequant(oracle.synth_f16(n, 0, SEED, 2, 1e-3, LOSS_SCALE))
    m = oracle.synth_f32(n, 0, SEED, 3, 1e-4)
    v = oracle.synth_f32(n, 0, SEED, 4, 1e-3, square=True)
    g_fresh = g32.copy()
    ts = (oracle.Tensor * k)()
    o = 0
    # reference order (optimizer.rs:185-227), contiguous host arrays as in memory.rs
    for i, t in enumerate(tensors):
        ts[i] = oracle.Tensor(w16[o:].ctypes.data, g32[o:].ctypes.data, m[o:].ctypes.data,
                              v[o:].ctypes.data, t.numel, EKO_HPARAMS["weight_decay"] if t.decay
                              else 0.0, 0 if t.name == "gamma_final" else 1)
        o += t.numel
    st = oracle.make_state(LOSS_SCALE, opt_step=START_STEP - 1)
    keep = (w16, g32, m, v, g_fresh)

    def step():
        np.copyto(g32, g_fresh)           # fresh grads each step (the backward's job; untimed)
        t0 = time.perf_counter()
        rc = oracle.lib().ork_ref_step_tensors(
            ts, k, st, EKO_HPARAMS["lr"], EKO_HPARAMS["beta1"], EKO_HPARAMS["beta2"],
            EKO_HPARAMS["eps"], EKO_HPARAMS["grad_clip"], 2.0 ** 24, 2000, threads)
        dt = time.perf_counter() - t0
        assert rc == 0
        return dt

    step.n_params = n
    step.n_tensors = k
    step.keep = keep
    return step


def needs_flush(n_total, world):
    """True when a rank's state (w, g, m, v of the mean shard) is below 4x
    the L2: such steps are timed one by one with the L2 flushed between
    them.  Decided on the mean shard so that every rank agrees."""
    return (n_total // world) * STATE_BYTES_PER_PARAM < 4 * L2_BYTES


def bounded_reference_step(L, threads, n_steps, budget_s):
    """A full-EKO step if n_steps of them fit in budget_s, else the longest
    prefix of the reference tensor order that does (a bounded sample)."""
    full = cpu_reference_step_setup(L, threads)
    t_full = min(full(), full())
    per_step = budget_s / max(n_steps, 1)
    if t_full <= per_step:
        return full, t_full
    target = L.n * per_step / t_full
    acc, k = 0, 0
    for t in L.tensors:
        if k > 0 and acc + t.numel > target:
            break
        acc += t.numel
        k += 1
    del full
    return cpu_reference_step_setup(L, threads, k), t_full


def run_reference(args):
    """--impl reference: the reference's CPU optimizer path (oracle port of
    opti.s + optimizer.rs + training.rs, per tensor, FP32 grads) with every
    host thread, on the same EKO-237M workload."""
    rank = int(os.environ.get("RANK", 0))
    if rank != 0:
        return
    from ark_b200 import layout
    from oracle import oracle
    oracle.build()
    # every host core this process may run on (torchrun sets OMP_NUM_THREADS=1)
    threads = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
    L = layout.eko_layout()
    step, t_full = bounded_reference_step(L, threads, args.steps + args.warmup, budget_s=150.0)
    for _ in range(args.warmup):
        step()
    times = [step() for _ in range(args.steps)]
    t = statistics.mean(times)
    value = BYTES_PER_PARAM * step.n_params / t / 1e9
    sample = (f"full EKO-237M step ({L.n} params, {L.n_tensors} tensors)" if step.n_tensors ==
              L.n_tensors else
              f"first {step.n_tensors} of {L.n_tensors} tensors in reference order "
              f"({step.n_params} params) per step; full step measured at {t_full * 1e3:.1f} ms")
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "GB/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(t * 1e3 * L.n / step.n_params, 3), "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded, BASELINE distributions)",
        "config": {"workload": "EKO-237M full optimizer step (BASELINE configs[0])",
                   "params": L.n, "tensors": L.n_tensors, "grads": "fp32 (reference layout)"},
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": threads,
                         "kind": "port", "sample": sample},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def cpu_baseline_single_thread(L, budget_s=20.0):
    """1-thread reference path (faithful to the reference's single thread)."""
    from oracle import oracle
    oracle.build()
    step = cpu_reference_step_setup(L, 1)
    times = []
    t_end = time.perf_counter() + budget_s
    while not times or (time.perf_counter() < t_end and len(times) < 3):
        times.append(step())
    t = min(times)
    return {"value": round(BYTES_PER_PARAM * L.n / t / 1e9, 3), "unit": "GB/s", "cores": 1,
            "kind": "port",
            "sample": f"full EKO-237M step x {len(times)} on 1 thread, best "
                      f"{t * 1e3:.0f} ms/step"}


def measure_aux(opt, L, w16, g16, m, v, stream, args, max_over_ranks, barrier):
    """Rows next to the path, timed with CUDA events on the step's stream:
    the step that also writes the forward's FP32 weights vs the step plus
    the reference's separate per-step dequant (legacy ark_dequant_f16_to_f32),
    and ARK4 checkpoint save / load of this rank's shard."""
    import torch

    import ark_b200 as ab
    from ark_b200 import checkpoint
    n = opt.n
    k = max(3, min(args.steps, 200))
    w32 = torch.empty(n, dtype=torch.float32, device=w16.device)
    ab.dequant_f16_to_f32(w16, w32)

    def timed(fn):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(k):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        barrier()
        return max_over_ranks(e0.elapsed_time(e1) / k)

    t_w32 = timed(lambda: opt.step_all_w32(w16, g16, m, v, w32))

    def step_then_dequant():
        opt.step_all(w16, g16, m, v)
        ab.dequant_f16_to_f32(w16, w32)     # legacy entry point: synchronous per call

    ab.legacy_set_async(True)
    t_sep = timed(step_then_dequant)
    ab.legacy_set_async(False)
    out = {"step_with_fp32_weights_ms": round(t_w32, 4),
           "step_then_dequant_ms": round(t_sep, 4),
           "fp32_copy_saving_ms": round(t_sep - t_w32, 4)}
    if args.ckpt_dir and L.tensors[0].name == "embed":
        import time
        path = os.path.join(args.ckpt_dir, f"ark_bench_{os.getpid() if opt.world == 1 else 'x'}.bin")
        if opt.world > 1:
            path = os.path.join(args.ckpt_dir, "ark_bench_sharded.bin")
        barrier()
        t0 = time.perf_counter()
        checkpoint.save(opt, path, w16, m, v, global_step=1)
        barrier()
        t_save = max_over_ranks(time.perf_counter() - t0)
        t0 = time.perf_counter()
        checkpoint.load(opt, path, w16, m, v)
        barrier()
        t_load = max_over_ranks(time.perf_counter() - t0)
        size = os.path.getsize(path)
        out["checkpoint"] = {"file_bytes": size, "save_s": round(t_save, 3),
                             "load_s": round(t_load, 3),
                             "save_gbs": round(size / t_save / 1e9, 2),
                             "load_gbs": round(size / t_load / 1e9, 2), "path": args.ckpt_dir}
        barrier()
        if opt.rank == 0:
            os.unlink(path)
    return out


def numa_local_cpus(device):
    """Host CPUs on the GPU's NUMA node (from its PCI address), or None."""
    import torch
    try:
        pr = torch.cuda.get_device_properties(device)
        bus = "%04x:%02x:%02x.0" % (pr.pci_domain_id, pr.pci_bus_id, pr.pci_device_id)
        txt = open(f"/sys/bus/pci/devices/{bus}/local_cpulist").read().strip()
    except (OSError, AttributeError, RuntimeError):
        return None
    cpus = set()
    for part in txt.split(","):
        a, _, b = part.partition("-")
        cpus.update(range(int(a), int(b or a) + 1))
    return cpus or None


def timed_loop(fn, k, stream, barrier, max_over_ranks):
    """k calls of fn between CUDA events on the step's stream; ms per call,
    max over ranks."""
    import torch
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(k):
        fn()
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    return max_over_ranks(e0.elapsed_time(e1) / k)


def measure_allgather(opt, L, w16, g16, m, v, stream, args, max_over_ranks, barrier):
    """The optional ZeRO-1 FP16 weight all-gather, timed separately: the
    NCCL all-gather alone and after the step, and the library's all-gather
    fused with the update (pass 2 stores the updated shard into every rank's
    full weight buffer over NVLink, ARK_STEP_GATHER_WEIGHTS)."""
    import torch
    world, n, dev = opt.world, opt.n, w16.device
    k = max(5, min(args.steps, 100))
    stride = -(-L.n // world) + 128
    w_pad = torch.zeros(stride, dtype=torch.float16, device=dev)
    w_pad[:n].copy_(w16)
    full_nccl = torch.empty(stride * world, dtype=torch.float16, device=dev)
    t_nccl = timed_loop(lambda: opt.allgather_weights(w_pad, full_nccl, stride), k, stream,
                        barrier, max_over_ranks)

    def step_then_nccl():
        opt.step_all(w_pad[:n], g16, m, v)
        opt.allgather_weights(w_pad, full_nccl, stride)

    t_seq = timed_loop(step_then_nccl, k, stream, barrier, max_over_ranks)
    del full_nccl
    full = opt.weight_buffer()                    # collective
    wf = full[opt.lo:opt.hi]
    wf.copy_(w_pad[:n])

    def fused():
        opt.step_gather(wf, g16, m, v)
        opt.weights_wait()

    for _ in range(3):
        fused()
    t_fused = timed_loop(fused, k, stream, barrier, max_over_ranks)
    t_step = timed_loop(lambda: opt.step_all(w_pad[:n], g16, m, v), k, stream, barrier,
                        max_over_ranks)
    bytes_in = 2 * (L.n - n)                      # every other rank's shard, into this GPU
    out = {"bytes_in_per_gpu": int(bytes_in), "steps": k,
           "nccl_allgather_ms": round(t_nccl, 4),
           "nccl_gbs_in_per_gpu": round(bytes_in / (t_nccl * 1e-3) / 1e9, 1),
           "step_ms": round(t_step, 4),
           "step_then_nccl_ms": round(t_seq, 4),
           "fused_step_gather_ms": round(t_fused, 4),
           "fused_gbs_in_per_gpu": round(bytes_in / (t_fused * 1e-3) / 1e9, 1),
           "peer_copy_gbs_measured": NVLINK_PEER_COPY_GBS,
           "fused_nvlink_frac": round(bytes_in / (t_fused * 1e-3) / 1e9 / NVLINK_PEER_COPY_GBS, 4),
           "nccl_nvlink_frac": round(bytes_in / (t_nccl * 1e-3) / 1e9 / NVLINK_PEER_COPY_GBS, 4),
           "fused_saving_vs_step_then_nccl_ms": round(t_seq - t_fused, 4),
           "how": "CUDA events over k iterations on the step's stream, max over ranks; fused = "
                  "step with ARK_STEP_GATHER_WEIGHTS + ark_cuda_opt_weights_wait"}
    full_ok = bool(torch.equal(full[opt.lo:opt.hi].view(torch.int16), wf.view(torch.int16)))
    out["own_slice_consistent"] = full_ok
    return out


LEGACY_KERNEL_N = 1 << 27     # elements per legacy-kernel measurement (state >> L2)


def measure_legacy(L, stream, args):
    """The drop-in path: the reference's per-tensor optimizer calls through
    the unchanged legacy symbols (272 x ark_asm_adam_step_f16 per EKO step,
    optimizer.rs:185-227, in the library's async mode with one wait per
    step), and each legacy kernel alone at 2^27 elements, as GB/s of its
    algorithmic bytes."""
    import torch

    import ark_b200 as ab
    from ark_b200 import synth
    dev = torch.device("cuda", torch.cuda.current_device())
    n = L.n
    w16 = torch.empty(n, dtype=torch.float16, device=dev)
    g32 = torch.empty(n, dtype=torch.float32, device=dev)
    m = torch.empty(n, dtype=torch.float32, device=dev)
    v = torch.empty(n, dtype=torch.float32, device=dev)
    synth.fill_f16(w16, 0, SEED, synth.STREAM_W, 0.02)
    synth.fill_f32(g32, 0, SEED, 9, 1e-3)
    synth.fill_f32(m, 0, SEED, synth.STREAM_M, 1e-4)
    synth.fill_f32(v, 0, SEED, synth.STREAM_V, 1e-3, square=True)
    lib = ab.lib()
    hp = EKO_HPARAMS
    calls = []
    o = 0
    for t in L.tensors:                          # reference order, per-tensor wd
        wd = hp["weight_decay"] if t.decay else 0.0
        calls.append((w16.data_ptr() + 2 * o, g32.data_ptr() + 4 * o, m.data_ptr() + 4 * o,
                      v.data_ptr() + 4 * o, t.numel, wd))
        o += t.numel
    step_no = [START_STEP]

    def legacy_step():
        t = step_no[0]
        for wp, gp, mp, vp, cnt, wd in calls:
            lib.ark_asm_adam_step_f16(wp, gp, mp, vp, cnt, hp["lr"], hp["beta1"], hp["beta2"],
                                      hp["eps"], wd, t)
        step_no[0] += 1

    nothing = lambda: None  # noqa: E731
    ab.legacy_set_async(True)
    try:
        for _ in range(3):
            legacy_step()
        ab.legacy_sync()
        k = max(3, min(args.steps, 50))
        t_leg = timed_loop(legacy_step, k, stream, nothing, lambda x: x)
        assert lib.ark_cuda_last_error() == 0
        # the same 272 calls captured once into a CUDA graph (the legacy
        # stream pointed at a capturing stream) and replayed: t is fixed in
        # the captured launches, which changes nothing in the time
        t_graph = None
        cap = torch.cuda.Stream(device=dev)
        graph = torch.cuda.CUDAGraph()
        lib.ark_cuda_legacy_set_stream(cap.cuda_stream)
        try:
            with torch.cuda.graph(graph, stream=cap):
                legacy_step()
        finally:
            lib.ark_cuda_legacy_set_stream(None)
        if lib.ark_cuda_last_error() == 0:
            for _ in range(3):
                graph.replay()
            t_graph = timed_loop(graph.replay, k, torch.cuda.current_stream(dev), nothing,
                                 lambda x: x)
        del graph
        del w16, g32, m, v
        torch.cuda.empty_cache()
        # each kernel alone
        N = LEGACY_KERNEL_N
        a32 = torch.empty(N, dtype=torch.float32, device=dev)
        b32 = torch.empty(N, dtype=torch.float32, device=dev)
        c32 = torch.empty(N, dtype=torch.float32, device=dev)
        d32 = torch.empty(N, dtype=torch.float32, device=dev)
        h16 = torch.empty(N, dtype=torch.float16, device=dev)
        synth.fill_f32(a32, 0, 1, 5, 0.02)
        synth.fill_f32(b32, 0, 1, 9, 1e-3)
        synth.fill_f32(c32, 0, 1, 3, 1e-4)
        synth.fill_f32(d32, 0, 1, 4, 1e-3, square=True)
        synth.fill_f16(h16, 0, 1, 1, 0.02)
        norm = torch.zeros(1, dtype=torch.float32, device=dev)
        sh = stream.cuda_stream
        kk = 20
        clip_no = [0]

        def clip_call():
            # the norm starts near 11.6 and each call clips it to a threshold
            # half the previous one, so every call applies the scale
            thr = 8.0 * 0.5 ** clip_no[0]
            clip_no[0] += 1
            lib.ark_cuda_grad_clip_noalloc(b32.data_ptr(), N, thr, norm.data_ptr(), sh)

        kern = {
            "adam_vec8_kernel<f16> (ark_asm_adam_step_f16)": (24, lambda: lib.ark_asm_adam_step_f16(
                h16.data_ptr(), b32.data_ptr(), c32.data_ptr(), d32.data_ptr(), N, 3e-4, 0.9,
                0.95, 1e-8, 0.1, 1000)),
            "adam_vec8_kernel<f32> (ark_asm_adam_step)": (32, lambda: lib.ark_asm_adam_step(
                a32.data_ptr(), b32.data_ptr(), c32.data_ptr(), d32.data_ptr(), N, 3e-4, 0.9,
                0.95, 1e-8, 0.1, 1000)),
            "clip_norm_kernel + clip_scale_kernel (grad clip, scale applied)": (
                12, clip_call),
            "quant_kernel (ark_quant_f32_to_f16)": (6, lambda: lib.ark_quant_f32_to_f16(
                a32.data_ptr(), h16.data_ptr(), N)),
            "dequant_kernel (ark_dequant_f16_to_f32)": (6, lambda: lib.ark_dequant_f16_to_f32(
                h16.data_ptr(), a32.data_ptr(), N)),
        }
        per = {}
        for name, (bpe, fn) in kern.items():
            for _ in range(3):
                fn()
            ms = timed_loop(fn, kk, stream, nothing, lambda x: x)
            per[name] = {"ms": round(ms, 4), "bytes_per_elem": bpe,
                         "gbs": round(bpe * N / (ms * 1e-3) / 1e9, 1)}
        assert lib.ark_cuda_last_error() == 0
    finally:
        ab.legacy_set_async(False)
    peak, _ = measured_peak()
    for d in per.values():
        d["frac"] = round(d["gbs"] / peak, 4)
    return {"legacy_step_ms": round(t_leg, 4), "legacy_step_calls": len(calls),
            "legacy_step_gbs": round(BYTES_PER_PARAM * n / (t_leg * 1e-3) / 1e9, 1),
            "legacy_step_graph_ms": round(t_graph, 4) if t_graph else None,
            "legacy_step_note": "272 x ark_asm_adam_step_f16 per step (FP32 grads, already "
                                "unscaled and clipped: the reference's unscale and clip are "
                                "host loops with no legacy symbol), async mode, events around "
                                "the calls",
            "kernels_elements": N, "kernels": per}


def _windows_of_shard(L, lo, hi, span=2048):
    """Windows of [lo, hi): the shard ends, its middle, the weight-decay
    boundary and the tensor boundaries that fall inside it."""
    cand = [lo, hi - span, (lo + hi) // 2, L.n_decay - span // 2]
    cand += [L.offsets[t.name] - span // 2 for t in L.flat]
    out = set()
    for a in cand:
        a = max(lo, min(a, hi - span))
        if lo <= a < hi:
            out.add((a, min(a + span, hi)))
    return sorted(out)


def parity_leg(opt, L, w16, g16, m, v, heavy, world, rank, dev, barrier):
    """Checker leg, after every timed region: the CPU oracle (test
    infrastructure, never the measured path) against one fresh device step.
    Every rank regenerates its shard's inputs, computes its oracle partial
    sum of squares, and the partials are all-gathered in rank order; each
    rank then compares windows of its shard (ends, middle, weight-decay and
    tensor boundaries) bit for bit with the oracle driven by the oracle's
    own global sum, and the replicated state across ranks."""
    import torch
    import torch.distributed as dist

    from ark_b200 import synth
    from oracle import oracle
    t0 = time.perf_counter()
    oracle.build()
    cores = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
    local_world = int(os.environ.get("LOCAL_WORLD_SIZE", world))
    oracle.lib().ork_set_threads(max(1, cores // max(local_world, 1)))
    lo, hi, n = opt.lo, opt.hi, opt.n
    # fresh inputs in the same buffers (the timed steps have moved w, m, v)
    synth.fill_f16(w16, lo, SEED, synth.STREAM_W, 0.02)
    synth.fill_grads(g16, lo, SEED, LOSS_SCALE, heavy=heavy)
    synth.fill_f32(m, lo, SEED, synth.STREAM_M, 1e-4)
    synth.fill_f32(v, lo, SEED, synth.STREAM_V, 1e-3, square=True)
    opt.set_status(opt_step=START_STEP - 1, loss_scale=LOSS_SCALE, clean_steps=0,
                   consecutive_nans=0, last_overflow=0, early_stop=0, error=0,
                   skipped_steps=0)
    g_host = oracle.synth_f16(n, lo, SEED, synth.STREAM_G, 1e-3, LOSS_SCALE,
                              synth.HEAVY_EVERY if heavy else 0,
                              synth.HEAVY_MULT if heavy else 1.0)
    cfg = oracle.make_cfg(n_decay=L.n_decay, scale_every=2000, scale_max=2.0 ** 24,
                          **{k: EKO_HPARAMS[k] for k in ("beta1", "beta2", "eps",
                                                         "weight_decay", "grad_clip")})
    sumsq, bad = oracle.partial_f16(cfg, oracle.make_state(LOSS_SCALE, START_STEP - 1), g_host,
                                    lo)
    if world > 1:
        parts = [torch.zeros(2, dtype=torch.float64, device=dev) for _ in range(world)]
        dist.all_gather(parts, torch.tensor([sumsq, float(bad)], dtype=torch.float64,
                                            device=dev))
        parts = [p.tolist() for p in parts]
    else:
        parts = [[sumsq, float(bad)]]
    g_sum = 0.0
    g_bad = 0
    for s_r, b_r in parts:                       # rank order
        g_sum += s_r
        g_bad += int(b_r)
    barrier()
    opt.step_all(w16, g16, m, v)
    st = opt.status()
    ok = g_bad == 0 and st["last_overflow"] == 0 and st["opt_step"] == START_STEP
    norm = np.float32(np.sqrt(g_sum))
    norm_err = abs(st["last_norm"] - float(norm)) / float(norm)
    sumsq_err = abs(st["last_sumsq"] - g_sum) / g_sum
    ok = ok and norm_err <= 1e-5 and sumsq_err <= 1e-12
    wins = _windows_of_shard(L, lo, hi)
    elems = 0
    for a, b in wins:
        w = oracle.synth_f16(b - a, a, SEED, synth.STREAM_W, 0.02)
        mm = oracle.synth_f32(b - a, a, SEED, synth.STREAM_M, 1e-4)
        vv = oracle.synth_f32(b - a, a, SEED, synth.STREAM_V, 1e-3, square=True)
        oracle.apply_f16(cfg, oracle.make_state(LOSS_SCALE, START_STEP - 1), w,
                         np.ascontiguousarray(g_host[a - lo:b - lo]), mm, vv, a, g_sum, g_bad)
        ok = ok and np.array_equal(g16[a - lo:b - lo].cpu().numpy().view(np.uint16),
                                   g_host[a - lo:b - lo])     # same generator on both sides
        ok = ok and np.array_equal(w16[a - lo:b - lo].cpu().numpy().view(np.uint16), w)
        ok = ok and np.array_equal(m[a - lo:b - lo].cpu().numpy().view(np.uint32),
                                   mm.view(np.uint32))
        ok = ok and np.array_equal(v[a - lo:b - lo].cpu().numpy().view(np.uint32),
                                   vv.view(np.uint32))
        elems += b - a
    # replicated state: every rank's 64-byte status identical
    keys = sorted(st)
    mine = torch.tensor([float(st[k]) for k in keys], dtype=torch.float64, device=dev)
    if world > 1:
        lo_t, hi_t = mine.clone(), mine.clone()
        dist.all_reduce(lo_t, op=dist.ReduceOp.MIN)
        dist.all_reduce(hi_t, op=dist.ReduceOp.MAX)
        same = bool(torch.equal(lo_t, hi_t))
        counts = torch.tensor([1.0 if ok else 0.0, float(len(wins)), float(elems)],
                              dtype=torch.float64, device=dev)
        okf = counts[:1].clone()
        dist.all_reduce(okf, op=dist.ReduceOp.MIN)
        dist.all_reduce(counts, op=dist.ReduceOp.SUM)
        ok_all = bool(okf.item() == 1.0)
        n_wins, n_elems = int(counts[1].item()), int(counts[2].item())
    else:
        same, ok_all, n_wins, n_elems = True, bool(ok), len(wins), elems
    return {"ok": bool(ok_all and same), "windows": n_wins, "elements": n_elems,
            "state_identical": same, "norm_rel_err": float(norm_err),
            "sumsq_rel_err": float(sumsq_err),
            "checker": "CPU oracle (oracle/ark_oracle.c) on every rank's shard after the timed "
                       "regions; one fresh device step; windows bit for bit",
            "leg_s": round(time.perf_counter() - t0, 2)}


def run_ours(args):
    import torch
    import torch.distributed as dist

    import ark_b200 as ab
    from ark_b200 import dist as adist
    from ark_b200 import layout, synth

    rank, world, local = adist.env_rank_world()
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    if args.params:
        L = layout.flat_layout(args.params)
        workload = f"flat buffer of {L.n} params (BASELINE configs[4])"
    else:
        L = layout.LAYOUTS[args.workload]()
        workload = {"eko": "EKO-237M full optimizer step (BASELINE configs[0])",
                    "1.3b": "1.3B decoder, ZeRO-1 sharded (BASELINE configs[2])",
                    "7b": "7B decoder, 1% of grads x100 so clipping is active, ZeRO-1 sharded "
                          "(BASELINE configs[3])"}[args.workload]
    heavy = args.workload == "7b" and not args.params
    comm = adist.nccl_comm(rank, world, local) if world > 1 else None
    adam = ab.AdamConfig(**EKO_HPARAMS)
    scale = ab.LossScaleConfig(init=LOSS_SCALE, every=2000, max=2.0 ** 24)
    stream = torch.cuda.current_stream(dev)
    opt = ab.Optimizer(L, adam, scale, device=local, rank=rank, world=world, comm=comm,
                       stream=stream, constant_lr=True, initial_step=START_STEP - 1,
                       use_graph=args.graph, nccl_exchange=args.nccl_exchange)
    lo, n = opt.lo, opt.n
    w16, g16, m, v = synth.make_state(n, lo, SEED, dev, loss_scale=LOSS_SCALE, heavy=heavy)
    if args.reduce:
        # gradient hand-off: each rank's full FP16 gradients (its own backward
        # output, scaled 1/world so the sum has the usual magnitude)
        full = opt.grad_buffer()
        synth.fill_grads(full, 0, SEED + 1 + rank, LOSS_SCALE / world, heavy=heavy)

        def do_step():
            opt.step_reduce(w16, g16, m, v)
    else:
        def do_step():
            opt.step_all(w16, g16, m, v)
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ---- timed region: K steps (the headline) ----
    # No event record between the kernels here: an event between pass 1 and
    # pass 2 would turn their programmatic dependency into a full one.  The
    # per-kernel split is timed in a second region of K steps right after,
    # with event-record nodes between the kernels.  A state below 4x the L2
    # is timed step by step instead, with the L2 flushed between steps.
    flush = {"auto": needs_flush(L.n, world), "flush": True, "none": False}[args.l2]
    # flush: write 256 MiB (evicts the L2), then read another 256 MiB, so that
    # the dirty flush lines are written back before the step, not during it
    scratch = torch.empty(FLUSH_BYTES // 4, dtype=torch.float32, device=dev) if flush else None
    scratch_r = torch.zeros(FLUSH_BYTES // 4, dtype=torch.float32, device=dev) if flush else None
    sink = torch.empty((), dtype=torch.float32, device=dev)
    tok = torch.zeros(1, dtype=torch.float32, device=dev)

    def flush_l2(k):
        scratch.fill_(float(k))
        torch.sum(scratch_r, dim=0, out=sink)
        if world > 1:
            # device-side barrier: every rank's stream passes this point
            # together, so no rank's step event includes waiting for a peer
            # that is still flushing
            dist.all_reduce(tok)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    step_evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                for _ in range(args.steps)] if flush else []
    sampled = list(range(world)) if rank == 0 else [local]
    with ClockSampler(nvidia_smi_ids(sampled)) as clocks:
        for _ in range(args.warmup):
            do_step()
        torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
        clocks.mark("t0")
        ev0.record(stream)
        for k in range(args.steps):
            if flush:
                flush_l2(k)
                step_evs[k][0].record(stream)
            do_step()
            if flush:
                step_evs[k][1].record(stream)
        ev1.record(stream)
        torch.cuda.synchronize()
        clocks.mark("t1")
        barrier()
        # ---- per-kernel region: K more steps with kernel events ----
        opt.profile_begin(args.steps)
        barrier()
        torch.cuda.synchronize()
        for k in range(args.steps):
            if flush:
                flush_l2(k)
            do_step()
        torch.cuda.synchronize()
        barrier()
    if flush:
        per_step = [a.elapsed_time(b) for a, b in step_evs]
        step_ms_local = float(np.mean(per_step))
    else:
        step_ms_local = ev0.elapsed_time(ev1) / args.steps
    prof = opt.profile_read(args.steps)
    # median / min per step: the flushed steps themselves, else the summed
    # kernel intervals of the per-kernel region
    per_step_src = per_step if flush else (prof.sum(axis=1).tolist() if len(prof) else [])
    step_stats = {"median_ms": round(float(np.median(per_step_src)), 4),
                  "min_ms": round(float(np.min(per_step_src)), 4),
                  "source": "per-step events around each flushed step" if flush else
                            "pass 1 + exchange + pass 2 event intervals per step, "
                            "per-kernel region"} if per_step_src else None
    step_ms = max_over_ranks(step_ms_local)
    st = opt.status()
    assert st["last_overflow"] == 0 and st["opt_step"] == START_STEP - 1 + args.warmup + 2 * args.steps
    e2e_steps = min(args.steps, 50)

    # ---- e2e: host grads -> device, step, status back, every step ----
    # the pinned host buffer is first touched by this process bound to the
    # GPU's NUMA node, so its pages sit on the node nearest the GPU
    cpus = numa_local_cpus(local) if hasattr(os, "sched_setaffinity") else None
    prev_aff = os.sched_getaffinity(0) if cpus else None
    if cpus and (cpus & prev_aff):
        os.sched_setaffinity(0, cpus & prev_aff)
    g_host = torch.empty(n, dtype=torch.float16, pin_memory=True)
    g_host.copy_(g16.cpu())
    if prev_aff:
        os.sched_setaffinity(0, prev_aff)
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    marks = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(e2e_steps)]
    e0.record(stream)
    for k in range(e2e_steps):
        marks[k][0].record(stream)
        opt.upload_grads(g16, g_host)
        marks[k][1].record(stream)
        opt.step_all(w16, g16, m, v)
        marks[k][2].record(stream)
        opt.status()
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / e2e_steps)
    e2e_h2d_ms = max_over_ranks(float(np.mean([a.elapsed_time(b) for a, b, _ in marks])))
    e2e_step_ms = max_over_ranks(float(np.mean([b.elapsed_time(c) for _, b, c in marks])))
    # the host->device ceiling: the same pinned copy alone, every rank at once
    h2d_alone_ms = timed_loop(lambda: opt.upload_grads(g16, g_host), min(e2e_steps, 20), stream,
                              barrier, max_over_ranks)
    e2e_split = {"h2d_ms": round(e2e_h2d_ms, 4), "step_ms": round(e2e_step_ms, 4),
                 "h2d_alone_ms": round(h2d_alone_ms, 4),
                 "h2d_aggregate_gbs": round(2 * L.n / (e2e_h2d_ms * 1e-3) / 1e9, 1),
                 "h2d_alone_aggregate_gbs": round(2 * L.n / (h2d_alone_ms * 1e-3) / 1e9, 1),
                 "pinned_numa_local": bool(cpus and (cpus & (prev_aff or set()))),
                 "note": "events around the upload and around the step of each e2e step; "
                         "the rest of e2e ms is the status read-back and host latency"}

    # ---- roofline of the dominant kernel (pass 2) ----
    peak, peak_src = measured_peak()
    roof = None
    if prof is not None and len(prof):
        p1 = float(np.mean(prof[:, 0]))
        ex = float(np.mean(prof[:, 1]))
        p2 = float(np.mean(prof[:, 2]))
        p2_max = max_over_ranks(p2)
        achieved = PASS2_BYTES_PER_PARAM * n / (p2 * 1e-3) / 1e9
        tpp = PASS2_DRAM_BYTES_PER_PARAM
        roof = {"kernel": "ark::pass2_kernel (fused unscale+clip+AdamW)", "bound": "hbm",
                "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4), "peak_source": peak_src,
                "traffic": round(tpp * n) if tpp else None,
                "algorithmic_bytes_per_launch": PASS2_BYTES_PER_PARAM * n,
                "pass2_ms": round(p2, 4), "pass2_ms_max_rank": round(p2_max, 4),
                "pass1_ms": round(p1, 4),
                "pass1_gbs": round(PASS1_BYTES_PER_PARAM * n / (p1 * 1e-3) / 1e9, 1),
                "exchange_ms": round(ex, 4), "launches_per_step": 2,
                "per_kernel_region": "K further steps with event-record nodes between the "
                                     "kernels (pass 2 then waits for pass 1 in full)",
                "kernels_ms_sum": round(p1 + ex + p2, 4)}
        if args.reduce:
            # pass 1 here is the reduce-scatter fused with the norm/flag pass:
            # every rank reads (world - 1) remote shards over NVLink
            roof["pass1_kernel"] = "ark::pass1_reduce_kernel (reduce-scatter over NVLink + norm/flag)"
            roof["nvlink_bytes_in_per_gpu"] = 2 * n * (world - 1)
            roof["nvlink_gbs_in_per_gpu"] = round(2 * n * (world - 1) / (p1 * 1e-3) / 1e9, 1)
            roof["nvlink_peer_copy_gbs_measured"] = NVLINK_PEER_COPY_GBS
    clk = clocks.summary()
    geom = opt.geometry()

    aux = measure_aux(opt, L, w16, g16, m, v, stream, args, max_over_ranks, barrier) \
        if args.aux else None
    allgather = None
    if world > 1 and not args.no_allgather:
        allgather = measure_allgather(opt, L, w16, g16, m, v, stream, args, max_over_ranks,
                                      barrier)
    legacy = None
    if world == 1 and not args.no_legacy and not args.params and args.workload == "eko":
        legacy = measure_legacy(L, stream, args)
    parity = None
    if not args.no_parity:
        parity = parity_leg(opt, L, w16, g16, m, v, heavy, world, rank, dev, barrier)

    cpu = None
    if (rank == 0 and world == 1 and not args.no_cpu_baseline and not args.params
            and args.workload == "eko"):
        cpu = cpu_baseline_single_thread(L)

    if rank == 0:
        value = BYTES_PER_PARAM * L.n / (step_ms * 1e-3) / 1e9
        e2e_val = BYTES_PER_PARAM * L.n / (e2e_ms * 1e-3) / 1e9
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(step_ms, 4),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded splitmix64 + Irwin-Hall normals with the BASELINE "
                    "distributions, generated on the device)",
            "config": {"workload": workload + (" + gradient hand-off (reduce-scatter over NVLink "
                                               "fused with pass 1)" if args.reduce else ""),
                       "params": L.n, "params_per_gpu": n, "tensors": L.n_tensors,
                       "parallelism": f"zero1-dp{world}", "t": START_STEP,
                       "loss_scale": LOSS_SCALE, "clip": "active",
                       "bytes_per_param": BYTES_PER_PARAM, "graph": bool(args.graph),
                       "exchange": ("none" if world == 1 else
                                    "nccl all-gather" if args.nccl_exchange else
                                    "p2p stores from pass 1 (nccl if unmappable)"),
                       "l2": ("L2 flushed between steps (256 MiB written, then another "
                              "256 MiB read so the dirty lines are written back first; both "
                              "outside the per-step events; state %.3f GB/GPU, mode %s)"
                              if flush else
                              "no flush between steps (state %.2f GB/GPU vs 126 MB L2, mode %s)")
                             % (n * STATE_BYTES_PER_PARAM / 1e9, args.l2),
                       "geometry": geom},
            "roofline": roof,
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e_val, 2), "unit": "GB/s", "ms_per_step": round(e2e_ms, 3),
                    "h2d_bytes_per_step": 2 * L.n, "d2h_bytes_per_step": 64 * world,
                    "steps": e2e_steps, "split": e2e_split,
                    "path": "Optimizer.upload_grads (pinned host fp16 grads) + step_all + "
                            "status() per step, through the C ABI"},
            "parity": parity,
            "allgather": allgather,
            "legacy": legacy,
            "step_stats": step_stats,
            "gpu_launches": 2 * args.steps,
            "aux": aux,
            "clocks": clk,
        }
        print(json.dumps(line), flush=True)
    opt.close()
    if comm:
        adist.nccl_comm_destroy(comm)
    if world > 1:
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--params", type=int, default=0,
                    help="flat-buffer workload of this many params instead of EKO-237M")
    ap.add_argument("--aux", action="store_true",
                    help="also time the FP32-weight-copy step and ARK4 checkpoint save/load")
    ap.add_argument("--ckpt-dir", default="",
                    help="directory for the --aux checkpoint files (default: none)")
    ap.add_argument("--reduce", action="store_true",
                    help="include the gradient hand-off: reduce-scatter of every rank's full "
                         "FP16 gradients over NVLink, fused with pass 1")
    ap.add_argument("--workload", choices=("eko", "1.3b", "7b"), default="eko",
                    help="model layout (BASELINE configs 0, 2, 3); the headline is eko")
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--no-graph", dest="graph", action="store_false",
                    help="launch the kernels directly instead of replaying a CUDA graph")
    ap.add_argument("--nccl-exchange", action="store_true",
                    help="N > 1: exchange the partials with NCCL instead of peer-to-peer stores")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-parity", action="store_true",
                    help="skip the oracle parity leg after the timed regions")
    ap.add_argument("--no-allgather", action="store_true",
                    help="N > 1: skip timing the FP16 weight all-gather (NCCL and fused)")
    ap.add_argument("--no-legacy", action="store_true",
                    help="N = 1: skip timing the legacy per-tensor entry points")
    ap.add_argument("--l2", choices=("auto", "flush", "none"), default="auto",
                    help="L2 handling between timed steps: flush below 4x L2 of state (auto), "
                         "always, or never")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
