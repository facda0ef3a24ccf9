#!/usr/bin/env python
"""Benchmark of the fused token sampler (one JSON line on rank 0).

Workload (configs[1] of the baseline): B=128 rows, V=151936, fp16 logits
N(0, 2.5^2) with 3% of ids per row shifted +6, four row groups (greedy,
top-k only, top-p only, temperature + top-k + top-p); seeded synthetic data.
A step is one sampler launch over the whole batch.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl native|reference]

native: K launches, replayed from CUDA graphs as a graph-captured decode step
launches them, timed with CUDA events on the replaying stream; inputs rotate
through enough device copies to hold 3x the 126 MB L2 (11 at C2, 408 MiB) so
every launch reads its logits from HBM.  ``e2e`` repeats the step through the public API with
the logits in pinned host memory: H2D copy, launch, D2H of the ids.
reference: the reference's CPU sampling path (torch port, all host threads).
flashinfer: the reference's own GPU step (torch divides by the gathered
mask_penalty rows and the temperature, then FlashInfer's
top_k_top_p_sampling_from_logits), timed the same way, for comparison.
Under torchrun each rank samples its own batch (batch-sharded, no collective);
time is the max over ranks.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "fused-sampler rows/sec & HBM GB/s at B=128,V=151936 fp16; µs/decode-step"
L2_BYTES = 126 * 1024 * 1024


def _peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def _traffic(workload):
    """DRAM bytes per launch from the committed ncu capture summary, if any."""
    p = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d.get(workload)
    return None


class ClockSampler:
    """Polls SM clock and clock-event reasons through NVML while running."""

    def __init__(self, index: int, period: float = 0.002):
        self.index, self.period = index, period
        self.samples, self.reasons = [], set()
        self.max_mhz = None
        self._stop = threading.Event()
        self._t = None

    def __enter__(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(self.index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self._nv = None
            return self
        names = {
            "hw_slowdown": getattr(self._nv, "nvmlClocksEventReasonHwSlowdown", 0x8),
            "hw_thermal_slowdown": getattr(self._nv, "nvmlClocksEventReasonHwThermalSlowdown", 0x40),
            "sw_thermal_slowdown": getattr(self._nv, "nvmlClocksEventReasonSwThermalSlowdown", 0x20),
            "sw_power_cap": getattr(self._nv, "nvmlClocksEventReasonSwPowerCap", 0x4),
            "hw_power_brake": getattr(self._nv, "nvmlClocksEventReasonHwPowerBrakeSlowdown", 0x80),
        }

        def run():
            while not self._stop.is_set():
                try:
                    self.samples.append(self._nv.nvmlDeviceGetClockInfo(self._h, self._nv.NVML_CLOCK_SM))
                    mask = self._nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                    for k, bit in names.items():
                        if mask & bit:
                            self.reasons.add(k)
                except Exception:
                    pass
                time.sleep(self.period)

        self._t = threading.Thread(target=run, daemon=True)
        self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._t is not None:
            self._t.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons),
                    "samples": 0}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


def _dist():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def _cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for ln in f:
                if ln.startswith("model name"):
                    return ln.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform
    return platform.processor() or "unknown"


def _all_cores():
    """Give torch every host core (torchrun sets OMP_NUM_THREADS=1 per rank)."""
    n = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
    torch.set_num_threads(n)
    return n


def cpu_reference_step(w):
    """One full step of the torch-CPU port of the reference path over every
    row of the workload, on all host cores; returns (rows, threads, step)."""
    from oracle.torch_port import sample_batch_torch
    threads = _all_cores()
    args = (w.logits, w.temperature, w.top_k, w.top_p, w.uniforms)
    return w.batch, threads, lambda: sample_batch_torch(*args)


def reference_logits_to_probs_c1(budget_s: float = 10.0):
    """The reference's own CPU sampler, ecahlang.utils.logits_to_probs
    (ecahlang/utils.py:3-18), run as-is on configs[0] (B=8, V=151936 fp32,
    T 0.7, k 50; it has no top-p stage) from the installed copy of the
    reference in baseline/_ref.  Returns a dict for the JSON line."""
    ref = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref, "ecahlang")):
        return {"unavailable": "baseline/_ref holds no installed reference"}
    if ref not in sys.path:
        sys.path.append(ref)
    from ecahlang.utils import logits_to_probs
    from ecahlang_b200 import workloads as W
    threads = _all_cores()
    w = W.config1(seed=0)
    B = w.batch
    mask = torch.ones_like(w.logits)
    T = w.temperature.reshape(B, 1)
    K = w.top_k.long()
    P = w.top_p
    with torch.no_grad():
        logits_to_probs(w.logits, mask, T, K, P)
        n, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < budget_s:
            logits_to_probs(w.logits, mask, T, K, P)
            n += 1
        dt = time.perf_counter() - t0
    return {"value": B * n / dt, "unit": "rows/s", "ms_per_call": 1e3 * dt / n, "calls": n, "cores": threads,
            "cpu_model": _cpu_model(),
            "workload": "configs[0]: B=8, V=151936 fp32 N(0,3^2) + 5 spikes at +12, T 0.7, k 50 "
                        "(logits_to_probs has no top-p)",
            "kind": "reference", "source": "ecahlang.utils.logits_to_probs from baseline/_ref, unmodified"}


def run_reference(a):
    ws, rank, _ = _dist()
    if rank != 0:
        return
    from ecahlang_b200 import workloads as W
    w = W.config2(seed=0)
    rows, threads, step = cpu_reference_step(w)
    t0 = time.perf_counter()
    step()
    t1 = time.perf_counter() - t0
    # every step is the whole 128-row batch; the number of timed steps is
    # capped so the run stays near two minutes of CPU work
    steps = max(1, min(a.steps, int(90.0 / max(t1, 1e-3))))
    warm = max(1, min(a.warmup, int(15.0 / max(t1, 1e-3))))
    for _ in range(warm):
        step()
    t0 = time.perf_counter()
    for _ in range(steps):
        step()
    dt = time.perf_counter() - t0
    rps = rows * steps / dt
    sample = (f"all {rows} rows of the workload per step; {steps} timed steps of the {a.steps} requested "
              f"(capped to about 90 s of CPU time), {warm} warm-up steps")
    line = {
        "impl": "reference", "metric": METRIC, "value": rps, "unit": "rows/s", "n_gpus": a.gpus,
        "steps": steps, "steps_requested": a.steps, "warmup": warm, "ms_per_step": 1e3 * dt / steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
        "data": "synthetic",
        "config": {"workload": "c2_mixed B=128 V=151936 fp16 (configs[1])", "batch": 128, "vocab": 151936,
                   "parallelism": "cpu"},
        "cpu_baseline": {"value": rps, "unit": "rows/s", "cores": threads, "cpu_model": _cpu_model(),
                         "kind": "port", "sample": sample},
        "e2e": {"value": rps, "unit": "rows/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "reference_logits_to_probs_c1": reference_logits_to_probs_c1(),
    }
    print(json.dumps(line), flush=True)


def run_native(a):
    ws, rank, local = _dist()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if ws > 1:
        import datetime
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=60),
                                             device_id=dev)
    from ecahlang_b200 import sampler as S
    from ecahlang_b200 import workloads as W

    w = W.config2(seed=rank)
    B, V = w.batch, w.vocab
    bytes_in = w.logits.numel() * w.logits.element_size()
    nbuf = max(2, -(-3 * L2_BYTES // bytes_in))
    bufs = [w.logits.to(dev) for _ in range(nbuf)]
    T, K, P = w.temperature.to(dev), w.top_k.to(dev), w.top_p.to(dev)
    smp = S.Sampler(B, V, w.logits.dtype, dev, seed=1234 + rank)
    stream = torch.cuda.current_stream(dev)

    def step(i):
        smp(bufs[i % nbuf], T, K, P)

    for i in range(a.warmup):
        step(i)
    torch.cuda.synchronize()
    # the timed steps run as CUDA-graph replays (how a graph-captured decode
    # step launches the sampler): `chunk` launches per graph on rotating
    # inputs, plus one graph for the remainder, exactly a.steps launches
    chunk = min(a.steps, 2 * nbuf)
    cap = torch.cuda.Stream(dev)
    cap.wait_stream(torch.cuda.current_stream(dev))

    def capture(n):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=cap):
            for i in range(n):
                step(i)
        return g

    g_full = capture(chunk)
    rem = a.steps % chunk
    g_rem = capture(rem) if rem else None
    g_full.replay()
    torch.cuda.synchronize()
    if ws > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        ev0.record(stream)
        for _ in range(a.steps // chunk):
            g_full.replay()
        if g_rem is not None:
            g_rem.replay()
        ev1.record(stream)
        torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1)
    if ws > 1:
        t = torch.tensor([ms], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        torch.distributed.barrier()
        ms = float(t.item())
    torch.cuda.synchronize()
    ms_step = ms / a.steps
    rows_total = B * ws * a.steps
    value = rows_total / (ms / 1e3)

    # ---- e2e through the drop-in API (SamplingManager, the reference manager's
    # methods): parameters through its pinned buffers, pinned host logits ->
    # device, sample, ids -> pinned host, every step
    from ecahlang_b200.manager import SamplingManager
    host = w.logits.pin_memory()
    dlog = torch.empty_like(bufs[0])
    mgr = SamplingManager(V, seq_lens=B, dtype=w.logits.dtype, device=dev, seed=4321 + rank)
    mgr.init_sampling_buffers(B)
    Tl, Kl, Pl = w.temperature.numpy(), w.top_k.numpy(), w.top_p.numpy()
    ids_host = torch.empty(B, dtype=torch.int32).pin_memory()
    ke = max(3, min(a.steps, 50))

    def e2e_step():
        mgr.fill_sampling_params(B, Tl, Kl, Pl)
        dlog.copy_(host, non_blocking=True)
        ids_host.copy_(mgr.sample(dlog), non_blocking=True)

    for _ in range(3):
        e2e_step()
    torch.cuda.synchronize()
    if ws > 1:
        torch.distributed.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(ke):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    ems = e0.elapsed_time(e1)
    if ws > 1:
        t = torch.tensor([ems], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ems = float(t.item())
    e2e_value = B * ws * ke / (ems / 1e3)
    h2d = bytes_in + 7 * 4 * B   # logits + the manager's seven parameter columns

    line = None
    if rank == 0:
        peak, peak_kind = _peaks()
        alg = w.algorithmic_bytes() + B * (4 + 4 + 4 + 4)   # logits + T/k/p + ids
        achieved = alg / (ms_step / 1e3) / 1e9
        line = {
            "metric": METRIC, "value": value, "unit": "rows/s", "n_gpus": ws, "steps": a.steps,
            "warmup": a.warmup, "ms_per_step": ms_step, "us_per_step": 1e3 * ms_step,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
            "data": "synthetic",
            "config": {"workload": "c2_mixed B=128 V=151936 fp16 (configs[1])", "batch_per_gpu": B,
                       "vocab": V, "l2": f"inputs rotate through {nbuf} device copies "
                       f"({nbuf * bytes_in / 2**20:.0f} MiB > 126 MiB L2)",
                       "parallelism": f"batch-sharded x{ws}" if ws > 1 else "single GPU",
                       "launch": f"CUDA-graph replays of {chunk} sampler launches"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "peak_kind": peak_kind,
                         "traffic": _traffic("c2_mixed"), "algorithmic_bytes_per_launch": alg},
            "e2e": {"value": e2e_value, "unit": "rows/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": B * 4, "ms_per_step": ems / ke, "steps": ke,
                    "api": "SamplingManager.fill_sampling_params + sample (pinned host buffers)",
                    "note": ("bound by the host-to-device copy of each rank's logits from pinned host memory "
                             f"({bytes_in / 1e6:.1f} MB per step and rank); at N > 1 the ranks copy at once and "
                             "share the host's memory and PCIe bandwidth, so the per-step time grows with N")},
            # one sampler kernel per step; no other kernels run in the timed region
            "gpu_launches": a.steps,
            "clocks": clk.summary(),
        }
        if ws == 1 and not a.no_cpu_baseline:
            rows, threads, cstep = cpu_reference_step(w)
            cstep()
            t0 = time.perf_counter()
            n = 0
            while time.perf_counter() - t0 < 15.0:
                cstep()
                n += 1
            dt = time.perf_counter() - t0
            line["cpu_baseline"] = {
                "value": rows * n / dt, "unit": "rows/s", "cores": threads, "cpu_model": _cpu_model(),
                "kind": "port",
                "sample": f"all {rows} rows of the workload, {n} steps in {dt:.1f} s "
                          f"(torch CPU port of the reference path, {threads} threads)",
                "reference_logits_to_probs_c1": reference_logits_to_probs_c1()}
    del g_full, g_rem
    # the other multi-GPU modes of configs[3] on the same ranks: the
    # vocab-parallel step (the one that moves data between GPUs: the fused
    # NVLink peer exchange) and the batch-sharded 8x batch
    extra = {}
    if not a.no_extra:
        ms_c4b, b_c4 = c4_batch_measure(a, ws, rank, local, dev, min(a.steps, 200))
        extra["batch_sharded_c4"] = {
            "workload": "configs[3] at 8x the batch: B=4096 V=128256 bf16 (k=64, p=0.9), split over the ranks",
            "rows_per_rank": b_c4, "us_per_step": 1e3 * ms_c4b, "rows_per_s": 4096 / (ms_c4b / 1e3),
            "scaling": "strong", "note": "row kernel per rank, no collective"}
        if ws > 1:
            vp = vp_measure(a, ws, rank, local, dev, "peer", min(a.steps, 1000))
            extra["vocab_parallel_c4"] = {
                "workload": "configs[3]: B=512 V=128256 bf16 split by vocabulary, fused NVLink peer exchange",
                "us_per_step": 1e3 * vp["ms_step"], "rows_per_s": vp["value"], "slice_per_rank": vp["loc"],
                "cand_cap": vp["cap"], "exchange": vp["how"], "wait_timeouts": vp["err"],
                "local_kernel_us": 1e3 * vp["ms_local"], "local_kernel_gbs": vp["roofline"]["achieved"],
                "local_kernel_frac": vp["roofline"]["frac"], "scaling": "strong"}
            vq = vp_measure(a, ws, rank, local, dev, "peer", min(a.steps, 200), no_top_k=True)
            extra["vocab_parallel_c4_no_top_k"] = {
                "workload": "configs[3] with top-k off (top_k=0, p=0.9, T=1): B=512 V=128256 bf16 split by "
                            "vocabulary; the rows take the exact distributed passes (5 slice passes, NCCL "
                            "all-gather / all-reduce between them)",
                "us_per_step": 1e3 * vq["ms_step"], "rows_per_s": vq["value"], "rows_refused": vq["rows_refused"],
                "scaling": "strong"}
        else:
            # the other single-GPU configs: configs[2] (penalised) and
            # configs[4] (what the sampler adds to a graph-captured decode step)
            us_rp, us_all, n3, _, _ = c3_measure(a, dev, min(a.steps, 400))
            extra["c3_penalised"] = {
                "workload": "configs[2]: B=128 V=151936 fp16, 384-token Zipf histories, T 0.8, top-p 0.95",
                "us_repetition_only": us_rp, "us_repetition_frequency_presence": us_all, "steps": n3}
            rows5, n5 = decode_measure(a, dev)
            extra["c5_decode_added_us"] = {
                "workload": "configs[4] shapes: LM head 2048 -> 151936 fp16 (random-init weights) in a CUDA graph, "
                            "with and without SamplingManager.sample + update_penalties (T 0.7, top-p 0.9, "
                            "repetition penalty 1.1); µs added per step by concurrency",
                "per_concurrency": {b: round(r["us_added"], 2) for b, r in rows5.items()},
                "us_head": {b: round(r["us_head"], 2) for b, r in rows5.items()}, "steps": n5}
    if ws > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    if line is not None:
        if extra:
            line["extra"] = extra
        print(json.dumps(line), flush=True)


def vp_measure(a, ws, rank, local, dev, exchange, steps, no_top_k=False):
    """configs[3] vocab-parallel step on an initialised process group (or
    one rank): B=512, V=128256 bf16 split by vocabulary; returns the timings
    (max over ranks) and the rank-0 summary fields.  no_top_k: every row
    with top-k off (top_k = 0, p = 0.9 kept), drawn by the distributed passes
    with NCCL collectives between them."""
    from ecahlang_b200 import workloads as W
    from ecahlang_b200.vocab_parallel import VocabParallelSampler, split_vocab
    w = W.config4(seed=0)
    B, V = w.batch, w.vocab
    off, loc = split_vocab(V, ws, rank)
    bytes_in = B * loc * 2
    nbuf = max(2, -(-3 * L2_BYTES // bytes_in))
    bufs = [w.logits[:, off:off + loc].contiguous().to(dev) for _ in range(nbuf)]
    T, K, P = w.temperature.to(dev), w.top_k.to(dev), w.top_p.to(dev)
    full = None
    if no_top_k:
        K = torch.zeros_like(K)
        full = torch.arange(B, dtype=torch.int32, device=dev)   # listed on the device: graph-capturable
    cap = min(256, 2048 // ws)
    peer = exchange == "peer" and ws > 1
    if peer:
        exch = "peer"
    elif ws > 1:
        exch = None   # NCCL all-gather
    else:
        exch = lambda c, n, ac, an: (ac[0].copy_(c), an[0].copy_(n))
    smp = VocabParallelSampler(B, V, ws, rank, torch.bfloat16, dev, seed=77, cand_cap=cap, exchange=exch)
    stream = torch.cuda.current_stream(dev)
    for i in range(a.warmup):
        smp(bufs[i % nbuf], T, K, P, full_rows=full)
    torch.cuda.synchronize()
    chunk = min(steps, 2 * nbuf)
    side = torch.cuda.Stream(dev)
    side.wait_stream(stream)

    def capture(n, fn):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=side):
            for i in range(n):
                fn(i)
        return g

    g_full = capture(chunk, lambda i: smp(bufs[i % nbuf], T, K, P, full_rows=full))
    rem = steps % chunk
    g_rem = capture(rem, lambda i: smp(bufs[i % nbuf], T, K, P, full_rows=full)) if rem else None
    g_full.replay()
    torch.cuda.synchronize()
    bad = int((smp.out[:B] < 0).sum().item())   # rows drawn by neither path
    if ws > 1:
        torch.distributed.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        e0.record(stream)
        for _ in range(steps // chunk):
            g_full.replay()
        if g_rem is not None:
            g_rem.replay()
        e1.record(stream)
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    err = smp.peer.error() if smp.peer is not None else 0
    # the local kernel alone (the step's HBM pass), on this rank
    g_loc = capture(chunk, lambda i: smp.local(bufs[i % nbuf], T, K, P))
    g_loc.replay()
    torch.cuda.synchronize()
    e0.record(stream)
    reps = max(1, min(20, steps // chunk))
    for _ in range(reps):
        g_loc.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    ms_local = e0.elapsed_time(e1) / (reps * chunk)
    if ws > 1:
        t = torch.tensor([ms, ms_local, float(err)], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms, ms_local, err = float(t[0].item()), float(t[1].item()), int(t[2].item())
        torch.distributed.barrier()
    del g_full, g_rem, g_loc
    smp.close()
    peak, peak_kind = _peaks()
    how = ("fused kernel, lists stored into every rank's buffer over NVLink (CUDA IPC)" if peer else
           "local kernel + NCCL all_gather + merge kernel" if ws > 1 else "local + merge kernels (1 rank)")
    ms_step = ms / steps
    achieved = bytes_in / (ms_local / 1e3) / 1e9
    return {
        "ms_step": ms_step, "value": B / (ms_step / 1e3), "B": B, "loc": loc, "cap": cap, "chunk": chunk,
        "rows_refused": bad,
        "nbuf": nbuf, "how": how, "err": err, "ms_local": ms_local, "peer": peer, "clocks": clk.summary(),
        "roofline": {"bound": "hbm", "kernel": "local step (vp_local_row_kernel)",
                     "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "peak_kind": peak_kind, "traffic": None, "algorithmic_bytes_per_launch": bytes_in,
                     "us_per_launch": 1e3 * ms_local},
    }


def run_vocab_parallel(a):
    """B=512, V=128256 bf16 split by vocabulary over the ranks; a
    step gives the same ids on every rank.  --exchange peer (default): one
    fused kernel per rank, lists stored straight into every rank's exchange
    buffer over NVLink; nccl: local kernel, NCCL all-gather, merge kernel.
    Steps are replayed from CUDA graphs; time = max over ranks of CUDA-event
    time; value = rows/s of the job."""
    ws, rank, local = _dist()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if ws > 1:
        import datetime
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
    r = vp_measure(a, ws, rank, local, dev, a.exchange, a.steps)
    if ws > 1:
        torch.distributed.destroy_process_group()
    if rank == 0:
        print(json.dumps({
            "metric": "vocab-parallel sampler rows/sec (configs[3]: B=512, V=128256 bf16, k=64, p=0.9)",
            "value": r["value"], "unit": "rows/s", "n_gpus": ws, "steps": a.steps, "warmup": a.warmup,
            "ms_per_step": r["ms_step"], "us_per_step": 1e3 * r["ms_step"], "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "c4_vocab_parallel B=512 V=128256 bf16", "slice_per_rank": r["loc"],
                       "cand_cap": r["cap"], "exchange": r["how"],
                       "launch": f"CUDA-graph replays of {r['chunk']} steps",
                       "l2": f"inputs rotate through {r['nbuf']} device copies"},
            "roofline": r["roofline"],
            "wait_timeouts": r["err"],
            "gpu_launches": a.steps * (1 if r["peer"] else 2),   # ours; NCCL and copy kernels not counted
            "clocks": r["clocks"],
        }), flush=True)


def c4_batch_measure(a, ws, rank, local, dev, steps):
    """configs[3]'s batch-sharded variant: the same rows at 8x the batch
    (B = 4096 of V = 128256 bf16, k=64, p=0.9, T=1), split over the ranks;
    each rank samples its 4096 / world rows with the row kernel, no
    collective.  Returns (ms per step, max over ranks; rows per rank)."""
    from ecahlang_b200 import sampler as S
    from ecahlang_b200 import workloads as W
    Bt = 4096
    b = Bt // ws
    w = W.config4(seed=rank, B=b)
    V = w.vocab
    bytes_in = b * V * 2
    nbuf = max(2, -(-3 * L2_BYTES // bytes_in))
    bufs = [w.logits.to(dev) for _ in range(nbuf)]
    T, K, P = w.temperature.to(dev), w.top_k.to(dev), w.top_p.to(dev)
    smp = S.Sampler(b, V, torch.bfloat16, dev, seed=99 + rank)
    for i in range(a.warmup):
        smp(bufs[i % nbuf], T, K, P)
    torch.cuda.synchronize()
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=side):
        for i in range(nbuf):
            smp(bufs[i], T, K, P)
    g.replay()
    torch.cuda.synchronize()
    if ws > 1:
        torch.distributed.barrier()
    reps = max(1, steps // nbuf)
    stream = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(reps):
        g.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / (reps * nbuf)
    if ws > 1:
        t = torch.tensor([ms], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
    del g
    return ms, b


def decode_measure(a, dev, concurrencies=(1, 8, 32, 128)):
    """What the sampling calls add to a CUDA-graph decode step at configs[4]
    shapes, per concurrency (see run_decode); returns the per-B rows and the
    replay count."""
    from ecahlang_b200.manager import SamplingManager
    H, V = 2048, 151936
    g = torch.Generator(device=dev).manual_seed(5)
    W = (torch.randn(V, H, device=dev, generator=g) * 0.02).to(torch.float16)
    stream = torch.cuda.current_stream(dev)
    side = torch.cuda.Stream(dev)
    per_graph = 10
    reps = max(3, min(50, a.steps // per_graph))
    rows = {}
    for B in concurrencies:
        h = torch.randn(B, H, device=dev, generator=g).to(torch.float16)
        logits = torch.empty(B, V, device=dev, dtype=torch.float16)
        # one request per row, each with a penalty slot (history capacity
        # for the 384 tokens configs[4] generates), parameters through the
        # bucket buffers
        mgr = SamplingManager(V, seq_lens=B, dtype=torch.float16, device=dev, history_capacity=512, seed=1)
        mgr.init_sampling_buffers(B)
        mgr.init_cuda_graph_buffers([B])
        reqs = [f"r{i}" for i in range(B)]
        for r in reqs:
            mgr.allocate(r)
        mgr.fill_cuda_graph_sampling_params(B, B, [0.7] * B, [V] * B, [0.9] * B, rep_pens=[1.1] * B,
                                            batch_ids=reqs)

        def head():
            torch.matmul(h, W.t(), out=logits)

        def step():
            head()
            ids = mgr.sample(logits, bucket_size=B)
            mgr.update_penalties(ids, bucket_size=B)

        for _ in range(a.warmup):
            step()
        torch.cuda.synchronize()
        side.wait_stream(stream)
        times = {}
        for name, fn in (("head", head), ("head+sampler", step)):
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr, stream=side):
                for _ in range(per_graph):
                    fn()
            gr.replay()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(reps):
                gr.replay()
            e1.record(stream)
            torch.cuda.synchronize()
            times[name] = 1e3 * e0.elapsed_time(e1) / (reps * per_graph)
            del gr
        rows[str(B)] = {"us_head": times["head"], "us_head_sampler": times["head+sampler"],
                        "us_added": times["head+sampler"] - times["head"]}
    return rows, reps * per_graph


def run_decode(a):
    """configs[4] shapes: what the sampler adds to a CUDA-graph decode step.
    Per concurrency B in {1, 8, 32, 128}: graph A = the LM head (fp16 GEMM,
    hidden 2048 -> V 151936, random-init weights N(0, 0.02^2) as the config's
    random-init model has, so the logits are nearly flat); graph B = the LM
    head, then the drop-in sampling calls on its logits, as decode_forward's
    graph would hold them: SamplingManager.sample (T 0.7, top_p 0.9, as the
    config, with the requests' repetition-penalty histories) and
    SamplingManager.update_penalties (ecahlang/main.py:159-171, :356-379,
    :691-694).  Added µs = B's replay time minus A's, CUDA events over graph
    replays.
    The 36 transformer layers before the head are not run: they do not touch
    the sampler's inputs, and the difference is what the sampler adds.  One
    GPU; other ranks exit."""
    ws, rank, local = _dist()
    if rank != 0:
        return
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    with ClockSampler(local) as clk:
        rows, n = decode_measure(a, dev)
    print(json.dumps({
        "metric": "µs the sampler adds to a CUDA-graph decode step (configs[4] shapes: LM head 2048 -> 151936 fp16)",
        "value": rows["128"]["us_added"], "unit": "us", "higher_is_better": False, "n_gpus": 1,
        "steps": n, "warmup": a.warmup, "dtype": "f16", "data": "synthetic",
        "config": {"workload": "c5 decode step: LM head GEMM (+ SamplingManager.sample + update_penalties), "
                               "random-init weights N(0, 0.02^2), T=0.7, top_p=0.9, repetition penalty 1.1 "
                               "with per-request histories", "launch": "CUDA-graph replays of 10 steps"},
        "per_concurrency": rows, "clocks": clk.summary(),
    }), flush=True)


def c3_measure(a, dev, steps):
    """configs[2] on one GPU: µs per launch with the repetition penalty alone
    and with frequency + presence penalties too (CUDA-graph replays over
    rotating input copies, CUDA events)."""
    from ecahlang_b200 import sampler as S
    from ecahlang_b200 import workloads as W
    w = W.config3(seed=0)
    B, V = w.batch, w.vocab
    bytes_in = B * V * 2
    nbuf = max(2, -(-3 * L2_BYTES // bytes_in))
    bufs = [w.logits.to(dev) for _ in range(nbuf)]
    T, K, P, U = w.temperature.to(dev), w.top_k.to(dev), w.top_p.to(dev), w.uniforms.to(dev)
    cap = max(len(t) for t, _ in w.history)
    pen = S.PenaltyState(B, cap, torch.float16, dev)
    for r, (t, c) in enumerate(w.history):
        pen.load(r, t, c, None)
    row_slot = torch.arange(B, dtype=torch.int32, device=dev)
    rf = torch.as_tensor(S.repetition_factor(w.rep_pen.numpy()), dtype=torch.float32).to(dev)
    fp, pp = w.freq_pen.to(dev), w.pres_pen.to(dev)
    wsb = S.new_workspace(B, V, torch.float16, dev)
    out = torch.zeros(B, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev)
    side = torch.cuda.Stream(dev)
    chunk = min(steps, 2 * nbuf)
    reps = max(1, steps // chunk)

    def timed(fn):
        for i in range(a.warmup):
            fn(i)
        torch.cuda.synchronize()
        side.wait_stream(stream)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=side):
            for i in range(chunk):
                fn(i)
        g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            g.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        del g
        return 1e3 * e0.elapsed_time(e1) / (reps * chunk)

    us_rp = timed(lambda i: S.launch(bufs[i % nbuf], T, K, P, out, wsb, uniforms=U, rep_factor=rf,
                                     penalty=pen, row_slot=row_slot))
    us_all = timed(lambda i: S.launch(bufs[i % nbuf], T, K, P, out, wsb, uniforms=U, rep_factor=rf,
                                      freq_pen=fp, pres_pen=pp, penalty=pen, row_slot=row_slot,
                                      freq_pres=True))
    return us_rp, us_all, reps * chunk, chunk, nbuf


def run_c3(a):
    """B=128, V=151936 fp16, Zipf histories, T 0.8, top-p 0.95.
    Two figures of one JSON object, both on the row kernel (a wide nucleus,
    so the dense top-p path): the repetition penalty alone, and repetition +
    frequency + presence penalties (the penalised logits stay fp16).  CUDA-
    graph replays over rotating input copies, CUDA events.  One GPU; other
    ranks exit."""
    ws, rank, local = _dist()
    if rank != 0:
        return
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    with ClockSampler(local) as clk:
        us_rp, us_all, n, chunk, nbuf = c3_measure(a, dev, a.steps)
    print(json.dumps({
        "metric": "penalised sampling step (configs[2]: B=128, V=151936 fp16, T 0.8, top-p 0.95)",
        "value": us_rp, "unit": "us", "higher_is_better": False, "n_gpus": 1, "steps": n,
        "warmup": a.warmup, "dtype": "f16", "data": "synthetic",
        "config": {"workload": "c3_penalised B=128 V=151936 fp16, 384-token Zipf histories",
                   "launch": f"CUDA-graph replays of {chunk} launches", "l2": f"{nbuf} rotating input copies"},
        "us_repetition_only": us_rp, "us_repetition_frequency_presence": us_all,
        "clocks": clk.summary(),
    }), flush=True)


def run_flashinfer(a):
    """The reference's own GPU sampling step on the C2 inputs, for comparison
    (ecahlang/main.py:481-491; the CUDA-graph path at :356-379 does the same
    work): gather the batch's rows of the dense mask_penalty table
    (manager.py:36, all ones here), divide the logits by them and by the
    temperature, then flashinfer.sampling.top_k_top_p_sampling_from_logits(
    ..., deterministic=True).  Timed like the native arm (CUDA-graph replays
    over rotating inputs, CUDA events); "kernel_only" times the FlashInfer
    call alone on pre-divided logits.  One GPU: other ranks exit at once."""
    ws, rank, local = _dist()
    if rank != 0:
        return
    import flashinfer
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    from ecahlang_b200 import workloads as W

    w = W.config2(seed=0)
    B, V = w.batch, w.vocab
    bytes_in = w.logits.numel() * w.logits.element_size()
    nbuf = max(2, -(-3 * L2_BYTES // bytes_in))
    bufs = [w.logits.to(dev) for _ in range(nbuf)]
    T, K, P = w.temperature.to(dev), w.top_k.to(dev), w.top_p.to(dev)
    mask_penalty = torch.ones(B, V, dtype=w.logits.dtype, device=dev)
    slots = torch.arange(B, device=dev)
    Tcol = T[:, None].to(w.logits.dtype)

    def full(i):
        y = bufs[i % nbuf] / mask_penalty.index_select(0, slots)
        y = y / Tcol
        return flashinfer.sampling.top_k_top_p_sampling_from_logits(y, top_k=K, top_p=P, deterministic=True)

    def kernel_only(i):
        return flashinfer.sampling.top_k_top_p_sampling_from_logits(bufs[i % nbuf], top_k=K, top_p=P,
                                                                     deterministic=True)

    stream = torch.cuda.current_stream(dev)

    def timed(fn):
        for i in range(a.warmup):
            fn(i)
        torch.cuda.synchronize()
        chunk = min(a.steps, 2 * nbuf)
        how = "CUDA-graph replays"
        try:
            cap = torch.cuda.Stream(dev)
            cap.wait_stream(stream)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=cap):
                for i in range(chunk):
                    fn(i)
            g.replay()
            torch.cuda.synchronize()
        except Exception as e:   # capture not supported: time eager launches queued back to back
            g, how = None, f"eager launches ({type(e).__name__} under graph capture)"
            torch.cuda.synchronize()
        n = (a.steps // chunk) * chunk if g is not None else a.steps
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        if g is not None:
            for _ in range(n // chunk):
                g.replay()
        else:
            for i in range(n):
                fn(i)
        e1.record(stream)
        torch.cuda.synchronize()
        del g
        return e0.elapsed_time(e1) / n, n, how

    ms_full, n_full, how_full = timed(full)
    ms_k, n_k, how_k = timed(kernel_only)
    peak, peak_kind = _peaks()
    alg = w.algorithmic_bytes() + B * (4 + 4 + 4 + 4)
    print(json.dumps({
        "impl": "flashinfer", "metric": METRIC, "value": B / (ms_full / 1e3), "unit": "rows/s", "n_gpus": 1,
        "steps": n_full, "warmup": a.warmup, "ms_per_step": ms_full, "us_per_step": 1e3 * ms_full,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
        "config": {"workload": "c2_mixed B=128 V=151936 fp16 (configs[1])", "batch_per_gpu": B, "vocab": V,
                   "l2": f"inputs rotate through {nbuf} device copies ({nbuf * bytes_in / 2**20:.0f} MiB > 126 MiB L2)",
                   "path": "mask_penalty row gather, / mask_penalty, / temperature, "
                           f"flashinfer {flashinfer.__version__} top_k_top_p_sampling_from_logits(deterministic=True)",
                   "launch": how_full},
        "roofline": {"bound": "hbm", "achieved": alg / (ms_full / 1e3) / 1e9, "peak": peak, "unit": "GB/s",
                     "frac": alg / (ms_full / 1e3) / 1e9 / peak, "peak_kind": peak_kind},
        "kernel_only": {"us_per_step": 1e3 * ms_k, "value": B / (ms_k / 1e3), "unit": "rows/s", "steps": n_k,
                        "launch": how_k, "achieved_gbs": alg / (ms_k / 1e3) / 1e9},
    }), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["native", "reference", "flashinfer"], default="native",
                    help="reference: the CPU port of the reference path; flashinfer: the reference's "
                         "own GPU path (torch divides + FlashInfer sampling), for comparison")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extra", action="store_true", help="batch mode: skip the configs[3] lines")
    ap.add_argument("--mode", choices=["batch", "vp", "decode", "c3"], default="batch",
                    help="batch: configs[1], rows sharded over the ranks; vp: configs[3], vocabulary split; "
                         "decode: configs[4], µs the sampler adds to a graph-captured decode step; "
                         "c3: configs[2], the penalised step")
    ap.add_argument("--exchange", choices=["peer", "nccl"], default="peer",
                    help="vp mode: fused kernel over NVLink peer memory, or NCCL all-gather between kernels")
    a = ap.parse_args()
    a.warmup = max(3, a.warmup)
    if a.impl == "reference":
        run_reference(a)
    elif a.impl == "flashinfer":
        run_flashinfer(a)
    elif a.mode == "vp":
        run_vocab_parallel(a)
    elif a.mode == "decode":
        run_decode(a)
    elif a.mode == "c3":
        run_c3(a)
    else:
        run_native(a)


if __name__ == "__main__":
    main()
