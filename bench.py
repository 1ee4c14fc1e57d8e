#!/usr/bin/env python
"""Benchmark of the B200 token sampler (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

N=1 runs configuration 3 (batch 256 x vocab 151,936 bf16, all penalties, top-k 20, top-p 0.8,
temperature 0.7): the north-star workload. N>1 (one process per GPU under torchrun, NCCL) runs
configuration 4 vocab-sharded: batch 1,024 x vocab 248,320 bf16 split evenly over the ranks,
local top-k 50 records, one all-gather, a merge on every rank. A step is one pass of the
sampler over one batch. Inputs are seeded synthetic logits resident in HBM; four rotating
logits buffers (more than 2x the 126 MB L2 in total) make every step read from HBM.

``value`` is rows/s for the whole job (device time, max over ranks). ``e2e`` is the same
metric through the public API with host (pinned) inputs copied in and the ids copied out in
every step. ``roofline`` relates the sampler kernel's algorithmic bytes to its CUDA-event
duration and the measured HBM copy bandwidth. ``cpu_baseline`` times vinfer's own sampler
restated in PyTorch (``oracle/reference_port.py``) on this host's cores over a bounded sample.
``--impl reference`` times only that CPU sampler, with the same metric and config.
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
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
L2_BYTES = 126 * 1024 * 1024
METRIC = "sampled rows/sec (logits HBM GB/s as % of B200 peak in roofline)"
CONFIG3_WORKLOAD = ("config3: batch 256 x vocab 151936 bf16, rep 1.1 / pres 0.5 / freq 0.3 over "
                    "4096-token Zipf(1.1) histories, temp 0.7, top-k 20, top-p 0.8")


def config4_workload(world: int) -> str:
    return ("config4: batch 1024 x vocab 248320 bf16 N(0,3) + 4 spikes, vocab-sharded over "
            f"{world} GPUs, local top-k 50 records, NCCL all-gather, merge on every rank, temp 1, "
            "top-k 50, top-p 0.9")


def workload_config(world: int, hist_nnz: int | None = None) -> dict:
    """The ``config`` object of a line: the workload alone (what both arms measure, so the two
    arms' objects are equal); how each arm measures it goes under ``method``."""
    if world == 1:
        return {"workload": CONFIG3_WORKLOAD, "batch": 256, "vocab": 151_936,
                "hist_nnz": hist_nnz}
    return {"workload": config4_workload(world), "batch": 1024, "vocab": 248_320}


SMI_FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")


# ----------------------------------------------------------------------------------------------
# helpers
# ----------------------------------------------------------------------------------------------
def dist_env() -> tuple[int, int, int]:
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)),
            int(os.environ.get("LOCAL_RANK", 0)))


class Clocks:
    """nvidia-smi sampling of SM clocks and throttle reasons around the timed region."""

    def __init__(self, gpu: int) -> None:
        self.gpu = gpu
        self.proc = None
        self.path = Path(tempfile.mkstemp(prefix="clocks", suffix=".csv")[1])

    def start(self) -> None:
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={SMI_FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=self.path.open("w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        for line in self.path.read_text().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                rows.append((float(f[1]), float(f[2]), float(f[3]), f[4:]))
            except ValueError:
                continue
        self.path.unlink(missing_ok=True)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"], "samples": 0}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[3][1:]) if v == "Active"})
        return {"sm_mhz": statistics.median(r[0] for r in rows),
                "sm_max_mhz": max(r[1] for r in rows), "reasons": reasons,
                "samples": len(rows), "power_w_max": max(r[2] for r in rows)}


def measured_peak() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except (KeyError, ValueError):
            pass
    return 6650.0, "fallback"


def ncu_traffic(workload: str) -> float | None:
    """DRAM bytes per launch of the sampler kernel, from the committed ncu summary."""
    p = ROOT / "profiles" / "roofline_traffic.txt"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        parts = line.split()
        if len(parts) >= 2 and parts[0] == workload:
            try:
                return float(parts[1])
            except ValueError:
                return None
    return None


def cpu_reference_rows_per_s(w, seconds: float, rows_cap: int | None = None) -> dict:
    """vinfer's sampler (restated in torch, with the build's penalty/min-p extensions) on this
    host, one row per call as the runtime calls it; time-bounded sample of the workload."""
    sys.path.insert(0, str(ROOT))
    from oracle.reference_port import extended_sample  # noqa: PLC0415
    from oracle.sampler_oracle import RowParams as OracleParams  # noqa: PLC0415

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    done = 0
    t0 = time.perf_counter()
    r = 0
    while True:
        p = OracleParams(temperature=float(w.temperature[r]), top_k=int(w.top_k[r]),
                         top_p=float(w.top_p[r]), min_p=float(w.min_p[r]),
                         repetition_penalty=float(w.repetition_penalty[r]),
                         presence_penalty=float(w.presence_penalty[r]),
                         frequency_penalty=float(w.frequency_penalty[r]))
        ids = cnt = None
        if w.hist_row_ptr is not None:
            a, b = int(w.hist_row_ptr[r]), int(w.hist_row_ptr[r + 1])
            ids, cnt = w.hist_ids[a:b], w.hist_counts[a:b]
        extended_sample(w.logits[r], p, seed=r, position=done, hist_ids=ids, hist_counts=cnt)
        done += 1
        r = (r + 1) % w.batch
        el = time.perf_counter() - t0
        if (rows_cap is not None and done >= rows_cap) or (rows_cap is None and el >= seconds):
            break
    el = time.perf_counter() - t0
    return {"value": done / el, "unit": "rows/s", "cores": threads, "kind": "port",
            "sample": f"{done} rows of {w.name} (one sample() call per row) in {el:.1f} s"}


# ----------------------------------------------------------------------------------------------
# single GPU: configuration 3
# ----------------------------------------------------------------------------------------------
def bench_single(args) -> dict:
    from vinfer_b200 import SAMPLER, BackendContext  # noqa: PLC0415
    from vinfer_b200.sampling import RowParams, TokenHistogram  # noqa: PLC0415
    from vinfer_b200.workloads import make  # noqa: PLC0415

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    w = make(3)
    B, V = w.batch, w.vocab
    topp = args.workload == "topp"
    if topp:  # configuration 3's logits, top-p only: the rows the candidates cannot decide
        w.top_k = np.zeros(B, np.int32)
        w.top_p = np.full(B, 0.9, np.float32)
        w.repetition_penalty = np.ones(B, np.float32)
        w.presence_penalty = np.zeros(B, np.float32)
        w.frequency_penalty = np.zeros(B, np.float32)
    backend = SAMPLER.resolve("b200", BackendContext(dev, torch.bfloat16))
    nbuf = max(4, int(np.ceil(2 * L2_BYTES / (w.logits.numel() * 2))) + 1)
    base = w.logits.to(dev)
    bufs = [base] + [base.clone() for _ in range(nbuf - 1)]
    params = RowParams.from_arrays(dev, **w.param_arrays())
    u = torch.from_numpy(w.uniforms).to(dev)
    hist = TokenHistogram.from_csr(w.hist_row_ptr, w.hist_ids, w.hist_counts, dev)
    out = torch.empty(B, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev)

    def step(i: int) -> None:
        backend.sample_batch(bufs[i % nbuf], params, u, hist, out=out)

    for i in range(max(args.warmup, 3)):
        step(i)
    torch.cuda.synchronize()
    backend.check()

    # CUDA graph of G steps (host launch cost out of the timed region); K = q * G + rem
    K = args.steps
    G = min(K, 64)
    graphs = []
    for n in ([G] if K % G == 0 else [G, K % G]):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for i in range(n):
                step(i)
        graphs.append(g)
    torch.cuda.synchronize()
    plan = [graphs[0]] * (K // G) + ([graphs[1]] if K % G else [])

    # per-launch kernel durations: events around single launches with the queue backed up
    torch.cuda._sleep(50_000_000)
    pairs = []
    for i in range(32):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(stream)
        step(i)
        e.record(stream)
        pairs.append((s, e))
    torch.cuda.synchronize()
    kernel_ms = statistics.mean(s.elapsed_time(e) for s, e in pairs)

    clocks = Clocks(0)
    clocks.start()
    t_end = time.time() + 0.6  # identical load before the timed region, for the clock samples
    while time.time() < t_end:
        for g in graphs[:1]:
            g.replay()
        torch.cuda.synchronize()
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for g in plan:
        g.replay()
    t1.record(stream)
    torch.cuda.synchronize()
    total_ms = t0.elapsed_time(t1)
    t_end = time.time() + 0.4
    while time.time() < t_end:
        graphs[0].replay()
        torch.cuda.synchronize()
    clk = clocks.stop()
    backend.check()

    # the other single-GPU configurations, timed the same way (outside the headline's timed
    # region): 2 (the reference's default request shape among its rows), 5 (adversarial rows,
    # top-k up to 1,000) and 4 unsharded (the reference point of the vocab-sharded lines)
    other_configs = {}
    if not topp:
        for n, k_n in ((2, min(K, 400)), (5, min(K, 20))):
            other_configs[str(n)] = config_rows_per_s(n, dev, k_n)
        c4_rows = unsharded_config4_rows_per_s(backend_c4(dev), dev, min(K, 200))
        other_configs["4_unsharded"] = {"rows_per_s": c4_rows, "ms_per_step": 1024 / c4_rows * 1e3,
                                        "batch": 1024, "vocab": 248_320, "dtype": "bf16"}
        other_configs["3_decode"] = decode_rows_per_s(w, dev, min(K, 300))

    # end to end through the public API: host inputs in, ids out, every step
    e2e_steps = max(3, min(K, 20))
    host_logits = w.logits.pin_memory()
    host_params = {k: torch.from_numpy(np.ascontiguousarray(v)).pin_memory()
                   for k, v in w.param_arrays().items()}
    host_u = torch.from_numpy(w.uniforms).pin_memory()
    host_hist = [torch.from_numpy(np.ascontiguousarray(a)).pin_memory()
                 for a in (w.hist_row_ptr, w.hist_ids, w.hist_counts)]
    host_ids = torch.empty(B, dtype=torch.int32).pin_memory()
    d_logits = torch.empty_like(base)
    d_params = RowParams.from_arrays(dev, **w.param_arrays())
    d_u = torch.empty_like(u)
    d_hist = TokenHistogram(*(torch.empty_like(t, device=dev) for t in host_hist))
    h2d = (host_logits.numel() * host_logits.element_size() + host_u.numel() * 4
           + sum(t.numel() * t.element_size() for t in host_params.values())
           + sum(t.numel() * t.element_size() for t in host_hist))

    def e2e_step() -> None:
        d_logits.copy_(host_logits, non_blocking=True)
        for k, t in host_params.items():
            getattr(d_params, k).copy_(t, non_blocking=True)
        d_u.copy_(host_u, non_blocking=True)
        for dst, src in zip((d_hist.row_ptr, d_hist.ids, d_hist.counts), host_hist):
            dst.copy_(src, non_blocking=True)
        ids = backend.sample_batch(d_logits, d_params, d_u, d_hist, out=out)
        host_ids.copy_(ids, non_blocking=True)

    e2e_step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / e2e_steps
    backend.check()
    if not np.array_equal(host_ids.numpy(), out.cpu().numpy()):
        raise RuntimeError("e2e ids differ from the device result")

    peak, peak_kind = measured_peak()
    algo = w.algorithmic_bytes() if not topp else B * V * 2 + 36 * B  # no penalties: no history
    achieved = algo / (kernel_ms * 1e-3) / 1e9
    traffic = ncu_traffic("config3") if not topp else None
    cpu = (None if args.no_cpu_baseline or topp
           else cpu_reference_rows_per_s(w, args.cpu_seconds))
    ms_step = total_ms / K
    return {
        "metric": METRIC,
        "value": B * K / (total_ms * 1e-3),
        "unit": "rows/s",
        "n_gpus": 1,
        "steps": K,
        "warmup": args.warmup,
        "ms_per_step": ms_step,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded, configuration 3)",
        "config": workload_config(1, w.hist_nnz) if not topp else
                  {"workload": "config3 logits, top-p only: batch 256 x vocab 151936 bf16, "
                               "temp 0.7, top-k 0, top-p 0.9, no penalties (rows that need the "
                               "exact search)", "batch": B, "vocab": V, "hist_nnz": 0},
        "method": {"l2": f"{nbuf} rotating logits buffers "
                         f"({nbuf * w.logits.numel() * 2 / 2**20:.0f} MiB > 2x L2)",
                   "parallelism": "single GPU", "graph_steps": G},
        "gb_per_s": algo / (ms_step * 1e-3) / 1e9,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "peak_kind": f"{peak_kind} (copy bandwidth)",
                     "traffic": traffic, "algorithmic_bytes": algo,
                     "kernel": "k_stream<bf16> + k_finish<bf16> (one sample_batch)",
                     "kernel_ms": kernel_ms},
        "clocks": clk,
        "e2e": {"value": B / (e2e_ms * 1e-3), "unit": "rows/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": B * 4, "steps": e2e_steps},
        "gpu_launches": 2 * K,  # k_stream and k_finish per step
        "cpu_baseline": cpu,
        "configs": other_configs,
    }


# ----------------------------------------------------------------------------------------------
# single GPU, --workload config4: configuration 4 unsharded (the strong-scaling reference for the
# vocab-sharded runs; not the default line)
# ----------------------------------------------------------------------------------------------
def bench_single_config4(args) -> dict:
    from vinfer_b200 import SAMPLER, BackendContext  # noqa: PLC0415
    from vinfer_b200.workloads import config4_shard  # noqa: PLC0415

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    B, V = 1024, 248_320
    backend = SAMPLER.resolve("b200", BackendContext(dev, torch.bfloat16))
    x, params, u = config4_shard(0, 1, dev, B, V)
    nbytes = x.numel() * x.element_size()
    nbuf = max(2, int(np.ceil(2 * L2_BYTES / nbytes)) + 1)
    bufs = [x] + [x.clone() for _ in range(nbuf - 1)]
    out = torch.empty(B, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev)

    def step(i: int) -> None:
        backend.sample_batch(bufs[i % nbuf], params, u, None, out=out)

    for i in range(max(args.warmup, 3)):
        step(i)
    torch.cuda.synchronize()
    backend.check()
    torch.cuda._sleep(20_000_000)
    pairs = []
    for i in range(16):
        s_, e_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s_.record(stream)
        step(i)
        e_.record(stream)
        pairs.append((s_, e_))
    torch.cuda.synchronize()
    kernel_ms = statistics.mean(a.elapsed_time(b) for a, b in pairs)

    K = args.steps
    clocks = Clocks(0)
    clocks.start()
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for i in range(K):
        step(i)
    t1.record(stream)
    torch.cuda.synchronize()
    total_ms = t0.elapsed_time(t1)
    clk = clocks.stop()
    backend.check()

    # end to end: the logits, the row parameters and the uniforms from pinned host memory
    host_x = x.cpu().pin_memory()
    host_p = {k: getattr(params, k).cpu().pin_memory() for k in
              ("temperature", "top_k", "top_p", "min_p", "repetition_penalty",
               "presence_penalty", "frequency_penalty")}
    host_u = u.cpu().pin_memory()
    host_ids = torch.empty(B, dtype=torch.int32).pin_memory()
    d_x, d_u = torch.empty_like(x), torch.empty_like(u)
    h2d = (nbytes + host_u.numel() * 4 + sum(t.numel() * t.element_size()
                                              for t in host_p.values()))

    def e2e_step() -> None:
        d_x.copy_(host_x, non_blocking=True)
        for k, t in host_p.items():
            getattr(params, k).copy_(t, non_blocking=True)
        d_u.copy_(host_u, non_blocking=True)
        ids = backend.sample_batch(d_x, params, d_u, None, out=out)
        host_ids.copy_(ids, non_blocking=True)

    e2e_steps = max(3, min(K, 20))
    e2e_step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / e2e_steps
    backend.check()

    peak, kind = measured_peak()
    algo = B * V * 2 + 36 * B
    achieved = algo / (kernel_ms * 1e-3) / 1e9
    return {
        "metric": METRIC,
        "value": B * K / (total_ms * 1e-3),
        "unit": "rows/s",
        "n_gpus": 1,
        "steps": K,
        "warmup": args.warmup,
        "ms_per_step": total_ms / K,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded on the device, configuration 4 distribution)",
        "config": {"workload": "config4 unsharded: batch 1024 x vocab 248320 bf16 N(0,3) + 4 "
                               "spikes on one GPU, temp 1, top-k 50, top-p 0.9",
                   "batch": B, "vocab": V,
                   "l2": f"{nbuf} rotating logits buffers "
                         f"({nbuf * nbytes / 2**20:.0f} MiB > 2x L2)",
                   "parallelism": "single GPU"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "peak_kind": f"{kind} (copy bandwidth)",
                     "traffic": None, "algorithmic_bytes": algo,
                     "kernel": "k_stream<bf16> + k_finish<bf16> (one sample_batch)",
                     "kernel_ms": kernel_ms},
        "clocks": clk,
        "e2e": {"value": B / (e2e_ms * 1e-3), "unit": "rows/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": B * 4, "steps": e2e_steps},
        "gpu_launches": 2 * K,  # k_stream and k_finish per step
        "cpu_baseline": None,
    }


# ----------------------------------------------------------------------------------------------
# N > 1: configuration 4, vocab-sharded (one process per GPU, NCCL)
# ----------------------------------------------------------------------------------------------
def graphed(step, K: int):
    """CUDA graphs of G = min(K, 64) calls of ``step(i)`` (and of K % G); replaying ``plan`` in
    order runs K steps with no host launch cost."""
    G = min(K, 64)
    graphs = []
    for n in ([G] if K % G == 0 else [G, K % G]):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for i in range(n):
                step(i)
        graphs.append(g)
    torch.cuda.synchronize()
    return graphs, [graphs[0]] * (K // G) + ([graphs[1]] if K % G else []), G


def config_rows_per_s(n: int, dev, K: int) -> dict:
    """Configuration ``n`` (2 or 5) on this GPU through ``sample_batch`` in CUDA graphs, with
    rotating logits buffers (more than 2x L2 in total): rows/s and the device time per batch."""
    from vinfer_b200 import SAMPLER, BackendContext  # noqa: PLC0415
    from vinfer_b200.sampling import RowParams, TokenHistogram  # noqa: PLC0415
    from vinfer_b200.workloads import make  # noqa: PLC0415

    w = make(n)
    B = w.batch
    backend = SAMPLER.resolve("b200", BackendContext(dev, w.logits.dtype))
    base = w.logits.to(dev)
    nb = base.numel() * base.element_size()
    nbuf = max(2, int(np.ceil(2 * L2_BYTES / nb)) + 1)
    bufs = [base] + [base.clone() for _ in range(nbuf - 1)]
    params = RowParams.from_arrays(dev, **w.param_arrays())
    u = torch.from_numpy(w.uniforms).to(dev)
    hist = (TokenHistogram.from_csr(w.hist_row_ptr, w.hist_ids, w.hist_counts, dev)
            if w.hist_row_ptr is not None else None)
    out = torch.empty(B, dtype=torch.int32, device=dev)

    def step(i: int) -> None:
        backend.sample_batch(bufs[i % nbuf], params, u, hist, out=out)

    for i in range(3):
        step(i)
    torch.cuda.synchronize()
    backend.check()
    graphs, plan, _ = graphed(step, K)
    stream = torch.cuda.current_stream(dev)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for g in plan:
        g.replay()
    t1.record(stream)
    torch.cuda.synchronize()
    backend.check()
    ms = t0.elapsed_time(t1) / K
    del graphs, plan, bufs
    return {"rows_per_s": B / (ms * 1e-3), "ms_per_step": ms, "batch": B, "vocab": w.vocab,
            "dtype": "bf16" if w.logits.dtype == torch.bfloat16 else "f32", "steps": K,
            "l2": f"{nbuf} rotating logits buffers"}


def decode_rows_per_s(w, dev, K: int) -> dict:
    """Configuration 3 as a decode loop: every step samples all 256 slots with their slotted
    histories (penalties) and counts the sampled ids into them in place (vinfer_hist_append),
    with nothing leaving the device; CUDA graphs, rotating logits buffers."""
    from vinfer_b200 import SAMPLER, BackendContext  # noqa: PLC0415
    from vinfer_b200.sampling import RowParams, SlotHistogram  # noqa: PLC0415

    B = w.batch
    backend = SAMPLER.resolve("b200", BackendContext(dev, torch.bfloat16))
    base = w.logits.to(dev)
    nbuf = max(2, int(np.ceil(2 * L2_BYTES / (base.numel() * 2))) + 1)
    bufs = [base] + [base.clone() for _ in range(nbuf - 1)]
    params = RowParams.from_arrays(dev, **w.param_arrays())
    u = torch.from_numpy(w.uniforms).to(dev)
    cap = 2048  # room for the longest history (1,646 entries) plus every step's new token
    slots = SlotHistogram.from_csr(w.hist_row_ptr, w.hist_ids, w.hist_counts, cap, dev)
    out = torch.empty(B, dtype=torch.int32, device=dev)

    def step(i: int) -> None:
        backend.decode_step(bufs[i % nbuf], params, u, slots, out=out)

    for i in range(3):
        step(i)
    torch.cuda.synchronize()
    backend.check()
    graphs, plan, _ = graphed(step, K)
    stream = torch.cuda.current_stream(dev)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for g in plan:
        g.replay()
    t1.record(stream)
    torch.cuda.synchronize()
    backend.check()
    ms = t0.elapsed_time(t1) / K
    del graphs, plan, bufs
    return {"rows_per_s": B / (ms * 1e-3), "ms_per_step": ms, "batch": B, "steps": K,
            "history": f"slotted, cap {cap} entries a slot, updated in place every step",
            "launches_per_step": 3}


def backend_c4(dev):
    from vinfer_b200 import SAMPLER, BackendContext  # noqa: PLC0415

    return SAMPLER.resolve("b200", BackendContext(dev, torch.bfloat16))


def unsharded_config4_rows_per_s(backend, dev, K: int) -> float:
    """Configuration 4 on this one GPU, unsharded (batch 1024 x vocab 248,320), through
    ``sample_batch`` in CUDA graphs: the strong-scaling reference of the sharded lines."""
    from vinfer_b200.workloads import config4_shard  # noqa: PLC0415

    B, V = 1024, 248_320
    x, params, u = config4_shard(0, 1, dev, B, V)
    nbuf = max(2, int(np.ceil(2 * L2_BYTES / (x.numel() * 2))) + 1)
    bufs = [x] + [x.clone() for _ in range(nbuf - 1)]
    out = torch.empty(B, dtype=torch.int32, device=dev)

    def step(i: int) -> None:
        backend.sample_batch(bufs[i % nbuf], params, u, None, out=out)

    for i in range(3):
        step(i)
    torch.cuda.synchronize()
    graphs, plan, _ = graphed(step, K)
    stream = torch.cuda.current_stream(dev)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for g in plan:
        g.replay()
    t1.record(stream)
    torch.cuda.synchronize()
    backend.check()
    del graphs, plan, bufs
    return B * K / (t0.elapsed_time(t1) * 1e-3)


def bench_sharded(args) -> dict | None:
    from datetime import timedelta  # noqa: PLC0415

    import torch.distributed as dist  # noqa: PLC0415

    from vinfer_b200 import SAMPLER, BackendContext  # noqa: PLC0415
    from vinfer_b200.sharded import B200ShardKernels, ShardedSampler, shard_range  # noqa: PLC0415
    from vinfer_b200.workloads import config4_shard  # noqa: PLC0415

    rank, world, local = dist_env()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))
    graphs = plan = None
    try:
        backend = SAMPLER.resolve("b200", BackendContext(dev, torch.bfloat16))
        sampler = ShardedSampler(B200ShardKernels(backend))
        B, V = 1024, 248_320
        lo, hi = shard_range(V, world, rank)
        x, params, u = config4_shard(rank, world, dev, B, V)
        shard_bytes = x.numel() * x.element_size()
        nbuf = max(2, int(np.ceil(2 * L2_BYTES / shard_bytes)) + 1)
        bufs = [x] + [x.clone() for _ in range(nbuf - 1)]
        out = torch.empty(B, dtype=torch.int32, device=dev)
        stream = torch.cuda.current_stream(dev)

        # the device steps of one batch (local records, NCCL all-gather, merge) issued back to
        # back with no host synchronisation, so the host runs ahead of the device and the timed
        # region is device time; the rows they leave unresolved are counted on the device and
        # read once after it. (CUDA graphs holding the NCCL call are not used: one such run
        # on this pool stalled at two GPUs; eager launches keep the collective under NCCL's
        # watchdog and the process group's timeout.)
        def step(i: int) -> None:
            sampler.sample_batch_async(bufs[i % nbuf], params, u, None, V, out=out)

        for i in range(max(args.warmup, 3)):
            sampler.sample_batch(bufs[i % nbuf], params, u, None, V, out=out)
        torch.cuda.synchronize()
        sampler.kernels.check()
        sampler.pending_unresolved(dev)
        for i in range(3):  # the asynchronous form once more, untimed
            step(i)
        torch.cuda.synchronize()
        sampler.pending_unresolved(dev)

        clocks = Clocks(local) if rank == 0 else None
        if clocks:
            clocks.start()
        dist.barrier()
        torch.cuda.synchronize()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        for i in range(args.steps):
            step(i)
        t1.record(stream)
        torch.cuda.synchronize()
        dist.barrier()
        ms = t0.elapsed_time(t1)
        clk = clocks.stop() if clocks else None
        unresolved = sampler.pending_unresolved(dev)
        sampler.kernels.check()

        # phases of one step: events around each device step on the launching stream
        bufd = sampler._buffers(B, dev)
        torch.cuda._sleep(20_000_000)
        ev = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(16)]
        for i in range(16):
            ev[i][0].record(stream)
            sampler.kernels.local(bufs[i % nbuf], params, u, None, lo, V, sampler.record_cap,
                                  bufd["local"], bufd["scratch_ids"])
            ev[i][1].record(stream)
            dist.all_gather_into_tensor(bufd["gathered"], bufd["local"])
            ev[i][2].record(stream)
            sampler.kernels.merge(bufs[i % nbuf], params, u, None, lo, V, sampler.record_cap,
                                  bufd["gathered"], world, out, bufd["unresolved"], None)
            ev[i][3].record(stream)
        torch.cuda.synchronize()
        phases = [statistics.mean(e[k].elapsed_time(e[k + 1]) for e in ev) for k in range(3)]
        local_ms = phases[0]

        # correctness of the timed configuration, checked on every rank: the same ids on all
        # ranks, and 16 rows assembled in full and sampled unsharded give the sharded ids
        ids = sampler.sample_batch(bufs[0], params, u, None, V, out=torch.empty_like(out))
        allids = torch.empty(world * B, dtype=torch.int32, device=dev)
        dist.all_gather_into_tensor(allids, ids)
        same = bool((allids.view(world, B) == ids.view(1, B)).all())
        idx = torch.arange(16, device=dev) * (B // 16) + 7
        spot = ids.clone()
        spot[idx] = -1
        sampler._resolve_rows(bufs[0], params, u, None, V, spot, None, idx)
        spot_ok = bool(torch.equal(spot, ids))

        # end to end through the public API: this rank's shard and the row parameters copied
        # from pinned host memory, the ids copied back, every step
        host_x = x.cpu().pin_memory()
        host_p = {k: getattr(params, k).cpu().pin_memory() for k in
                  ("temperature", "top_k", "top_p", "min_p", "repetition_penalty",
                   "presence_penalty", "frequency_penalty")}
        host_u = u.cpu().pin_memory()
        host_ids = torch.empty(B, dtype=torch.int32).pin_memory()
        d_x = torch.empty_like(x)
        d_u = torch.empty_like(u)
        h2d = (host_x.numel() * host_x.element_size() + host_u.numel() * 4
               + sum(t.numel() * t.element_size() for t in host_p.values()))

        def e2e_step() -> None:
            d_x.copy_(host_x, non_blocking=True)
            for k, t in host_p.items():
                getattr(params, k).copy_(t, non_blocking=True)
            d_u.copy_(host_u, non_blocking=True)
            r = sampler.sample_batch(d_x, params, d_u, None, V, out=out)
            host_ids.copy_(r, non_blocking=True)

        e2e_steps = max(3, min(args.steps, 20))
        e2e_step()
        torch.cuda.synchronize()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(e2e_steps):
            e2e_step()
        e1.record(stream)
        torch.cuda.synchronize()
        e2e_ms = e0.elapsed_time(e1) / e2e_steps
        sampler.kernels.check()

        # the strong-scaling reference: configuration 4 unsharded on rank 0's GPU alone
        ref = unsharded_config4_rows_per_s(backend, dev, args.steps) if rank == 0 else 0.0
        dist.barrier()

        t = torch.tensor([ms, local_ms, e2e_ms, float(unresolved), *phases,
                          0.0 if same else 1.0, 0.0 if spot_ok else 1.0],
                         dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, local_ms, e2e_ms, unresolved = float(t[0]), float(t[1]), float(t[2]), int(t[3])
        phases = [float(v) for v in t[4:7]]
        same, spot_ok = float(t[7]) == 0.0, float(t[8]) == 0.0
    finally:
        del graphs, plan
        dist.destroy_process_group()
    if rank != 0:
        return None
    peak, kind = measured_peak()
    shard_algo = B * (hi - lo) * 2 + 36 * B  # local-record pass: this rank's logits and params
    achieved = shard_algo / (local_ms * 1e-3) / 1e9
    value = B * args.steps / (ms * 1e-3)
    return {
        "metric": METRIC,
        "value": value,
        "unit": "rows/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms / args.steps,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded on the device, configuration 4 distribution)",
        "config": workload_config(world),
        "method": {"shard_vocab": hi - lo,
                   "record_bytes_per_row": sampler.rec_bytes,
                   "allgather_bytes_per_rank": B * sampler.rec_bytes,
                   "l2": f"{nbuf} rotating shard buffers per rank "
                         f"({nbuf * shard_bytes / 2**20:.0f} MiB > 2x L2)",
                   "parallelism": f"vocab-sharded over {world} ranks",
                   "timed_steps": "eager, back to back, no host synchronisation",
                   "unresolved_rows_in_timed_steps": unresolved},
        "strong_scaling_ref": {"value": ref, "unit": "rows/s",
                               "what": "configuration 4 unsharded on one GPU (rank 0's), "
                                       "sample_batch in CUDA graphs",
                               "speedup": value / ref if ref else None},
        "phase_ms": {"local_records": phases[0], "all_gather": phases[1], "merge": phases[2],
                     "how": "CUDA events around each device step, mean of 16 eager steps, "
                            "max over ranks"},
        "ids_equal_across_ranks": same,
        "spot_rows_match": spot_ok,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "peak_kind": f"{kind} (copy bandwidth)",
                     "traffic": None, "algorithmic_bytes": shard_algo,
                     "kernel": "k_stream<bf16> + k_finish<bf16> (local records, one rank)",
                     "kernel_ms": local_ms},
        "clocks": clk,
        "e2e": {"value": B / (e2e_ms * 1e-3), "unit": "rows/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": B * 4, "steps": e2e_steps},
        "gpu_launches": 3 * args.steps,  # k_stream, k_finish (records), k_merge per step
        "cpu_baseline": None,
    }


# ----------------------------------------------------------------------------------------------
# reference arm: vinfer's CPU sampler on this host
# ----------------------------------------------------------------------------------------------
def bench_reference(args, world: int) -> dict:
    from vinfer_b200.workloads import make  # noqa: PLC0415

    config = 3 if world == 1 else 4
    w = make(config, batch=None if config == 3 else 64)
    K, W = args.steps, args.warmup
    budget = args.ref_seconds
    t0 = time.perf_counter()
    est = cpu_reference_rows_per_s(w, 0.0, rows_cap=max(1, min(W, 3)))
    per_row = 1.0 / est["value"]
    rows_per_step = max(1, int(budget / max(K, 1) / per_row))
    cpu_reference_rows_per_s(w, 0.0, rows_cap=max(1, W))  # warm-up steps (1 row each)
    t1 = time.perf_counter()
    res = cpu_reference_rows_per_s(w, 0.0, rows_cap=K * rows_per_step)
    el = time.perf_counter() - t1
    value = res["value"]
    return {
        "impl": "reference",
        "metric": METRIC,
        "value": value,
        "unit": "rows/s",
        "n_gpus": world,
        "steps": K,
        "warmup": W,
        "ms_per_step": el * 1e3 / K,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": f"synthetic (seeded, configuration {config})",
        "config": workload_config(world, w.hist_nnz if config == 3 else None),
        "method": {"rows_per_step": rows_per_step,
                   "note": "each step samples rows_per_step rows of the configuration on the CPU "
                           "(the whole row, unsharded), one sample() call per row as "
                           "generate() makes them; the metric is rows per second"},
        "cpu_baseline": {"value": value, "unit": "rows/s", "cores": res["cores"], "kind": "port",
                         "sample": res["sample"]},
        "e2e": {"value": value, "unit": "rows/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "wall_s": time.perf_counter() - t0,
    }


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--ref-seconds", type=float, default=60.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", choices=["default", "config4", "config5", "topp"],
                    default="default",
                    help="one GPU only: config4 times configuration 4 unsharded (the reference "
                         "for the vocab-sharded runs); config5 times configuration 5 (adversarial "
                         "rows, mostly the exact search); topp times configuration 3's logits "
                         "with top-p only (the exact search); the default line is configuration 3")
    args = ap.parse_args()
    rank, world, local = dist_env()
    if args.impl == "reference":
        if rank == 0:
            print(json.dumps(bench_reference(args, world)), flush=True)
        return
    if world > 1:
        line = bench_sharded(args)
    elif args.gpus > 1:
        raise SystemExit("--gpus N > 1 runs one process per GPU: launch bench.py under "
                         "torch.distributed.run with --nproc-per-node N")
    elif args.workload == "config4":
        line = bench_single_config4(args)
    elif args.workload == "config5":
        dev = torch.device("cuda", 0)
        torch.cuda.set_device(dev)
        r = config_rows_per_s(5, dev, max(1, args.steps))
        line = {"metric": METRIC, "value": r["rows_per_s"], "unit": "rows/s", "n_gpus": 1,
                "steps": r["steps"], "warmup": 3, "ms_per_step": r["ms_per_step"],
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "f32", "data": "synthetic (seeded, configuration 5)",
                "config": {"workload": "config5: batch 512 x vocab 151936 f32, flat / one +30 "
                                       "token / 1000-way tie / N(0,1) rows, top-k U{1..1000}, "
                                       "top-p U[0.1,1], temp U[0.1,2], 512-token histories",
                           "batch": r["batch"], "vocab": r["vocab"]},
                "method": {"l2": r["l2"], "timing": "sample_batch in CUDA graphs"}}
    else:
        line = bench_single(args)
    if line is not None and rank == 0:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
