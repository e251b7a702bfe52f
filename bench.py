#!/usr/bin/env python
"""Benchmark of the paged-KV decode hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload ``decode`` (default): one decode step of the north-star shape --
per GPU, B=32 requests with 2048-token contexts (2047 cached + 1 appended),
16 query / 8 KV heads, head_dim 128, bf16, block_size 16, pages from a seeded
permutation of a pool 1.1x the pages used (BASELINE configs 2-3 family).  A
step is the reference's per-layer decode hot path: ``write_kv_cache_batch``
(append) followed by ``paged_attention``.  Request-sharded: every rank owns an
independent pool and batch (weak scaling, no collective on the data path).

Metric: paged-decode KV-read GB/s (algorithmic KV bytes read by the step /
step time), summed over GPUs; decode tok/s is reported beside it.  Timed with
CUDA events around K replays of a CUDA graph of one step; the inputs (295 MB
per GPU) exceed the 126 MB L2.  ``e2e`` repeats the step through the public
Python API with host buffers: every step copies q/k/v/tables/lengths from
pinned host memory and reads the output back.  ``--impl reference`` times the
reference algorithm's CPU path (the oracle restatement) on the host cores.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from datetime import timedelta
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "paged-decode KV-read GB/s (% HBM peak); decode tok/s at 1/2/4/8 B200"
HQ, HKV, D, BS = 16, 8, 128, 16


def parse_args(argv=None):
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=20000)
    parser.add_argument("--warmup", type=int, default=20)
    parser.add_argument("--impl", choices=("ours", "reference"), default="ours")
    parser.add_argument("--batch", type=int, default=32, help="requests per GPU")
    parser.add_argument("--context", type=int, default=2048, help="attended tokens per request")
    parser.add_argument("--cpu-seconds", type=float, default=10.0, help="CPU baseline sample budget")
    return parser.parse_args(argv)


# ----------------------------------------------------------------------- setup
def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and not torch.distributed.is_initialized():
        backend = "nccl" if args.impl == "ours" else "gloo"
        if backend == "nccl":
            torch.cuda.set_device(local)
        torch.distributed.init_process_group(backend, timeout=timedelta(seconds=300))
    elif args.impl == "ours":
        torch.cuda.set_device(local)
    return world, rank, local


def kv_bytes(lengths, esize=2):
    return sum(lengths) * 2 * HKV * D * esize


def decode_bytes(lengths, batch, esize=2):
    """Algorithmic bytes of one decode call: KV read once + q and out + page-table entries."""
    return kv_bytes(lengths, esize) + 2 * batch * HQ * D * esize + 8 * sum(math.ceil(n / BS) for n in lengths)


def make_inputs(batch, context, device, seed):
    gen = torch.Generator(device=device).manual_seed(seed)
    pages = math.ceil(context / BS)
    pool = math.ceil(1.1 * batch * pages)
    kc = torch.randn(pool, BS, HKV, D, device=device, dtype=torch.bfloat16, generator=gen)
    vc = torch.randn(pool, BS, HKV, D, device=device, dtype=torch.bfloat16, generator=gen)
    perm = torch.randperm(pool, device=device, generator=gen)
    tables = perm[: batch * pages].view(batch, pages).contiguous()
    q = torch.randn(batch, HQ, D, device=device, dtype=torch.bfloat16, generator=gen)
    k = torch.randn(batch, HKV, D, device=device, dtype=torch.bfloat16, generator=gen)
    v = torch.randn(batch, HKV, D, device=device, dtype=torch.bfloat16, generator=gen)
    offsets = torch.full((batch,), context - 1, dtype=torch.int64, device=device)
    lens = offsets + 1
    return {"query": q, "key_cache": kc, "value_cache": vc, "block_tables": tables, "token_offsets": offsets,
            "context_lens": lens, "key": k, "value": v}


# ---------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi samples of this GPU while the timed region runs."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index):
        uuid = str(torch.cuda.get_device_properties(device_index).uuid)
        self.gpu = uuid if uuid.startswith("GPU-") else f"GPU-{uuid}"
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        return False

    def summary(self):
        sm, mx, reasons = [], [], set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[0]))
                mx.append(float(parts[1]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[4:8]):
                if flag.lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


def measured_peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.is_file():
        data = json.loads(path.read_text())
        return float(data["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def ncu_traffic(name):
    """DRAM bytes per launch of the decode op from the committed ncu summary, if any."""
    path = ROOT / "profiles" / "traffic.json"
    if path.is_file():
        value = json.loads(path.read_text()).get(name)
        return None if value is None else float(value)
    return None


# ---------------------------------------------------------------- CPU baseline
class CpuReference:
    """Reference algorithm on the host cores: oracle append + decode on a bounded sample."""

    SAMPLE_BATCH = 2

    def __init__(self, context):
        sys.path.insert(0, str(ROOT / "tests" / "golden"))
        import cases
        from oracle import kv_write, paged_decode

        self.kv_write, self.paged_decode = kv_write, paged_decode
        self.context = context
        self.case = cases.append_decode_case(torch.bfloat16, batch=self.SAMPLE_BATCH,
                                             contexts=[context - 1] * self.SAMPLE_BATCH, block_size=BS,
                                             seed=404, pool_slack=1.0)
        self.nbytes = decode_bytes(self.case["context_lens"].tolist(), self.SAMPLE_BATCH)

    def step(self):
        c = self.case
        self.kv_write.write_kv_cache_batch(c["key_cache"], c["value_cache"], c["block_tables"],
                                           c["token_offsets"], c["key"], c["value"], BS)
        self.paged_decode.paged_attention(c["query"], c["key_cache"], c["value_cache"], c["block_tables"],
                                          c["context_lens"], BS)

    def timed(self, seconds=0.0, min_steps=1):
        done, start = 0, time.perf_counter()
        while done < min_steps or time.perf_counter() - start < seconds:
            self.step()
            done += 1
        return (time.perf_counter() - start) / done, done

    def describe(self, per_step, done):
        threads = torch.get_num_threads()
        return {"value": self.nbytes / per_step / 1e9, "unit": "GB/s", "cores": threads, "kind": "port",
                "sample": f"{done} steps of the oracle's append+decode (restating mini_engine/kernels "
                          f"fallback.py:27-64 and data.py:67-81) on {self.SAMPLE_BATCH} requests x "
                          f"{self.context} tokens, bf16, {per_step * 1e3:.1f} ms/step, torch threads={threads}"}


def cpu_baseline(context, seconds):
    ref = CpuReference(context)
    ref.timed(0.0, 1)
    per_step, done = ref.timed(seconds, 3)
    return ref.describe(per_step, done)


def run_reference(args, world, rank):
    if rank != 0:
        return None
    torch.set_num_threads(os.cpu_count() or 1)
    ref = CpuReference(args.context)
    ref.timed(0.0, min(args.warmup, 3))
    # each step is a bounded CPU sample; stop after ~60 s so the run ends in minutes
    done, start = 0, time.perf_counter()
    while done < args.steps and (done < 3 or time.perf_counter() - start < 60.0):
        ref.step()
        done += 1
    per_step = (time.perf_counter() - start) / done
    base = ref.describe(per_step, done)
    value = base["value"]
    return {"metric": METRIC, "value": value, "unit": "GB/s", "impl": "reference", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": per_step * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic",
            "config": {"workload": f"decode step (KV append + paged attention), {args.batch} x {args.context} "
                                   f"tokens per GPU; each CPU step is a {CpuReference.SAMPLE_BATCH}-request sample",
                       "parallelism": "rank 0 only, host cores"},
            "cpu_baseline": base,
            "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


# ------------------------------------------------------------------- GPU arm
def run_ours(args, world, rank, local):
    from myvllm_mini_engine_b200 import _lib
    from myvllm_mini_engine_b200.kernels import paged_attention, write_kv_cache_batch

    device = torch.device("cuda", local)
    x = make_inputs(args.batch, args.context, device, seed=1234 + rank)
    lengths = [args.context] * args.batch
    step_bytes = decode_bytes(lengths, args.batch)
    stream = torch.cuda.current_stream(device)

    def step(out_holder=None):
        write_kv_cache_batch(x["key_cache"], x["value_cache"], x["block_tables"], x["token_offsets"], x["key"],
                             x["value"], BS, validate=False)
        return paged_attention(x["query"], x["key_cache"], x["value_cache"], x["block_tables"],
                               x["context_lens"], BS, validate=False)

    # warm up on the capture stream, so the per-stream decode workspace exists
    # before capture and its one-time zero fill is not part of the graph
    capture_stream = torch.cuda.Stream(device)
    capture_stream.wait_stream(stream)
    with torch.cuda.stream(capture_stream):
        for _ in range(3):
            step()
    torch.cuda.synchronize(device)
    # one step captured as a graph, with external timing events around the decode op
    ev_a = torch.cuda.Event(enable_timing=True, external=True)
    ev_b = torch.cuda.Event(enable_timing=True, external=True)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=capture_stream):
        write_kv_cache_batch(x["key_cache"], x["value_cache"], x["block_tables"], x["token_offsets"], x["key"],
                             x["value"], BS, validate=False)
        ev_a.record()
        out = paged_attention(x["query"], x["key_cache"], x["value_cache"], x["block_tables"], x["context_lens"],
                              BS, validate=False)
        ev_b.record()
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize(device)

    def barrier():
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize(device)

    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    kernel_ms = []
    with ClockSampler(local) as clocks:
        barrier()
        start.record(stream)
        for _ in range(args.steps):
            graph.replay()
        end.record(stream)
        barrier()
        # per-launch decode time: the same graph, reading the inner events after each replay
        for _ in range(min(args.steps, 50)):
            graph.replay()
            ev_b.synchronize()
            kernel_ms.append(ev_a.elapsed_time(ev_b))
    elapsed_ms = start.elapsed_time(end)
    if world > 1:
        t = torch.tensor([elapsed_ms], device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        elapsed_ms = float(t.item())
    ms_per_step = elapsed_ms / args.steps
    value = world * step_bytes / (ms_per_step * 1e-3) / 1e9
    kernel_avg_ms = statistics.mean(kernel_ms)
    achieved = step_bytes / (kernel_avg_ms * 1e-3) / 1e9
    peak, peak_kind = measured_peaks()

    # ---- end to end through the public API, host buffers in and out
    host = {k: x[k].cpu().pin_memory() for k in ("query", "key", "value", "block_tables", "token_offsets",
                                                 "context_lens")}
    dev = {k: torch.empty_like(x[k]) for k in host}
    out_host = torch.empty(out.shape, dtype=out.dtype, pin_memory=True)
    h2d = sum(t.numel() * t.element_size() for t in host.values())
    d2h = out_host.numel() * out_host.element_size()

    def e2e_step():
        for k, t in host.items():
            dev[k].copy_(t, non_blocking=True)
        write_kv_cache_batch(x["key_cache"], x["value_cache"], dev["block_tables"], dev["token_offsets"],
                             dev["key"], dev["value"], BS, validate=False)
        result = paged_attention(dev["query"], x["key_cache"], x["value_cache"], dev["block_tables"],
                                 dev["context_lens"], BS, validate=False)
        out_host.copy_(result, non_blocking=True)

    for _ in range(args.warmup):
        e2e_step()
    barrier()
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e_start.record(stream)
    for _ in range(args.steps):
        e2e_step()
    e_end.record(stream)
    barrier()
    e2e_ms = e_start.elapsed_time(e_end)
    if world > 1:
        t = torch.tensor([e2e_ms], device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e_value = world * step_bytes / (e2e_ms / args.steps * 1e-3) / 1e9
    status = _lib.device_status(device)
    if status:
        raise RuntimeError(f"device status bits set during the benchmark: {status}")
    del graph
    if rank != 0:
        return None
    line = {
        "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"decode step (KV append + paged attention) of {args.batch} requests x "
                               f"{args.context} tokens per GPU, Hq16/Hkv8/D128, block 16",
                   "global_batch": args.batch * world, "seq_len": args.context,
                   "parallelism": f"request-sharded x{world} (independent KV pools)",
                   "l2": f"inputs {2 * x['key_cache'].numel() * 2 / 1e6:.0f} MB per GPU > 126 MB L2"},
        "decode_tok_s": world * args.batch / (ms_per_step * 1e-3),
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "peak_source": peak_kind,
                     "traffic": ncu_traffic("decode_b32_ctx2048_bf16"),
                     "kernel": "paged decode (split kernel + combine kernel) per launch",
                     "bytes_per_launch": step_bytes, "launch_ms": kernel_avg_ms},
        "e2e": {"value": e2e_value, "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "ms_per_step": e2e_ms / args.steps},
        "gpu_launches": 3 * args.steps,
        "clocks": clocks.summary(),
    }
    if world == 1:
        line["cpu_baseline"] = cpu_baseline(args.context, args.cpu_seconds)
    return line


def main(argv=None):
    args = parse_args(argv)
    world, rank, local = dist_setup(args)
    try:
        line = run_reference(args, world, rank) if args.impl == "reference" else run_ours(args, world, rank, local)
        if line is not None and rank == 0:
            print(json.dumps(line), flush=True)
    finally:
        if world > 1 and torch.distributed.is_initialized():
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
