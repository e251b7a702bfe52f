#!/usr/bin/env python
"""Benchmark of the paged-KV decode hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload ``decode`` (default): one decode step of the north-star shape --
per GPU, B=32 requests with 2048-token contexts (2047 cached + 1 appended),
16 query / 8 KV heads, head_dim 128, bf16, block_size 16, pages from a seeded
permutation of a pool 1.1x the pages used (BASELINE configs 2-3 family).  A
step is the reference's per-layer decode hot path: ``write_kv_cache_batch``
(append) followed by ``paged_attention`` (native_qwen3.py:188-196), run as one
fused launch (``paged_attention_with_append``).  Request-sharded: every rank owns an
independent pool and batch (weak scaling, no collective on the data path).

Metric: paged-decode KV-read GB/s (algorithmic KV bytes read by the step /
step time), summed over GPUs.  Timed with CUDA events around K replays of a
CUDA graph of one step, in ``--repeats`` windows (median reported, min and max
beside it); the inputs (295 MB per GPU) exceed the 126 MB L2.  ``e2e`` repeats
the step through the public Python API with host buffers: every step copies
q/k/v/tables/lengths from pinned host memory and reads the output back.
``--impl reference`` times the reference algorithm's CPU path (the oracle
restatement) on the host cores.

The same JSON line also carries every BASELINE config (unless
``--headline-only``): ``config1``..``config3`` (decode, one GPU, L2 flushed
before every step), ``config4`` (copy-on-write + scatter + ragged prefill, one
GPU) and ``qwen3`` (config 5, the whole Qwen3 decode step, 256 requests x 4096
split over the N ranks: strong scaling, its ``value`` is the model's decode
tok/s), each with its roofline fraction and the CPU path timed beside it.
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
    parser.add_argument("--steps", type=int, default=200)
    parser.add_argument("--warmup", type=int, default=20)
    parser.add_argument("--repeats", type=int, default=25,
                        help="decode: timed windows of --steps steps each; ms_per_step is their median")
    parser.add_argument("--headline-only", action="store_true",
                        help="decode: skip the per-config fields (configs 1-4 at one GPU, config 5 at every N)")
    parser.add_argument("--impl", choices=("ours", "reference"), default="ours")
    parser.add_argument("--workload", choices=("decode", "qwen3", "prefill"), default="decode",
                        help="decode: append + paged attention per GPU (weak scaling); qwen3: the full "
                             "Qwen3-0.6B decode step of BASELINE config 5 (strong scaling over --batch); "
                             "prefill: BASELINE config 4 (copy-on-write + slot scatter + ragged paged prefill)")
    parser.add_argument("--batch", type=int, default=None,
                        help="requests per GPU (decode, default 32) or in total (qwen3, default 256)")
    parser.add_argument("--context", type=int, default=None,
                        help="attended tokens per request (decode, default 2048) or cached tokens (qwen3, 4096)")
    parser.add_argument("--cpu-seconds", type=float, default=10.0, help="CPU baseline sample budget")
    parser.add_argument("--projections", choices=("fused", "cublas"), default="fused",
                        help="qwen3: tcgen05 projections with the element-wise steps fused in for per-GPU batches "
                             "up to Qwen3DecodeStep.FUSED_MAX_BATCH (default), or cuBLAS projections around the "
                             "element-wise kernels")
    parser.add_argument("--kv-dtype", choices=("bf16", "fp8", "fp8_e5m2"), default="bf16",
                        help="decode / prefill: the KV pool format; fp8 = E4M3 pool, fp8_e5m2 = E5M2 pool, with "
                             "per-pool scales (decode: fused quantising KV append + fp8 paged attention, "
                             "device-timed only; prefill: config 4 with a quantising scatter and the fp8 prefill)")
    args = parser.parse_args(argv)
    if args.batch is None:
        args.batch = 32 if args.workload == "decode" else 256
    if args.context is None:
        args.context = 2048 if args.workload == "decode" else 4096
    return args


# ----------------------------------------------------------------------- setup
def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and not torch.distributed.is_initialized():
        backend = "nccl" if args.impl == "ours" else "gloo"
        if backend == "nccl":
            torch.cuda.set_device(local)
        kwargs = {"device_id": torch.device("cuda", local)} if backend == "nccl" else {}
        torch.distributed.init_process_group(backend, timeout=timedelta(seconds=300), **kwargs)
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


def packed_buffers(tensors, device, align=256):
    """One pinned host buffer and one device buffer holding every tensor, with typed views.

    Returns (host, dev): dicts of views by name plus "_buffer", the flat uint8
    storage; host views are filled with the tensors' current values.
    """
    offsets, total = {}, 0
    for k, t in tensors.items():
        offsets[k] = total
        total += (t.numel() * t.element_size() + align - 1) // align * align
    host_buf = torch.empty(total, dtype=torch.uint8, pin_memory=True)
    dev_buf = torch.empty(total, dtype=torch.uint8, device=device)
    host, dev = {"_buffer": host_buf}, {"_buffer": dev_buf}
    for k, t in tensors.items():
        n = t.numel() * t.element_size()
        host[k] = host_buf[offsets[k]:offsets[k] + n].view(t.dtype).view(t.shape)
        dev[k] = dev_buf[offsets[k]:offsets[k] + n].view(t.dtype).view(t.shape)
        host[k].copy_(t.cpu())
    return host, dev


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
    from myvllm_mini_engine_b200.kernels import paged_attention_with_append

    device = torch.device("cuda", local)
    x = make_inputs(args.batch, args.context, device, seed=1234 + rank)
    lengths = [args.context] * args.batch
    step_bytes = decode_bytes(lengths, args.batch)
    stream = torch.cuda.current_stream(device)

    def step():
        # the append of the step's new K/V rows and the decode over context + 1, one launch
        # (paged_attention_with_append); chained: the offsets and tables predate the previous
        # kernel, so each launch's prologue overlaps the tail of the one before
        return paged_attention_with_append(x["query"], x["key_cache"], x["value_cache"], x["block_tables"],
                                           x["token_offsets"], x["key"], x["value"], BS, validate=False,
                                           chained=True)

    # warm up on the capture stream, so the per-stream decode workspace exists
    # before capture and its one-time zero fill is not part of the graph
    capture_stream = torch.cuda.Stream(device)
    capture_stream.wait_stream(stream)
    with torch.cuda.stream(capture_stream):
        for _ in range(3):
            step()
    torch.cuda.synchronize(device)
    # the timed workload: K consecutive steps, captured as graphs of at most 256 steps
    per_graph = max(1, min(args.steps, 256))
    full, rest = divmod(args.steps, per_graph)
    graphs = []
    for count in [per_graph] * min(full, 1) + ([rest] if rest else []):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=capture_stream):
            for _ in range(count):
                out = step()
        graphs.append((g, count))
    big = graphs[0][0] if full else None
    tail = graphs[-1][0] if rest else None

    def run_steps():
        for _ in range(full):
            big.replay()
        if tail is not None:
            tail.replay()

    # one launch alone between external events (no overlap with a neighbour): its isolated duration
    ev_a = torch.cuda.Event(enable_timing=True, external=True)
    ev_b = torch.cuda.Event(enable_timing=True, external=True)
    probe = torch.cuda.CUDAGraph()
    with torch.cuda.graph(probe, stream=capture_stream):
        ev_a.record()
        paged_attention_with_append(x["query"], x["key_cache"], x["value_cache"], x["block_tables"],
                                    x["token_offsets"], x["key"], x["value"], BS, validate=False)
        ev_b.record()
    for _ in range(max(1, math.ceil(args.warmup / args.steps))):  # at least W untimed steps
        run_steps()
    torch.cuda.synchronize(device)

    def barrier():
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize(device)

    # R windows of exactly K steps, each bracketed by a barrier and a synchronize; a window's
    # time is the max over ranks, and ms_per_step is the median window
    repeats = max(1, args.repeats)
    windows = []
    kernel_ms = []
    with ClockSampler(local) as clocks:
        for _ in range(repeats):
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            barrier()
            start.record(stream)
            run_steps()
            end.record(stream)
            barrier()
            windows.append(start.elapsed_time(end))
        # isolated duration of one launch: the probe graph, reading its events after each replay
        for _ in range(min(args.steps, 50)):
            probe.replay()
            ev_b.synchronize()
            kernel_ms.append(ev_a.elapsed_time(ev_b))
    if world > 1:
        t = torch.tensor(windows, device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        windows = [float(x) for x in t.tolist()]
    per_step = sorted(w / args.steps for w in windows)
    ms_per_step = statistics.median(per_step)
    value = world * step_bytes / (ms_per_step * 1e-3) / 1e9
    kernel_avg_ms = statistics.mean(kernel_ms)
    # the step is one launch of the kernel: its average duration in the timed region is the step time
    achieved = step_bytes / (ms_per_step * 1e-3) / 1e9
    peak, peak_kind = measured_peaks()

    # ---- end to end through the public API, host buffers in and out: every step
    # copies its inputs (q, k, v, tables, offsets: one pinned host buffer, one
    # copy) to the GPU, runs the fused append + decode and copies the output back
    # to pinned host memory.  As a serving loop would, the copies run on a second
    # stream, pipelined across steps: step k+1's inputs go up into the other of
    # two device input buffers while step k computes, and step k's output comes
    # down while step k+1 computes.  The steps (copies and kernels) are captured
    # in CUDA graphs of up to 256 steps, as the decode loop of a serving engine
    # is, so the host issues one graph launch per window instead of a Python
    # call per copy and kernel.
    names = ("query", "key", "value", "block_tables", "token_offsets")
    host, dev_a = packed_buffers({k: x[k] for k in names}, device)
    _, dev_b = packed_buffers({k: x[k] for k in names}, device)
    devs = (dev_a, dev_b)
    outs_host = [torch.empty(x["query"].shape, dtype=x["query"].dtype, pin_memory=True) for _ in range(2)]
    h2d = host["_buffer"].numel()
    d2h = outs_host[0].numel() * outs_host[0].element_size()
    copies = torch.cuda.Stream(device)
    # the copies go straight to the CUDA runtime (cuda-python): plain memcpy nodes in the graph
    from cuda.bindings import runtime as cudart

    def memcpy(dst, src, nbytes, kind, on):
        err = cudart.cudaMemcpyAsync(dst, src, nbytes, kind, cudart.cudaStream_t(on.cuda_stream))[0]
        if err != cudart.cudaError_t.cudaSuccess:
            raise RuntimeError(f"cudaMemcpyAsync failed: {err}")

    to_dev, to_host = cudart.cudaMemcpyKind.cudaMemcpyHostToDevice, cudart.cudaMemcpyKind.cudaMemcpyDeviceToHost

    def e2e_steps(count):
        """``count`` steps with their copies, issued on the current (capturing) stream and ``copies``."""
        compute = torch.cuda.current_stream(device)
        copied = [torch.cuda.Event() for _ in range(count)]
        done = [torch.cuda.Event() for _ in range(count)]
        results = []  # every step's output stays allocated until its download is ordered before later work
        copies.wait_stream(compute)
        memcpy(devs[0]["_buffer"].data_ptr(), host["_buffer"].data_ptr(), h2d, to_dev, copies)
        copied[0].record(copies)
        for k in range(count):
            d = devs[k % 2]
            compute.wait_event(copied[k])
            result = paged_attention_with_append(d["query"], x["key_cache"], x["value_cache"], d["block_tables"],
                                                 d["token_offsets"], d["key"], d["value"], BS, validate=False,
                                                 chained=True)
            done[k].record(compute)
            if k + 1 < count:
                if k >= 1:  # step k-1 has finished reading the buffer of step k+1
                    copies.wait_event(done[k - 1])
                memcpy(devs[(k + 1) % 2]["_buffer"].data_ptr(), host["_buffer"].data_ptr(), h2d, to_dev, copies)
                copied[k + 1].record(copies)
            copies.wait_event(done[k])
            memcpy(outs_host[k % 2].data_ptr(), result.data_ptr(), d2h, to_host, copies)
            results.append(result)
        compute.wait_stream(copies)

    with torch.cuda.stream(capture_stream):
        e2e_steps(2)  # eager warm-up of the copy path
    torch.cuda.synchronize(device)
    e2e_graphs = []
    for count in [per_graph] * min(full, 1) + ([rest] if rest else []):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=capture_stream):
            e2e_steps(count)
        e2e_graphs.append(g)
    e2e_big = e2e_graphs[0] if full else None
    e2e_tail = e2e_graphs[-1] if rest else None

    def run_e2e():
        for _ in range(full):
            e2e_big.replay()
        if e2e_tail is not None:
            e2e_tail.replay()

    for _ in range(max(1, math.ceil(args.warmup / args.steps))):
        run_e2e()
    barrier()
    e2e_windows = []
    for _ in range(min(repeats, 5)):
        e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        e_start.record(stream)
        run_e2e()
        e_end.record(stream)
        barrier()
        e2e_windows.append(e_start.elapsed_time(e_end))
    if world > 1:
        t = torch.tensor(e2e_windows, device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        e2e_windows = [float(v) for v in t.tolist()]
    e2e_ms = statistics.median(e2e_windows)
    del e2e_graphs, e2e_big, e2e_tail
    e2e_value = world * step_bytes / (e2e_ms / args.steps * 1e-3) / 1e9
    status = _lib.device_status(device)
    if status:
        raise RuntimeError(f"device status bits set during the benchmark: {status}")
    del graphs, big, tail, probe
    if rank != 0:
        return None
    line = {
        "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"decode step (KV append + paged attention, one fused launch) of {args.batch} "
                               f"requests x {args.context} tokens per GPU, Hq16/Hkv8/D128, block 16",
                   "global_batch": args.batch * world, "seq_len": args.context,
                   "parallelism": f"request-sharded x{world} (independent KV pools)",
                   "l2": f"inputs {2 * x['key_cache'].numel() * 2 / 1e6:.0f} MB per GPU > 126 MB L2",
                   "timing": f"CUDA graphs of up to {per_graph} consecutive steps (chained launches), "
                             f"{repeats} windows of exactly {args.steps} steps"},
        "windows": {"count": repeats, "steps_each": args.steps, "ms_per_step_median": ms_per_step,
                    "ms_per_step_min": per_step[0], "ms_per_step_max": per_step[-1]},
        "layer_op_tok_s": world * args.batch / (ms_per_step * 1e-3),
        "layer_op_tok_s_note": "requests served per second by ONE layer's append + decode (an operator rate); "
                               "the model's decode tok/s is qwen3.value (BASELINE config 5, all 28 layers)",
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "peak_source": peak_kind,
                     "traffic": ncu_traffic("decode_b32_ctx2048_bf16"),
                     "kernel": "fused KV append + split-KV paged decode (merge in the same launch); one launch per "
                               "step, so its average duration in the timed region is the step time",
                     "bytes_per_launch": step_bytes, "launch_ms": ms_per_step,
                     "launch_isolated_ms": kernel_avg_ms,
                     "frac_isolated": step_bytes / (kernel_avg_ms * 1e-3) / 1e9 / peak,
                     "isolated_note": "one launch alone in a graph between events: its prologue and merge tail "
                                      "are not overlapped with a neighbouring launch"},
        "e2e": {"value": e2e_value, "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "ms_per_step": e2e_ms / args.steps,
                "path": "paged_attention_with_append (Python API), one H2D copy of the packed inputs and one D2H "
                        "copy of the output per step, pinned host buffers; copies on a second stream, pipelined "
                        "across steps (double-buffered device inputs); steps and copies captured in CUDA graphs "
                        "of up to 256 steps, median of the timed windows"},
        "gpu_launches": args.steps * repeats,
        "gpu_launches_note": "one fused append + decode launch per step, in each of the timed windows",
        "clocks": clocks.summary(),
    }
    if world == 1:
        line["cpu_baseline"] = cpu_baseline(args.context, args.cpu_seconds)
    return line


# ------------------------------------------------- BASELINE configs 1-3 (decode)
def config_decode_bytes(c):
    """Algorithmic bytes of one decode call of a case: KV read once + q and out + page-table entries."""
    q, kc = c["query"], c["key_cache"]
    batch, heads, dim = q.shape
    _, bs, kv_heads, _ = kc.shape
    lengths = [int(n) for n in c["context_lens"].tolist()]
    es = q.element_size()
    return (sum(lengths) * 2 * kv_heads * dim * es + 2 * batch * heads * dim * es
            + 8 * sum(math.ceil(n / bs) for n in lengths))


class CpuConfigReference:
    """The reference's CPU path (oracle append + decode, restating data.py:67-81 and fallback.py:27-64) on a case."""

    def __init__(self, c, label):
        from oracle import kv_write, paged_decode

        self.kv_write, self.paged_decode, self.c, self.label = kv_write, paged_decode, c, label
        self.kc, self.vc = c["key_cache"].clone(), c["value_cache"].clone()
        self.nbytes = config_decode_bytes(c)

    def step(self):
        c = self.c
        self.kv_write.write_kv_cache_batch(self.kc, self.vc, c["block_tables"], c["token_offsets"], c["key"],
                                           c["value"], c["block_size"])
        self.paged_decode.paged_attention(c["query"], self.kc, self.vc, c["block_tables"], c["context_lens"],
                                          c["block_size"])

    def describe(self, seconds):
        self.step()
        done, start = 0, time.perf_counter()
        while done < 2 or time.perf_counter() - start < seconds:
            self.step()
            done += 1
        per_step = (time.perf_counter() - start) / done
        threads = torch.get_num_threads()
        return {"value": self.nbytes / per_step / 1e9, "unit": "GB/s", "cores": threads, "kind": "port",
                "ms_per_step": per_step * 1e3,
                "sample": f"{done} steps of the oracle's append + decode on the whole of {self.label}, "
                          f"torch threads={threads}"}


def measure_decode_config(label, c, device, steps, warmup, cpu_seconds, peak):
    """One BASELINE decode config at one GPU: KV append + paged decode, L2 flushed before every step.

    Each replay of a CUDA graph writes a 256 MB buffer (more than the 126 MB L2), then runs the
    step between events; a second graph times the decode launch alone (not chained to the append).
    """
    from myvllm_mini_engine_b200.kernels import paged_attention, write_kv_cache_batch

    g = {k: (v.to(device) if isinstance(v, torch.Tensor) else v) for k, v in c.items()}
    bs = g["block_size"]
    nbytes = config_decode_bytes(c)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)
    events = [torch.cuda.Event(enable_timing=True, external=True) for _ in range(4)]

    def append():
        write_kv_cache_batch(g["key_cache"], g["value_cache"], g["block_tables"], g["token_offsets"], g["key"],
                             g["value"], bs, validate=False)

    def decode(chained):
        return paged_attention(g["query"], g["key_cache"], g["value_cache"], g["block_tables"], g["context_lens"],
                               bs, validate=False, chained=chained)

    side = torch.cuda.Stream(device)
    side.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(side):
        for _ in range(3):
            append()
            out = decode(True)
    side.synchronize()
    step_graph, launch_graph = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
    with torch.cuda.graph(step_graph, stream=side):
        flush.fill_(1)
        events[0].record()
        append()
        out = decode(True)
        events[1].record()
    with torch.cuda.graph(launch_graph, stream=side):
        flush.fill_(1)
        append()
        events[2].record()
        decode(False)
        events[3].record()
    for _ in range(warmup):
        step_graph.replay()
        launch_graph.replay()
    torch.cuda.synchronize(device)
    step_ms, launch_ms = [], []
    for _ in range(max(1, min(steps, 200))):
        step_graph.replay()
        events[1].synchronize()
        step_ms.append(events[0].elapsed_time(events[1]))
        launch_graph.replay()
        events[3].synchronize()
        launch_ms.append(events[2].elapsed_time(events[3]))
    del step_graph, launch_graph
    step_avg, launch_avg = statistics.median(step_ms), statistics.median(launch_ms)
    cpu = CpuConfigReference(c, label).describe(cpu_seconds)
    achieved = nbytes / (launch_avg * 1e-3) / 1e9
    return {"workload": label, "dtype": str(c["query"].dtype).replace("torch.", ""),
            "value": nbytes / (step_avg * 1e-3) / 1e9, "unit": "GB/s (KV-read bytes / step time)",
            "us_per_step": step_avg * 1e3, "decode_launch_us": launch_avg * 1e3, "bytes_per_launch": nbytes,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "frac": achieved / peak,
                         "unit": "GB/s"},
            "l2": "flushed (256 MB write) before every step", "steps": len(step_ms),
            "cpu_baseline": cpu, "vs_cpu": (nbytes / (step_avg * 1e-3) / 1e9) / cpu["value"]}


def run_configs(args, world, rank, local):
    """BASELINE configs 1-3 (decode) and 4 (prefill) at one GPU, and config 5 (Qwen3 step) at every N.

    Returns the fields to add to the headline line (rank 0), or None on other ranks.  Config 5 runs on
    every rank, strong-scaled: 256 requests split over the ranks, each with its own KV pool.
    """
    import copy

    sys.path.insert(0, str(ROOT / "tests" / "golden"))
    import cases

    extra = {}
    device = torch.device("cuda", local)
    peak, _ = measured_peaks()
    if world == 1:
        budget = min(args.cpu_seconds, 3.0)
        for name, build, label in (
                ("config1", cases.config1, "BASELINE config 1: fp32, 1 request, 128 cached + 1 appended, bs16"),
                ("config2", cases.config2, "BASELINE config 2: fp16, 8 requests x 512 + 1, bs256"),
                ("config3", cases.config3, "BASELINE config 3: bf16, 32 requests, contexts U[1,2048] seeded + 1, "
                                           "bs16, pool 1.1x")):
            extra[name] = measure_decode_config(label, build(), device, args.steps, args.warmup, budget, peak)
        sub = copy.copy(args)
        sub.workload, sub.steps, sub.cpu_seconds = "prefill", max(1, min(args.steps, 200)), min(args.cpu_seconds, 5.0)
        line = run_prefill(sub, world, rank, local)
        extra["config4"] = {k: line[k] for k in ("value", "unit", "ms_per_step", "prefill_tokens_s", "roofline", "e2e",
                                                 "cpu_baseline", "clocks")}
        extra["config4"]["workload"] = line["config"]["workload"]
        extra["config4"]["vs_cpu"] = line["value"] / line["cpu_baseline"]["value"]
    sub = copy.copy(args)
    sub.workload, sub.batch, sub.context, sub.kv_dtype = "qwen3", 256, 4096, "bf16"
    sub.steps = max(1, min(args.steps, 30))
    try:
        line = run_qwen3(sub, world, rank, local)
    except SystemExit as error:
        line = {"skipped": str(error)} if rank == 0 else None
    if rank == 0 and line is not None:
        keep = ("value", "unit", "ms_per_step", "scaling", "roofline", "step_roofline", "e2e", "projections",
                "cpu_baseline", "gpu_launches", "clocks", "skipped")
        extra["qwen3"] = {k: line[k] for k in keep if k in line}
        if "config" in line:
            extra["qwen3"]["workload"] = line["config"]["workload"] + f"; {256 // world} requests per GPU"
        if "cpu_baseline" in line:
            extra["qwen3"]["vs_cpu"] = line["value"] / line["cpu_baseline"]["value"]
    return extra if rank == 0 else None


def run_fp8(args, world, rank, local):
    """Decode step over an FP8 pool: the fused quantising KV append + fp8 paged attention, one launch.

    The bf16 pools of the decode workload are quantised once (untimed) by the
    quantising slot scatter; the timed steps are chained fused launches captured
    as graphs of up to 256 steps, as in the bf16 headline.  Bytes per step count
    the KV pool at one byte per element, q and the output at two.
    """
    from myvllm_mini_engine_b200 import _lib
    from myvllm_mini_engine_b200.kernels import paged_attention_fp8_with_append, write_kv_cache_slots_fp8

    device = torch.device("cuda", local)
    x = make_inputs(args.batch, args.context, device, seed=1234 + rank)
    fmt = "e5m2" if args.kv_dtype == "fp8_e5m2" else "e4m3"
    k_scale, v_scale = 4.5 / 448, 4.5 / 448
    pool_rows = x["key_cache"].shape[0] * BS
    kq = torch.empty(x["key_cache"].shape, dtype=torch.uint8, device=device)
    vq = torch.empty_like(kq)
    write_kv_cache_slots_fp8(kq, vq, torch.arange(pool_rows, device=device), x["key_cache"].view(-1, HKV, D),
                             x["value_cache"].view(-1, HKV, D), k_scale, v_scale, kv_format=fmt, validate=False)
    del x["key_cache"], x["value_cache"]
    offsets = (x["context_lens"] - 1).contiguous()
    lengths = [args.context] * args.batch
    step_bytes = kv_bytes(lengths, 1) + 2 * args.batch * HQ * D * 2 + 8 * sum(math.ceil(n / BS) for n in lengths)
    stream = torch.cuda.current_stream(device)

    def step(chained=True):
        return paged_attention_fp8_with_append(x["query"], kq, vq, x["block_tables"], offsets, x["key"], x["value"],
                                               BS, k_scale, v_scale, kv_format=fmt, validate=False, chained=chained)

    capture_stream = torch.cuda.Stream(device)
    capture_stream.wait_stream(stream)
    with torch.cuda.stream(capture_stream):
        for _ in range(3):
            step()
    torch.cuda.synchronize(device)
    per_graph = max(1, min(args.steps, 256))
    full, rest = divmod(args.steps, per_graph)
    graphs = []
    for count in [per_graph] * min(full, 1) + ([rest] if rest else []):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=capture_stream):
            for _ in range(count):
                step()
        graphs.append(g)
    big = graphs[0] if full else None
    tail = graphs[-1] if rest else None

    def run_steps():
        for _ in range(full):
            big.replay()
        if tail is not None:
            tail.replay()

    ev_a = torch.cuda.Event(enable_timing=True, external=True)
    ev_b = torch.cuda.Event(enable_timing=True, external=True)
    probe = torch.cuda.CUDAGraph()
    with torch.cuda.graph(probe, stream=capture_stream):
        ev_a.record()
        step(chained=False)
        ev_b.record()
    for _ in range(max(1, math.ceil(args.warmup / args.steps))):  # at least W untimed steps
        run_steps()
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
        run_steps()
        end.record(stream)
        barrier()
        for _ in range(min(args.steps, 50)):
            probe.replay()
            ev_b.synchronize()
            kernel_ms.append(ev_a.elapsed_time(ev_b))
    elapsed_ms = start.elapsed_time(end)
    if world > 1:
        t = torch.tensor([elapsed_ms], device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        elapsed_ms = float(t.item())
    ms_per_step = elapsed_ms / args.steps
    kernel_avg_ms = statistics.mean(kernel_ms)
    peak, peak_kind = measured_peaks()
    achieved = step_bytes / (kernel_avg_ms * 1e-3) / 1e9
    status = _lib.device_status(device)
    if status:
        raise RuntimeError(f"device status bits set during the benchmark: {status}")
    del graphs, big, tail, probe
    if rank != 0:
        return None
    return {
        "metric": f"fp8 paged-decode KV-read GB/s ({fmt.upper()} pool)", "value": world * step_bytes / (ms_per_step * 1e-3) / 1e9,
        "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": f"{fmt} KV, bf16 q/out",
        "data": "synthetic",
        "config": {"workload": f"decode step (fused quantising KV append + fp8 paged attention) of {args.batch} "
                               f"requests x {args.context} tokens per GPU, Hq16/Hkv8/D128, block 16",
                   "global_batch": args.batch * world, "seq_len": args.context,
                   "parallelism": f"request-sharded x{world} (independent KV pools)",
                   "l2": f"inputs {2 * kq.numel() / 1e6:.0f} MB per GPU > 126 MB L2"},
        "layer_op_tok_s": world * args.batch / (ms_per_step * 1e-3),
        "layer_op_tok_s_note": "requests served per second by ONE layer's append + decode (an operator rate); "
                               "the model's decode tok/s is qwen3.value (BASELINE config 5, all 28 layers)",
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "peak_source": peak_kind, "traffic": None,
                     "kernel": "fused fp8 KV append + paged decode, one launch timed alone between events",
                     "bytes_per_launch": step_bytes, "launch_ms": kernel_avg_ms,
                     "step_frac": step_bytes / (ms_per_step * 1e-3) / 1e9 / peak},
        "e2e": None, "gpu_launches": args.steps, "clocks": clocks.summary(),
    }


# ------------------------------------------------- config 5: Qwen3 decode step
QWEN3_SEED = 2025


def qwen3_config():
    from myvllm_mini_engine_b200.engine.qwen3 import Qwen3Config
    return Qwen3Config.qwen3_0_6b()


def qwen3_weight_bytes(cfg, esize=2):
    """Weights one step reads: every projection of every layer, the norms, and the tied LM head once."""
    h, d, i = cfg.hidden_size, cfg.head_dim, cfg.intermediate_size
    per_layer = ((cfg.num_attention_heads + 2 * cfg.num_key_value_heads) * d * h + h * cfg.num_attention_heads * d
                 + 2 * i * h + h * i + 2 * h + 2 * d)
    return esize * (cfg.num_hidden_layers * per_layer + cfg.vocab_size * h + h)


def qwen3_tables(batch, pages, device, seed):
    """Seeded permutation of a pool holding exactly ``batch * pages`` pages."""
    gen = torch.Generator(device=device).manual_seed(seed)
    perm = torch.randperm(batch * pages, device=device, generator=gen)
    return perm.view(batch, pages).contiguous()


class CpuQwen3Reference:
    """The reference model's decode step on the host cores (oracle restatement) on a bounded sample."""

    SAMPLE_BATCH = 1

    def __init__(self, context, threads=None):
        from myvllm_mini_engine_b200.engine.qwen3 import Qwen3Weights
        from oracle import qwen3 as oracle_qwen3

        if threads:
            torch.set_num_threads(threads)
        self.oracle = oracle_qwen3
        self.cfg = cfg = qwen3_config()
        self.context = context
        self.weights = Qwen3Weights.random(cfg, dtype=torch.bfloat16, device="cpu", seed=QWEN3_SEED)
        pages = math.ceil((context + 1) / BS)
        shape = (cfg.num_hidden_layers, self.SAMPLE_BATCH * pages, BS, cfg.num_key_value_heads, cfg.head_dim)
        gen = torch.Generator().manual_seed(QWEN3_SEED + 7)
        self.key = torch.randn(shape, generator=gen).to(torch.bfloat16)
        self.value = torch.randn(shape, generator=gen).to(torch.bfloat16)
        self.tables = torch.arange(self.SAMPLE_BATCH * pages, dtype=torch.int64).view(self.SAMPLE_BATCH, pages)
        self.ids = torch.randint(0, cfg.vocab_size, (self.SAMPLE_BATCH,), generator=gen)
        self.positions = torch.full((self.SAMPLE_BATCH,), context, dtype=torch.int64)

    def step(self):
        self.oracle.decode_step(self.cfg, self.weights, self.ids, self.key, self.value, self.tables, self.positions)

    def timed(self, seconds=0.0, min_steps=1, max_steps=None):
        done, start = 0, time.perf_counter()
        while done < min_steps or (time.perf_counter() - start < seconds and (max_steps is None or done < max_steps)):
            self.step()
            done += 1
        return (time.perf_counter() - start) / done, done

    def describe(self, per_step, done):
        threads = torch.get_num_threads()
        return {"value": self.SAMPLE_BATCH / per_step, "unit": "tok/s", "cores": threads, "kind": "port",
                "sample": f"{done} decode steps of the oracle restating NativeQwen3.forward_decode_batch "
                          f"(native_qwen3.py:423-456, torch backends, bf16) on {self.SAMPLE_BATCH} request x "
                          f"{self.context} cached tokens, 28 layers, {per_step * 1e3:.0f} ms/step, "
                          f"torch threads={threads}"}


def qwen3_line_base(args, world, kind):
    return {"metric": METRIC, "unit": "tok/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (random N(0,0.02) weights, N(0,1) KV history, uniform token ids)",
            "config": {"workload": f"Qwen3-0.6B-architecture batch decode step (BASELINE config 5): "
                                   f"{args.batch} requests x {args.context} cached tokens (+1 appended), 28 layers, "
                                   f"hidden 1024, 16/8 heads x 128, SwiGLU 3072, vocab 151936 tied, block 16, "
                                   f"greedy", "model": "qwen3-0.6b-arch", "global_batch": args.batch,
                       "seq_len": args.context, "parallelism": kind,
                       "l2": "KV pool per GPU >> 126 MB L2"}}


def run_qwen3_reference(args, world, rank):
    if rank != 0:
        return None
    ref = CpuQwen3Reference(args.context, threads=os.cpu_count() or 1)
    ref.timed(0.0, min(args.warmup, 1))
    per_step, done = ref.timed(60.0, 2, args.steps)
    base = ref.describe(per_step, done)
    line = qwen3_line_base(args, world, "rank 0 only, host cores")
    line.update({"value": base["value"], "impl": "reference", "ms_per_step": per_step * 1e3, "cpu_baseline": base,
                 "e2e": {"value": base["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}})
    return line


def run_qwen3(args, world, rank, local):
    from myvllm_mini_engine_b200 import _lib
    from myvllm_mini_engine_b200.cache.kv_cache import FP8KVCachePool, PagedKVPool
    from myvllm_mini_engine_b200.engine.qwen3 import DecodeGraph, Qwen3DecodeStep, Qwen3Weights
    from myvllm_mini_engine_b200.kernels import paged_attention, paged_attention_fp8

    fmt = {"fp8": "e4m3", "fp8_e5m2": "e5m2"}.get(args.kv_dtype)  # None: bf16 pool
    kv_es = 1 if fmt else 2
    if args.batch % world:
        raise SystemExit(f"--batch {args.batch} does not split over {world} GPUs")
    device = torch.device("cuda", local)
    cfg = qwen3_config()
    batch = args.batch // world
    pages = math.ceil((args.context + 1) / BS)
    blocks = batch * pages
    pool_bytes = 2 * cfg.num_hidden_layers * blocks * BS * cfg.num_key_value_heads * cfg.head_dim * kv_es
    free, _ = torch.cuda.mem_get_info(device)
    if pool_bytes + (4 << 30) > free:
        raise SystemExit(f"KV pool of {pool_bytes / 1e9:.1f} GB does not fit the {free / 1e9:.1f} GB free on "
                         f"GPU {local}")
    weights = Qwen3Weights.random(cfg, dtype=torch.bfloat16, device=device, seed=QWEN3_SEED)
    gen = torch.Generator(device=device).manual_seed(QWEN3_SEED + 1 + rank)
    if fmt:
        # FP8 pool: N(0,1) history quantised by the pool's own scatter (scale 1/32: |x| < 14 fits E4M3)
        pool = FP8KVCachePool(cfg.num_hidden_layers, blocks, BS, cfg.num_key_value_heads, cfg.head_dim,
                              k_scale=1 / 32, v_scale=1 / 32, kv_format=fmt, device=device)
        rows = torch.empty(blocks * BS, cfg.num_key_value_heads, cfg.head_dim, dtype=torch.bfloat16, device=device)
        slots = torch.arange(blocks * BS, device=device)
        for layer in range(cfg.num_hidden_layers):
            rows.normal_(generator=gen)
            pool.write_slots(layer, slots, rows, rows.flip(0), validate=False)
        del rows, slots
    else:
        pool = PagedKVPool(cfg.num_hidden_layers, blocks, BS, cfg.num_key_value_heads, cfg.head_dim,
                           dtype=torch.bfloat16, device=device)
        for layer in range(cfg.num_hidden_layers):
            pool.key[layer].normal_(generator=gen)
            pool.value[layer].normal_(generator=gen)
    tables = qwen3_tables(batch, pages, device, QWEN3_SEED + 100 + rank)
    ids = torch.randint(0, cfg.vocab_size, (batch,), device=device, generator=gen)
    positions = torch.full((batch,), args.context, dtype=torch.int64, device=device)
    step = Qwen3DecodeStep(cfg, weights, pool, fused_projections=args.projections == "fused")
    fused = step.fused_projections and batch <= step.FUSED_MAX_BATCH  # the path this batch takes
    graph = DecodeGraph(step, batch, pages)
    graph.load(ids, positions, tables)
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize(device)
    stream = torch.cuda.current_stream(device)

    def barrier():
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize(device)

    def max_over_ranks(ms):
        if world > 1:
            t = torch.tensor([ms], device=device)
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        barrier()
        start.record(stream)
        for _ in range(args.steps):
            graph.replay()
        end.record(stream)
        barrier()
    ms_per_step = max_over_ranks(start.elapsed_time(end)) / args.steps

    # the dominant kernel alone: paged decode over this rank's batch, one launch per layer, graph-replayed
    lengths = [args.context + 1] * batch
    launch_bytes = kv_bytes(lengths, kv_es) + 2 * batch * HQ * D * 2 + 8 * sum(math.ceil(n / BS) for n in lengths)
    q = torch.randn(batch, HQ, D, device=device, dtype=torch.bfloat16, generator=gen)
    lens = positions + 1

    def attend(layer):
        if fmt:
            return pool.attend(layer, q, tables, lens, validate=False)
        return paged_attention(q, pool.key[layer], pool.value[layer], tables, lens, BS, validate=False)

    side = torch.cuda.Stream(device)
    side.wait_stream(stream)
    with torch.cuda.stream(side):
        attend(0)
    side.synchronize()
    decode_graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(decode_graph, stream=side):
        for layer in range(cfg.num_hidden_layers):
            attend(layer)
    decode_graph.replay()
    torch.cuda.synchronize(device)
    d_start, d_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = max(1, min(args.steps, 20))
    d_start.record(stream)
    for _ in range(reps):
        decode_graph.replay()
    d_end.record(stream)
    torch.cuda.synchronize(device)
    launch_ms = d_start.elapsed_time(d_end) / (reps * cfg.num_hidden_layers)
    achieved = launch_bytes / (launch_ms * 1e-3) / 1e9
    peak, peak_kind = measured_peaks()

    # end to end through the graph API: host metadata in, host token ids out, every step
    host_ids, host_pos, host_tables = (t.cpu().pin_memory() for t in (ids, positions, tables))
    out_host = torch.empty(batch, dtype=torch.int64, pin_memory=True)
    h2d = sum(t.numel() * t.element_size() for t in (host_ids, host_pos, host_tables))
    d2h = out_host.numel() * out_host.element_size()

    def e2e_step():
        graph.load(host_ids, host_pos, host_tables)
        out_host.copy_(graph.replay(), non_blocking=True)

    for _ in range(min(args.warmup, 3)):
        e2e_step()
    barrier()
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e_start.record(stream)
    for _ in range(args.steps):
        e2e_step()
    e_end.record(stream)
    barrier()
    e2e_ms = max_over_ranks(e_start.elapsed_time(e_end)) / args.steps
    status = _lib.device_status(device)
    if status:
        raise RuntimeError(f"device status bits set during the benchmark: {status}")
    del graph, decode_graph
    if rank != 0:
        return None
    step_bytes = cfg.num_hidden_layers * (launch_bytes + 2 * batch * HKV * D * kv_es) + qwen3_weight_bytes(cfg)
    line = qwen3_line_base(args, world, f"request-sharded x{world} ({batch} requests and an independent KV "
                                        f"pool per GPU, weights replicated, no collective)")
    line["config"]["kv_pool"] = fmt or "bf16"
    if fmt:
        line["dtype"] = f"bf16 compute, {fmt} KV pool (scales 1/32)"
    line.update({
        "value": args.batch / (ms_per_step * 1e-3), "ms_per_step": ms_per_step,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "peak_source": peak_kind, "traffic": ncu_traffic("qwen3_decode_b256_ctx4097_bf16"),
                     "kernel": f"paged decode, {batch} requests x {args.context + 1} tokens per launch",
                     "bytes_per_launch": launch_bytes, "launch_ms": launch_ms},
        "step_roofline": {"bytes_per_step": step_bytes, "achieved": step_bytes / (ms_per_step * 1e-3) / 1e9,
                          "frac": step_bytes / (ms_per_step * 1e-3) / 1e9 / peak, "unit": "GB/s",
                          "decode_share": cfg.num_hidden_layers * launch_ms / ms_per_step},
        "e2e": {"value": args.batch / (e2e_ms * 1e-3), "unit": "tok/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms},
        "gpu_launches": ((5 * cfg.num_hidden_layers + 4) if fused else (5 * cfg.num_hidden_layers + 3)) * args.steps,
        "gpu_launches_note": ("libminikv kernels only: per layer the q|k|v, o, gate|up and down projections "
                              "(tcgen05, element-wise steps fused) and the paged decode, plus the first and the "
                              "final RMSNorm and the greedy argmax (two launches); the LM head is cuBLAS" if fused else
                              "libminikv kernels only (RMSNorm x2, qk-norm+RoPE+append, paged decode, SiLU*up per "
                              "layer, plus the first RMSNorm and the greedy argmax, two launches); the 4 projections per layer "
                              "and the LM head are cuBLAS"),
        "projections": "fused tcgen05" if fused else "cublas",
        "clocks": clocks.summary(),
    })
    if world == 1:
        ref = CpuQwen3Reference(args.context)
        ref.timed(0.0, 1)
        per_step, done = ref.timed(args.cpu_seconds, 2)
        line["cpu_baseline"] = ref.describe(per_step, done)
    return line


# ------------------------------------------- config 4: ragged chunked prefill
def prefill_flops(starts, chunk, heads=HQ, dim=D):
    """Causal (query, key) pairs x 4 Hq D: query i of a chunk starting at s attends s + i + 1 keys."""
    return sum(4 * heads * dim * (chunk * s + chunk * (chunk + 1) // 2) for s in starts)


def config4_inputs(device):
    sys.path.insert(0, str(ROOT / "tests" / "golden"))
    import cases
    return cases.config4()


class CpuPrefillReference:
    """The reference's torch prefill path on the host cores (oracle restatement), whole config 4."""

    def __init__(self, threads=None):
        from oracle import kv_write, metadata, prefill

        if threads:
            torch.set_num_threads(threads)
        c = config4_inputs("cpu")
        self.c, self.prefill = c, prefill
        self.kc, self.vc = c["key_cache"].clone(), c["value_cache"].clone()
        meta = metadata.prefill_metadata(c["tokens"], c["cow_tables"], c["starts"], block_size=c["block_size"],
                                         num_blocks=c["num_blocks"])
        self.t = {k: torch.tensor(v, dtype=torch.int64) for k, v in meta.items()}
        kv_write.copy_blocks(self.kc.unsqueeze(0), self.vc.unsqueeze(0), [c["cow_pair"]])
        kv_write.write_kv_cache_slots(self.kc, self.vc, self.t["slot_mapping"], c["key"], c["value"])
        self.flops = prefill_flops(c["starts"], 128)

    def step(self):
        t = self.t
        self.prefill.paged_prefill_fp32(self.c["q"], self.kc, self.vc, t["cu_seqlens_q"], t["query_starts"],
                                        t["block_tables"], t["context_lens"], self.c["block_size"])

    def timed(self, seconds, min_steps, max_steps=None):
        done, start = 0, time.perf_counter()
        while done < min_steps or (time.perf_counter() - start < seconds and (max_steps is None or done < max_steps)):
            self.step()
            done += 1
        return (time.perf_counter() - start) / done, done

    def describe(self, per_step, done):
        threads = torch.get_num_threads()
        return {"value": self.flops / per_step / 1e12, "unit": "TFLOP/s", "cores": threads, "kind": "port",
                "sample": f"{done} runs of the oracle's paged prefill (restating kernels/prefill.py:114-131, "
                          f"torch path in fp32) over all of config 4 (16 x 128-token chunks), "
                          f"{per_step * 1e3:.0f} ms/run, torch threads={threads}"}


PREFILL_METRIC = "paged-prefill TFLOP/s (BASELINE config 4: CoW + slot scatter + ragged prefill)"


def prefill_line_base(args, world):
    return {"metric": PREFILL_METRIC, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "BASELINE config 4: copy-on-write of a shared prefix page, slot scatter of "
                                   "16 x 128-token chunks, ragged causal paged prefill over prefixes U[0,1024] "
                                   "(8 requests share 32 pages), Hq16/Hkv8/D128, bf16, block 16",
                       "global_batch": 16 * world, "seq_len": 128, "parallelism": f"independent x{world}",
                       "l2": "L2 flushed (256 MB write) before every timed step"}}


def run_prefill_reference(args, world, rank):
    if rank != 0:
        return None
    ref = CpuPrefillReference(threads=os.cpu_count() or 1)
    ref.timed(0.0, 1)
    per_step, done = ref.timed(60.0, 3, args.steps)
    base = ref.describe(per_step, done)
    line = prefill_line_base(args, world)
    line.update({"value": base["value"], "impl": "reference", "ms_per_step": per_step * 1e3, "cpu_baseline": base,
                 "e2e": {"value": base["value"], "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                         "d2h_bytes_per_step": 0}})
    return line


def run_prefill(args, world, rank, local):
    """BASELINE config 4 as one step: copy-on-write, slot scatter, ragged prefill.  With
    ``--kv-dtype fp8`` / ``fp8_e5m2`` the pool holds E4M3 / E5M2 codes: the CoW moves bytes, the
    scatter quantises, and the prefill is ``paged_prefill_attention_fp8``."""
    from myvllm_mini_engine_b200 import _lib
    from myvllm_mini_engine_b200.engine import PrefillBatch
    from myvllm_mini_engine_b200.kernels import (copy_blocks, paged_prefill_attention, paged_prefill_attention_fp8,
                                                 write_kv_cache_slots, write_kv_cache_slots_fp8)

    device = torch.device("cuda", local)
    c = config4_inputs(device)
    bs, chunk = c["block_size"], 128
    flops = prefill_flops(c["starts"], chunk)
    fmt = {"fp8": "e4m3", "fp8_e5m2": "e5m2"}.get(args.kv_dtype)  # None: 16-bit pool
    k_scale = v_scale = 4.5 / 448
    gk, gv = c["key_cache"].to(device), c["value_cache"].to(device)
    if fmt is not None:
        rows = gk.shape[0] * bs
        kq, vq = (torch.empty(gk.shape, dtype=torch.uint8, device=device) for _ in range(2))
        write_kv_cache_slots_fp8(kq, vq, torch.arange(rows, device=device), gk.view(rows, HKV, D),
                                 gv.view(rows, HKV, D), k_scale, v_scale, kv_format=fmt, validate=False)
        gk, gv = kq, vq
    words = (lambda t: t.view(torch.float16)) if fmt is not None else (lambda t: t)  # CoW moves 16-bit words
    q, key, value = (c[k].to(device) for k in ("q", "key", "value"))
    pairs = torch.tensor([list(c["cow_pair"])], dtype=torch.int64, device=device)
    batch = PrefillBatch.from_sequences(c["tokens"], c["cow_tables"], c["starts"], block_size=bs,
                                        num_blocks=c["num_blocks"], device=device)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)
    events = [torch.cuda.Event(enable_timing=True, external=True) for _ in range(3)]

    def scatter(k_rows, v_rows):
        if fmt is None:
            write_kv_cache_slots(gk, gv, batch.slot_mapping, k_rows, v_rows, validate=False)
        else:
            write_kv_cache_slots_fp8(gk, gv, batch.slot_mapping, k_rows, v_rows, k_scale, v_scale, kv_format=fmt,
                                     validate=False)

    def attend(q_rows):
        meta = (batch.cu_seqlens_q, batch.query_starts, batch.block_tables, batch.context_lens)
        if fmt is None:
            return paged_prefill_attention(q_rows, gk, gv, *meta, bs, validate=False, max_query_len=chunk)
        return paged_prefill_attention_fp8(q_rows, gk, gv, *meta, bs, k_scale, v_scale, kv_format=fmt,
                                           validate=False, max_query_len=chunk)

    def step(timed=False):
        copy_blocks(words(gk).unsqueeze(0), words(gv).unsqueeze(0), pairs, validate=False)
        scatter(key, value)
        if timed:
            events[1].record()
        return attend(q)

    side = torch.cuda.Stream(device)
    side.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(side):
        for _ in range(3):
            step()
    side.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        flush.fill_(1)
        events[0].record()
        out = step(timed=True)
        events[2].record()
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize(device)
    steps = max(1, min(args.steps, 2000))
    step_ms, prefill_ms = [], []
    with ClockSampler(local) as clocks:
        for _ in range(steps):
            graph.replay()
            events[2].synchronize()
            step_ms.append(events[0].elapsed_time(events[2]))
            prefill_ms.append(events[1].elapsed_time(events[2]))
    step_avg, prefill_avg = statistics.mean(step_ms), statistics.mean(prefill_ms)
    if world > 1:
        t = torch.tensor([step_avg, prefill_avg], device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        step_avg, prefill_avg = (float(x) for x in t.tolist())
    peak = 1630.4
    path = ROOT / "MEASURED_PEAKS.json"
    peak_kind = "fallback"
    if path.is_file():
        peak, peak_kind = float(json.loads(path.read_text())["bf16_tflops"]), "measured (burst)"

    # end to end: the chunk's q/k/v from pinned host memory, the output back to the host, every step
    host = {k: c[k].pin_memory() for k in ("q", "key", "value")}
    dev = {k: torch.empty_like(v, device=device) for k, v in host.items()}
    out_host = torch.empty(out.shape, dtype=out.dtype, pin_memory=True)

    def e2e_step():
        for k, t in host.items():
            dev[k].copy_(t, non_blocking=True)
        copy_blocks(words(gk).unsqueeze(0), words(gv).unsqueeze(0), pairs, validate=False)
        scatter(dev["key"], dev["value"])
        out_host.copy_(attend(dev["q"]), non_blocking=True)

    for _ in range(3):
        e2e_step()
    torch.cuda.synchronize(device)
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    stream = torch.cuda.current_stream(device)
    e_start.record(stream)
    for _ in range(steps):
        flush.fill_(1)
        e2e_step()
    e_end.record(stream)
    torch.cuda.synchronize(device)
    e2e_ms = e_start.elapsed_time(e_end) / steps
    status = _lib.device_status(device)
    if status:
        raise RuntimeError(f"device status bits set during the benchmark: {status}")
    del graph
    if rank != 0:
        return None
    line = prefill_line_base(args, world)
    achieved = flops / (prefill_avg * 1e-3) / 1e12
    kv_read = sum(min(len(t) * bs, s + chunk) for t, s in zip(c["cow_tables"], c["starts"])) * 2 * HKV * D * \
        (1 if fmt is not None else 2)
    if fmt is not None:
        line["dtype"] = f"{fmt} KV codes, fp16 MMAs (fp32 accumulate)"
        line["metric"] = PREFILL_METRIC.replace("ragged prefill", f"ragged prefill over an {fmt.upper()} pool")
        line["config"]["workload"] = line["config"]["workload"].replace(
            "bf16, block 16", f"bf16 query, {fmt.upper()} KV pool (per-pool scales), block 16")
    line.update({
        "value": world * flops / (step_avg * 1e-3) / 1e12, "ms_per_step": step_avg, "steps": steps,
        "prefill_tokens_s": world * 16 * chunk / (step_avg * 1e-3),
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": achieved / peak, "peak_source": peak_kind,
                     "traffic": ncu_traffic("prefill_config4_bf16" if fmt is None else f"prefill_config4_{fmt}"),
                     "kernel": "paged prefill (tcgen05 + TMEM, TMA page boxes) per launch" if fmt is None else
                               "paged prefill (tcgen05 + TMEM; FP8 page boxes converted to fp16 in shared memory) "
                               "per launch",
                     "flops_per_launch": flops, "kv_bytes_per_launch": kv_read,
                     "launch_ms": prefill_avg},
        "e2e": {"value": world * flops / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
                "h2d_bytes_per_step": sum(t.numel() * t.element_size() for t in host.values()),
                "d2h_bytes_per_step": out_host.numel() * out_host.element_size(), "ms_per_step_with_flush": e2e_ms},
        "gpu_launches": 3 * steps,
        "clocks": clocks.summary(),
    })
    if world == 1:
        ref = CpuPrefillReference()
        ref.timed(0.0, 1)
        per_step, done = ref.timed(args.cpu_seconds, 2)
        line["cpu_baseline"] = ref.describe(per_step, done)
    return line


def main(argv=None):
    args = parse_args(argv)
    world, rank, local = dist_setup(args)
    try:
        if args.workload == "qwen3":
            line = run_qwen3_reference(args, world, rank) if args.impl == "reference" else \
                run_qwen3(args, world, rank, local)
        elif args.workload == "prefill":
            line = run_prefill_reference(args, world, rank) if args.impl == "reference" else \
                run_prefill(args, world, rank, local)
        else:
            if args.impl == "reference":
                line = run_reference(args, world, rank)
            elif args.kv_dtype in ("fp8", "fp8_e5m2"):
                line = run_fp8(args, world, rank, local)
            else:
                line = run_ours(args, world, rank, local)
                if not args.headline_only:
                    extra = run_configs(args, world, rank, local)
                    if rank == 0:
                        line.update(extra)
        if line is not None and rank == 0:
            print(json.dumps(line), flush=True)
    finally:
        if world > 1 and torch.distributed.is_initialized():
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
