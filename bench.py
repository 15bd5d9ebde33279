#!/usr/bin/env python
"""Benchmark of the fused packed-KV dequantize + decode-attention path on B200.

Metric: packed-KV GB/s (K+V codes plus K+V FP16 scales of the selected blocks, per decode)
and microseconds per layer-decode, for the 128K-token INT4 GQA configuration: 1 layer,
131072 tokens, 8 KV heads x 128 dims, 32 query heads, block 128, group 32.

  python bench.py [--gpus N] [--steps K] [--warmup W]           # this implementation
  python bench.py --impl reference [--steps K] [--warmup W]      # reference CPU decode

N > 1 runs one rank per GPU (launched by torch.distributed.run): the context is N x 131072
tokens split by token-block ranges; each rank decodes its 1024 blocks, and the same kernel
pushes its combined (out, lse) slices to every rank over NVLink peer stores and merges all
ranks' slices exactly, so a step is one kernel per rank (weak scaling; at N = 8 this is the
1M-token configuration).
"""

from __future__ import annotations

import argparse
import csv
import datetime
import io
import json
import math
import os
import shutil
import statistics
import subprocess
import sys
import tempfile
import time
from dataclasses import replace
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "kvssd-attention_b200"))

import numpy as np  # noqa: E402
import torch  # noqa: E402

METRIC = "packed-KV GB/s & us/layer-decode (128K INT4 GQA), % HBM peak"
WORKLOAD = "c2"
FALLBACK_HBM_GBS = 6650.0


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--copies", type=int, default=3,
                    help="input copies rotated between steps so no step reads from L2")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-pipeline", action="store_true",
                    help="skip the KVSSDPipeline and record-decode legs")
    ap.add_argument("--path", choices=["auto", "stream", "cpasync", "regs", "generic"],
                    default="auto",
                    help="A/B: force the tensor-core family (TMA-fed streaming where it "
                         "qualifies), the cp.async-fed streaming, register-fed or CUDA-core kernel")
    ap.add_argument("--eager", action="store_true",
                    help="launch the timed device-resident steps one by one instead of "
                         "replaying them from a CUDA graph")
    ap.add_argument("--kernel-only", action="store_true",
                    help="profiling aid: only the device-timed decode loop (no roofline leg, "
                         "e2e leg or CPU baseline)")
    ap.add_argument("--cpu-seconds", type=float, default=10.0,
                    help="target duration of the CPU-baseline sample")
    return ap.parse_args()


def peaks() -> tuple[float, str]:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        try:
            return float(json.loads(path.read_text())["hbm_gbs"]), "measured"
        except (KeyError, ValueError):
            pass
    return FALLBACK_HBM_GBS, "fallback"


class ClockSampler:
    """nvidia-smi clock/throttle samples every 200 ms while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=self.file, stderr=subprocess.DEVNULL)
        except (FileNotFoundError, OSError):
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict | None:
        if self.proc is None:
            return None
        self.file.flush()
        text = Path(self.file.name).read_text()
        rows = [r for r in csv.reader(io.StringIO(text)) if len(r) >= 9]
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].strip().replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].strip().replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].strip() == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(rows)}


def cpu_threads() -> int:
    """Host threads the oracle uses: one worker per logical CPU (see kvssd_oracle.decode)."""
    return os.cpu_count() or 1


def sample_blocks() -> int:
    """Blocks per CPU sample: 8-block chunks, several per host thread, at most a full layer."""
    return min(1024, max(64, 8 * cpu_threads()))


def cpu_oracle_run(seconds: float, blocks: int | None = None, min_runs: int = 1) -> dict:
    """Times the oracle (numpy restatement of kvssd's reference backend) on a bounded sample
    of the benchmark workload with the same shapes and distributions."""
    from kvssd_b200.workloads import WORKLOADS, make_layer
    from oracle import kvssd_oracle as orc

    blocks = blocks or sample_blocks()
    w = replace(WORKLOADS[WORKLOAD], tokens=blocks * WORKLOADS[WORKLOAD].block_tokens)
    layer = make_layer(w, 0, "cpu")
    args = [t.numpy() for t in (layer.packed_k, layer.packed_v, layer.scales_k, layer.scales_v,
                                layer.valid_tokens)]
    q = layer.query.float().numpy()
    nbytes = blocks * w.bytes_per_block
    runs, t0 = 0, time.perf_counter()
    while runs < min_runs or time.perf_counter() - t0 < seconds:
        orc.decode(q, *args, w.bits, w.group_size, 1 / math.sqrt(w.head_dim))
        runs += 1
    dt = time.perf_counter() - t0
    return {"value": nbytes * runs / dt / 1e9, "unit": "GB/s", "cores": cpu_threads(),
            "kind": "port", "seconds": dt, "runs": runs,
            "sample": f"{blocks} of 1024 blocks ({blocks * w.block_tokens} tokens) of the c2 "
                      f"workload shape per run, {runs} runs; numpy restatement of "
                      "src/kvssd/backends/reference.py, 8-block chunks on "
                      f"{cpu_threads()} host threads merged exactly"}


def workload_text(world: int) -> str:
    """The workload both arms report (the reference arm measures a bounded sample of it)."""
    return (f"{WORKLOAD}: 1 layer x 131072 tokens per GPU, INT4 group 32 FP16 scales, 8 KV heads "
            "x 128, 32 query heads (GQA 4), block 128, AllBlocks"
            + (f"; {world} GPUs split one {world * 131072}-token context by token-block ranges; "
               "each rank's decode kernel pushes its combined slices to every rank over NVLink "
               "peer stores and merges them exactly (one kernel per rank per step)"
               if world > 1 else ""))


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from kvssd_b200.workloads import WORKLOADS, make_layer
    from oracle import kvssd_oracle as orc

    blocks = sample_blocks()
    w = replace(WORKLOADS[WORKLOAD], tokens=blocks * WORKLOADS[WORKLOAD].block_tokens)
    layer = make_layer(w, 0, "cpu")
    tensors = [t.numpy() for t in (layer.packed_k, layer.packed_v, layer.scales_k,
                                   layer.scales_v, layer.valid_tokens)]
    q = layer.query.float().numpy()
    step = lambda: orc.decode(q, *tensors, w.bits, w.group_size, 1 / math.sqrt(w.head_dim))  # noqa: E731
    for _ in range(max(args.warmup, 0)):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = (time.perf_counter() - t0) / args.steps
    nbytes = blocks * w.bytes_per_block
    value = nbytes / dt / 1e9
    emit({
        "impl": "reference", "metric": METRIC, "value": value, "unit": "GB/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": dt * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": workload_text(1),
                   "sample": f"{blocks} of the 1024 blocks per step, timed on the host cores",
                   "kv_heads": w.kv_heads, "head_dim": w.head_dim, "query_heads": w.query_heads,
                   "block_tokens": w.block_tokens, "bits": w.bits, "group_size": w.group_size},
        "cpu_baseline": {"value": value, "unit": "GB/s", "cores": cpu_threads(), "kind": "port",
                         "sample": f"{blocks} blocks ({blocks * w.block_tokens} tokens) of the c2 "
                                   "shape per step; numpy restatement of kvssd's reference "
                                   "backend, 8-block chunks on all host threads merged exactly "
                                   "(the reference is Python and is not installed on the GPU "
                                   "host)"},
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    })


def pipeline_legs(w, base, q, scale, device, rank, args) -> dict:
    """Times KVSSDPipeline.decode end to end from a store file of the layer, and the on-GPU
    record decode alone on the layer's records in HBM."""
    from kvssd_b200 import CacheSpec, KVCacheStore, KVSSDPipeline, ops
    from kvssd_b200.format import PackedKVBlock
    from kvssd_b200.quant import QuantizedTensor

    spec = CacheSpec(1, w.kv_heads, w.head_dim, w.block_tokens, w.bits, w.group_size)
    shape = (w.block_tokens, w.kv_heads, w.head_dim)
    kp, vp = base.packed_k.cpu(), base.packed_v.cpu()
    ks, vs, valid = base.scales_k.cpu(), base.scales_v.cpu(), base.valid_tokens.cpu()
    blocks = (PackedKVBlock(0, b, int(valid[b]),
                            QuantizedTensor(kp[b], ks[b], shape, w.bits, w.group_size),
                            QuantizedTensor(vp[b], vs[b], shape, w.bits, w.group_size))
              for b in range(kp.shape[0]))
    root = Path(tempfile.mkdtemp(prefix=f"kvssd_bench_r{rank}_", dir="/dev/shm"
                                 if Path("/dev/shm").is_dir() else None))
    store = KVCacheStore.from_blocks(root, spec, blocks)
    record_bytes = kp.shape[0] * spec.record_bytes
    try:
        pipe = KVSSDPipeline(store, device=device, io_depth=8, stage_blocks=128,
                             require_cuda_kernel=True)
        qh = q.float()
        for _ in range(2):
            pipe.decode(qh, 0)
        torch.cuda.synchronize(device)
        steps = max(2, min(args.steps, 5))
        t0 = time.perf_counter()
        for _ in range(steps):
            out = pipe.decode(qh, 0)
            out.cpu()
        pipe_s = (time.perf_counter() - t0) / steps
        raw = store.read_records(0, store.blocks_for_layer(0)).to(device)
        for _ in range(3):
            ops.decode_records(raw, spec, 0)
        torch.cuda.synchronize(device)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(10):
            ops.decode_records(raw, spec, 0)
        e1.record()
        torch.cuda.synchronize(device)
        rec_ms = e0.elapsed_time(e1) / 10
        pipe.close()
    finally:
        store.close()
        shutil.rmtree(root, ignore_errors=True)
    nbytes = w.blocks_per_layer * w.bytes_per_block
    return {
        "KVSSDPipeline_decode": {
            "value": nbytes / pipe_s / 1e9, "unit": "GB/s", "ms_per_step": pipe_s * 1e3,
            "path": "KVSSDPipeline(store, stage_blocks=128, io_depth=8).decode(query, 0): "
                    "store file in /dev/shm (page cache), native record reads, H2D, on-GPU "
                    "record decode with CRC-32, fused decode, chunk merge; host wall clock"},
        "record_decode_on_gpu": {
            "value": record_bytes / (rec_ms * 1e-3) / 1e9, "unit": "GB/s of records",
            "us_per_layer": rec_ms * 1e3,
            "note": "1024 raw records resident in HBM -> PackedBatch + CRC-32 check"},
    }


def graph_time(fn, device, reps: int = 20) -> float:
    """Device ms per call of ``fn``: ``reps`` calls captured in one CUDA graph (after 3 eager
    warm-up calls and one on the capture stream), one warm replay, then one timed replay."""
    stream = torch.cuda.current_stream(device)
    for _ in range(3):
        fn()
    side = torch.cuda.Stream(device)
    side.wait_stream(stream)
    with torch.cuda.stream(side):
        fn()
    stream.wait_stream(side)
    torch.cuda.synchronize(device)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=side):
        for _ in range(reps):
            fn()
    g.replay()
    torch.cuda.synchronize(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    g.replay()
    e1.record(stream)
    torch.cuda.synchronize(device)
    del g
    return e0.elapsed_time(e1) / reps


def c4_legs(w, base, device, args) -> dict:
    """The multi-layer step of c4 on one GPU: 32 layers x 65536 tokens (each layer 512 blocks of
    distinct memory: halves of 16 copies of this workload's pool), each with its own query,
    decoded by one batched launch and by 32 single decodes; CUDA-graph replays, device time."""
    from kvssd_b200 import ops

    layers, per = 32, w.blocks_per_layer // 2
    copies = [[t.clone() for t in (base.packed_k, base.packed_v, base.scales_k, base.scales_v,
                                   base.valid_tokens)] for _ in range(layers // 2)]
    pools = [[t[h * per:(h + 1) * per] for t in copies[i // 2]] for i, h in
             ((i, i % 2) for i in range(layers))]
    gen = torch.Generator().manual_seed(4)
    queries = [torch.randn(w.query_heads, w.head_dim, generator=gen).half().to(device)
               for _ in range(layers)]
    problems = [(q, *p, None) for q, p in zip(queries, pools)]
    scale = 1 / math.sqrt(w.head_dim)
    batch = ops.BatchedDecode(problems, w.bits, w.group_size, scale)
    batched_ms = graph_time(batch.run, device)
    single_ms = graph_time(lambda: [ops.decode(q, *p, w.bits, w.group_size, scale)
                                    for q, p in zip(queries, pools)], device)
    step_bytes = layers * per * w.bytes_per_block
    return {
        "workload": "c4 on 1 GPU: 32 layers x 65536 tokens, INT4 g32, 8 KV heads, GQA 4",
        "batched_one_launch": {"us_per_layer": batched_ms * 1e3 / layers,
                               "GB/s": step_bytes / (batched_ms * 1e-3) / 1e9},
        "one_decode_per_layer": {"us_per_layer": single_ms * 1e3 / layers,
                                 "GB/s": step_bytes / (single_ms * 1e-3) / 1e9},
        "bytes_per_step": step_bytes,
    }


def small_config_legs(device) -> dict:
    """Latency of the other single-GPU configurations (device time per decode, CUDA-graph
    replays): c1 (8192 tokens, INT4, all 64 blocks) and c3 (INT2 with 1 % outlier channels x8,
    RecentSinkBlocks(1, 32) over 1024 blocks: 33 blocks through a block table)."""
    from kvssd_b200 import RecentSinkBlocks, ops
    from kvssd_b200.workloads import WORKLOADS, make_layer

    res = {}
    for name in ("c1", "c3"):
        w = WORKLOADS[name]
        lay = make_layer(w, 0, "cpu")
        t = [x.to(device) for x in (lay.query, lay.packed_k, lay.packed_v, lay.scales_k,
                                    lay.scales_v, lay.valid_tokens)]
        sel = list(range(lay.packed_k.shape[0]))
        table = None
        if w.sink is not None:
            sel = RecentSinkBlocks(w.sink, w.recent).select(sel)
            table = torch.tensor(sel, dtype=torch.int32, device=device)
        scale = 1 / math.sqrt(w.head_dim)
        us = graph_time(lambda: ops.decode(*t, w.bits, w.group_size, scale, block_table=table),
                        device, reps=50) * 1e3
        nbytes = len(sel) * w.bytes_per_block
        plan = ops.decode_plan(len(sel), w.block_tokens, w.query_heads, w.kv_heads, w.head_dim,
                               w.bits, w.group_size)
        res[name] = {"us_per_decode": us, "GB/s": nbytes / (us * 1e-6) / 1e9,
                     "inputs": "resident, L2-warm between replays (a latency figure)",
                     "selected_blocks": len(sel), "packed_kv_bytes": nbytes,
                     "kernel": plan["kernel"]}
    return res


def run_ours(args) -> None:
    from kvssd_b200 import B200AttentionBackend, PackedBatch, ops
    from kvssd_b200.sharding import ShardedDecoder
    from kvssd_b200.workloads import WORKLOADS, make_layer

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.gpus != world:
        raise SystemExit(f"--gpus {args.gpus} needs {args.gpus} ranks (got WORLD_SIZE={world}); "
                         "launch with torch.distributed.run")
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    from kvssd_b200 import _native
    ops.set_path_override({"auto": _native.PATH_AUTO, "stream": _native.PATH_TENSOR_CORE,
                           "cpasync": _native.PATH_TENSOR_CORE_CPASYNC,
                           "regs": _native.PATH_TENSOR_CORE_REGS,
                           "generic": _native.PATH_GENERIC}[args.path])
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=device,
                                timeout=datetime.timedelta(seconds=120))

    w = WORKLOADS[WORKLOAD]
    # Rank r owns token-block range r of an (N x 131072)-token context (distinct data per rank).
    base = make_layer(w, layer=rank, device=device)
    q = base.query
    pools = [base]
    for _ in range(1, max(args.copies, 1)):
        pools.append(type(base)(base.query, base.packed_k.clone(), base.packed_v.clone(),
                                base.scales_k.clone(), base.scales_v.clone(),
                                base.valid_tokens.clone()))
    nbytes = w.blocks_per_layer * w.bytes_per_block
    qh, d = q.shape
    scale = 1 / math.sqrt(d)
    out_v = torch.empty((qh, d), dtype=torch.float32, device=device)
    lse_v = torch.empty((qh,), dtype=torch.float32, device=device)
    batches = [PackedBatch(p.packed_k, p.packed_v, p.scales_k, p.scales_v, p.valid_tokens,
                           w.bits, w.group_size) for p in pools]
    # N > 1: this rank's 1024 blocks are its token-block shard of the N x 1024-block context;
    # the library's ShardedDecoder decodes it, all-gathers (out, lse) over NCCL and merges.
    sharded = ShardedDecoder("tokens") if world > 1 else None

    def step(i: int):
        if sharded is not None:
            sharded.run(q, batches[i % len(batches)], scale)
            return
        p = pools[i % len(pools)]
        ops.decode(q, p.packed_k, p.packed_v, p.scales_k, p.scales_v, p.valid_tokens, w.bits,
                   w.group_size, scale, out=out_v, lse=lse_v)

    stream = torch.cuda.current_stream(device)

    graphs = []  # CUDA graphs of timed steps; released before the process group is destroyed

    def timed(fn, steps: int, warmup: int, graph: bool = False) -> float:
        """Device time per step (max over ranks). graph=True captures the `steps` steps into one
        CUDA graph after the eager warm-up and replays it once more untimed before the timed
        replay: the same kernels and collectives, without the per-launch host latency."""
        for i in range(warmup):
            fn(i)
        run = None
        if graph:
            side = torch.cuda.Stream(device)
            side.wait_stream(stream)
            with torch.cuda.stream(side):
                for i in range(3):
                    fn(i)
            stream.wait_stream(side)
            torch.cuda.synchronize(device)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=side):
                for i in range(steps):
                    fn(i)
            graphs.append(g)
            g.replay()
            run = g.replay
        if dist:
            dist.barrier()
        torch.cuda.synchronize(device)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        if run is not None:
            run()
        else:
            for i in range(steps):
                fn(i)
        e1.record(stream)
        torch.cuda.synchronize(device)
        if dist:
            dist.barrier()
        ms = e0.elapsed_time(e1) / steps
        if dist:
            t = torch.tensor([ms], device=device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    def busy(seconds: float) -> None:
        """Untimed steps that keep the GPU under the same load while clocks are sampled."""
        t_end = time.perf_counter() + seconds
        i = 0
        while time.perf_counter() < t_end:
            for _ in range(50):
                step(i)
                i += 1
            torch.cuda.synchronize(device)

    # ---- device-timed whole step (inputs resident in HBM); clocks sampled around it
    with ClockSampler(device.index) as clocks:
        busy(0.0 if args.kernel_only else 1.0)
        ms = timed(step, args.steps, max(args.warmup, 3), graph=not args.eager)
        busy(0.0 if args.kernel_only else 0.5)
    clock_summary = clocks.summary()
    value = world * nbytes / (ms * 1e-3) / 1e9
    if args.kernel_only:
        torch.cuda.synchronize(device)
        graphs.clear()
        if dist:
            dist.destroy_process_group()
        if rank == 0:
            emit({"metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world,
                  "steps": args.steps, "ms_per_step": ms, "kernel_only": True, "path": args.path})
        return

    # ---- roofline leg: the dominant kernel alone on this rank, same inputs and rotation. The
    # streaming kernel folds its own split-KV parts (fused combine), so one launch is the
    # whole decode; the other kernels are timed without their separate combine launch.
    plan = ops.decode_plan(w.blocks_per_layer, w.block_tokens, w.query_heads, w.kv_heads,
                           w.head_dim, w.bits, w.group_size)
    fused = plan["kernel"] in ops.STREAMING_KERNELS

    def local_decode(i: int):
        p = pools[i % len(pools)]
        ops.decode(q, p.packed_k, p.packed_v, p.scales_k, p.scales_v, p.valid_tokens, w.bits,
                   w.group_size, scale, out=out_v, lse=lse_v)

    def split_only(i: int):
        p = pools[i % len(pools)]
        ops.decode_split(q, p.packed_k, p.packed_v, p.scales_k, p.scales_v, p.valid_tokens,
                         w.bits, w.group_size, scale)

    split_ms = timed(split_only, args.steps, 3, graph=not args.eager)
    peer = sharded is not None and sharded._peer is not None
    if peer:  # the timed step is exactly one kernel per rank: decode + combine + exchange
        kernel_ms = ms
    elif fused:
        kernel_ms = timed(local_decode, args.steps, 3, graph=not args.eager)
    else:
        kernel_ms = split_ms
    kernel_name = {"tensor_core_tma": "tma_decode_kernel",
                   "tensor_core_stream": "async_decode_kernel",
                   "tensor_core_regs": "tc_decode_kernel",
                   "generic": "simt_decode_kernel"}[plan["kernel"]]
    peak, peak_kind = peaks()
    achieved = nbytes / (kernel_ms * 1e-3) / 1e9
    traffic = None
    tfile = ROOT / "profiles" / "decode_c2_traffic.json"
    if tfile.exists():  # the ncu capture of the same kernel (null if it was another kernel)
        tinfo = json.loads(tfile.read_text())
        if kernel_name in tinfo.get("kernel", ""):
            traffic = tinfo.get("dram_bytes_per_launch")

    # ---- end to end through the plugin with host buffers (H2D + decode + D2H each step)
    backend = B200AttentionBackend()
    host = [t.cpu().pin_memory() for t in (base.packed_k, base.packed_v, base.scales_k,
                                            base.scales_v, base.valid_tokens, base.query)]
    dev_bufs = [torch.empty_like(t, device=device) for t in host]
    out_host = torch.empty((qh, d), dtype=torch.float32).pin_memory()
    h2d = sum(t.numel() * t.element_size() for t in host)
    d2h = out_host.numel() * 4

    def e2e_step(i: int):
        for src, dst in zip(host, dev_bufs):
            dst.copy_(src, non_blocking=True)
        batch = PackedBatch(*dev_bufs[:5], w.bits, w.group_size)
        if sharded is not None:
            out, lse = sharded.run(dev_bufs[5], batch, scale)
        else:
            out, lse = backend.run(dev_bufs[5], batch, scale)
        out_host.copy_(out, non_blocking=True)

    e2e_steps = max(3, min(args.steps, 20))
    e2e_ms = timed(e2e_step, e2e_steps, 3)
    e2e_value = world * nbytes / (e2e_ms * 1e-3) / 1e9

    # ---- the reference's own entry point, KVSSDPipeline.decode(query, layer), from a store file
    # of this rank's layer: native record reads (page cache), chunked host-to-device copies,
    # on-GPU record decode (headers + CRC-32) and the fused decode; plus the GPU record decode
    # alone on the layer's records resident in HBM.
    pipeline = None
    c4 = None
    small = None
    if not args.no_pipeline and world == 1:
        pipeline = pipeline_legs(w, base, q, scale, device, rank, args)
        c4 = c4_legs(w, base, device, args)
        small = small_config_legs(device)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_oracle_run(args.cpu_seconds)
    torch.cuda.synchronize(device)
    graphs.clear()  # graphs that hold NCCL calls go before the process group
    if sharded is not None:
        sharded.close()  # collective: unmaps the peers' exchange buffers
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    launches_per_step = 1 if fused else 2 + (1 if world > 1 else 0)
    record = {
        "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": max(args.warmup, 3), "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
        "config": {
            "workload": workload_text(world),
            "us_per_layer_decode": ms * 1e3,
            "packed_kv_bytes_per_gpu": nbytes,
            "hbm_peak_gbs": peak,
            "hbm_frac": value / world / peak,
            "kv_bits": w.bits,
            "l2": f"inputs rotated over {len(pools)} copies ({len(pools) * nbytes / 1e6:.0f} MB > 126 MB L2)",
            "parallelism": f"token-range split x{world}" if world > 1 else "single GPU",
            "launch": ("eager: one host call per step" if args.eager else
                       "the K timed steps replayed from one CUDA graph (captured after the "
                       "warm-up; same kernels and collectives, no per-call host latency); "
                       "e2e is eager through the public API"),
        },
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "traffic": traffic,
                     "kernel": f"{kernel_name}<{w.kv_heads},{w.group_size}> "
                               f"({plan['n_splits']} CTAs, split-KV stream"
                               + ("; combine and NVLink exchange fused in the kernel tail)"
                                  if peer else "; combine fused in the kernel tail)" if fused
                                  else "; combine kernel excluded)"),
                     "kernel_us": kernel_ms * 1e3,
                     "split_only_us": split_ms * 1e3,
                     "peak_kind": f"{peak_kind} (burst copy)"},
        "e2e": {"value": e2e_value, "unit": "GB/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms,
                "path": ("ShardedDecoder.run (C ABI kvssd_b200_decode_exchange over NVLink)"
                         if world > 1 else "B200AttentionBackend.run (C ABI)")
                        + " from pinned host buffers"},
        "gpu_launches": args.steps * launches_per_step,
        "clocks": clock_summary,
    }
    if cpu is not None:
        record["cpu_baseline"] = cpu
    if pipeline is not None:
        record["pipeline"] = pipeline
    if c4 is not None:
        record["c4_multi_layer"] = c4
    if small is not None:
        record["c1_c3_latency"] = small
    emit(record)


_RESULT_FD = 1


def emit(record: dict) -> None:
    """Writes the one JSON result line to the process's original standard output."""
    os.write(_RESULT_FD, (json.dumps(record) + "\n").encode())


def main() -> None:
    global _RESULT_FD
    args = parse_args()
    # Everything else that reaches file descriptor 1 (e.g. NCCL's version banner, printed by
    # the C library) goes to stderr, so standard output carries exactly one JSON line.
    sys.stdout.flush()
    _RESULT_FD = os.dup(1)
    os.dup2(2, 1)
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
