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
    ap.add_argument("--no-c4", action="store_true", help="skip the c4 multi-layer leg")
    ap.add_argument("--records-only", action="store_true",
                    help="profiling aid: only the on-GPU record decode of the c2 layer's 1024 "
                         "records (one JSON line with its timing)")
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


def cpu_layer():
    """The benchmark layer (all 1024 blocks of the c2 workload) as numpy arrays for the oracle."""
    from kvssd_b200.workloads import WORKLOADS, make_layer

    w = WORKLOADS[WORKLOAD]
    layer = make_layer(w, 0, "cpu")
    arrays = [t.numpy() for t in (layer.packed_k, layer.packed_v, layer.scales_k,
                                  layer.scales_v, layer.valid_tokens)]
    return w, layer.query.float().numpy(), arrays


def cpu_oracle_run(seconds: float, min_runs: int = 1) -> dict:
    """Times the oracle (numpy restatement of kvssd's reference backend) on the benchmark's own
    workload -- one whole c2 layer per run -- repeated for about ``seconds``."""
    from oracle import kvssd_oracle as orc

    w, q, arrays = cpu_layer()
    nbytes = w.blocks_per_layer * w.bytes_per_block
    runs, t0 = 0, time.perf_counter()
    while runs < min_runs or time.perf_counter() - t0 < seconds:
        orc.decode(q, *arrays, w.bits, w.group_size, 1 / math.sqrt(w.head_dim))
        runs += 1
    dt = time.perf_counter() - t0
    return {"value": nbytes * runs / dt / 1e9, "unit": "GB/s", "cores": cpu_threads(),
            "kind": "port", "seconds": dt, "runs": runs, "sample_blocks": w.blocks_per_layer,
            "sample": f"the whole c2 layer ({w.blocks_per_layer} blocks, {w.tokens} tokens) per "
                      f"run, {runs} runs; numpy restatement of src/kvssd/backends/reference.py, "
                      f"8-block chunks on {cpu_threads()} host threads merged exactly"}


def workload_text(world: int) -> str:
    """The workload both arms report."""
    return (f"{WORKLOAD}: 1 layer x 131072 tokens per GPU, INT4 group 32 FP16 scales, 8 KV heads "
            "x 128, 32 query heads (GQA 4), block 128, AllBlocks"
            + (f"; {world} GPUs split one {world * 131072}-token context by token-block ranges; "
               "each rank's decode kernel pushes its combined slices to every rank over NVLink "
               "peer stores and merges them exactly (one kernel per rank per step)"
               if world > 1 else ""))


def run_reference(args) -> None:
    """The reference arm: kvssd's reference backend algorithm (the oracle port) on the host
    cores, on the same workload as the measured arm (the whole c2 layer per step)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle import kvssd_oracle as orc

    w, q, arrays = cpu_layer()
    step = lambda: orc.decode(q, *arrays, w.bits, w.group_size, 1 / math.sqrt(w.head_dim))  # noqa: E731
    for _ in range(max(args.warmup, 0)):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = (time.perf_counter() - t0) / args.steps
    nbytes = w.blocks_per_layer * w.bytes_per_block
    value = nbytes / dt / 1e9
    emit({
        "impl": "reference", "metric": METRIC, "value": value, "unit": "GB/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": dt * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": workload_text(1),
                   "sample": f"the whole layer ({w.blocks_per_layer} blocks) per step, timed on "
                             "the host cores (rank 0 only when launched on several GPUs)",
                   "sample_blocks": w.blocks_per_layer,
                   "kv_heads": w.kv_heads, "head_dim": w.head_dim, "query_heads": w.query_heads,
                   "block_tokens": w.block_tokens, "bits": w.bits, "group_size": w.group_size},
        "cpu_baseline": {"value": value, "unit": "GB/s", "cores": cpu_threads(), "kind": "port",
                         "sample_blocks": w.blocks_per_layer,
                         "sample": f"the whole c2 layer ({w.blocks_per_layer} blocks, {w.tokens} "
                                   "tokens) per step; numpy restatement of kvssd's reference "
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
        io_depth = 8  # measured: 16 reader threads made the step slower (10.7 vs 9.9 ms)
        pipe = KVSSDPipeline(store, device=device, io_depth=io_depth, stage_blocks=128,
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
        ref_out = out.clone()
        pipe.close()
        # the same store opened with the "mapped" backend: page-locked mapping, DMA copies
        mapped_s, mapped_note = None, None
        try:
            mstore = KVCacheStore.open(root, storage_backend="mapped")
        except RuntimeError as exc:  # the driver would not page-lock the mapping
            mapped_note = str(exc)
        else:
            try:
                mpipe = KVSSDPipeline(mstore, device=device, stage_blocks=128,
                                      require_cuda_kernel=True)
                for _ in range(2):
                    mout = mpipe.decode(qh, 0)
                torch.cuda.synchronize(device)
                if not torch.equal(mout, ref_out):
                    raise BenchFailure("the mapped-store pipeline differs from the default one")
                t0 = time.perf_counter()
                for _ in range(steps):
                    mout = mpipe.decode(qh, 0)
                    mout.cpu()
                mapped_s = (time.perf_counter() - t0) / steps
                mpipe.close()
            finally:
                mstore.close()
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
    finally:
        store.close()
        shutil.rmtree(root, ignore_errors=True)
    nbytes = w.blocks_per_layer * w.bytes_per_block
    return {
        "KVSSDPipeline_decode": {
            "value": nbytes / pipe_s / 1e9, "unit": "GB/s", "ms_per_step": pipe_s * 1e3,
            "path": f"KVSSDPipeline(store, stage_blocks=128, io_depth={io_depth}).decode(query, 0): "
                    "store file in /dev/shm (page cache), native record reads, H2D, on-GPU "
                    "record decode with CRC-32, fused decode, chunk merge; host wall clock"},
        "KVSSDPipeline_decode_mapped": (
            {"value": nbytes / mapped_s / 1e9, "unit": "GB/s", "ms_per_step": mapped_s * 1e3,
             "path": "the same store opened with storage_backend='mapped' (file mapped "
                     "read-only and page-locked; records copied to the device by DMA, one "
                     "copy per run of records), same pipeline; host wall clock"}
            if mapped_s is not None else {"unavailable": mapped_note}),
        "record_decode_on_gpu": {
            "value": record_bytes / (rec_ms * 1e-3) / 1e9, "unit": "GB/s of records",
            "us_per_layer": rec_ms * 1e3,
            "hbm_bytes_per_layer": record_bytes + nbytes,
            "hbm_frac": (record_bytes + nbytes) / (rec_ms * 1e-3) / 1e9 / peaks()[0],
            "note": "1024 raw records resident in HBM -> PackedBatch + CRC-32 check (reads the "
                    "records, writes the packed KV: hbm_frac counts both)"},
    }


def records_only(args) -> None:
    """The record-decode leg alone: the c2 layer written as a store in /dev/shm, its 1024 raw
    records read into HBM, then ``args.warmup`` + ``args.steps`` ops.decode_records calls (the
    timed ones between CUDA events on the current stream)."""
    from kvssd_b200 import CacheSpec, KVCacheStore, ops
    from kvssd_b200.format import PackedKVBlock
    from kvssd_b200.quant import QuantizedTensor
    from kvssd_b200.workloads import WORKLOADS, make_layer

    device = torch.device("cuda", 0)
    w = WORKLOADS[WORKLOAD]
    lay = make_layer(w, 0, "cpu")
    spec = CacheSpec(1, w.kv_heads, w.head_dim, w.block_tokens, w.bits, w.group_size)
    shape = (w.block_tokens, w.kv_heads, w.head_dim)
    blocks = (PackedKVBlock(0, b, int(lay.valid_tokens[b]),
                            QuantizedTensor(lay.packed_k[b], lay.scales_k[b], shape, w.bits,
                                            w.group_size),
                            QuantizedTensor(lay.packed_v[b], lay.scales_v[b], shape, w.bits,
                                            w.group_size))
              for b in range(lay.packed_k.shape[0]))
    root = Path(tempfile.mkdtemp(prefix="kvssd_records_", dir="/dev/shm"
                                 if Path("/dev/shm").is_dir() else None))
    try:
        store = KVCacheStore.from_blocks(root, spec, blocks)
        raw = store.read_records(0, store.blocks_for_layer(0)).to(device)
        store.close()
        for _ in range(max(3, args.warmup)):
            out = ops.decode_records(raw, spec, 0)
        torch.cuda.synchronize(device)
        if int((out[5] != 0).sum()) or not torch.equal(out[0].cpu(), lay.packed_k):
            raise BenchFailure("record decode does not reproduce the layer")
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            ops.decode_records(raw, spec, 0)
        e1.record()
        torch.cuda.synchronize(device)
        us = e0.elapsed_time(e1) / args.steps * 1e3
    finally:
        shutil.rmtree(root, ignore_errors=True)
    moved = raw.numel() + w.blocks_per_layer * w.bytes_per_block
    emit({"records_only": {"us_per_layer": us, "hbm_bytes_per_layer": moved,
                           "GB/s": moved / (us * 1e-6) / 1e9,
                           "hbm_frac": moved / (us * 1e-6) / 1e9 / peaks()[0],
                           "steps": args.steps, "warmup": max(3, args.warmup)}})


def graph_time(fn, device, reps: int = 20, rotate: int = 1) -> float:
    """Device ms per call of ``fn(i)``: ``reps`` calls captured in one CUDA graph (after 3 eager
    warm-up calls and one on the capture stream), one warm replay, then one timed replay."""
    stream = torch.cuda.current_stream(device)
    for i in range(3):
        fn(i)
    side = torch.cuda.Stream(device)
    side.wait_stream(stream)
    with torch.cuda.stream(side):
        fn(0)
    stream.wait_stream(side)
    torch.cuda.synchronize(device)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=side):
        for i in range(reps):
            fn(i)
    g.replay()
    torch.cuda.synchronize(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    g.replay()
    e1.record(stream)
    torch.cuda.synchronize(device)
    del g
    return e0.elapsed_time(e1) / reps


def c4_step(w, base, device, rank: int, world: int, dist):
    """The c4 multi-layer step, KV-head sharded over ``world`` ranks: 32 layers x 65536 tokens
    (each layer 512 blocks of distinct memory, halves of 16 copies of this rank's c2 pool), each
    with its own query. Rank r owns KV heads [r*8/N, (r+1)*8/N) of every layer and their query
    heads (kvssd's GQA map), re-laid head-contiguous; a step is one batched launch over its 32
    layers plus, for N > 1, one NCCL all-gather of the output rows of all layers."""
    from kvssd_b200 import ops
    from kvssd_b200.sharding import head_shard

    layers, per = 32, w.blocks_per_layer // 2
    kv_lo, kv_hi, q_lo, q_hi = head_shard(w.kv_heads, w.query_heads, rank, world)
    cut = lambda t: t[:, :, kv_lo:kv_hi].contiguous()  # noqa: E731
    copies = [[cut(t) for t in (base.packed_k, base.packed_v, base.scales_k, base.scales_v)]
              + [base.valid_tokens.clone()] for _ in range(layers // 2)]
    pools = [[t[h * per:(h + 1) * per] for t in copies[i // 2]] for i, h in
             ((i, i % 2) for i in range(layers))]
    gen = torch.Generator().manual_seed(4)
    queries = [torch.randn(w.query_heads, w.head_dim, generator=gen).half()[q_lo:q_hi]
               .contiguous().to(device) for _ in range(layers)]
    rows = q_hi - q_lo
    out = torch.empty((layers, rows, w.head_dim), dtype=torch.float32, device=device)
    lse = torch.empty((layers, rows), dtype=torch.float32, device=device)
    batch = ops.BatchedDecode([(q, *p, None) for q, p in zip(queries, pools)], w.bits,
                              w.group_size, 1 / math.sqrt(w.head_dim), out=out, lse=lse)
    gathered = None
    if world > 1:
        gathered = torch.empty((world, layers, rows, w.head_dim), dtype=torch.float32,
                               device=device)

    def step(i: int):
        batch.run()
        if gathered is not None:
            dist.all_gather_into_tensor(gathered.view(-1), out.view(-1))

    return step, batch, layers * per * w.bytes_per_block * (kv_hi - kv_lo) // w.kv_heads


def small_config_legs(device) -> dict:
    """Latency of the other single-GPU configurations, CUDA-graph replays, device time per
    decode, both with the inputs L2-warm and cold: c1 (8192 tokens, INT4, all 64 blocks) and
    c3 (INT2 with 1 % outlier channels x8, RecentSinkBlocks(1, 32) over 1024 blocks: 33 blocks
    through a block table). Cold: the selected blocks are replicated into R distinct copies
    (R x selected bytes > 126 MB L2) and step i reads copy i % R (c1: the pool view of copy r;
    c3: one pool of R x 33 blocks with one block table per copy, the RecentSink order kept)."""
    from kvssd_b200 import RecentSinkBlocks, ops
    from kvssd_b200.workloads import WORKLOADS, make_layer

    res = {}
    for name in ("c1", "c3"):
        w = WORKLOADS[name]
        lay = make_layer(w, 0, device)
        q = lay.query
        pool = [lay.packed_k, lay.packed_v, lay.scales_k, lay.scales_v, lay.valid_tokens]
        sel = list(range(lay.packed_k.shape[0]))
        table = None
        if w.sink is not None:
            sel = RecentSinkBlocks(w.sink, w.recent).select(sel)
            table = torch.tensor(sel, dtype=torch.int32, device=device)
        scale = 1 / math.sqrt(w.head_dim)
        warm_us = graph_time(lambda i: ops.decode(q, *pool, w.bits, w.group_size, scale,
                                                  block_table=table), device, reps=50) * 1e3
        nbytes = len(sel) * w.bytes_per_block
        reps = -(-int(1.2 * 126e6) // nbytes)  # copies whose bytes exceed L2 by 20 %
        idx = torch.tensor(sel, device=device, dtype=torch.long)
        picked = [t.index_select(0, idx) for t in pool]
        big = [t.repeat(reps, *([1] * (t.ndim - 1))) for t in picked]
        n_sel = len(sel)
        if table is None:
            views = [[t[r * n_sel:(r + 1) * n_sel] for t in big] for r in range(reps)]
            cold = lambda i: ops.decode(q, *views[i % reps], w.bits, w.group_size, scale)  # noqa: E731
        else:
            tables = [torch.arange(r * n_sel, (r + 1) * n_sel, dtype=torch.int32, device=device)
                      for r in range(reps)]
            cold = lambda i: ops.decode(q, *big, w.bits, w.group_size, scale,  # noqa: E731
                                        block_table=tables[i % reps])
        cold_us = graph_time(cold, device, reps=max(50, 2 * reps)) * 1e3
        plan = ops.decode_plan(n_sel, w.block_tokens, w.query_heads, w.kv_heads, w.head_dim,
                               w.bits, w.group_size)
        res[name] = {"us_per_decode": cold_us, "GB/s": nbytes / (cold_us * 1e-6) / 1e9,
                     "us_per_decode_l2_warm": warm_us,
                     "GB/s_l2_warm": nbytes / (warm_us * 1e-6) / 1e9,
                     "inputs": f"cold: {reps} copies of the selected blocks "
                               f"({reps * nbytes / 1e6:.0f} MB > 126 MB L2) rotated step by "
                               "step; warm: the same blocks every step",
                     "selected_blocks": n_sel, "packed_kv_bytes": nbytes,
                     "kernel": plan["kernel"], "ctas": plan["n_splits"]}
        del big, picked
    return res


def int2_leg(device, copies: int = 3) -> dict:
    """INT2 over the whole c3 cache (131072 tokens, 1 % outlier channels x8, AllBlocks),
    inputs rotated over ``copies`` copies (> L2), CUDA-graph replays."""
    from kvssd_b200 import ops
    from kvssd_b200.workloads import WORKLOADS, make_layer

    w = WORKLOADS["c3"]
    lay = make_layer(w, 0, device)
    pools = [[lay.packed_k, lay.packed_v, lay.scales_k, lay.scales_v, lay.valid_tokens]]
    for _ in range(1, copies):
        pools.append([t.clone() for t in pools[0]])
    scale = 1 / math.sqrt(w.head_dim)
    us = graph_time(lambda i: ops.decode(lay.query, *pools[i % copies], w.bits, w.group_size,
                                         scale), device, reps=30) * 1e3
    nbytes = w.blocks_per_layer * w.bytes_per_block
    plan = ops.decode_plan(w.blocks_per_layer, w.block_tokens, w.query_heads, w.kv_heads,
                           w.head_dim, w.bits, w.group_size)
    peak = peaks()[0]
    return {"workload": "INT2 g32, 131072 tokens (1024 blocks), 8 KV heads x 128, 32 query "
                        "heads, 1 % outlier channels x8, AllBlocks",
            "us_per_decode": us, "GB/s": nbytes / (us * 1e-6) / 1e9,
            "frac": nbytes / (us * 1e-6) / 1e9 / peak, "packed_kv_bytes": nbytes,
            "l2": f"inputs rotated over {copies} copies ({copies * nbytes / 1e6:.0f} MB)",
            "kernel": plan["kernel"]}


class BenchFailure(RuntimeError):
    pass


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
    # the library's ShardedDecoder runs one fused decode + NVLink exchange kernel per rank.
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

    def check_status(where: str) -> None:
        """Every rank waits for its kernels and reads its device status word; any flagged
        failure (on any rank) ends the run with an error instead of a number."""
        torch.cuda.synchronize(device)
        if sharded is not None:
            sharded.check()  # collective: all ranks raise together
            return
        value = ops.read_device_status_all(device)
        if value:
            raise BenchFailure(f"{where}: device status {value:#x} "
                               f"({ops.describe_status(value)})")

    def barrier() -> None:
        if dist:
            dist.barrier()

    def timed(fn, steps: int, warmup: int, graph: bool = False) -> float:
        """Device time per step (max over ranks). graph=True captures the `steps` steps into one
        CUDA graph after the eager warm-up and replays it once more untimed before the timed
        replay: the same kernels and collectives, without the per-launch host latency. Every
        rank runs exactly the same number of steps."""
        barrier()
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
        barrier()
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
        barrier()
        ms = e0.elapsed_time(e1) / steps
        if dist:
            t = torch.tensor([ms], device=device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    def busy(calls: int) -> None:
        """Untimed steps that keep the GPU under the same load while clocks are sampled: a
        fixed number of calls, the same on every rank (each multi-GPU step is an exchange that
        every rank must join), in batches of 50 with a synchronisation after each."""
        barrier()
        for start in range(0, calls, 50):
            for i in range(start, min(calls, start + 50)):
                step(i)
            torch.cuda.synchronize(device)
        barrier()

    # ---- device-timed whole step (inputs resident in HBM); clocks sampled around it
    busy_calls = 0 if args.kernel_only else 20000  # ~1 s of decodes at ~45 us
    with ClockSampler(device.index) as clocks:
        busy(busy_calls)
        ms = timed(step, args.steps, max(args.warmup, 3), graph=not args.eager)
        busy(busy_calls // 2)
    clock_summary = clocks.summary()
    check_status("timed decode steps")
    value = world * nbytes / (ms * 1e-3) / 1e9
    if args.kernel_only:
        torch.cuda.synchronize(device)
        graphs.clear()
        if sharded is not None:
            sharded.close()
        if dist:
            dist.destroy_process_group()
        if rank == 0:
            emit({"metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world,
                  "steps": args.steps, "ms_per_step": ms, "kernel_only": True, "path": args.path,
                  "device_status": 0})
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
    check_status("roofline legs")
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

    # ---- N > 1: every rank must hold the same result, equal to the ranks' local decodes
    # merged by the NCCL path (all-gather + N-way merge kernel).
    agree = None
    if sharded is not None:
        ox, lx = sharded.run(q, batches[0], scale)
        ox, lx = ox.clone(), lx.clone()
        torch.cuda.synchronize(device)
        got = torch.empty((world, qh * d + qh), dtype=torch.float32, device=device)
        dist.all_gather_into_tensor(got.view(-1), torch.cat([ox.view(-1), lx]))
        same = all(torch.equal(got[r], got[0]) for r in range(world))
        nccl = ShardedDecoder("tokens", transport="nccl")
        on, ln = nccl.run(q, batches[0], scale)
        finite = bool(torch.isfinite(ox).all()) and bool(torch.isfinite(lx).all())
        diff = torch.tensor([float((on - ox).abs().max()), float((ln - lx).abs().max()),
                             0.0 if finite else 1.0], device=device)
        dist.all_reduce(diff, op=dist.ReduceOp.MAX)
        agree = {"ranks_agree": bool(same), "exchange_vs_nccl_merge_max_abs_out": float(diff[0]),
                 "exchange_vs_nccl_merge_max_abs_lse": float(diff[1]),
                 "finite": bool(diff[2] == 0.0)}
        check_status("rank agreement check")
        if not same or diff[0] > 1e-5 or diff[1] > 1e-5 or diff[2] != 0.0:
            raise BenchFailure(f"multi-GPU results disagree: {agree}")

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
    if sharded is None:
        backend.check(device)
    check_status("end-to-end steps")
    e2e_value = world * nbytes / (e2e_ms * 1e-3) / 1e9

    # ---- the c4 multi-layer step: KV-head sharded over the ranks (one batched launch over the
    # rank's 32 layers + one NCCL all-gather of the output rows per step).
    c4 = None
    if not args.no_c4:
        c4_fn, c4_batch, c4_bytes = c4_step(w, base, device, rank, world, dist)
        c4_ms = timed(c4_fn, max(3, min(args.steps, 20)), 3, graph=not args.eager)
        if c4_batch.read_status():
            raise BenchFailure("c4 batched decode flagged a device failure")
        check_status("c4 steps")
        total = 32 * (w.blocks_per_layer // 2) * w.bytes_per_block
        c4 = {"workload": f"c4: 32 layers x 65536 tokens, INT4 g32, 8 KV heads, GQA 4; KV heads "
                          f"sharded over {world} GPU(s) ({w.kv_heads // world} per GPU), one "
                          "batched launch over the rank's 32 layers"
                          + (" + one NCCL all-gather of all layers' output rows" if world > 1
                             else "") + " per step (strong scaling: the step's work is fixed)",
              "n_gpus": world, "us_per_step": c4_ms * 1e3, "us_per_layer": c4_ms * 1e3 / 32,
              "GB/s": total / (c4_ms * 1e-3) / 1e9, "bytes_per_step": total,
              "bytes_per_gpu": c4_bytes, "per_gpu_hbm_frac": c4_bytes / (c4_ms * 1e-3) / 1e9 / peak}
        del c4_fn, c4_batch

    # ---- the reference's own entry point, KVSSDPipeline.decode(query, layer), from a store file
    # of this rank's layer, plus the GPU record decode alone; other single-GPU configurations.
    pipeline = small = int2 = None
    if not args.no_pipeline and world == 1:
        pipeline = pipeline_legs(w, base, q, scale, device, rank, args)
        small = small_config_legs(device)
        int2 = int2_leg(device)
        check_status("single-GPU legs")

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_oracle_run(args.cpu_seconds)
    torch.cuda.synchronize(device)
    graphs.clear()  # graphs that hold NCCL calls go before the process group
    if sharded is not None:
        sharded.close()  # collective: final status check, unmaps the peers' exchange buffers
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    launches_per_step = 1 if fused else 2
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
        "device_status": 0,
        "clocks": clock_summary,
    }
    if agree is not None:
        record.update(agree)
    if cpu is not None:
        record["cpu_baseline"] = cpu
    if c4 is not None:
        record["c4_multi_layer"] = c4
    if int2 is not None:
        record["int2_128k"] = int2
    if small is not None:
        record["c1_c3_latency"] = small
    if pipeline is not None:
        record["pipeline"] = pipeline
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
        return
    try:
        if args.records_only:
            records_only(args)
            return
        run_ours(args)
    except Exception as exc:  # a failed check prints no result line and exits non-zero
        from kvssd_b200.ops import DeviceFailure

        if isinstance(exc, (BenchFailure, DeviceFailure)):
            print(f"bench failed: {exc}", file=sys.stderr)
            raise SystemExit(3) from exc
        raise


if __name__ == "__main__":
    main()
