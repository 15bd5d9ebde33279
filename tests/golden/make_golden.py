"""Generates the golden fixtures in this directory from the reference implementation.

Run where the reference project is checked out (its path in --reference or $KVSSD_REFERENCE):

    python tests/golden/make_golden.py [--reference /path/to/kvssd-attention]

Every expected value is produced by the reference's own code (kvssd.quant, kvssd.format,
kvssd.store, kvssd.selectors, kvssd.attention, kvssd.backends.reference); inputs are seeded.
The fixtures are small .npz/.json files plus one tiny store directory, so the tests that
read them run anywhere without the reference.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import math
import os
import shutil
import sys
import tempfile
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]


def sha(t: torch.Tensor) -> str:
    return hashlib.sha256(t.contiguous().cpu().view(torch.uint8).numpy().tobytes()).hexdigest()


def u16(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("KVSSD_REFERENCE"), required="KVSSD_REFERENCE" not in os.environ)
    ap.add_argument("--skip-large", action="store_true", help="skip the full-size configs")
    args = ap.parse_args()
    sys.path.insert(0, str(Path(args.reference) / "src"))
    sys.path.insert(0, str(REPO / "kvssd-attention_b200"))
    from kvssd.attention import merge_attention_chunks, packed_attention
    from kvssd.backends import PackedBatch
    from kvssd.backends.reference import ReferenceAttentionBackend
    from kvssd.format import CacheSpec
    from kvssd.quant import dequantize_tensor, quantize_tensor, unpack_codes
    from kvssd.selectors import RecentSinkBlocks
    from kvssd.store import KVCacheStore

    from kvssd_b200.workloads import WORKLOADS, raw_layer  # seeded raw K/V only

    torch.set_num_threads(8)
    backend = ReferenceAttentionBackend()

    # ---- quantizer: round trips, edge groups (all-zero, huge, tiny, fp16 input)
    for bits in (2, 4):
        for group in (16, 32):
            gen = torch.Generator().manual_seed(100 + bits * 10 + group)
            x = torch.randn(5, 3, 128, generator=gen)
            x[0, 0, :group] = 0.0
            x[0, 1, :group] *= 1e4
            x[0, 2, :group] *= 1e-6
            x[1, 0, group : 2 * group] = -x[1, 0, group : 2 * group].abs()
            xh = x.half()
            out = {}
            for tag, inp in (("f32", x), ("f16", xh)):
                q = quantize_tensor(inp, bits, group)
                out[f"x_{tag}"] = inp.float().numpy()
                out[f"packed_{tag}"] = q.packed.numpy()
                out[f"scales_{tag}"] = u16(q.scales)
                out[f"codes_{tag}"] = unpack_codes(q.packed, bits, 128).numpy()
                out[f"deq32_{tag}"] = dequantize_tensor(q, torch.float32).numpy()
                out[f"deq16_{tag}"] = u16(dequantize_tensor(q, torch.float16))
            np.savez_compressed(HERE / f"quant_b{bits}_g{group}.npz", **out)

    # ---- backend matrix (make_batch-style fixtures plus the configs' head layout)
    cases = [
        # name, bits, qh, kvh, d, nb, bt, group, valid, qdtype
        ("mk_b{b}_1_1_32", 1, 1, 32, 2, 8, 16, [8, 5], "f32"),
        ("mk_b{b}_4_1_64", 4, 1, 64, 2, 8, 16, [8, 5], "f32"),
        ("mk_b{b}_4_2_128", 4, 2, 128, 2, 8, 16, [8, 5], "f32"),
        ("gqa4_b{b}_32_8_128", 32, 8, 128, 3, 128, 32, [128, 128, 77], "f16"),
        ("mha_b{b}_8_8_64", 8, 8, 64, 3, 16, 32, [16, 0, 9], "f16"),
        ("mqa_b{b}_8_1_128", 8, 1, 128, 4, 32, 32, [32, 1, 32, 17], "bf16"),
        ("gqa12_b{b}_24_2_64", 24, 2, 64, 2, 32, 16, [32, 20], "f32"),
        ("d256_b{b}_16_2_256", 16, 2, 256, 2, 16, 64, [16, 11], "f16"),
        ("g128_b{b}_8_2_128", 8, 2, 128, 2, 16, 128, [16, 16], "f64"),
        ("bt40_b{b}_8_4_128", 8, 4, 128, 3, 40, 32, [40, 33, 40], "f16"),
    ]
    dt = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16, "f64": torch.float64}
    for bits in (2, 4):
        for name, qh, kvh, d, nb, bt, group, valid, qdt in cases:
            name = name.format(b=bits)
            gen = torch.Generator().manual_seed(41)
            q = torch.randn(qh, d, generator=gen).to(dt[qdt])
            k = torch.randn(nb, bt, kvh, d, generator=gen)
            v = torch.randn(nb, bt, kvh, d, generator=gen)
            kq, vq = quantize_tensor(k, bits, group), quantize_tensor(v, bits, group)
            vt = torch.tensor(valid, dtype=torch.int32)
            batch = PackedBatch(kq.packed, vq.packed, kq.scales, vq.scales, vt, bits, group)
            scale = 1.0 / math.sqrt(d)
            o, l = backend.run(q, batch, scale)
            np.savez_compressed(
                HERE / f"backend_{name}.npz",
                query=q.double().numpy(), query_dtype=np.array(qdt), packed_k=kq.packed.numpy(),
                packed_v=vq.packed.numpy(), scales_k=u16(kq.scales), scales_v=u16(vq.scales),
                valid=vt.numpy(), bits=bits, group=group, sm_scale=scale, out=o.numpy(),
                lse=l.numpy(),
            )

    # ---- exact chunk merge (attention.py:91-102), including an empty (-inf) chunk
    gen = torch.Generator().manual_seed(17)
    lo, ro = torch.randn(6, 32, generator=gen), torch.randn(6, 32, generator=gen)
    ll, rl = torch.randn(6, generator=gen) * 5, torch.randn(6, generator=gen) * 5
    ll[2] = -math.inf
    mo, ml = merge_attention_chunks(lo, ll, ro, rl)
    np.savez_compressed(HERE / "merge.npz", lo=lo.numpy(), ll=ll.numpy(), ro=ro.numpy(),
                        rl=rl.numpy(), out=mo.numpy(), lse=ml.numpy())

    # ---- record format: a small store written by the reference
    store_dir = HERE / "store_small"
    if store_dir.exists():
        shutil.rmtree(store_dir)
    gen = torch.Generator().manual_seed(3)
    keys, values = torch.randn(2, 19, 2, 32, generator=gen), torch.randn(2, 19, 2, 32, generator=gen)
    spec = CacheSpec(2, 2, 32, block_tokens=8, bits=4, group_size=16)
    st = KVCacheStore.create(store_dir, keys, values, spec, storage_backend="buffered")
    st.close()
    np.savez_compressed(HERE / "store_small_inputs.npz", keys=keys.numpy(), values=values.numpy())
    specs = []
    for layers, kvh, d, bt, bits, group in [(1, 8, 128, 128, 4, 32), (1, 8, 128, 128, 2, 32),
                                            (2, 2, 32, 8, 4, 16), (1, 4, 64, 16, 2, 16)]:
        s = CacheSpec(layers, kvh, d, bt, bits, group)
        specs.append(dict(spec=[layers, kvh, d, bt, bits, group], packed_dim=s.packed_dim,
                          scale_count=s.scale_count, packed_count=s.packed_count,
                          payload_bytes=s.payload_bytes, record_bytes=s.record_bytes))
    (HERE / "cachespec.json").write_text(json.dumps(specs, indent=1) + "\n")

    # ---- selectors
    sel = []
    for n, sink, recent in [(10, 1, 2), (10, 0, 3), (10, 3, 0), (4, 3, 3), (3, 1, 5), (1024, 1, 32),
                            (0, 1, 1), (5, 5, 5)]:
        sel.append(dict(available=list(range(n)), sink=sink, recent=recent,
                        chosen=RecentSinkBlocks(sink, recent).select(list(range(n)))))
    (HERE / "selectors.json").write_text(json.dumps(sel) + "\n")

    # ---- packed_attention over a store (tests/test_attention.py setup: seed 5, 13 tokens)
    for bits in (2, 4):
        with tempfile.TemporaryDirectory() as tmp:
            gen = torch.Generator().manual_seed(5)
            k = torch.randn(1, 13, 2, 32, generator=gen)
            v = torch.randn(1, 13, 2, 32, generator=gen)
            q = torch.randn(4, 32, generator=gen)
            s = CacheSpec(1, 2, 32, block_tokens=8, bits=bits, group_size=16)
            st = KVCacheStore.create(tmp, k, v, s, storage_backend="buffered")
            blocks = [st.read(0, i) for i in st.blocks_for_layer(0)]
            out = packed_attention(q, blocks, attention_backend="reference")
            st.close()
        np.savez_compressed(HERE / f"packed_attention_b{bits}.npz", keys=k.numpy(),
                            values=v.numpy(), query=q.numpy(), out=out.numpy())

    if args.skip_large:
        return
    # ---- full-size configurations: reference quantizer hashes + reference decode output
    for cname in ("c1", "c3", "c2"):
        w = WORKLOADS[cname]
        k, v, q, channels = raw_layer(w, 0, "cpu")
        nb = w.blocks_per_layer
        kq = quantize_tensor(k.reshape(nb, w.block_tokens, w.kv_heads, w.head_dim), w.bits, w.group_size)
        vq = quantize_tensor(v.reshape(nb, w.block_tokens, w.kv_heads, w.head_dim), w.bits, w.group_size)
        sel = w.selected_blocks()
        idx = torch.tensor(sel)
        valid = torch.full((len(sel),), w.block_tokens, dtype=torch.int32)
        batch = PackedBatch(kq.packed[idx], vq.packed[idx], kq.scales[idx], vq.scales[idx], valid,
                            w.bits, w.group_size)
        o, l = backend.run(q, batch, 1.0 / math.sqrt(w.head_dim))
        np.savez_compressed(
            HERE / f"config_{cname}.npz", query=u16(q), out=o.numpy(), lse=l.numpy(),
            selected=np.array(sel), sha_packed_k=sha(kq.packed), sha_packed_v=sha(vq.packed),
            sha_scales_k=sha(kq.scales), sha_scales_v=sha(vq.scales),
            outlier_channels=np.array([] if channels is None else channels.tolist()),
        )
        print(cname, "done", flush=True)


if __name__ == "__main__":
    main()
