"""Shared test configuration: the ``gpu`` marker, import paths and golden-fixture helpers.

Tests marked ``gpu`` need a B200 (sm_100a) and the built libkvssd_b200.so; all others run on
any CPU host. The oracle (oracle/kvssd_oracle.py) is imported here only as the checker.
"""

from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = ROOT / "tests" / "golden"
for p in (ROOT / "kvssd-attention_b200", ROOT):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU and the built native library")


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device in this environment")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def load_npz(name: str) -> dict:
    with np.load(GOLDEN / name, allow_pickle=False) as z:
        return {k: z[k] for k in z.files}


def load_json(name: str):
    return json.loads((GOLDEN / name).read_text())


def f16(bits: np.ndarray) -> np.ndarray:
    """uint16 bit patterns -> float16 array."""
    return np.asarray(bits, dtype=np.uint16).view(np.float16)


def golden_names(prefix: str) -> list[str]:
    return sorted(p.name for p in GOLDEN.glob(f"{prefix}*.npz"))


QUERY_DTYPES = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16,
                "f64": torch.float64}
