"""The reference arm of bench.py (kvssd's reference decode, restated in numpy, timed on the host
cores) keeps the driver's JSON contract: one line, the measured arm's metric, unit and workload,
a cpu_baseline describing the run and an e2e key with no host-device traffic; ranks other than 0
exit 0 without output. Runs on CPU (about 15 s: one whole c2 layer per step)."""

from __future__ import annotations

import json
import os
import subprocess
import sys

from conftest import ROOT


def _bench(*args: str, env: dict | None = None) -> subprocess.CompletedProcess:
    return subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], cwd=ROOT,
                          env={**os.environ, **(env or {})}, capture_output=True, text=True,
                          timeout=600)


def test_reference_arm_prints_one_contract_line():
    done = _bench("--impl", "reference", "--steps", "1", "--warmup", "3")
    assert done.returncode == 0, done.stderr[-2000:]
    lines = [ln for ln in done.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1
    rec = json.loads(lines[0])
    assert rec["impl"] == "reference" and rec["unit"] == "GB/s" and rec["value"] > 0
    assert (rec["n_gpus"], rec["steps"], rec["warmup"]) == (1, 1, 3)
    assert rec["higher_is_better"] is True and rec["scaling"] == "weak"
    assert rec["vs_baseline"] is None and rec["data"] == "synthetic"
    assert rec["config"]["workload"].startswith("c2: 1 layer x 131072 tokens")
    assert "model" not in rec["config"]
    base = rec["cpu_baseline"]
    assert base["value"] == rec["value"] and base["kind"] in ("port", "reference")
    assert base["cores"] >= 1 and base["sample"]
    assert rec["e2e"] == {"value": rec["value"], "unit": "GB/s", "h2d_bytes_per_step": 0,
                          "d2h_bytes_per_step": 0}
    assert abs(rec["ms_per_step"] - 150994944 / (rec["value"] * 1e9) * 1e3) < 1e-6 * rec["ms_per_step"]


def test_reference_arm_other_ranks_exit_quietly():
    done = _bench("--impl", "reference", "--steps", "1", "--warmup", "3",
                  env={"RANK": "1", "WORLD_SIZE": "2"})
    assert done.returncode == 0, done.stderr[-2000:]
    assert done.stdout.strip() == ""
