"""bench.py's reference arm -- the reference's CPU path, which the round-end run times beside the CUDA path -- prints
the benchmark contract's JSON line on a host without a GPU."""

from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def test_reference_arm_prints_the_contract_line():
    run = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "1"],
                         cwd=ROOT, capture_output=True, text=True, timeout=900)  # fmt: skip
    assert run.returncode == 0, run.stderr[-2000:]
    line = json.loads(run.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference"
    assert line["metric"] == "latent-descent sample-steps/s (L=900, B=128)" and line["unit"] == "sample-steps/s"
    assert line["higher_is_better"] is True and line["steps"] == 1 and line["n_gpus"] == 1
    assert line["value"] > 0
    assert line["e2e"] == {"value": line["value"], "unit": line["unit"], "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}  # fmt: skip
    cpu = line["cpu_baseline"]
    assert cpu["value"] == line["value"] and cpu["cores"] >= 1 and cpu["kind"] in ("port", "reference") and cpu["sample"]
