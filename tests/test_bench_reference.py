"""bench.py's reference arm (`--impl reference`): the oracle -- the reference's
CPU kernels restated -- timed on this host's cores, printing one JSON line on
the same metric, unit and workload as the CUDA arm of the same config, with
the cpu_baseline and e2e blocks the bench contract asks for.  CPU only."""
from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))
import bench  # noqa: E402


def _line(*args: str) -> dict:
    out = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1",
                          "--warmup", "0", *args], cwd=ROOT, capture_output=True, text=True,
                         timeout=600, check=True).stdout
    return json.loads(out.strip().splitlines()[-1])


@pytest.mark.parametrize("config,metric", [("2", bench.METRIC), ("3", bench.METRIC3),
                                           ("4", bench.METRIC4), ("5", bench.METRIC5)])
def test_reference_arm_line(config, metric):
    d = _line("--config", config)
    assert d["impl"] == "reference"
    assert d["metric"] == metric and d["unit"] == "tokens/s" and d["higher_is_better"] is True
    assert d["value"] > 0 and d["ms_per_step"] > 0
    assert d["config"]["workload"].startswith(f"config {config}")
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["sample"]
    assert cb["value"] == d["value"]
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["unit"] == d["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
