"""bench.py's reference arm on the CPU: the reference's own operators timed
on a bounded sample, printed as the one JSON line the bench contract asks
for (same metric, unit and config keys as the GPU arm)."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.parametrize("gpus", [1, 4])
def test_reference_arm_prints_one_contract_line(gpus):
    res = subprocess.run(
        [sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference",
         "--workload", "qwen2-0.5b-t256", "--gpus", str(gpus), "--steps", "2",
         "--warmup", "1", "--cpu-budget", "0.5"],
        capture_output=True, text=True, timeout=300, cwd=ROOT)
    assert res.returncode == 0, res.stderr[-2000:]
    lines = [l for l in res.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    line = json.loads(lines[0])
    assert line["impl"] == "reference"
    assert line["unit"] == "tokens/s" and line["value"] > 0
    assert line["higher_is_better"] is True and line["steps"] == 2 and line["warmup"] == 1
    assert line["scaling"] == "strong"
    assert line["config"]["workload"] == "qwen2-0.5b-t256"
    assert line["config"]["global_tokens"] == 256
    assert line["e2e"]["h2d_bytes_per_step"] == 0
    cpu = line["cpu_baseline"]
    assert cpu["cores"] >= 1 and cpu["kind"] in ("reference", "port")
    assert cpu["spread_tokens_per_s"]["min"] <= cpu["spread_tokens_per_s"]["max"]
