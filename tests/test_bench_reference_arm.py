"""bench.py's reference arm (`--impl reference`) on the host cores: the JSON
line carries the keys the benchmark contract asks of it.  Runs on CPU only
(the arm uses no GPU); skipped where the reference build oracle/_ref is
absent."""
import json
import os
import subprocess
import sys

import pytest

import ref_oracle

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.skipif(not (ref_oracle.available("bench_sdf3d")
                         and ref_oracle.available("static")),
                    reason="oracle/_ref not built")
def test_reference_arm_line():
    env = dict(os.environ, TMNN_REF_BUDGET_S="1")
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"),
                          "--impl", "reference", "--steps", "1", "--warmup", "3"],
                         cwd=ROOT, env=env, capture_output=True, text=True,
                         timeout=300, check=True)
    lines = [l for l in out.stdout.splitlines() if l.strip()]
    assert len(lines) == 1, out.stdout
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert d["value"] > 0 and d["higher_is_better"] is True
    assert d["unit"] == "steps/s (2^18-point batches)"
    assert d["steps"] == 1 and d["warmup"] == 3
    cb = d["cpu_baseline"]
    assert cb["kind"] == "reference" and cb["value"] == d["value"]
    assert cb["cores"] >= 1 and "threadgroups at once" in cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"],
                        "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    n = d["config"]["sample_points_per_step"]
    assert 2048 <= n <= 1 << 18 and n & (n - 1) == 0
    assert d["config"]["same_config"] == (n == 1 << 18)
