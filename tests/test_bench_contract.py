"""bench.py's reference arm on the host cores (`--impl reference`: the CPU restatement of
the decode path) prints the one JSON line the benchmark contract asks for.  Runs on CPU
with a 2-layer model so that it takes seconds."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_json_line():
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--layers", "2",
                        "--steps", "1", "--warmup", "1", "--cpu-seconds", "2"],
                       cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, r.stdout
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["value"] > 0 and d["n_gpus"] == 1 and d["steps"] == 1
    for k in ("metric", "unit", "higher_is_better", "scaling", "dtype", "data", "config", "ms_per_step"):
        assert k in d, k
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["sample"] and cb["value"] == d["value"]
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
