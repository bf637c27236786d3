"""The reference arm of bench.py (the oracle port timed on the host cores)
prints one well-formed JSON line with the keys the bench contract names, on a
small workload, without a GPU."""
from __future__ import annotations

import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_prints_one_json_line():
    p = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--workload", "c1",
                        "--steps", "1", "--warmup", "0"], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert p.returncode == 0, p.stderr[-2000:]
    lines = [l for l in p.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["unit"] == "tokens/s" and d["value"] > 0
    assert d["higher_is_better"] is True and d["n_gpus"] == 1
    assert d["dtype"] == "f64 (oracle arithmetic on f32 inputs)"  # c1 is an f32 workload
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == d["value"]
    assert d["e2e"] == {"value": d["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    # ms_per_step is the measured wall time of the sampled work, the whole-prefill
    # figure sits under its own key; config equals the GPU arm's dict
    assert d["extrapolated"]["extrapolated"] is True
    assert d["extrapolated"]["value"] == d["value"]
    assert d["ms_per_step"] <= d["extrapolated"]["ms_per_prefill"]
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "edge-prefill_b200"))
    import bench
    import workloads as W

    assert d["config"] == bench.config_of(W.CONFIGS["c1"], 1, False)
