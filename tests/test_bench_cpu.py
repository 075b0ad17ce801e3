"""The reference arm of bench.py on the host cores (no GPU): one JSON line per run with the
contract's keys, the metric and unit of the matching B200 workload, a positive value,
and a cpu_baseline / e2e that describe the same run."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
KEYS = {"metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
        "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config", "impl",
        "cpu_baseline", "e2e"}


@pytest.mark.parametrize("workload,unit", [("decode_8b", "committed tok/s"),
                                           ("entropy_select", "GB/s"),
                                           ("block_attention", "TFLOP/s")])
def test_reference_arm_line(workload, unit):
    sys.path.insert(0, ROOT)
    import bench
    # decode_8b: a 2-layer model keeps this contract check to seconds (the driver's run
    # uses all 36 layers)
    extra = ["--layers", "2"] if workload == "decode_8b" else []
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference",
                        "--workload", workload, "--steps", "2", "--warmup", "0"] + extra,
                       capture_output=True, text=True, timeout=300, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, r.stdout[-2000:]
    d = json.loads(lines[0])
    assert KEYS <= set(d), KEYS - set(d)
    assert d["impl"] == "reference" and d["metric"] == bench.METRIC and d["unit"] == unit
    assert d["value"] > 0 and d["n_gpus"] == 1 and d["warmup"] >= 3
    assert d["higher_is_better"] is True
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["kind"] in ("port", "reference")
    assert cb["cores"] >= 1 and cb["sample"]
    assert d["e2e"]["value"] == d["value"] and d["e2e"]["h2d_bytes_per_step"] == 0
    if workload == "decode_8b":
        # the B200 arm's line carries the same workload config (decode_8b_config())
        assert d["config"] == bench.decode_8b_config(2)
