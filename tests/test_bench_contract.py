"""The bench's reference arm runs on CPU: check that its single JSON line
carries the keys the bench contract requires (metric, value, unit, the
cpu_baseline description and an e2e object with no host-device bytes), that
it times the reference's own src/reference.py when its offline install is
present, and that its config object is the one our arm prints."""

import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_json_line():
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "2",
                          "--warmup", "1"], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.strip().splitlines() if l.startswith("{")]
    assert len(lines) == 1, out.stdout
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "higher_is_better", "config"):
        assert key in d, key
    assert d["value"] > 0 and d["unit"] == "TB/s" and d["higher_is_better"] is True
    cb = d["cpu_baseline"]
    ref_installed = os.path.isfile(os.path.join(ROOT, "baseline", "_ref", "reference.py"))
    assert cb["kind"] == ("reference" if ref_installed else "port") and cb["cores"] >= 1 and cb["sample"] and cb["value"] == d["value"]
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["unit"] == d["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
    # both arms print the same config object for the same workload
    sys.path.insert(0, ROOT)
    import bench

    assert d["config"] == bench.workload_config("c2", 1)
    assert d["metric"] == bench.metric_name("c2")
