"""The benchmark's reference arm on CPU (no GPU needed): one JSON line with
the contract's keys, the same metric and unit as the GPU arm, and the
reference-arm fields (impl, cpu_baseline, e2e with no host-device bytes)."""

import json
import pathlib
import subprocess
import sys

ROOT = pathlib.Path(__file__).resolve().parents[1]


def test_reference_arm_line():
    out = subprocess.run(
        [sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "1",
         "--workload", "c1"],
        cwd=str(ROOT), capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config"):
        assert key in d, key
    assert d["impl"] == "reference"
    assert d["metric"] == "KV store/retrieve GB/s (HBM & pinned-host MemoryObj)"
    assert d["unit"] == "GB/s" and d["higher_is_better"] is True
    assert d["n_gpus"] == 1 and d["steps"] == 1 and d["warmup"] == 1
    assert d["value"] > 0
    assert d["config"]["workload"].startswith("c1")
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["kind"] in ("port", "reference") and cb["cores"] >= 1
    assert d["e2e"] == {"value": d["value"], "unit": "GB/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}
    # the reference arm maps none of the product's native libraries
    assert d["product_libraries_loaded"] == []
    assert "full paged buffers" in cb["sample"]
