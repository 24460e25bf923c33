"""The benchmark's reference arm on the CPU: one JSON line with the contract's keys, the same
metric, unit and config as the GPU arm's (config 1), and nothing that needs a GPU."""

from __future__ import annotations

import json
import subprocess
import sys

from conftest import ROOT


def test_reference_arm_line_matches_the_gpu_arm_contract():
    out = subprocess.run(
        [sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1", "--warmup", "0",
         "--extra-cpu-seconds", "0.5"],
        capture_output=True, text=True, timeout=600, cwd=ROOT, check=True,
    ).stdout.strip().splitlines()
    assert len(out) == 1
    line = json.loads(out[0])
    sys.path.insert(0, str(ROOT))
    import bench

    assert line["impl"] == "reference"
    assert line["metric"] == bench.Letterbox.metric and line["unit"] == bench.Letterbox.unit
    assert line["higher_is_better"] is True and line["n_gpus"] == 1
    assert line["config"] == bench.Letterbox.static_config()  # the same config as the GPU arm's
    assert line["value"] > 0 and line["e2e"]["value"] == line["value"]
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["cores"] >= 1
    # the extras: every other config of the metric, timed on the same host cores
    assert set(line["extras"]) == set(bench.EXTRAS)
    for key, entry in line["extras"].items():
        assert entry["value"] > 0 and entry["unit"] == bench.WORKLOADS[key].unit, key
        assert entry["metric"] == bench.WORKLOADS[key].metric
    ref = line.get("cpu_baseline_reference")
    if ref is not None and "unavailable" not in ref:  # the reference's offline install is present
        assert ref["kind"] == "reference" and ref["value"] > 0
