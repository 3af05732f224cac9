"""bench.py's CPU arm on CPU: it prints one JSON line whose metric, unit,
direction and config are those of the GPU arm at the same N, so the two arms
describe the same workload (the GPU arm builds its config with the same
helper, decode_config)."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402


def test_cpu_arm_line_matches_the_gpu_arm_config():
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference",
                          "--steps", "1", "--warmup", "3", "--cpu-seconds", "1"],
                         capture_output=True, text=True, timeout=600, check=True).stdout
    lines = [json.loads(l) for l in out.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    line = lines[0]
    assert line["impl"] == "reference"
    assert line["metric"] == bench.METRIC and line["unit"] == "tok/s"
    assert line["higher_is_better"] is True and line["scaling"] == "strong"
    assert line["config"] == bench.decode_config(bench.CFG, 1)
    assert line["value"] > 0 and line["e2e"]["value"] == line["value"]
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["cores"] >= 1


def test_decode_config_names_the_tensor_parallel_split_at_n_gpus():
    one, eight = bench.decode_config(bench.CFG, 1), bench.decode_config(bench.CFG, 8)
    assert one["parallelism"] == "single" and eight["parallelism"].startswith("tp8")
    assert {k: v for k, v in one.items() if k != "parallelism"} == \
        {k: v for k, v in eight.items() if k != "parallelism"}
    per_layer, head = bench.algorithmic_bytes(bench.CFG)
    assert one["bytes_per_step"] == bench.CFG["n_layer"] * sum(per_layer) + head == 4224983044
