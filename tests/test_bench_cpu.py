"""bench.py's reference arm (the CPU port of the reference's torch path) on a tiny sample: the JSON line the driver
parses carries every key of the contract, and ranks other than 0 exit quietly."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CMD = [sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1", "--warmup", "3",
       "--cpu-sample-tokens", "1", "--prompt", "16"]


def test_reference_arm_json_line():
    run = subprocess.run(CMD, capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert run.returncode == 0, run.stderr[-2000:]
    line = json.loads(run.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["unit"] == "tok/s" and line["value"] > 0
    assert line["n_gpus"] == 1 and line["steps"] == 1 and line["warmup"] == 1
    assert line["higher_is_better"] is True and line["vs_baseline"] is None and line["data"] == "synthetic"
    for key in ("metric", "ms_per_step", "scaling", "dtype", "config"):
        assert key in line
    assert line["config"]["workload"].startswith("BASELINE configs[3]")
    cpu = line["cpu_baseline"]
    assert cpu["value"] == line["value"] and cpu["kind"] == "port" and cpu["cores"] >= 1 and cpu["sample"]
    assert line["e2e"] == {"value": line["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_print_nothing():
    run = subprocess.run(CMD, capture_output=True, text=True, timeout=120, cwd=ROOT,
                         env=dict(os.environ, RANK="1", WORLD_SIZE="2"))
    assert run.returncode == 0 and run.stdout.strip() == "", (run.stdout, run.stderr[-1000:])
