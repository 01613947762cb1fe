"""The JSON line of `bench.py --impl reference` (the reference arm: the CPU path timed on the host
cores), checked against the bench contract on the CPU.  The b200 arm needs a GPU and is run by
the GPU jobs."""
import json
import os
import subprocess
import sys

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_json_line():
  # --sample-n keeps the CPU block small here; the driver's run times exact blocks of the workload
  out = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "0",
                        "--sample-n", "64"], cwd=REPO, capture_output=True, text=True, timeout=600)
  assert out.returncode == 0, out.stderr[-2000:]
  lines = [l for l in out.stdout.splitlines() if l.startswith("{")]
  assert len(lines) == 1, out.stdout
  d = json.loads(lines[0])
  for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
              "vs_baseline", "dtype", "data", "config"):
    assert key in d, key
  assert d["impl"] == "reference"
  assert d["metric"] == "pairformer_ms_per_block" and d["unit"] == "ms/block"
  assert d["higher_is_better"] is False and d["value"] > 0 and d["steps"] == 1 and d["n_gpus"] == 1
  assert "workload" in d["config"]
  sys.path.insert(0, REPO)
  import bench
  assert d["config"] == bench.workload_config(512, 475, 1)   # the b200 arm prints the same object
  cb = d["cpu_baseline"]
  assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["value"] == d["value"] and cb["sample"]
  assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
