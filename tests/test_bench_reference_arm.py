"""The reference arm of bench.py (`--impl reference`): the CPU oracle port timed on the host
cores, one JSON line on rank 0 with the contract's keys and the repo arm's config entry;
other ranks print nothing.  A reduced grid keeps the CPU work to seconds."""
import json
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
ARGS = [sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1", "--warmup", "3",
        "--cpu-sample-blocks", "2", "--grid", "4,16,32", "--heads", "4"]


def test_reference_arm_prints_one_contract_line():
    run = subprocess.run(ARGS, cwd=ROOT, capture_output=True, text=True, timeout=600,
                         env={**os.environ, "RANK": "0", "WORLD_SIZE": "1"})
    assert run.returncode == 0, run.stderr
    lines = [ln for ln in run.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1
    line = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["impl"] == "reference"
    assert line["value"] > 0 and line["warmup"] >= 3
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["cores"] >= 1
    assert line["cpu_baseline"]["value"] == line["value"]
    assert line["e2e"] == {"value": line["value"], "unit": line["unit"], "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}
    assert "workload" in line["config"]
    sys.path.insert(0, str(ROOT))
    import bench

    bench.GRID, bench.HEADS = (4, 16, 32), 4
    T = 4 * 16 * 32
    assert line["config"] == json.loads(json.dumps(bench.config1_dict(1, bench.ops_target_topk(T), T)))
    assert line["extrapolated"]["attention_extrapolation_factor"] == line["cpu_baseline"]["attention_extrapolation_factor"]
    assert "route of all 4 heads in full" in line["cpu_baseline"]["sample"]
    assert line["cpu_baseline"]["summary_extrapolation_factor"] == 2


def test_reference_arm_other_ranks_stay_silent():
    run = subprocess.run(ARGS, cwd=ROOT, capture_output=True, text=True, timeout=600,
                         env={**os.environ, "RANK": "1", "WORLD_SIZE": "2"})
    assert run.returncode == 0, run.stderr
    assert run.stdout.strip() == ""
