"""bench.py's reference arm on the CPU: the JSON line it prints keeps the bench contract (one line, the arm's metric and
unit, a config that states the batch x sequence it actually timed, cpu_baseline and e2e describing the same run), and
under torchrun only rank 0 times and prints."""
import json
import os
import subprocess
import sys

from conftest import ROOT


def run_reference(extra_env=None):
    env = dict(os.environ, **(extra_env or {}))
    return subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--config", "tiny",
                           "--steps", "2", "--warmup", "1"], cwd=ROOT, env=env, capture_output=True, text=True,
                          timeout=600)


def test_reference_arm_prints_one_honest_line():
    r = run_reference()
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, r.stdout
    line = json.loads(lines[0])
    assert line["impl"] == "reference" and line["unit"] == "tokens/s" and line["higher_is_better"] is True
    assert line["value"] > 0 and line["steps"] == 2 and line["warmup"] == 1
    cfg = line["config"]
    # the config names what was timed: one sequence of the sampled length per step, not the GPU workload's batch
    assert cfg["batch_per_gpu"] == 1 and cfg["global_batch"] == 1 and cfg["seq_len"] >= 1
    cb = line["cpu_baseline"]
    assert cb["value"] == line["value"] and cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["sample"]
    assert line["e2e"] == {"value": line["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_runs_on_rank_zero_only():
    r = run_reference({"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"})
    assert r.returncode == 0, r.stderr[-2000:]
    assert not [l for l in r.stdout.splitlines() if l.startswith("{")]
