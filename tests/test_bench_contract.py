"""bench.py's reference arm on the CPU: one JSON line with the keys the
benchmark contract names, for the training step and the evaluation workload
(small samples so the test runs in seconds)."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
KEYS = {"metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
        "vs_baseline", "dtype", "data", "config", "impl", "cpu_baseline", "e2e"}


@pytest.mark.parametrize("workload,config", [("train", "resnet20"), ("eval", "resnet20")])
def test_reference_arm_line(workload, config):
    env = dict(os.environ, RNN_REF_SAMPLE="2")
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--workload",
                          workload, "--config", config, "--steps", "1", "--warmup", "3"],
                         capture_output=True, text=True, env=env, timeout=600, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert KEYS <= set(d), KEYS - set(d)
    assert d["impl"] == "reference" and d["value"] > 0 and d["higher_is_better"] is True
    assert d["e2e"]["value"] == d["value"] and d["e2e"]["h2d_bytes_per_step"] == 0
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["cores"] >= 1
    assert "workload" in d["config"]


def test_reference_arm_uses_every_host_core_under_torchrun_env():
    """torchrun exports OMP_NUM_THREADS=1 to every rank; the CPU arm must still
    time the restatement on all host cores, so its value is the same at every N."""
    env = dict(os.environ, RNN_REF_SAMPLE="2", OMP_NUM_THREADS="1", RANK="0", WORLD_SIZE="4")
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--config",
                          "resnet20", "--steps", "1", "--warmup", "3", "--gpus", "4"],
                         capture_output=True, text=True, env=env, timeout=600, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    d = json.loads([l for l in out.stdout.splitlines() if l.startswith("{")][0])
    assert d["cpu_baseline"]["cores"] == len(os.sched_getaffinity(0))
