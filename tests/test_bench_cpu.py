"""The bench's reference arm on the CPU: the one JSON line the driver reads.

`bench.py --impl reference` times the C restatement of the reference's CPU
mixer path (the Rust reference is not buildable here) and prints one line
with the same metric, unit and config as the GPU arm, plus `cpu_baseline` and
an `e2e` with zero host-device bytes.  Under torchrun only rank 0 runs it;
the other ranks exit 0 without output."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(extra_env=None, *args):
    env = dict(os.environ)
    env.update(extra_env or {})
    return subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", *args],
                          cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)


def test_reference_arm_prints_one_contract_line():
    p = _run(None, "--steps", "1", "--warmup", "3")
    assert p.returncode == 0, p.stderr[-2000:]
    lines = [ln for ln in p.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert d["value"] > 0 and d["unit"] == "tok/s" and d["higher_is_better"] is True
    assert d["steps"] == 1 and d["warmup"] >= 3 and d["n_gpus"] == 1
    assert d["config"]["workload"].startswith("mixer-stack decode")
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["sample"] and cb["value"] == d["value"]
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_exit_quietly():
    p = _run({"RANK": "1", "LOCAL_RANK": "1", "WORLD_SIZE": "2"}, "--steps", "1", "--warmup", "3")
    assert p.returncode == 0, p.stderr[-2000:]
    assert not [ln for ln in p.stdout.splitlines() if ln.startswith("{")]
