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
    # the same config dict as the GPU arm's at this world size (a sample of it is timed)
    import importlib.util
    spec = importlib.util.spec_from_file_location("bench_mod", os.path.join(ROOT, "bench.py"))
    bm = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bm)
    assert d["config"] == bm.decode_config(1, bm.B_PER_GPU, bm.CTX)
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["sample"] and cb["value"] == d["value"]
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_exit_quietly():
    p = _run({"RANK": "1", "LOCAL_RANK": "1", "WORLD_SIZE": "2"}, "--steps", "1", "--warmup", "3")
    assert p.returncode == 0, p.stderr[-2000:]
    assert not [ln for ln in p.stdout.splitlines() if ln.startswith("{")]


def test_clock_samples_summary():
    """The clocks record of the JSON line, from nvidia-smi CSV samples: median SM clock under load, the
    max clock, and every throttle reason seen Active (sw_power_cap is kept and noted; the hw/thermal ones
    make a run invalid)."""
    sys.path.insert(0, ROOT)
    import bench

    lines = [
        "0, 1965, 1965, 700.1, 0x0000000000000000, Not Active, Not Active, Not Active, Not Active",
        "0, 1890, 1965, 990.5, 0x0000000000000004, Not Active, Not Active, Not Active, Active",
        "0, 1950, 1965, 995.0, 0x0000000000000004, Not Active, Not Active, Not Active, Active",
        "0, [N/A], 1965, 0, 0x0, Not Active, Not Active, Not Active, Not Active",
        "garbage",
    ]
    d = bench.Clocks.summarize(lines)
    assert d == {"sm_mhz": 1950.0, "sm_max_mhz": 1965.0, "reasons": ["sw_power_cap"], "samples": 3}
    hot = bench.Clocks.summarize([lines[0].replace("Not Active, Not Active, Not Active, Not Active",
                                                   "Active, Not Active, Active, Not Active")])
    assert hot["reasons"] == ["hw_slowdown", "sw_thermal_slowdown"]
    assert bench.Clocks.summarize([])["sm_mhz"] is None
