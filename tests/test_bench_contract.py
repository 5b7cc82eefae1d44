"""bench.py's JSON line, as the driver reads it, from the arm that runs here
without a GPU: `--impl reference` times the reference's own CPU engine
(oracle/_ref) on a small sample and prints one line with the contract's keys,
its cpu_baseline and an e2e of no copies; or, where the reference build is
missing, the contract's `unavailable` line.
"""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _last_json(out: str) -> dict:
    lines = [l for l in out.splitlines() if l.startswith("{")]
    assert lines, out[-2000:]
    return json.loads(lines[-1])


def test_reference_arm_line():
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "3",
                        "--no-selfplay"], cwd=ROOT, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    line = _last_json(r.stdout)
    assert line["impl"] == "reference"
    if "unavailable" in line:   # no reference build on this machine
        assert isinstance(line["unavailable"], str) and line["unavailable"]
        return
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "higher_is_better", "scaling", "dtype",
                "data", "config", "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["metric"] == "19x19 net positions/sec" and line["unit"] == "positions/s"
    assert line["value"] > 0 and line["higher_is_better"] is True and line["steps"] == 1 and line["warmup"] >= 3
    cb = line["cpu_baseline"]
    assert cb["kind"] == "reference" and cb["cores"] >= 1 and cb["value"] == line["value"] and cb["sample"]
    e2e = line["e2e"]
    assert e2e["value"] == line["value"] and e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
    assert "workload" in line["config"]


def test_engine_arm_fails_loudly_without_a_gpu():
    """The engine arm has no CPU fallback: without a usable GPU it exits
    non-zero with the reason and prints no measurement line."""
    import azb200

    ok, _ = azb200.cuda_available(0)
    if ok:
        return   # a GPU is present; the GPU tests cover the engine arm
    r = subprocess.run([sys.executable, "bench.py", "--steps", "1", "--warmup", "3", "--no-cpu-baseline",
                        "--no-selfplay"], cwd=ROOT, capture_output=True, text=True, timeout=300)
    assert r.returncode != 0
    assert "no usable GPU" in (r.stdout + r.stderr)
    assert not [l for l in r.stdout.splitlines() if l.startswith("{") and '"value"' in l]
