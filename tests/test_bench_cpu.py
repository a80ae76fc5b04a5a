"""The reference arm of bench.py on CPU: `bench.py --impl reference` times the
reference's own decode (oracle/_ref, main.c compiled unchanged) and prints one
JSON line with the contract's keys; under torchrun only rank 0 prints it."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(args, env_extra=None, timeout=600):
    env = dict(os.environ)
    env.update(env_extra or {})
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *args], cwd=ROOT, env=env,
                       capture_output=True, text=True, timeout=timeout)
    assert r.returncode == 0, r.stderr[-2000:]
    return [ln for ln in r.stdout.splitlines() if ln.startswith("{")]


def test_reference_arm_json_line():
    lines = _run(["--impl", "reference", "--steps", "2", "--warmup", "3"])
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    if "unavailable" in d:  # the reference tree was absent when oracle/_ref was built
        return
    assert d["metric"] == "decode tok/s" and d["unit"] == "tok/s" and d["higher_is_better"] is True
    assert d["steps"] == 2 and d["warmup"] == 3 and d["value"] > 0
    assert abs(d["ms_per_step"] - 1e3 / d["value"]) < 1e-6 * d["ms_per_step"] + 1e-9
    cb = d["cpu_baseline"]
    assert cb["kind"] == "reference" and cb["cores"] >= 1 and cb["value"] == d["value"]
    assert d["e2e"] == {"value": d["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert d["config"]["sequences"] == 64


def test_reference_arm_other_ranks_print_nothing():
    assert _run(["--impl", "reference", "--steps", "1", "--warmup", "3"], {"RANK": "1"}) == []
