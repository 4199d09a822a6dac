"""bench.py's reference arm on the CPU: the JSON contract of its one line, and
that ranks other than 0 of a multi-rank launch print nothing and exit 0."""

import json
import os
import subprocess
import sys

from conftest import ROOT


def run_bench(args, env_extra=None):
    env = dict(os.environ)
    env.update(env_extra or {})
    return subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *args],
                          capture_output=True, text=True, timeout=600, cwd=ROOT, env=env)


def test_reference_arm_json_line():
    r = run_bench(["--impl", "reference", "--size", "384", "--steps", "1", "--warmup", "1"])
    assert r.returncode == 0, r.stderr
    lines = [ln for ln in r.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config"):
        assert key in d, key
    assert d["impl"] == "reference" and d["value"] > 0 and d["higher_is_better"] is True
    assert d["steps"] == 1 and d["warmup"] == 1 and d["config"]["N"] == 384
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == d["value"] and cb["sample"]
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["unit"] == d["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0


def test_reference_arm_other_ranks_are_silent():
    r = run_bench(["--impl", "reference", "--size", "384", "--gpus", "2", "--steps", "1",
                   "--warmup", "1"], {"RANK": "1", "WORLD_SIZE": "2"})
    assert r.returncode == 0, r.stderr
    assert r.stdout.strip() == ""
