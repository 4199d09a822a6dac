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


def test_parity_blocks_are_blocks_of_the_full_reference_result():
    """bench.py's parity report runs the oracle on blocks of the full-size
    input.  That is only valid because rows of A and columns of B (lines of A
    for gram) are extracted independently: a block of the oracle's output on
    the block's rows and columns must equal that block of the full result,
    bit for bit.  Checked here on small cases of each kind."""
    import numpy as np
    sys.path.insert(0, ROOT)
    import bench
    import ozaki_oracle as O
    rng = np.random.RandomState(5)
    A, B = rng.randn(300, 1000), rng.randn(1000, 520)
    blocks = bench.sample_blocks(300, 520, rows=64, cols=256)
    assert blocks == [(0, 64, 0, 256), (236, 300, 264, 520)]
    fused, numpy_, exact = bench.reference_blocks("matmul", {"A": A, "B": B}, blocks, 4, 1)
    full_f = O.fused_ondevice(A, B, 4, 1)[2]
    full_n = O.ondevice_numpy(A, B, 4, 1)
    for (r0, r1, c0, c1), f, nn in zip(blocks, fused, numpy_):
        assert np.array_equal(f, full_f[r0:r1, c0:c1])
        assert np.array_equal(nn, full_n[r0:r1, c0:c1])
    # gram: G = (P + P^T) / 2, P = ozaki(A^T, A)
    G = rng.randn(1500, 300) * np.exp(rng.randn(1, 300))
    gb = bench.sample_blocks(300, 300, rows=40, cols=100)
    fused, _, exact = bench.reference_blocks("gram", {"A": G}, gb, 4, 1)
    full = O.gram_ozaki(G, 4, 1)
    for (r0, r1, c0, c1), f in zip(gb, fused):
        assert np.array_equal(f, full[r0:r1, c0:c1])
    # residual: b - ozaki(A, x)
    X, Bv = rng.randn(1000, 16), rng.randn(300, 16)
    rb = bench.sample_blocks(300, 16, rows=64, cols=256)
    fused, _, _ = bench.reference_blocks("residual", {"A": A, "x": X, "b": Bv}, rb, 4, 1)
    full = O.residual_ozaki(A, X, Bv, 4, 1)
    for (r0, r1, c0, c1), f in zip(rb, fused):
        assert np.array_equal(f, full[r0:r1, c0:c1])
    # the report on the reference's own blocks: ratio 1
    rep = bench.parity_report("matmul", {"A": A, "B": B},
                              [full_f[r0:r1, c0:c1] for r0, r1, c0, c1 in blocks], blocks, 4, 1)
    assert rep["within_1p5x_ref"] and rep["rel_err_ours"] == rep["rel_err_ref_fused"]
