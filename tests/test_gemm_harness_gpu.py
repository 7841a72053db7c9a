"""The harness protocol on the GPU: gemm_bench over the reference tuner's problems with random
verified schedules (the gemm/fuzz.py pattern), and the check catching a wrong reference."""

import json
import subprocess

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_fuzz_reference_shapes(tmp_path):
    from q4b.gemm import REF_SHAPES, fuzz
    tot, failures = fuzz.run(REF_SHAPES, 5, tmp_path, "fuzz", seed=11, target_ms=1.0, reps=1)
    assert not failures, failures
    assert tot["n"] >= 8 * 6


def test_harness_reports_a_mismatch(tmp_path):
    """Plant the mistake in the reference file (CPU side): the harness must report ok=false."""
    from q4b.gemm import BY_ID, make_data
    from q4b.gemm.harness import BENCH
    s = BY_ID["S8"]
    d = make_data(s, tmp_path / s.id)
    c = np.fromfile(d / "Cref.bin", dtype=np.float32)
    c[len(c) // 2] += 10.0
    c.tofile(d / "Cref.bin")
    man = tmp_path / "m.txt"
    man.write_text(f"bad {d} 1:bn=128,stages=0,split=1\n# a comment line\nnan_free {d} 2:\n")
    out = subprocess.run([str(BENCH), f"--manifest={man}", "--target-ms=1", "--reps=1", "--warmup-ms=10"],
                         capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stderr
    lines = [json.loads(x) for x in out.stdout.splitlines()]
    assert [r["name"] for r in lines] == ["bad", "nan_free"]
    assert all(r["ok"] is False and 1e-3 < r["err"] < 1.0 for r in lines)
    assert all(r["us"] > 0 and r["iters"] >= 1 for r in lines)
