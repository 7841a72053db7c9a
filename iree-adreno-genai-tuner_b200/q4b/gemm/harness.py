"""Runs batches of GEMM candidates through the harness binary (the CUDA counterpart of
gemm/device.py:68-126's run_batch; the transport is a local process instead of adb).

A batch is written as one manifest (<name> <shape_dir> <candidate> per line); the harness prints
one JSON line per candidate. Recovery follows the reference's protocol: when the harness exits 3
(a sticky device error, reported as "device_lost" for the candidate being run) that candidate is
blamed and recorded as failed, and the candidates it had not reached are run again in a fresh
process (bounded retries); any other non-zero exit fails the candidates without a result line.
"""

from __future__ import annotations

import json
import os
import pathlib
import subprocess

BENCH = pathlib.Path(__file__).resolve().parents[1] / "bin" / "gemm_bench"


def run_batch(cands, out_dir, tag, *, bench=None, target_ms=30.0, reps=5, cold=False, timeout=900, retries=2,
              extra_args=()):
    """cands: [{"name", "shape_dir", "candidate"}] -> {name: result dict}."""
    bench = pathlib.Path(bench or os.environ.get("Q4B_GEMM_BENCH") or BENCH)
    out_dir = pathlib.Path(out_dir)
    out_dir.mkdir(parents=True, exist_ok=True)
    results = {}
    todo = list(cands)
    attempt = 0
    while todo:
        manifest = out_dir / f"{tag}.{attempt}.manifest"
        manifest.write_text("".join(f"{c['name']} {c['shape_dir']} {c['candidate']}\n" for c in todo))
        cmd = [str(bench), f"--manifest={manifest}", f"--target-ms={target_ms}", f"--reps={reps}", *extra_args]
        if cold:
            cmd.append("--cold")
        try:
            p = subprocess.run(cmd, capture_output=True, text=True, timeout=timeout)
            out, rc, err = p.stdout, p.returncode, p.stderr
        except subprocess.TimeoutExpired as e:
            out = e.stdout.decode() if isinstance(e.stdout, bytes) else (e.stdout or "")
            rc, err = -9, "timeout"
        blamed = None
        for line in out.splitlines():
            try:
                r = json.loads(line)
            except ValueError:
                continue
            if "name" in r:
                results[r["name"]] = r
                if r.get("error") == "device_lost":
                    blamed = r["name"]
        remaining = [c for c in todo if c["name"] not in results]
        if rc == 0 or not remaining:
            break
        if rc == 3 and attempt < retries:
            attempt += 1
            todo = [c for c in remaining if c["name"] != blamed]
            continue
        for c in remaining:
            results[c["name"]] = {"name": c["name"], "ok": False, "error": f"harness exit {rc}: {err.strip()[-200:]}"}
        break
    return results
