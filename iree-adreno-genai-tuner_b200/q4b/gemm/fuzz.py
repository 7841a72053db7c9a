"""Correctness fuzz for the GEMM schedule space (gemm/fuzz.py:1-59 of the reference): per shape,
random verified schedules plus fixed corner schedules and the library default must all match Cref
in the harness.

  python -m q4b.gemm.fuzz --shapes S1 S2 --per-shape 8 --tag fuzz1 [--out gemm_runs]
"""

from __future__ import annotations

import argparse
import collections
import pathlib
import random

from .schedule import Schedule, default_schedule
from .search import Recorder, admissible, run_candidates
from .shapes import BY_ID, REF_SHAPES, make_data
from .verifier import library_accepts, verify

FIXED = [Schedule(kernel=2), Schedule(kernel=1, bn=64, stages=2, split=1), Schedule(kernel=1, bn=256, stages=2, split=1),
         Schedule(kernel=1, bn=128, stages=0, split=3), Schedule(kernel=1, bn=256, stages=0, split=2)]


def pick_schedules(s, n, rng):
    """n admissible schedules drawn at random, plus the corners and the library default."""
    pool, _ = admissible(s)
    picks = rng.sample(pool, min(n, len(pool)))
    seen = {sc.key() for sc in picks}
    for sc in FIXED + [default_schedule(s)]:
        if sc.key() not in seen and verify(s, sc).ok and library_accepts(s, sc):
            seen.add(sc.key())
            picks.append(sc)
    return picks


def run(shapes, per_shape, out, tag, seed=7, **hkw):
    out = pathlib.Path(out)
    data = out / "data"
    log_dir = out / tag
    log_dir.mkdir(parents=True, exist_ok=True)
    rec, rng, tot = Recorder(log_dir / "log.jsonl"), random.Random(seed), collections.Counter()
    failures = []
    for s in shapes:
        if not (data / s.id / "meta.txt").exists():
            make_data(s, data / s.id)
        picks = pick_schedules(s, per_shape, rng)
        res = run_candidates(s, picks, data, log_dir, tag, rec, "fuzz", **hkw)
        ok = sum(1 for sc in picks if res.get(sc.key()))
        tot["ok"] += ok
        tot["n"] += len(picks)
        bad = [sc.short() for sc in picks if not res.get(sc.key())]
        failures += [(s.id, b) for b in bad]
        print(f"{s.id}: {ok}/{len(picks)} correct", ("FAILED: " + " | ".join(bad)) if bad else "", flush=True)
    print("TOTAL", dict(tot))
    return tot, failures


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--shapes", nargs="+", default=[s.id for s in REF_SHAPES])
    ap.add_argument("--per-shape", type=int, default=8)
    ap.add_argument("--tag", default="fuzz")
    ap.add_argument("--out", default="gemm_runs")
    ap.add_argument("--seed", type=int, default=7)
    a = ap.parse_args(argv)
    tot, failures = run([BY_ID[i] for i in a.shapes], a.per_shape, a.out, a.tag, a.seed, target_ms=2.0, reps=1)
    return 0 if not failures else 1


if __name__ == "__main__":
    raise SystemExit(main())
