"""Schedule search for q4b_gemm_f16 (the CUDA counterpart of the reference's gemm/search.py:148-215
propose -> verify -> rank -> measure -> refit loop).

  python -m q4b.gemm.search --shapes B1 B2 --budget 48 --batch 12 --method ranked random --tag run1

The CUDA schedule space of one shape is small (tile width x ring depth x k split, a few hundred
points), so it is enumerated whole and filtered once by the verifier and by the library's own
plan check; the search then spends its GPU budget in batches over that admissible set:

  ranked  each batch is the unmeasured schedules the cost model predicts fastest, except that a
          quarter of it goes to the best-predicted schedule of each tile width neither measured
          nor in the batch yet (the strata the model knows least about); after each batch the
          residual model is refitted on every measurement so far (all shapes) and the remainder
          re-ranked.
  random  the same budget on admissible schedules in a seeded random order (the control).

Every measurement and every batch summary is one JSON object in <out>/<tag>/log.jsonl (see
Recorder); the fastest correct schedule per shape goes to <out>/<tag>/best.json as
{shape id: {"candidate", "us", "tflops"}}.
"""

from __future__ import annotations

import argparse
import itertools
import json
import pathlib
import random
import time
import zlib

import numpy as np

from . import harness
from .cost_model import ResidualModel
from .schedule import Schedule, default_schedule, domains
from .shapes import BY_ID, SHAPES, make_data
from .verifier import library_accepts, verify


def space(s):
    """Every tcgen05 schedule the domains of shape s name (unverified), one per distinct kernel:
    kernel 1 over tile width x ring depth x k split, kernel 3 (stream-K) over tile width x ring depth."""
    d = domains(s)
    out, keys = [], set()
    cands = [Schedule(kernel=1, bn=bn, stages=st, split=sp)
             for bn, st, sp in itertools.product(d["bn"], d["stages"], d["split"])]
    cands += [Schedule(kernel=3, bn=bn, stages=st) for bn, st in itertools.product(d["bn"], d["stages"])]
    for sc in cands:
        if sc.key() not in keys:
            keys.add(sc.key())
            out.append(sc)
    return out


def admissible(s):
    """(schedules the verifier passes and the library plans, {reason: count} of the rest)."""
    ok, why = [], {}
    for sc in space(s):
        v = verify(s, sc)
        reasons = list(v.reasons) if not v.ok else ([] if library_accepts(s, sc) else ["library-rejects"])
        if reasons:
            for r in reasons:
                why[r] = why.get(r, 0) + 1
        else:
            ok.append(sc)
    return ok, why


class Recorder:
    """Append-only JSON-lines record of a search: {"t": seconds since start, "event": ..., ...}."""

    def __init__(self, path):
        self.path = pathlib.Path(path)
        self.t0 = time.time()

    def __call__(self, event: str, **fields):
        with self.path.open("a") as f:
            f.write(json.dumps({"t": round(time.time() - self.t0, 3), "event": event, **fields}) + "\n")


def run_candidates(s, scheds, data_dir, out_dir, tag, rec, strategy, round_i=0, predicted=None, **hkw):
    """Measure schedules of shape s in one harness process. Returns {schedule key: us or None};
    a wrong result, a launch error or a lost device counts as None."""
    names = [f"{s.id}_{tag}_{i}" for i in range(len(scheds))]
    cands = [{"name": n, "shape_dir": str(pathlib.Path(data_dir) / s.id), "candidate": sc.candidate()}
             for n, sc in zip(names, scheds)]
    results = harness.run_batch(cands, out_dir, f"{s.id}_{tag}", **hkw) if cands else {}
    out = {}
    for i, (n, sc) in enumerate(zip(names, scheds)):
        r = results.get(n, {"ok": False, "error": "no result"})
        good = bool(r.get("ok")) and r.get("us") is not None
        status = "ok" if good else ("wrong" if r.get("err") is not None and not r.get("ok") else "failed")
        out[sc.key()] = float(r["us"]) if good else None
        rec("measurement", shape=s.id, strategy=strategy, round=round_i, schedule=sc.candidate(),
            predicted_us=None if predicted is None else round(float(predicted[i]), 3),
            us=r.get("us"), us_min=r.get("us_min"), rel_err=r.get("err"), status=status, error=r.get("error"),
            tflops=round(s.flops / (r["us"] * 1e6), 2) if good else None)
    return out


def rank_corr(a, b):
    """Spearman correlation of two equal-length sequences (ties broken by position)."""
    if len(a) < 3:
        return None
    ra = np.argsort(np.argsort(np.asarray(a, dtype=float)))
    rb = np.argsort(np.argsort(np.asarray(b, dtype=float)))
    if ra.std() == 0 or rb.std() == 0:
        return None
    return float(np.corrcoef(ra, rb)[0, 1])


def pick_ranked(pool, pred, take, measured_bn):
    """take schedules from pool: the best predicted, except that a quarter of the batch (at least
    one) goes to the best-predicted schedule of each tile width that is neither measured yet nor
    already in the batch, strata taken in order of their best prediction."""
    order = sorted(range(len(pool)), key=lambda i: pred[i])
    quota = max(1, take // 4)
    chosen = order[: max(0, take - quota)]
    covered = measured_bn | {pool[i].bn for i in chosen}
    for i in order:  # stratum leaders: first (best-predicted) schedule of each uncovered width
        if len(chosen) >= take:
            break
        if pool[i].bn not in covered:
            covered.add(pool[i].bn)
            chosen.append(i)
    for i in order:  # fill the rest of the batch by prediction
        if len(chosen) >= take:
            break
        if i not in chosen:
            chosen.append(i)
    return chosen


def tune(s, strategy, budget, batch, model, data_dir, out_dir, rec, seed=0, **hkw):
    """Spend `budget` measurements of shape s with `strategy`. Returns {key: (schedule, us or None)}."""
    pool, rejected = admissible(s)
    rng = random.Random(zlib.crc32(f"{s.id}/{strategy}/{seed}".encode()))
    if strategy == "random":
        rng.shuffle(pool)
    done = {}
    round_i = 0
    while len(done) < budget and pool:
        take = min(batch, budget - len(done), len(pool))
        if strategy == "random":
            idx = list(range(take))
            pred = None
        else:
            pred_all = model.predict_us(s, pool)
            idx = pick_ranked(pool, pred_all, take, {sc.bn for sc, _ in done.values()})
            pred = [pred_all[i] for i in idx]
        scheds = [pool[i] for i in idx]
        t0 = time.time()
        res = run_candidates(s, scheds, data_dir, out_dir, f"{strategy}{round_i}", rec, strategy, round_i, pred, **hkw)
        for sc in scheds:
            done[sc.key()] = (sc, res.get(sc.key()))
            if res.get(sc.key()):
                model.add(s, sc, res[sc.key()])
        taken = set(idx)
        pool = [sc for j, sc in enumerate(pool) if j not in taken]
        model.fit()
        ok = [(p, res[sc.key()]) for sc, p in zip(scheds, pred or [None] * len(scheds)) if res.get(sc.key()) and p]
        best = min((us for _, us in done.values() if us), default=None)
        corr = rank_corr([p for p, _ in ok], [m for _, m in ok]) if ok else None
        rec("round", shape=s.id, strategy=strategy, round=round_i, measured=len(done), remaining=len(pool),
            best_us=best, best_tflops=round(s.flops / (best * 1e6), 2) if best else None, rank_corr=corr,
            model=model.kind, rejected=rejected, gpu_s=round(time.time() - t0, 1))
        print(f"  {s.id} {strategy:6s} batch {round_i}: {len(done):3d} measured, best "
              f"{(s.flops / (best * 1e6)) if best else 0:8.1f} TFLOP/s, rank corr "
              f"{'-' if corr is None else f'{corr:.2f}'} [{model.kind}]", flush=True)
        round_i += 1
    return done


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--shapes", nargs="+", default=[s.id for s in SHAPES])
    ap.add_argument("--method", nargs="+", default=["ranked", "random"], choices=["ranked", "random"])
    ap.add_argument("--budget", type=int, default=48)
    ap.add_argument("--batch", type=int, default=12)
    ap.add_argument("--tag", default="run1")
    ap.add_argument("--out", default="gemm_runs")
    ap.add_argument("--target-ms", type=float, default=20.0)
    ap.add_argument("--reps", type=int, default=5)
    ap.add_argument("--cold", action="store_true", help="flush L2 before every timed call")
    a = ap.parse_args(argv)
    out = pathlib.Path(a.out) / a.tag
    out.mkdir(parents=True, exist_ok=True)
    data = pathlib.Path(a.out) / "data"
    rec = Recorder(out / "log.jsonl")
    model = ResidualModel()  # one model for every shape: residuals transfer through the features
    hkw = dict(target_ms=a.target_ms, reps=a.reps, cold=a.cold)
    best = {}
    for sid in a.shapes:
        s = BY_ID[sid]
        if not (data / s.id / "meta.txt").exists():
            make_data(s, data / s.id)
        print(f"== {s.id} {s.name} M={s.M} N={s.N} K={s.K} {s.layout}", flush=True)
        anchors = [Schedule(kernel=2), default_schedule(s)]
        base = run_candidates(s, anchors, data, out, "anchor", rec, "anchor", **hkw)
        seen = {sc.key(): (sc, base.get(sc.key())) for sc in anchors}
        for sc in anchors:
            us = base.get(sc.key())
            print(f"  {sc.short():24s}: {us and s.flops / (us * 1e6):8.1f} TFLOP/s ({us} us)", flush=True)
        for m in a.method:
            seen.update(tune(s, m, a.budget, a.batch, model, data, out, rec, **hkw))
        fastest = min(((us, sc) for sc, us in seen.values() if us), key=lambda t: t[0], default=None)
        if fastest:
            us, sc = fastest
            best[s.id] = {"candidate": sc.candidate(), "us": us, "tflops": s.flops / (us * 1e6)}
            print(f"  best {sc.short()}: {best[s.id]['tflops']:.1f} TFLOP/s ({us:.2f} us)", flush=True)
    (out / "best.json").write_text(json.dumps(best, indent=1) + "\n")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
