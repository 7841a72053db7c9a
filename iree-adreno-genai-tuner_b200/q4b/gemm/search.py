"""Schedule search for q4b_gemm_f16: propose -> verify -> rank (cost model) -> measure the top k
through the harness -> learn (the CUDA counterpart of gemm/search.py:1-275 of the reference).

  python -m q4b.gemm.search --shapes B1 B2 --budget 48 --batch 12 --method model random --tag run1

method=model   evolutionary search: each round pools random schedules plus mutations / crossovers of
               the best measured ones, keeps the verifier-approved ones the library also accepts,
               ranks them with the cost model, measures the top `batch` (25% exploration picks) in
               one harness call, refits the model.
method=random  the same GPU budget spent on verifier-approved schedules in random order.
Every candidate's verdict, prediction and measurement goes to <out>/<tag>/log.jsonl; the best
schedule per shape goes to <out>/<tag>/best.json ({shape id: candidate string}).
"""

from __future__ import annotations

import argparse
import collections
import dataclasses
import json
import pathlib
import random
import time

from . import harness
from .cost_model import Learned
from .schedule import Schedule, default_schedule, domains
from .shapes import BY_ID, SHAPES, make_data
from .verifier import library_accepts, verify


def random_sched(s, rng):
    d = domains(s)
    return Schedule(kernel=1, bn=rng.choice(d["bn"]), stages=rng.choice(d["stages"]), split=rng.choice(d["split"]))


def mutate(s, sc, rng):
    d = domains(s)
    k = dataclasses.asdict(sc)
    for name in rng.sample(list(d), rng.choice([1, 1, 2])):
        k[name] = rng.choice(d[name])
    k["kernel"] = 1
    return Schedule(**k)


def crossover(a, b, rng):
    ka, kb = dataclasses.asdict(a), dataclasses.asdict(b)
    return Schedule(**{n: (ka if rng.random() < 0.5 else kb)[n] for n in ka})


class Log:
    def __init__(self, path):
        self.f = open(path, "a")

    def write(self, **kw):
        self.f.write(json.dumps(kw) + "\n")
        self.f.flush()


def measure(s, scheds, data_dir, out_dir, tag, log, meta, metric="us", **hkw):
    """Run a batch through the harness. Returns {key: time or None}."""
    cands, by_name = [], {}
    for i, sc in enumerate(scheds):
        name = f"{s.id}_{tag}_{i}"
        cands.append({"name": name, "shape_dir": str(data_dir / s.id), "candidate": sc.candidate()})
        by_name[name] = sc
    res = harness.run_batch(cands, out_dir, f"{s.id}_{tag}", **hkw) if cands else {}
    out = {}
    for name, sc in by_name.items():
        r = res.get(name, {"ok": False, "error": "missing"})
        good = bool(r.get("ok")) and r.get("us") is not None
        out[sc.key()] = r[metric] if good else None
        log.write(**meta, shape=s.id, sched=dataclasses.asdict(sc), stage="gpu", ok=good, us=r.get("us"),
                  us_min=r.get("us_min"), err=r.get("err"), error=r.get("error"),
                  tflops=(s.flops / (r["us"] * 1e6)) if good else None)
    return out


def tune(s, method, budget, batch, model, data_dir, out_dir, log, seed=0, pool=400, init=None, **hkw):
    rng = random.Random(seed * 1000 + int(s.id[1:]) + (0 if method == "model" else 7))
    measured = dict(init or {})  # key -> (sched, us or None)
    budget += len(measured)
    rejected = collections.Counter()
    round_i = 0
    while len(measured) < budget:
        props = [random_sched(s, rng) for _ in range(pool)]
        if method == "model":
            good = sorted(((us, sc) for sc, us in measured.values() if us), key=lambda t: t[0])[:8]
            for _ in range(pool if good else 0):
                p = rng.choice(good)[1]
                props.append(mutate(s, p, rng) if rng.random() < 0.75 else crossover(p, rng.choice(good)[1], rng))
        seen, valid = set(measured), []
        for sc in props:
            k = sc.key()
            if k in seen:
                continue
            seen.add(k)
            v = verify(s, sc)
            if v.ok and not library_accepts(s, sc):
                v.ok, v.reasons = False, ["library-rejects"]
            if v.ok:
                valid.append(sc)
            else:
                rejected.update(v.reasons)
        if not valid:
            break
        take = min(batch, budget - len(measured))
        meta = dict(method=method, round=round_i, model=model.kind if method == "model" else "none")
        if method == "random":
            rng.shuffle(valid)
            pick, preds = valid[:take], [None] * min(take, len(valid))
        else:
            preds_all = model.predict_us(s, valid)
            order = sorted(range(len(valid)), key=lambda i: preds_all[i])
            n_exploit = max(1, int(take * 0.75))
            exploit = [valid[i] for i in order[:n_exploit]]
            rest = [valid[i] for i in order[n_exploit:]]
            pick = exploit + rng.sample(rest, min(len(rest), take - n_exploit))
            idx = {sc.key(): i for i, sc in enumerate(valid)}
            preds = [float(preds_all[idx[sc.key()]]) for sc in pick]
        t0 = time.time()
        res = measure(s, pick, data_dir, out_dir, f"{method}{round_i}", log, meta, **hkw)
        for sc in pick:
            us = res.get(sc.key())
            measured[sc.key()] = (sc, us)
            if us:
                model.add(s, sc, us)
        pairs = [(pr, res.get(sc.key())) for sc, pr in zip(pick, preds) if pr and res.get(sc.key())]
        rho = None
        if len(pairs) >= 5 and len({p for p, _ in pairs}) > 1 and len({m for _, m in pairs}) > 1:
            from scipy.stats import spearmanr
            rho = float(spearmanr([p for p, _ in pairs], [m for _, m in pairs]).correlation)
        model.fit()
        best = min((us for _, us in measured.values() if us), default=None)
        log.write(kind="round", shape=s.id, method=method, round=round_i, n=len(measured), best_us=best, rho=rho,
                  valid=len(valid), proposed=len(props), gpu_s=round(time.time() - t0, 1), model=meta["model"],
                  rejected=dict(rejected))
        print(f"  {s.id} {method:6s} round {round_i}: measured {len(measured):3d}  best "
              f"{best and s.flops / (best * 1e6):8.1f} TFLOP/s  rank-rho {rho if rho is None else round(rho, 2)}  "
              f"[{meta['model']}] valid {len(valid)}/{len(props)}", flush=True)
        round_i += 1
    return measured, rejected


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--shapes", nargs="+", default=[s.id for s in SHAPES])
    ap.add_argument("--method", nargs="+", default=["model", "random"])
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
    log = Log(out / "log.jsonl")
    model = Learned()  # shared across shapes: knowledge transfers from earlier shapes
    hkw = dict(target_ms=a.target_ms, reps=a.reps, cold=a.cold)
    best = {}
    for sid in a.shapes:
        s = BY_ID[sid]
        if not (data / s.id / "meta.txt").exists():
            make_data(s, data / s.id)
        print(f"== {s.id} {s.name} M={s.M} N={s.N} K={s.K} {s.layout}", flush=True)
        base = measure(s, [Schedule(kernel=2), default_schedule(s)], data, out, "baseline", log,
                       dict(method="baseline", round=0, model="none"), **hkw)
        for sc in (Schedule(kernel=2), default_schedule(s)):
            us = base.get(sc.key())
            print(f"  {sc.short():24s}: {us and s.flops / (us * 1e6):8.1f} TFLOP/s ({us} us)", flush=True)
        results = {sc.key(): (sc, base.get(sc.key())) for sc in (Schedule(kernel=2), default_schedule(s))}
        for m in a.method:
            measured, _ = tune(s, m, a.budget, a.batch, model, data, out, log, **hkw)
            results.update(measured)
        top = min(((us, sc) for sc, us in results.values() if us), key=lambda t: t[0], default=None)
        if top:
            best[s.id] = {"candidate": top[1].candidate(), "us": top[0], "tflops": s.flops / (top[0] * 1e6)}
            print(f"  best {top[1].short()}: {best[s.id]['tflops']:.1f} TFLOP/s ({top[0]:.2f} us)", flush=True)
    (out / "best.json").write_text(json.dumps(best, indent=1) + "\n")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
