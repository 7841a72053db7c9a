"""CPU checks of the GEMM tuner (q4b.gemm): problem files, verifier vs the library's own plan
check, the verifier's replay catching planted index errors, the harness driver's device_lost
recovery (against a fake harness), the cost model and one search run end to end on the fake
harness. No GPU: the library's plan check runs on the host."""

import json
import pathlib
import random
import stat
import sys

import numpy as np
import pytest

from oracle import q4_oracle as O


def _gemm():
    from q4b import gemm
    return gemm


def test_shapes_cover_the_sweep():
    g = _gemm()
    got = {(s.M, s.N, s.K, s.layout) for s in g.SHAPES}
    want = {(m, n, k, "NN") for m in (128, 2048) for n, k in [(5120, 3072), (3072, 3072), (16384, 3072), (3072, 8192)]}
    assert got == want and len(g.SHAPES) == 8
    assert {s.M for s in g.EXTRA} == {1}
    assert len(g.REF_SHAPES) == 8 and g.TOL == 5e-3


@pytest.mark.parametrize("sid", ["S3", "S5", "S8"])
def test_make_data_files_match_the_oracle(tmp_path, sid):
    g = _gemm()
    s = g.BY_ID[sid]
    d = g.make_data(s, tmp_path / sid, seed=0)
    assert g.read_meta(d) == (s.M, s.N, s.K, s.la, s.lb, g.TOL)
    a, b, c = O.gemm_make_data(s.M, s.N, s.K, s.la, s.lb, seed=int(sid[1:]))
    assert np.array_equal(np.fromfile(d / "A.bin", dtype=np.float16), a.ravel())
    assert np.array_equal(np.fromfile(d / "B.bin", dtype=np.float16), b.ravel())
    cref = np.fromfile(d / "Cref.bin", dtype=np.float32).reshape(s.M, s.N)
    assert O.rel_err(cref, c) < 1e-6


def test_verifier_never_passes_what_the_library_rejects():
    g = _gemm()
    from q4b.gemm import search
    ragged = [g.Shape("R1", "r", 100, 200, 136, "NN"), g.Shape("R2", "r", 37, 100, 64, "TN"),
              g.Shape("R3", "r", 3, 5, 7, "TT"), g.Shape("R4", "r", 257, 264, 8, "NT")]
    n_ok = 0
    for s in g.SHAPES + g.EXTRA + g.REF_SHAPES + ragged:
        for sc in search.space(s):
            v = g.verify(s, sc)
            lib_ok = g.library_accepts(s, sc)
            assert not (v.ok and not lib_ok), (s, sc, v)
            n_ok += v.ok
        assert g.verify(s, g.Schedule(kernel=2)).ok
    assert n_ok > 500


def test_verifier_reason_codes():
    g = _gemm()
    s = g.BY_ID["B5"]
    assert "tile-width" in g.verify(s, g.Schedule(kernel=1, bn=96)).reasons
    assert "ring-depth" in g.verify(s, g.Schedule(kernel=1, bn=256, stages=9)).reasons
    assert "split-range" in g.verify(g.BY_ID["S6"], g.Schedule(kernel=1, bn=128, split=2)).reasons
    assert "tma-pitch-B" in g.verify(g.Shape("X1", "x", 64, 100, 64, "NN"), g.Schedule(kernel=1, bn=64)).reasons
    assert "tile-exceeds-problem" in g.verify(g.BY_ID["S3"], g.Schedule(kernel=1, bn=256)).reasons


def test_mapping_check_catches_planted_errors(monkeypatch):
    """Plant index mistakes in the replayed algebra (CPU only) and see the verifier object."""
    g = _gemm()
    from q4b.gemm import schedule, verifier
    s = g.BY_ID["B2"]
    sc = g.Schedule(kernel=1, bn=128, stages=0, split=4)
    assert g.verify(s, sc).ok
    # overlapping k splits
    monkeypatch.setattr(verifier, "k_range", lambda s_, sc_, z: (0, schedule.k_steps(s_) // sc_.split + 1))
    assert "reduction-coverage" in g.verify(s, sc).reasons
    monkeypatch.undo()
    # a B box shifted by 8 elements: misaligned and not covering the tile
    real = schedule.tma_loads

    def shifted(s_, sc_, mt, nt, ks):
        return [(op, x + 8 if op == "B" else x, y, w, h) for op, x, y, w, h in real(s_, sc_, mt, nt, ks)]
    monkeypatch.setattr(verifier, "tma_loads", shifted)
    r = g.verify(s, sc).reasons
    assert "tile-coverage" in r
    # a box of the wrong height: expect_tx no longer matches
    monkeypatch.setattr(verifier, "tma_loads",
                        lambda *a: [(op, x, y, w, h // 2) for op, x, y, w, h in real(*a)])
    assert "expect-tx-mismatch" in g.verify(s, sc).reasons


def test_default_schedule_matches_the_library():
    """The Python restatement of plan_gemm's default agrees with the library's workspace size."""
    import ctypes

    from q4b import _lib
    from q4b.gemm.schedule import workspace_bytes
    g = _gemm()
    L = _lib.lib()
    for s in g.SHAPES + g.EXTRA + g.REF_SHAPES:
        sc = g.default_schedule(s)
        ws = L.q4b_gemm_f16_workspace(s.M, s.N, s.K, s.la.encode(), s.lb.encode(), None)
        assert ws == workspace_bytes(s, sc), (s, sc)
        c = _lib.GemmCfg(**sc.cfg())
        assert L.q4b_gemm_f16_workspace(s.M, s.N, s.K, s.la.encode(), s.lb.encode(), ctypes.byref(c)) == ws


def test_tuned_schedules_are_the_library_default():
    """For the config-2 shapes the library's default plan is the schedule the B200 search measured
    fastest (q4b/gemm/tuned_b200.json, compiled into plan_gemm's table)."""
    import ctypes

    from q4b import _lib
    from q4b.gemm.schedule import tuned_schedules
    L = _lib.lib()
    t = tuned_schedules()
    assert len(t) == 8
    for (m, n, k, lay), sc in t.items():
        out = _lib.GemmCfg()
        assert L.q4b_gemm_f16_plan(m, n, k, lay[0].encode(), lay[1].encode(), None, ctypes.byref(out)) == 0
        assert (out.kernel, out.bn, out.stages, out.split) == (1, sc.bn, sc.stages, sc.split), (m, n, k)
    # a problem outside the table keeps the built-in plan: 256-wide tiles over many rows -> 2 stages
    out = _lib.GemmCfg()
    assert L.q4b_gemm_f16_plan(4096, 4096, 4096, b"N", b"N", None, ctypes.byref(out)) == 0
    assert (out.bn, out.stages) == (256, 2)


def test_cost_model_sanity():
    g = _gemm()
    from q4b.gemm import cost_model
    s = g.BY_ID["B7"]  # 2048 x 16384 x 3072
    t_tc = cost_model.analytic_us(s, g.Schedule(kernel=1, bn=256))
    t_simt = cost_model.analytic_us(s, g.Schedule(kernel=2))
    assert 0 < t_tc < t_simt
    # bounded below by the compulsory DRAM bytes and the tensor peak
    assert t_tc >= s.flops / (cost_model.TENSOR_TFLOPS * 1e6)
    # the residual model: no data = the analytic estimate; a consistent bias is learned (and transfers
    # to schedules it has not seen), noise is not amplified
    m = cost_model.ResidualModel()
    from q4b.gemm import search
    pool, _ = search.admissible(s)
    assert m.kind == "analytic"
    assert abs(m.predict_us(s, pool[:1])[0] / cost_model.analytic_us(s, pool[0]) - 1) < 1e-12
    rng = random.Random(0)
    train, test = pool[::2], pool[1::2]
    for sc in train:
        m.add(s, sc, cost_model.analytic_us(s, sc) * 1.5 * rng.uniform(0.97, 1.03))
    m.fit()
    assert m.kind.startswith("analytic+residual")
    ratio = m.predict_us(s, test) / np.array([cost_model.analytic_us(s, sc) for sc in test])
    assert np.all(np.abs(ratio / 1.5 - 1) < 0.15), ratio


FAKE = r'''#!{py}
import json, sys
man = [a.split("=", 1)[1] for a in sys.argv[1:] if a.startswith("--manifest=")][0]
bad = "{bad}"
for line in open(man):
    name, shape_dir, cand = line.split()
    if name == bad:
        print(json.dumps({{"name": name, "ok": False, "error": "device_lost"}}), flush=True)
        sys.exit(3)
    bn = int(cand.split("bn=")[1].split(",")[0]) if "bn=" in cand else 64
    print(json.dumps({{"name": name, "ok": True, "err": 1e-4, "us": 100.0 / bn, "us_min": 90.0 / bn,
                       "iters": 1, "reps": 1}}), flush=True)
'''


def _fake_bench(tmp_path, bad="none"):
    p = tmp_path / "fake_bench"
    p.write_text(FAKE.format(py=sys.executable, bad=bad))
    p.chmod(p.stat().st_mode | stat.S_IEXEC)
    return p


def test_harness_blames_device_lost_and_reruns_the_rest(tmp_path):
    from q4b.gemm import harness
    bench = _fake_bench(tmp_path, bad="c1")
    cands = [{"name": f"c{i}", "shape_dir": "x", "candidate": f"1:bn={64 << (i % 3)},stages=0,split=1"}
             for i in range(4)]
    res = harness.run_batch(cands, tmp_path / "out", "t", bench=bench)
    assert res["c1"]["ok"] is False and res["c1"]["error"] == "device_lost"
    assert all(res[f"c{i}"]["ok"] for i in (0, 2, 3))
    # the rerun manifest holds only what the failed process had not reached, minus the blamed one
    rerun = (tmp_path / "out" / "t.1.manifest").read_text().split()
    assert "c1" not in rerun and "c2" in rerun and "c0" not in rerun


def test_search_runs_end_to_end_on_a_fake_harness(tmp_path, monkeypatch):
    from q4b.gemm import search
    monkeypatch.setenv("Q4B_GEMM_BENCH", str(_fake_bench(tmp_path)))
    rc = search.main(["--shapes", "B1", "--budget", "10", "--batch", "4", "--tag", "t", "--out", str(tmp_path / "r")])
    assert rc == 0
    best = json.loads((tmp_path / "r" / "t" / "best.json").read_text())
    assert best["B1"]["candidate"].startswith("1:bn=256")  # the fake harness rewards wide tiles
    log = [json.loads(x) for x in (tmp_path / "r" / "t" / "log.jsonl").read_text().splitlines()]
    meas = [r for r in log if r["event"] == "measurement"]
    assert sum(1 for r in meas if r["strategy"] in ("ranked", "random")) == 20
    assert sum(1 for r in meas if r["strategy"] == "anchor") == 2
    # the ranked strategy's stratum leaders reach every tile width within its first two batches
    from q4b.gemm.schedule import Schedule
    early = {Schedule.parse(r["schedule"]).bn for r in meas if r["strategy"] == "ranked" and r["round"] < 2}
    assert early == {64, 128, 256}
    assert all(r["status"] == "ok" for r in meas)
    rounds = [r for r in log if r["event"] == "round"]
    assert [r["round"] for r in rounds if r["strategy"] == "ranked"] == [0, 1, 2]


def test_stream_k_plan_and_workspace():
    """Kernel 3 (persistent stream-K): tile width 256 once there are 8 row tiles (else 128), the
    deepest ring that fits (one CTA per SM, two TMEM accumulators), a shallower ring on request; the
    workspace is the per-tile counters plus two [128][bn] fp32 part-tile slots per CTA (148 CTAs on
    a B200, or one per unit when there are fewer units); split > 1 is rejected."""
    import ctypes

    from q4b import _lib
    L = _lib.lib()

    def plan(m, n, k, **cfg):
        out = _lib.GemmCfg()
        rc = L.q4b_gemm_f16_plan(m, n, k, b"N", b"N", ctypes.byref(_lib.GemmCfg(kernel=3, **cfg)), ctypes.byref(out))
        return rc, (out.kernel, out.bn, out.stages, out.split)

    def ws(m, n, k, **cfg):
        return L.q4b_gemm_f16_workspace(m, n, k, b"N", b"N", ctypes.byref(_lib.GemmCfg(kernel=3, **cfg)))

    assert plan(2048, 5120, 3072) == (0, (3, 256, 4, 1))
    assert plan(128, 5120, 3072) == (0, (3, 128, 6, 1))
    assert plan(128, 5120, 3072, bn=64) == (0, (3, 64, 8, 1))
    assert plan(128, 5120, 3072, stages=3) == (0, (3, 128, 3, 1))
    counters = 64 * 1024
    assert ws(2048, 5120, 3072) == counters + 2 * 148 * 128 * 256 * 4
    # 2 tiles x 2 k steps = 4 units: four CTAs
    assert ws(128, 256, 128) == counters + 2 * 4 * 128 * 128 * 4
    assert plan(128, 5120, 3072, split=2)[0] != 0
    assert plan(128, 5120, 3072, bn=96)[0] != 0


def test_bench_reports_the_plan():
    """bench.py's gemm rows name the schedule each shape ran (the default or --gemm-cfg)."""
    import bench
    assert bench.gemm_plan(128, 16384, 3072) == "1:bn=128,stages=5,split=1"
    assert bench.gemm_plan(2048, 5120, 3072, {"kernel": 3}) == "3:bn=256,stages=4,split=1"
    assert bench.gemm_plan(8, 8, 8, {"kernel": 2}) == "2:bn=0,stages=0,split=1"


def test_stream_k_schedules_in_the_space():
    """Kernel 3 (stream-K) schedules: candidate strings round-trip, the verifier's replay of the
    run / segment / part-tile algebra is clean on the config-2 and ragged shapes, and its workspace
    restatement equals the library's."""
    import ctypes

    from q4b import _lib
    from q4b.gemm import schedule, search
    g = _gemm()
    sc = schedule.Schedule.parse("3:bn=256,stages=4")
    assert (sc.kernel, sc.bn, sc.stages, sc.split) == (3, 256, 4, 1) and sc.candidate() == "3:bn=256,stages=4"
    assert sc.cfg() == dict(kernel=3, bn=256, stages=4)
    L = _lib.lib()
    shapes = g.SHAPES + [g.Shape("R1", "r", 100, 200, 136, "NN"), g.Shape("R5", "r", 4096, 4096, 128, "NN"),
                         g.Shape("R6", "r", 136, 200, 4160, "TT")]
    n3 = 0
    for s in shapes:
        for sc in (x for x in search.space(s) if x.kernel == 3):
            v = g.verify(s, sc)
            if not v.ok:
                assert set(v.reasons) <= {"ring-depth", "shared-memory", "tile-exceeds-problem"}, (s, sc, v)
                continue
            n3 += 1
            ws = L.q4b_gemm_f16_workspace(s.M, s.N, s.K, s.la.encode(), s.lb.encode(),
                                          ctypes.byref(_lib.GemmCfg(**sc.cfg())))
            assert ws == schedule.workspace_bytes(s, sc), (s, sc)
    assert n3 > 50


def test_stream_k_mapping_catches_planted_errors(monkeypatch):
    """Plant mistakes in kernel 3's replayed algebra (CPU only): an owner search one CTA off, a
    fix-up reading the other slot of a contributor, runs that overlap."""
    from q4b.gemm import schedule, verifier
    g = _gemm()
    s, sc = g.BY_ID["B5"], g.Schedule(kernel=3, bn=256)
    assert g.verify(s, sc).ok
    monkeypatch.setattr(verifier, "sk_cta_of", lambda u, U, G: min(G - 1, schedule.sk_cta_of(u, U, G) + 1))
    assert "run-owner" in g.verify(s, sc).reasons
    monkeypatch.undo()
    real = schedule.sk_fixup_slots
    monkeypatch.setattr(verifier, "sk_fixup_slots", lambda *a: [(c, slot ^ 1) for c, slot in real(*a)])
    assert "fixup-slots" in g.verify(s, sc).reasons
    monkeypatch.undo()
    monkeypatch.setattr(verifier, "sk_run", lambda U, G, c: (max(0, U * c // G - 1), U * (c + 1) // G))
    assert "run-partition" in g.verify(s, sc).reasons
