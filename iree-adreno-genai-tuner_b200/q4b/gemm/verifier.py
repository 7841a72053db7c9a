"""Verifier: a schedule must pass this before it is allowed onto the GPU (the CUDA counterpart of
gemm/verifier.py:1-189 of the reference).

  1. static rules   legality against the B200's limits and the kernel's own rules, each failure
                    with a reason code (shared memory, TMEM columns per SM, TMA row-pitch and
                    coordinate alignment, split-K counters, grid limits, waste)
  2. mapping check  replay the kernel's tile / k-split / TMA index algebra (q4b.gemm.schedule) and
                    prove: every output tile is owned exactly once, every k step is reduced
                    exactly once, each ring slot's TMA boxes deliver exactly the bytes the
                    producer announces (expect_tx) with 16-byte-aligned inner coordinates,
                    out-of-range rows / cols are covered by the kernel's guards
  3. the library    q4b_gemm_f16_workspace() runs the C++ plan check on the host (no GPU) right
                    before a candidate is measured; disagreement with stages 1-2 is a verifier bug

After measurement the harness still compares C with Cref; a candidate that passes here but fails
there counts against the verifier.
"""

from __future__ import annotations

import collections
import dataclasses

from .schedule import (BK, BM, COUNTER_TILES, SMEM_BUDGET, Schedule, eff_stages, grid, k_range, k_steps, max_stages,
                       sk_accumulators, sk_cta_of, sk_fixup_slots, sk_occupancy, sk_run, sk_segments, sk_tiles,
                       sk_units, smem_bytes, stage_bytes, tma_loads, workspace_bytes)

DEVICES = {
    # B200 (sm_100a): 148 SMs, 227 KB shared memory per CTA (228 KB per SM), 512 TMEM columns per SM
    "b200": dict(sms=148, smem_per_cta=232448, smem_per_sm=233472, tmem_cols=512, max_grid_yz=65535,
                 max_ws_bytes=4 << 30),
}


def static_check(s, sc: Schedule, device="b200"):
    d = DEVICES[device]
    v = []
    if sc.kernel not in (1, 2, 3):
        return ["kernel-id"]
    if sc.kernel == 2:
        return v  # any size and alignment
    if sc.kernel == 3:
        return static_check_sk(s, sc, d)
    if sc.bn not in (64, 128, 256):
        return ["tile-width"]
    # TMA: row pitches must be multiples of 16 bytes (8 fp16) for both stored operands
    lda = s.K if s.la == "N" else s.M
    ldb = s.N if s.lb == "N" else s.K
    if lda % 8:
        v.append("tma-pitch-A")
    if ldb % 8:
        v.append("tma-pitch-B")
    st = eff_stages(sc)
    if sc.stages and not 2 <= sc.stages <= max_stages(sc):
        v.append("ring-depth")
    if st * stage_bytes(sc) > SMEM_BUDGET or smem_bytes(sc) > d["smem_per_cta"]:
        v.append("shared-memory")
    # TMEM: CTAs that fit on one SM by shared memory must fit their accumulators in 512 columns,
    # otherwise later CTAs block in tcgen05.alloc until earlier ones finish
    ctas_per_sm = max(1, d["smem_per_sm"] // (smem_bytes(sc) + 1024))
    if ctas_per_sm * sc.bn > d["tmem_cols"]:
        v.append("tmem-columns")
    kt = k_steps(s)
    if not 1 <= sc.split <= kt:
        v.append("split-range")
    gx, gy, gz = grid(s, sc)
    if gy > d["max_grid_yz"] or gz > d["max_grid_yz"]:
        v.append("grid-size")
    if sc.split > 1 and gx * gy > COUNTER_TILES:
        v.append("split-counters")
    if workspace_bytes(s, sc) > d["max_ws_bytes"]:
        v.append("workspace-size")
    # waste: tiles far wider than the problem (all-padding columns)
    if sc.bn > 64 and sc.bn >= 2 * s.N:
        v.append("tile-exceeds-problem")
    # splits of fewer than two k steps only add partial traffic
    if sc.split > 1 and kt // sc.split < 2:
        v.append("split-too-fine")
    return v


def static_check_sk(s, sc: Schedule, d):
    """Kernel 3's static rules: the kernel-1 tile / TMA / ring rules, no k split (it balances k
    itself), TMEM for its accumulators on every CTA an SM holds, one counter per tile."""
    v = []
    if sc.bn not in (64, 128, 256):
        return ["tile-width"]
    lda = s.K if s.la == "N" else s.M
    ldb = s.N if s.lb == "N" else s.K
    if lda % 8:
        v.append("tma-pitch-A")
    if ldb % 8:
        v.append("tma-pitch-B")
    if sc.stages and not 2 <= sc.stages <= max_stages(sc):
        v.append("ring-depth")
    if eff_stages(sc) * stage_bytes(sc) > SMEM_BUDGET or smem_bytes(sc) > d["smem_per_cta"]:
        v.append("shared-memory")
    if sk_occupancy(sc) * sk_accumulators(sc) * sc.bn > d["tmem_cols"]:
        v.append("tmem-columns")
    if sc.split != 1:
        v.append("split-range")
    tm, tn = sk_tiles(s, sc)
    if tm * tn > COUNTER_TILES:
        v.append("split-counters")
    if workspace_bytes(s, sc) > d["max_ws_bytes"]:
        v.append("workspace-size")
    if sc.bn > 64 and sc.bn >= 2 * s.N:
        v.append("tile-exceeds-problem")
    return v


def mapping_check_sk(s, sc: Schedule):
    """Replay kernel 3's run / segment / part-tile algebra: the runs partition the units with none
    empty; sk_cta_of finds each run's owner; a CTA's segments cover its run in order, whole tiles
    except possibly the first and the last; every tile's units are covered once, by one whole
    segment or by the contiguous CTAs the fix-up finds, whose partial slots are the ones they write."""
    v = []
    U, kt = sk_units(s, sc), k_steps(s)
    G = grid(s, sc)[0]
    if G < 1 or G > U:
        return ["empty-run"]
    prev = 0
    written = {}  # tile -> [(cta, slot, k0, k1)] from the CTAs' own segments
    whole = collections.Counter()
    for c in range(G):
        u0, u1 = sk_run(U, G, c)
        if u0 != prev or u1 <= u0:
            v.append("run-partition")
        prev = u1
        if sk_cta_of(u0, U, G) != c or sk_cta_of(u1 - 1, U, G) != c:
            v.append("run-owner")
        segs = sk_segments(s, sc, c, G)
        if sum(k1 - k0 for _, k0, k1, _ in segs) != u1 - u0:
            v.append("segment-coverage")
        for i, (t, k0, k1, slot) in enumerate(segs):
            if slot is None:
                whole[t] += 1
            else:
                if 0 < i < len(segs) - 1:
                    v.append("partial-middle-segment")
                written.setdefault(t, []).append((c, slot, k0, k1))
    if prev != U:
        v.append("run-partition")
    tm, tn = sk_tiles(s, sc)
    for t in range(tm * tn):
        parts = written.get(t, [])
        if whole[t] + (1 if parts else 0) != 1 or whole[t] > 1:
            v.append("tile-ownership")
            continue
        if not parts:
            continue
        if [(c, slot) for c, slot, _, _ in parts] != sk_fixup_slots(s, sc, t, G):
            v.append("fixup-slots")
        ks = [(k0, k1) for _, _, k0, k1 in parts]
        if ks[0][0] != 0 or ks[-1][1] != kt or any(a[1] != b[0] for a, b in zip(ks, ks[1:])):
            v.append("reduction-coverage")
    return sorted(set(v))


def mapping_check(s, sc: Schedule):
    """Replay the kernel's index algebra for the first, an interior and the last tile."""
    v = []
    if sc.kernel == 3:
        v = mapping_check_sk(s, sc)
        tm, tn = sk_tiles(s, sc)
        sc = Schedule(kernel=1, bn=sc.bn, stages=sc.stages, split=1)  # the same TMA boxes per unit
        gx, gy = tm, tn
        return sorted(set(v + tma_check(s, sc, gx, gy)))
    if sc.kernel == 2:
        gx, gy, _ = grid(s, sc)
        if gx * 64 < s.N or gy * 64 < s.M:
            v.append("output-coverage")
        return v
    gx, gy, gz = grid(s, sc)
    # output tiles: (m_tile, n_tile) -> rows [128 m, 128 m + 128) x cols [bn n, bn n + bn)
    if gx * BM < s.M or gy * sc.bn < s.N or (gx - 1) * BM >= s.M or (gy - 1) * sc.bn >= s.N:
        v.append("output-coverage")
    # every k step reduced exactly once over the splits, each split non-empty
    kcount = collections.Counter()
    for z in range(gz):
        lo, hi = k_range(s, sc, z)
        if hi <= lo:
            v.append("empty-split")
            break
        kcount.update(range(lo, hi))
    if sorted(kcount) != list(range(k_steps(s))) or any(c != 1 for c in kcount.values()):
        v.append("reduction-coverage")
    v += tma_check(s, sc, gx, gy)
    return sorted(set(v))


def tma_check(s, sc: Schedule, gx: int, gy: int):
    """Ring slots: the boxes of one slot deliver exactly stage_bytes (the expect_tx count); the
    innermost coordinate of every box is a multiple of 16 bytes; boxes of one operand tile the
    operand's shared-memory region without overlap (first, an interior and the last tile)."""
    v = []
    tiles = {(0, 0), (gx // 2, gy // 2), (gx - 1, gy - 1)}
    for (mt, nt) in tiles:
        for ks in {0, k_steps(s) - 1}:
            boxes = tma_loads(s, sc, mt, nt, ks)
            total = sum(w * h * 2 for _, _, _, w, h in boxes)
            if total != stage_bytes(sc):
                v.append("expect-tx-mismatch")
            if any((x * 2) % 16 for _, x, _, _, _ in boxes):
                v.append("tma-inner-alignment")
            if any(h > 256 or w * 2 != 128 for _, _, _, w, h in boxes):
                v.append("tma-box")
            # each box covers a run of tile rows (M rows of A, N rows of B) times the slot's 64 k
            rows = {"A": [], "B": []}
            for op, x, y, w, h in boxes:
                mn_major = (op == "A" and s.la == "T") or (op == "B" and s.lb == "N")
                row0 = (x if mn_major else y) - (mt * BM if op == "A" else nt * sc.bn)
                nrow = w if mn_major else h
                k0, nk = (y, h) if mn_major else (x, w)
                if k0 != ks * BK or nk != BK:
                    v.append("tile-coverage")
                rows[op].append((row0, row0 + nrow))
            for op, extent in (("A", BM), ("B", sc.bn)):
                runs = sorted(rows[op])
                if runs[0][0] != 0 or runs[-1][1] != extent or any(a[1] != b[0] for a, b in zip(runs, runs[1:])):
                    v.append("tile-coverage")
    return sorted(set(v))


@dataclasses.dataclass
class Verdict:
    ok: bool
    reasons: list


def verify(s, sc: Schedule, device="b200") -> Verdict:
    r = static_check(s, sc, device)
    if not r:
        r = mapping_check(s, sc)
    return Verdict(not r, r)


def library_accepts(s, sc: Schedule) -> bool:
    """Stage 3: the library's own plan check (host only, no GPU)."""
    import ctypes

    from .._lib import GemmCfg, lib
    c = GemmCfg(**sc.cfg())
    return lib().q4b_gemm_f16_workspace(s.M, s.N, s.K, s.la.encode(), s.lb.encode(), ctypes.byref(c)) >= 0
