"""Cost model: ranks verified schedules before any of them touches the GPU (the CUDA counterpart of
gemm/cost_model.py:1-198 of the reference).

  analytic_us(s, sc)  roofline estimate on the B200: per CTA, k steps x max(tcgen05 time, operand
                      load time at the SM's share of L2 bandwidth) + ring fill + epilogue, times
                      the number of waves; bounded below by the DRAM time of the compulsory bytes
                      plus split-K partial traffic; + reduction and launch overheads. Peaks come
                      from MEASURED_PEAKS.json when present (driver-measured copy GB/s and dense
                      bf16 TFLOP/s), else the pool's earlier measurement.
  ResidualModel       the analytic estimate corrected by a ridge regression of log(measured /
                      analytic) on schedule + shape features, refitted after every batch of
                      measurements and shared across shapes.
"""

from __future__ import annotations

import json
import math
import os
import pathlib

import numpy as np

from .schedule import BK, BM, Schedule, eff_stages, grid, k_steps, sk_occupancy, sk_units, smem_bytes


def _peaks():
    for p in (os.environ.get("Q4B_PEAKS"), pathlib.Path.cwd() / "MEASURED_PEAKS.json",
              pathlib.Path(__file__).resolve().parents[3] / "MEASURED_PEAKS.json"):
        if p and pathlib.Path(p).is_file():
            try:
                d = json.loads(pathlib.Path(p).read_text())
                return float(d.get("hbm_gbs", 6650.0)), float(d.get("bf16_tflops", 1590.0))
            except (ValueError, OSError):
                pass
    return 6650.0, 1590.0


HBM_GBS, TENSOR_TFLOPS = _peaks()
SMS = 148
L2_GBS = 20000.0     # aggregate L2 -> SM operand bandwidth assumed for tile re-reads
LAUNCH_US = 3.0      # launch + prologue of one kernel
FILL_US = 0.8        # first ring slot in flight (DRAM latency) + TMEM allocation
EPI_US_PER_KB = 0.004  # TMEM -> registers -> global per KB of output tile


def ctas_per_sm(sc: Schedule) -> int:
    if sc.kernel == 2:
        return 8
    if sc.kernel == 3:
        return sk_occupancy(sc)
    by_smem = max(1, 233472 // (smem_bytes(sc) + 1024))
    return max(1, min(by_smem, 512 // sc.bn))


def analytic_us(s, sc: Schedule) -> float:
    gx, gy, gz = grid(s, sc)
    ctas = gx * gy * gz
    if sc.kernel == 2:
        # CUDA cores: ~1/16 of the tensor peak, operands through L1
        flops = 2.0 * gy * 64 * gx * 64 * s.K
        return flops / (TENSOR_TFLOPS * 1e6 / 16) + s.min_bytes / (HBM_GBS * 1e3) + LAUNCH_US
    per_sm = ctas_per_sm(sc)
    waves = math.ceil(ctas / (SMS * per_sm))
    nk = k_steps(s) / sc.split
    fixup = 0.0
    if sc.kernel == 3:  # one wave of equal runs; part-tiles written and added back by the last CTA
        waves, nk = 1, sk_units(s, sc) / ctas
        fixup = 2.0 * BM * sc.bn * 4 * 2 / (L2_GBS * 1e3 / SMS) + 2 * FILL_US
    step_flops = 2.0 * BM * sc.bn * BK
    t_mma = step_flops / (TENSOR_TFLOPS * 1e6 / SMS)                    # us per k step
    step_bytes = (BM + sc.bn) * BK * 2.0
    active = min(ctas, SMS * per_sm)
    t_load = step_bytes * active / (L2_GBS * 1e3) if active else 0.0     # SMs share L2 bandwidth
    # a shallow ring exposes part of the DRAM latency on every k step
    depth = eff_stages(sc)
    t_step = max(t_mma * per_sm, t_load) * (1.0 + 0.6 / depth)
    t_cta = nk * t_step + FILL_US + EPI_US_PER_KB * BM * sc.bn * 2 / 1024 + fixup
    t_waves = waves * t_cta
    part = 2.0 * sc.split * gx * gy * BM * sc.bn * 4 if sc.split > 1 else 0.0
    t_dram = (s.min_bytes + part) / (HBM_GBS * 1e3)
    red = (part / 2) / (HBM_GBS * 1e3) if sc.split > 1 else 0.0  # the last CTA re-reads partials
    return max(t_waves, t_dram) + red + LAUNCH_US


FEATURE_NAMES = ["logM", "logN", "logK", "A_T", "B_T", "simt", "logBN", "stages", "logSplit", "logCTAs", "waves",
                 "ctas_per_sm", "tile_eff", "k_per_split", "log_analytic", "ai"]


def features(s, sc: Schedule) -> np.ndarray:
    gx, gy, gz = grid(s, sc)
    ctas = gx * gy * gz
    simt = sc.kernel == 2
    bn = 64 if simt else sc.bn
    bm = 64 if simt else BM
    f = [math.log2(s.M), math.log2(s.N), math.log2(s.K), s.la == "T", s.lb == "T", simt, math.log2(bn),
         0 if simt else eff_stages(sc), math.log2(sc.split if not simt else 1), math.log2(ctas),
         ctas / (SMS * ctas_per_sm(sc)), ctas_per_sm(sc), (s.M * s.N) / (gx * bm * gy * bn) if not simt else
         (s.M * s.N) / (gx * 64 * gy * 64), k_steps(s) / (1 if simt else sc.split), math.log(analytic_us(s, sc)),
         s.flops / s.min_bytes]
    return np.array([float(x) for x in f])


class ResidualModel:
    """Analytic estimate times a learned correction: log(us) = log(analytic_us) + w . z(features),
    where z standardises the features over the measurements seen so far and w is a ridge
    regression of the log residuals (closed form, numpy). With no measurements w = 0 and the
    prediction is the analytic estimate; the ridge penalty shrinks the correction towards zero
    while measurements are few, so the model moves away from the analytic ranking only as far as
    the data supports. One instance is shared across shapes: the features are shape-relative, so
    residuals measured on one shape correct the ranking on the next."""

    def __init__(self, ridge: float = 4.0):
        self.ridge = ridge
        self.rows, self.resid = [], []
        self.w = None
        self.mu = self.sd = None

    def add(self, s, sc: Schedule, us: float):
        self.rows.append(features(s, sc))
        self.resid.append(math.log(us) - math.log(analytic_us(s, sc)))

    def fit(self):
        if not self.rows:
            self.w = None
            return
        X = np.stack(self.rows)
        self.mu = X.mean(0)
        self.sd = X.std(0)
        self.sd[self.sd < 1e-9] = 1.0
        Z = np.hstack([np.ones((len(X), 1)), (X - self.mu) / self.sd])
        r = np.asarray(self.resid)
        A = Z.T @ Z + self.ridge * np.eye(Z.shape[1])
        self.w = np.linalg.solve(A, Z.T @ r)

    def correction(self, s, sc: Schedule) -> float:
        if self.w is None:
            return 0.0
        z = np.concatenate([[1.0], (features(s, sc) - self.mu) / self.sd])
        return float(z @ self.w)

    def predict_us(self, s, scheds) -> np.ndarray:
        return np.array([analytic_us(s, sc) * math.exp(self.correction(s, sc)) for sc in scheds])

    @property
    def kind(self) -> str:
        return "analytic" if self.w is None else f"analytic+residual({len(self.rows)})"
