"""The GEMM problems of the tuner and their on-disk form (gemm/shapes.py:1-66 of the reference).

C[M,N] = op(A) @ op(B), fp16 in / out, fp32 accumulation. Layout letters follow BLAS:
  A "N": stored [M][K] row-major      A "T": stored [K][M]
  B "N": stored [K][N] row-major      B "T": stored [N][K]  (a torch Linear weight)

A shape directory holds meta.txt ("M N K LA LB TOL"), A.bin and B.bin (fp16, stored layout) and
Cref.bin (fp32 row-major [M][N]) -- the files the harness (q4b/bin/gemm_bench) reads.

SHAPES are the B200 sweep: M in {128, 2048} x the Llama-3.2-3B projections (N, K) in
{(5120, 3072), (3072, 3072), (16384, 3072), (3072, 8192)}, row-major A [M,K] and B [K,N] ("NN");
the M = 1 rows of the same projections are EXTRA (memory-bound). REF_SHAPES are the reference
tuner's own eight problems (gemm/shapes.py:41-50), kept for the correctness fuzz.
"""

from __future__ import annotations

import dataclasses
import pathlib

import numpy as np


@dataclasses.dataclass(frozen=True)
class Shape:
    id: str
    name: str
    M: int
    N: int
    K: int
    layout: str  # "NN" | "NT" | "TN" | "TT"
    note: str = ""

    @property
    def la(self):
        return self.layout[0]

    @property
    def lb(self):
        return self.layout[1]

    @property
    def flops(self):
        return 2.0 * self.M * self.N * self.K

    @property
    def min_bytes(self):  # compulsory traffic: A and B read once, C written once (fp16)
        return 2.0 * (self.M * self.K + self.K * self.N + self.M * self.N)


_PROJ = [("qkv", 5120, 3072), ("o", 3072, 3072), ("gate_up", 16384, 3072), ("down", 3072, 8192)]

SHAPES = [Shape(f"B{i + 1}", f"{p}_m{m}", m, n, k, "NN", "3B projection" + (" (prefill chunk)" if m == 128 else ""))
          for i, (m, (p, n, k)) in enumerate((m, pnk) for m in (128, 2048) for pnk in _PROJ)]
EXTRA = [Shape(f"B{9 + i}", f"{p}_m1", 1, n, k, "NN", "3B projection, batch-1 decode (HBM-bound)")
         for i, (p, n, k) in enumerate(_PROJ)]
REF_SHAPES = [
    Shape("S1", "square_nn", 1024, 1024, 1024, "NN", "regular square"),
    Shape("S2", "prefill_nt", 128, 3072, 3072, "NT", "prefill: 128 tokens x Linear(3072, 3072)"),
    Shape("S3", "skinny_tn", 4096, 64, 1024, "TN", "tall-skinny"),
    Shape("S4", "flat_nt", 16, 4096, 4096, "NT", "short-wide: batch-16 decode"),
    Shape("S5", "largek_tt", 256, 256, 8192, "TT", "large K"),
    Shape("S6", "smallk_nn", 2048, 2048, 32, "NN", "small K (rank-32 update)"),
    Shape("S7", "gemv_nt", 1, 4096, 4096, "NT", "matrix-vector"),
    Shape("S8", "regular_tn", 768, 768, 768, "TN", "regular, A transposed"),
]
BY_ID = {s.id: s for s in SHAPES + EXTRA + REF_SHAPES}

TOL = 5e-3  # max|C - Cref| / max|Cref| (gemm/shapes.py:53)


def make_data(s: Shape, out: pathlib.Path, seed: int = 0) -> pathlib.Path:
    """Write meta.txt, A.bin, B.bin (fp16 U(-1, 1), stored layout) and Cref.bin (fp32 A @ B).

    Seeded per shape (seed + the shape's number), so every run regenerates identical files."""
    out = pathlib.Path(out)
    out.mkdir(parents=True, exist_ok=True)
    rng = np.random.default_rng(seed + int(s.id[1:]))
    a = rng.uniform(-1, 1, (s.M, s.K)).astype(np.float16)  # logical A [M][K]
    b = rng.uniform(-1, 1, (s.K, s.N)).astype(np.float16)  # logical B [K][N]
    c = a.astype(np.float32) @ b.astype(np.float32)
    (a if s.la == "N" else np.ascontiguousarray(a.T)).tofile(out / "A.bin")
    (b if s.lb == "N" else np.ascontiguousarray(b.T)).tofile(out / "B.bin")
    c.astype(np.float32).tofile(out / "Cref.bin")
    (out / "meta.txt").write_text(f"{s.M} {s.N} {s.K} {s.la} {s.lb} {TOL}\n")
    return out


def read_meta(d: pathlib.Path):
    m, n, k, la, lb, tol = (pathlib.Path(d) / "meta.txt").read_text().split()
    return int(m), int(n), int(k), la, lb, float(tol)
