"""The CUDA schedule space of q4b_gemm_f16 (the counterpart of gemm/schedule.py:43-103's Schedule)
and the index algebra of its kernels, restated here so the verifier can replay it.

Kernel 1 (tcgen05): a CTA computes one 128 x bn tile of C over the k steps [k_begin, k_end) of its
split z (64 wide each); grid = (ceil(M/128), ceil(N/bn), split); a shared-memory ring of `stages`
slots, each holding A's 128 x 64 tile (16 KB) and B's bn x 64 tile; a TMEM accumulator of bn
columns. Kernel 2 (CUDA cores): 64 x 64 tiles, no options. Kernel 3 (tcgen05, persistent stream-K):
the U = tiles x k-steps units split into G equal runs [c U / G, (c + 1) U / G), G = min(U, 148 x
CTAs per SM); the same ring and TMA boxes per unit as kernel 1; a CTA's run cuts into one segment per
tile, only its first and last possibly part of a tile, written to partial slots 2c and 2c + 1.

A schedule's candidate string is what the harness manifest carries: "1:bn=128,stages=6,split=2",
"3:bn=256,stages=4".
"""

from __future__ import annotations

import dataclasses
import math

BM, BK = 128, 64
SMEM_BUDGET = 200 * 1024  # ring bytes the kernel may use (csrc/gemm_f16.cu kGemmSmemBudget)
COUNTER_TILES = 16384     # split-K arrival counters in the workspace (64 KB of u32)
SMS = 148                 # the B200's SMs (kernel 3's persistent grid)


@dataclasses.dataclass(frozen=True)
class Schedule:
    kernel: int = 1   # 1 = tcgen05 + TMA + TMEM, 2 = CUDA-core tiles, 3 = tcgen05 persistent stream-K
    bn: int = 128     # output tile width (64 | 128 | 256)
    stages: int = 0   # ring depth (0 = as many as fit)
    split: int = 1    # k splits

    def key(self):
        # stages 0 means "as many as fit": the same kernel as naming that depth
        st = self.stages or SMEM_BUDGET // ((BM + self.bn) * BK * 2)
        if self.kernel == 2:
            return (2,)
        return (3, self.bn, st) if self.kernel == 3 else (self.kernel, self.bn, st, self.split)

    def candidate(self) -> str:
        if self.kernel == 2:
            return "2:"
        if self.kernel == 3:
            return f"3:bn={self.bn},stages={self.stages}"
        return f"1:bn={self.bn},stages={self.stages},split={self.split}"

    def short(self) -> str:
        if self.kernel == 2:
            return "simt"
        if self.kernel == 3:
            return f"streamk bn{self.bn} st{self.stages or 'max'}"
        return f"tc bn{self.bn} st{self.stages or 'max'} sk{self.split}"

    def cfg(self) -> dict:
        if self.kernel == 2:
            return dict(kernel=2)
        if self.kernel == 3:
            return dict(kernel=3, bn=self.bn, stages=self.stages)
        return dict(kernel=1, bn=self.bn, stages=self.stages, split=self.split)

    @staticmethod
    def parse(text: str) -> "Schedule":
        kern, _, rest = text.partition(":")
        kw = dict(kernel=int(kern))
        for item in filter(None, rest.split(",")):
            k, _, v = item.partition("=")
            kw[k] = int(v)
        return Schedule(**kw)


def stage_bytes(sc: Schedule) -> int:
    return (BM + sc.bn) * BK * 2


def max_stages(sc: Schedule) -> int:
    return SMEM_BUDGET // stage_bytes(sc)


def eff_stages(sc: Schedule) -> int:
    return sc.stages or max_stages(sc)


def smem_bytes(sc: Schedule) -> int:
    """Dynamic shared memory of one CTA (ring + 1 KB alignment slack)."""
    if sc.kernel == 2:
        return 2 * 16 * 65 * 4
    return eff_stages(sc) * stage_bytes(sc) + 1024


def k_steps(s) -> int:
    return -(-s.K // BK)


def grid(s, sc: Schedule):
    if sc.kernel == 2:
        return (-(-s.N // 64), -(-s.M // 64), 1)
    if sc.kernel == 3:
        return (sk_ctas(s, sc), 1, 1)
    return (-(-s.M // BM), -(-s.N // sc.bn), sc.split)


# ---- kernel 3 (stream-K): the index algebra of gemm_f16_sk and plan_sk ----------------------------

def sk_occupancy(sc: Schedule) -> int:
    """CTAs per SM: by shared memory (228 KB an SM, 1 KB reserved per CTA), at most 2 (register cap)."""
    return max(1, min(2, 233472 // (smem_bytes(sc) + 2048)))


def sk_accumulators(sc: Schedule) -> int:
    """TMEM accumulators per CTA: one when two CTAs share an SM, else two."""
    return 1 if sk_occupancy(sc) >= 2 else 2


def sk_tiles(s, sc: Schedule):
    return -(-s.M // BM), -(-s.N // sc.bn)


def sk_units(s, sc: Schedule) -> int:
    tm, tn = sk_tiles(s, sc)
    return tm * tn * k_steps(s)


def sk_ctas(s, sc: Schedule, sms: int = SMS) -> int:
    return min(sk_units(s, sc), sms * sk_occupancy(sc))


def sk_run(U: int, G: int, c: int):
    """Units [u0, u1) of CTA c."""
    return U * c // G, U * (c + 1) // G


def sk_cta_of(u: int, U: int, G: int) -> int:
    """The CTA whose run contains unit u (G <= U: no run is empty)."""
    return ((u + 1) * G + U - 1) // U - 1


def sk_segments(s, sc: Schedule, c: int, G: int):
    """CTA c's segments in order: (tile, k0, k1, slot) with slot None for a whole tile, else the
    partial slot 2c (its first segment) or 2c + 1."""
    U, kt = sk_units(s, sc), k_steps(s)
    u0, u1 = sk_run(U, G, c)
    out, u = [], u0
    while u < u1:
        t, k0 = divmod(u, kt)
        k1 = min(kt, k0 + (u1 - u))
        whole = k0 == 0 and k1 == kt
        out.append((t, k0, k1, None if whole else 2 * c + (0 if u == u0 else 1)))
        u += k1 - k0
    return out


def sk_fixup_slots(s, sc: Schedule, t: int, G: int):
    """The contributors of tile t and the slot the last of them reads for each, in k order (the
    kernel's fix-up: slot 2cc if t is cc's first tile, else 2cc + 1)."""
    U, kt = sk_units(s, sc), k_steps(s)
    c0, c1 = sk_cta_of(t * kt, U, G), sk_cta_of((t + 1) * kt - 1, U, G)
    return [(cc, 2 * cc + (0 if t == (U * cc // G) // kt else 1)) for cc in range(c0, c1 + 1)]


def k_range(s, sc: Schedule, z: int):
    """The k steps split z reduces: [z*kt/split, (z+1)*kt/split), as the kernel computes them."""
    kt = k_steps(s)
    return (z * kt) // sc.split, ((z + 1) * kt) // sc.split


def tma_loads(s, sc: Schedule, m_tile: int, n_tile: int, k_step: int):
    """The TMA boxes one ring slot receives: (operand, x, y, box_w, box_h) with x the innermost
    (contiguous) coordinate, as gemm_f16_tc issues them."""
    m0, n0, kx = m_tile * BM, n_tile * sc.bn, k_step * BK
    out = []
    if s.la == "N":
        out.append(("A", kx, m0, 64, BM))
    else:
        out += [("A", m0, kx, 64, 64), ("A", m0 + 64, kx, 64, 64)]
    if s.lb == "T":
        out.append(("B", kx, n0, 64, sc.bn))
    else:
        out += [("B", n0 + 64 * j, kx, 64, 64) for j in range(sc.bn // 64)]
    return out


def workspace_bytes(s, sc: Schedule) -> int:
    if sc.kernel == 3:
        return 64 * 1024 + 2 * sk_ctas(s, sc) * BM * sc.bn * 4
    if sc.kernel == 2 or sc.split == 1:
        return 0
    gx, gy, _ = grid(s, sc)
    return 64 * 1024 + sc.split * gx * gy * BM * sc.bn * 4


def domains(s):
    kt = k_steps(s)
    return {
        "bn": [64, 128, 256],
        "stages": [0, 2, 3, 4, 5, 6, 8],
        "split": sorted({x for x in (1, 2, 3, 4, 6, 8, 12, 16) if x <= kt}),
    }


def tuned_schedules() -> dict:
    """{(M, N, K, layout): Schedule} from tuned_b200.json: the schedules a search on a B200 measured
    fastest for the config-2 shapes, which plan_gemm takes as its default for exactly those problems."""
    import json
    import pathlib

    from .shapes import BY_ID
    out = {}
    for sid, rec in json.loads((pathlib.Path(__file__).with_name("tuned_b200.json")).read_text()).items():
        sh = BY_ID[sid]
        kv = dict(p.split("=") for p in rec["candidate"].split(":", 1)[1].split(","))
        out[(sh.M, sh.N, sh.K, sh.layout)] = Schedule(kernel=1, bn=int(kv["bn"]), stages=int(kv["stages"]),
                                                       split=int(kv["split"]))
    return out


def default_schedule(s) -> Schedule:
    """The library's built-in choice (plan_gemm in csrc/gemm_f16.cu): the searched schedule for the
    config-2 problems (tuned_b200.json); otherwise the widest tile that still gives 148 tiles, then
    split-K while that fills more SMs and each split keeps >= 4 k steps (stages: as many as fit, or
    2 for 256-wide tiles over 8 or more row tiles)."""
    if s.la == "N" and s.K % 8 or s.la == "T" and s.M % 8 or s.lb == "N" and s.N % 8 or s.lb == "T" and s.K % 8:
        return Schedule(kernel=2)
    tuned = tuned_schedules().get((s.M, s.N, s.K, s.layout))
    if tuned is not None:
        return tuned
    tm = -(-s.M // BM)
    bn = 256
    while bn > 64 and tm * -(-s.N // bn) < 148:
        bn //= 2
    tn = -(-s.N // bn)
    kt = k_steps(s)
    split = 1
    while tm * tn * split < 148 and kt // (split * 2) >= 4:
        split *= 2
    return Schedule(kernel=1, bn=bn, stages=0, split=split)


def log2i(x: int) -> float:
    return math.log2(max(1, x))
