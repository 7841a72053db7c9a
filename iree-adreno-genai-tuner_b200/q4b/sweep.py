"""Batched int4 projection sweep: q4_linear over the 3B projection shapes at
M in {1, 4, 16, 64}, each timed as CUDA-graph replays over enough distinct weight copies that the
weights come from HBM (more than the 126 MB L2), against the HBM roofline.

    python -m q4b.sweep [--shapes qkv o gu down lm] [--m 1 4 16 64] [--reps 20]

Prints one JSON line per (shape, M): algorithmic bytes = N K / 2 + 2 N K / G + 2 M K + 2 M N
(int4 weights, fp16 scales, fp16 x and y), GB/s, fraction of the measured HBM copy bandwidth, the
kernel the planner picked. One GPU (the tensor-parallel split of a projection is the same call on a
smaller shape).
"""

from __future__ import annotations

import argparse
import json
import math
import pathlib

import torch

from . import _lib, ops

SHAPES = {"qkv": (5120, 3072), "o": (3072, 3072), "gu": (16384, 3072), "down": (3072, 8192), "lm": (128256, 3072)}
G = 128
L2_BYTES = 126 * 2**20


def _peak_gbs() -> tuple[float, str]:
    p = pathlib.Path(__file__).resolve().parents[2] / "MEASURED_PEAKS.json"
    if p.exists():
        return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def algorithmic_bytes(n: int, k: int, m: int) -> int:
    return n * k // 2 + 2 * n * (k // G) + 2 * m * k + 2 * m * n


def measure(n: int, k: int, m: int, reps: int = 20, dev=None) -> dict:
    dev = dev or torch.device("cuda", torch.cuda.current_device())
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    wbytes = n * k // 2 + 2 * n * (k // G)
    copies = max(1, math.ceil(2 * L2_BYTES / wbytes))  # the weights a replay reads exceed L2 twice over
    qws = [torch.randint(-2**31, 2**31 - 1, (n, k // 8), dtype=torch.int32, device=dev, generator=g)
           for _ in range(copies)]
    scs = [(torch.randn(n, k // G, device=dev, generator=g) * 0.02).abs().half() for _ in range(copies)]
    x = torch.randn(m, k, device=dev, generator=g).half()
    ys = [torch.empty(m, n, dtype=torch.float16, device=dev) for _ in range(copies)]
    stream = torch.cuda.Stream(device=dev)
    with torch.cuda.stream(stream):
        for i in range(copies):
            ops.q4_linear(x, qws[i], scs[i], G, out=ys[i])
        graph = torch.cuda.CUDAGraph()
        graph.capture_begin()
        for i in range(copies):
            ops.q4_linear(x, qws[i], scs[i], G, out=ys[i])
        graph.capture_end()
        for _ in range(3):
            graph.replay()
    stream.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(reps):
            graph.replay()
        e1.record(stream)
    e1.synchronize()
    if _lib.lib().q4b_device_status(1) != 0:
        raise RuntimeError("q4b: a bounded device wait gave up during the sweep")
    per_call = e0.elapsed_time(e1) / 1e3 / (reps * copies)
    peak, src = _peak_gbs()
    b = algorithmic_bytes(n, k, m)
    gbs = b / per_call / 1e9
    ws = _lib.lib().q4b_q4_linear_workspace(m, n, k, G, 0, None)
    return {"N": n, "K": k, "M": m, "bytes": b, "us_per_call": round(per_call * 1e6, 3), "GB_s": round(gbs, 1),
            "frac": round(gbs / peak, 4), "peak_GB_s": peak, "peak_source": src, "weight_copies": copies,
            "workspace_bytes": int(ws), "kernel": "tcgen05 GEMM (kernel 5)" if m > 32 else "int4 GEMV (kernel 1)"}


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--shapes", nargs="*", default=list(SHAPES))
    ap.add_argument("--m", nargs="*", type=int, default=[1, 4, 16, 64])
    ap.add_argument("--reps", type=int, default=20)
    a = ap.parse_args(argv)
    for name in a.shapes:
        n, k = SHAPES[name]
        for m in a.m:
            print(json.dumps({"shape": name, **measure(n, k, m, a.reps)}), flush=True)


if __name__ == "__main__":
    main()
