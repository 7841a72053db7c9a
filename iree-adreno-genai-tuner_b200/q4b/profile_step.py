"""Run a few single-token decode steps of a 3B-shaped model with few layers (a short, fixed launch
sequence for profilers): embed, per layer q|k|v+RoPE, attention, o, gate/up, down, final norm,
lm_head+argmax.

    python -m q4b.profile_step [--layers 1] [--steps 3] [--ctx 128] [--prefill C]

--prefill C first runs one C-row prefill chunk at position 0 (the tcgen05 GEMM path for C > 32).
"""

from __future__ import annotations

import argparse
import time


def main(argv=None):
    import torch

    from . import SYNTHETIC, LlamaQ4, SyntheticStateDict
    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--ctx", type=int, default=128, help="position of the first decode step")
    ap.add_argument("--bucket", type=int, default=256)
    ap.add_argument("--prefill", type=int, default=0, help="rows of one prefill chunk run first")
    a = ap.parse_args(argv)
    cfg = dict(SYNTHETIC["3b"], num_hidden_layers=a.layers)
    model = LlamaQ4(None, group=128, max_ctx=max(a.bucket, a.ctx + a.steps + 1), sd=SyntheticStateDict(cfg), cfg=cfg,
                    max_chunk=max(8, a.prefill))
    caches = model.new_caches()
    if a.prefill:
        toks = torch.arange(a.prefill, dtype=torch.int32).reshape(1, -1) * 7 + 3
        L = max(a.bucket, a.prefill)
        model.step(toks, torch.tensor([0]), torch.tensor([a.prefill - 1]), caches, L)
    tok = torch.tensor([[17]], dtype=torch.int32)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for i in range(a.steps):
        nxt, _ = model.step(tok, torch.tensor([a.ctx + i]), torch.tensor([0]), caches, a.bucket)
        tok = nxt.reshape(1, 1)
    torch.cuda.synchronize()
    print(f"{a.steps} steps of {a.layers} layer(s): {(time.perf_counter() - t0) * 1e3:.2f} ms, last token {int(tok)}")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
