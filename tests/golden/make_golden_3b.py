"""Golden greedy stream of the Llama-3.2-3B-shape LlamaQ4 from the REFERENCE.

    python tests/golden/make_golden_3b.py [--ref /path/to/reference] [--new 256] [--layers 28]

Builds the reference's own ``LlamaQ4`` (``scripts/llm/llama_q4.py``, imported unchanged) from
``q4b.SyntheticStateDict(SYNTHETIC["3b"], seed=0)`` on the CPU. That generator is integer hashing
plus one fp32 multiply, so the GPU test regenerates bit-identical weights without the reference.
The reference step is driven by the runner schedule of ``runner/llm_runner.c:143-246`` (restated in
``oracle.q4_oracle.generate``) with the bench's request: the 512-id prompt of
``numpy.random.default_rng(0).integers(0, vocab, 512)``, chunk 128, buckets 256..4096, bucketed.

Stored in ``model_3b_ref.npz`` (small: the full logits are 128256 floats per step):
  tokens [new]            greedy ids (tokens[0] from the prefill, then one per decode step)
  margin [new]            top-1 minus top-2 logit of each step
  top1 [new]              the winning logit of each step
  logit_idx [S, n]        per checked step, the vocab indices kept: the top 64 and every 32nd id
  logit_val [S, n]        the reference logits at those indices (S = the first --keep steps)
  chunk_buckets, step_buckets, prompt, n_layers
Decode steps use the reference's fused GEMV form (EXPORT_FUSED_GEMV, ``llama_q4.py:56-90``), the
formulation its export compiles for M == 1; prefill chunks use dequantise + F.linear (``:72``).
"""

from __future__ import annotations

import argparse
import os
import pathlib
import sys
import time

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "iree-adreno-genai-tuner_b200"))

PROMPT_LEN, CHUNK, BUCKETS = 512, 128, [256, 512, 1024, 2048, 4096]
KEEP_TOP, KEEP_STRIDE = 64, 32


def kept_indices(logits: np.ndarray) -> np.ndarray:
    top = np.argsort(-logits, kind="stable")[:KEEP_TOP]
    return np.unique(np.concatenate([top, np.arange(0, logits.shape[0], KEEP_STRIDE)])).astype(np.int32)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", type=pathlib.Path, default=pathlib.Path(os.environ.get("Q4B_REFERENCE", "reference")))
    ap.add_argument("--new", type=int, default=256)
    ap.add_argument("--keep", type=int, default=8)
    ap.add_argument("--layers", type=int, default=None, help="fewer layers, for a timing probe only")
    ap.add_argument("--out", type=pathlib.Path, default=HERE / "model_3b_ref.npz")
    a = ap.parse_args()
    import torch

    from oracle import q4_oracle as O
    from q4b.llama import SyntheticStateDict
    from q4b.runner import SYNTHETIC
    torch.set_num_threads(8)
    sys.dont_write_bytecode = True
    sys.path.insert(0, str(a.ref / "scripts" / "llm"))
    import llama_q4 as R  # the reference module, unmodified

    cfg = dict(SYNTHETIC["3b"])
    t0 = time.time()
    sd = SyntheticStateDict(cfg, seed=0, device="cpu")
    with torch.no_grad():
        model = R.LlamaQ4(None, group=128, max_ctx=4096, vocab_chunk=32064, n_layers=a.layers, sd=sd, cfg=cfg).eval()
    print(f"reference model built in {time.time() - t0:.0f} s", flush=True)
    prompt = np.random.default_rng(0).integers(0, cfg["vocab_size"], PROMPT_LEN)
    caches = model.new_caches()
    log = []

    def step(tokens, start, last, L):
        R.EXPORT_FUSED_GEMV[0] = len(tokens) == 1
        t = time.time()
        with torch.no_grad():
            nxt, lg = model.step(torch.from_numpy(np.asarray(tokens, dtype=np.int32)).reshape(1, -1),
                                 torch.tensor([start], dtype=torch.int32), torch.tensor([last], dtype=torch.int32),
                                 caches, L)
        if len(tokens) > 1 and start + len(tokens) < PROMPT_LEN:  # a prefill chunk whose token is unused
            print(f"prefill chunk at {start}: {time.time() - t:.1f} s", flush=True)
            return int(nxt)
        lg = lg[0].numpy().astype(np.float32)
        top2 = np.sort(lg)[-2:]
        entry = {"margin": float(top2[1] - top2[0]), "top1": float(top2[1])}
        if len(log) < a.keep:
            idx = kept_indices(lg)
            entry["idx"], entry["val"] = idx, lg[idx]
        log.append(entry)
        print(f"step {len(log) - 1}: token {int(nxt)} margin {entry['margin']:.4g} ({time.time() - t:.1f} s)",
              flush=True)
        return int(nxt)

    toks, chunks, steps = O.generate(step, prompt.tolist(), a.new, CHUNK, BUCKETS, schedule="bucketed",
                                     max_ctx=4096)
    kept = [e for e in log if "idx" in e]
    n = max(len(e["idx"]) for e in kept)
    idx = np.full((len(kept), n), -1, dtype=np.int32)
    val = np.zeros((len(kept), n), dtype=np.float32)
    for i, e in enumerate(kept):
        idx[i, : len(e["idx"])], val[i, : len(e["val"])] = e["idx"], e["val"]
    np.savez_compressed(a.out, tokens=np.array(toks, dtype=np.int32),
                        margin=np.array([e["margin"] for e in log], dtype=np.float32),
                        top1=np.array([e["top1"] for e in log], dtype=np.float32),
                        logit_idx=idx, logit_val=val, chunk_buckets=np.array(chunks, dtype=np.int32),
                        step_buckets=np.array(steps, dtype=np.int32), prompt=prompt.astype(np.int32),
                        n_layers=np.int32(model.n_layers))
    print(f"{a.out.name}: {a.out.stat().st_size / 1e3:.0f} kB, {time.time() - t0:.0f} s total")


if __name__ == "__main__":
    main()
