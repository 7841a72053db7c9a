"""Runner: the scheduler of runner/llm_runner.c over the native model (q4b_runner_* in libq4b.so).

    python -m q4b.runner [--prompt ids.txt] [--max_new_tokens 32] [--chunk 128]
        [--buckets 256,512,1024,2048,4096] [--schedule bucketed|max] [--stop_ids 1,2] [--warmup 1]
        (--model-dir DIR | --synthetic tiny|3b [--seed 0]) [--n_layers N] [--max_ctx 4096]

--model-dir takes a Hugging Face checkpoint directory (quantised at load) or a q4b export
(python -m q4b.export: packed weights + meta.json, whose prompt is the default).

Flag names and the printed JSON object follow runner/llm_runner.c:35-45 and :249-262.
"""

from __future__ import annotations

import argparse
import ctypes
import json
import pathlib
import sys

from . import _lib


class Runner:
    """llm_runner.c's generation loop. One CUDA graph per used (phase, bucket), captured during the
    untimed warm-up; decode steps run back to back on the device unless sync_every_step."""

    def __init__(self, model, chunk: int, buckets, schedule: str = "bucketed", graphs: bool = True, warmup: int = 1,
                 sync_every_step: bool = False, caches=None):
        import torch
        self.model = model
        self.caches = caches if caches is not None else model.new_caches()
        model.bind_caches(self.caches)
        self.buckets = (ctypes.c_int * len(buckets))(*buckets)
        opts = _lib.RunnerOpts(chunk, ctypes.cast(self.buckets, ctypes.c_void_p), len(buckets),
                               {"bucketed": 0, "max": 1}[schedule], int(graphs), warmup, int(sync_every_step))
        self.chunk, self.schedule = chunk, schedule
        h = ctypes.c_void_p()
        with torch.cuda.device(model.device):
            _lib.check(_lib.lib().q4b_runner_create(model.native(), ctypes.byref(opts), ctypes.byref(h)),
                       "runner_create")
        self._h = h

    def generate(self, prompt, max_new: int, stop_ids=()):
        """Returns (tokens, report) where report is llm_runner.c's JSON object as a dict."""
        import torch
        p = (ctypes.c_int32 * len(prompt))(*[int(t) for t in prompt])
        s = (ctypes.c_int32 * max(1, len(stop_ids)))(*[int(t) for t in stop_ids] or [0])
        out = (ctypes.c_int32 * max(1, max_new))()
        n_out = ctypes.c_int()
        rep = _lib.Report()
        with torch.cuda.device(self.model.device):
            _lib.check(_lib.lib().q4b_runner_generate(self._h, p, len(prompt), max_new, s, len(stop_ids), out,
                                                      ctypes.byref(n_out), ctypes.byref(rep)), "runner_generate")
        report = json.loads(_lib.lib().q4b_runner_report_json(self._h).decode())
        report["decode_wall_ms"] = rep.decode_wall_ms
        return list(out[: n_out.value]), report

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None:
            try:
                _lib.lib().q4b_runner_destroy(h)
            except Exception:
                pass


def _parse_ints(s):
    return [int(t) for t in s.replace(",", " ").split()] if s else []


def main(argv=None):
    from . import LlamaQ4, SyntheticStateDict
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--prompt", default=None, help="file with whitespace-separated prompt token ids "
                    "(default: the prompt in the export's meta.json)")
    ap.add_argument("--max_new_tokens", type=int, default=32)
    ap.add_argument("--chunk", type=int, default=128)
    ap.add_argument("--buckets", default="256,512,1024,2048,4096")
    ap.add_argument("--schedule", default="bucketed", choices=["bucketed", "max"])
    ap.add_argument("--n_layers", type=int, default=None)
    ap.add_argument("--max_ctx", type=int, default=4096)
    ap.add_argument("--stop_ids", default="")
    ap.add_argument("--warmup", type=int, default=1)
    ap.add_argument("--group", type=int, default=128)
    ap.add_argument("--model-dir", type=pathlib.Path, default=None)
    ap.add_argument("--synthetic", choices=["tiny", "3b"], default=None)
    ap.add_argument("--seed", type=int, default=0)
    a = ap.parse_args(argv)
    meta = None
    if a.model_dir and (a.model_dir / "meta.json").exists():  # a q4b export (q4b.export): packed weights
        from . import export
        meta = json.loads((a.model_dir / "meta.json").read_text())
    if a.prompt:
        prompt = _parse_ints(pathlib.Path(a.prompt).read_text())
    elif meta and meta.get("prompt"):
        prompt = [int(t) for t in meta["prompt"]]
    else:
        ap.error("--prompt is required (the model has no exported prompt)")
    if meta:
        model = export.load(a.model_dir, max_ctx=a.max_ctx, max_chunk=a.chunk)
    elif a.model_dir:
        model = LlamaQ4(a.model_dir, group=a.group, max_ctx=a.max_ctx, n_layers=a.n_layers, max_chunk=a.chunk,
                        per_linear_group=True)
    else:
        cfg = SYNTHETIC[a.synthetic or "tiny"]
        model = LlamaQ4(None, group=a.group, max_ctx=a.max_ctx, n_layers=a.n_layers,
                        sd=SyntheticStateDict(cfg, seed=a.seed), cfg=cfg, max_chunk=a.chunk, per_linear_group=True)
    r = Runner(model, a.chunk, _parse_ints(a.buckets), a.schedule, warmup=a.warmup)
    _, report = r.generate(prompt, a.max_new_tokens, _parse_ints(a.stop_ids))
    report.pop("decode_wall_ms", None)
    print(json.dumps(report, separators=(",", ":")))
    return 0


# model configurations without checkpoints: BASELINE's tiny config and the Llama-3.2-3B shape
SYNTHETIC = {
    "tiny": dict(hidden_size=256, num_hidden_layers=4, num_attention_heads=8, num_key_value_heads=2, head_dim=32,
                 intermediate_size=688, vocab_size=1024, rms_norm_eps=1e-5, rope_theta=500000.0,
                 max_position_embeddings=4096, tie_word_embeddings=True, hidden_act="silu", initializer_range=0.2),
    "3b": dict(hidden_size=3072, num_hidden_layers=28, num_attention_heads=24, num_key_value_heads=8, head_dim=128,
               intermediate_size=8192, vocab_size=128256, rms_norm_eps=1e-5, rope_theta=500000.0,
               rope_scaling={"rope_type": "llama3", "factor": 32.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
                             "original_max_position_embeddings": 8192},
               max_position_embeddings=131072, tie_word_embeddings=True, hidden_act="silu", initializer_range=0.02),
}

if __name__ == "__main__":
    sys.exit(main())
