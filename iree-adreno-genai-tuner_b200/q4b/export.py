"""Export / pack cache: the contract of scripts/llm/export_llama.py for the B200 build.

The reference exports a compiled module with one static-shape entry point per (phase, KV bucket)
and writes the quantised weights plus a meta.json next to it (export_llama.py:25-54); the runner
(runner/llm_runner.c) calls the entry points by name. Here the entry points are the same functions
of the native model (`entry_points`: names -> StepFn), and the on-disk export is the packed int4
weights in the reference's QLinear layout (qweight [N, K/8] int32, scales [N, K/G] fp16) in one
safetensors file, the HF config, and the reference's meta.json keys:

    <out>/weights.safetensors   l{i}_{wqkv|wo|wgu|wdown}_{qweight|scales|group}, l{i}_ln_in,
                                l{i}_ln_post, embed_qweight, embed_scales, embed_group, ln_f
    <out>/config.json           the model's HF config
    <out>/meta.json             n_layers, n_kv_heads, head_dim, max_ctx, vocab, chunk, buckets,
                                prompt, ref_tokens (export_llama.py:51-54), plus entry_points and
                                format

Loading an export needs no quantisation, so the directory doubles as a pack cache: `cached` keys a
directory by the model's config, the weight source and the group rule, and fills it on first use.

    python -m q4b.export --out DIR (--model-dir HF_DIR | --synthetic tiny|3b [--seed 0])
                         [--chunk 128] [--buckets 256 512 1024 2048 4096] [--layers N] [--group 128]
"""

from __future__ import annotations

import argparse
import hashlib
import json
import pathlib

import numpy as np

FORMAT = "q4b-packed-v1"
WEIGHTS, CONFIG, META = "weights.safetensors", "config.json", "meta.json"


def entry_names(chunk: int, buckets) -> list[str]:
    """export_llama.py:44-48: prefill_c{C}_l{L} for every bucket L >= C, decode_l{L} for every
    bucket, and decode_logits_l{L0} (logits instead of the token) for the smallest bucket."""
    names = []
    for L in buckets:
        if L >= chunk:
            names.append(f"prefill_c{chunk}_l{L}")
        names.append(f"decode_l{L}")
    names.append(f"decode_logits_l{buckets[0]}")
    return names


def entry_points(model, chunk: int, buckets) -> dict:
    """The entry points by the reference's names, each a StepFn of `model` (a fixed KV bucket;
    decode_logits_* returns the logits)."""
    from .llama import StepFn
    out = {}
    for name in entry_names(chunk, buckets):
        L = int(name.rsplit("_l", 1)[1])
        out[name] = StepFn(model, L, return_logits=name.startswith("decode_logits"))
    return out


def packed_state(model) -> dict:
    """The model's packed tensors as host numpy arrays in the layout LlamaQ4.from_packed reads."""
    t = lambda a: a.detach().cpu().numpy()  # noqa: E731
    out = {}
    for i, ly in enumerate(model.layers):
        for nm in ("wqkv", "wo", "wgu", "wdown"):
            q = getattr(ly, nm)
            out[f"l{i}_{nm}_qweight"] = t(q.qweight)
            out[f"l{i}_{nm}_scales"] = t(q.scales)
            out[f"l{i}_{nm}_group"] = np.array(q.group, dtype=np.int32)
        out[f"l{i}_ln_in"], out[f"l{i}_ln_post"] = t(ly.ln_in), t(ly.ln_post)
    out["embed_qweight"], out["embed_scales"] = t(model.embed.qweight), t(model.embed.scales)
    out["embed_group"] = np.array(model.embed.group, dtype=np.int32)
    out["ln_f"] = t(model.ln_f)
    return out


def meta_dict(cfg: dict, packed: dict, max_ctx: int, chunk: int, buckets, prompt=None, ref_tokens=None) -> dict:
    n_layers = sum(1 for k in packed if k.endswith("_wqkv_qweight"))
    hd = cfg.get("head_dim") or cfg["hidden_size"] // cfg["num_attention_heads"]
    return dict(n_layers=n_layers, n_kv_heads=cfg["num_key_value_heads"], head_dim=hd, max_ctx=max_ctx,
                vocab=int(packed["embed_qweight"].shape[0]), chunk=chunk, buckets=list(buckets),
                prompt=None if prompt is None else [int(v) for v in prompt],
                ref_tokens=None if ref_tokens is None else [int(v) for v in ref_tokens],
                entry_points=entry_names(chunk, buckets), format=FORMAT)


def write(out, cfg: dict, packed: dict, max_ctx: int, chunk: int, buckets, prompt=None, ref_tokens=None):
    """Write an export directory from packed host arrays (no GPU needed)."""
    from safetensors.numpy import save_file
    out = pathlib.Path(out)
    out.mkdir(parents=True, exist_ok=True)
    arrays = {k: np.ascontiguousarray(np.asarray(v)) for k, v in packed.items()}
    arrays = {k: (v.reshape(1) if v.ndim == 0 else v) for k, v in arrays.items()}
    save_file(arrays, str(out / (WEIGHTS + ".tmp")))
    (out / (WEIGHTS + ".tmp")).replace(out / WEIGHTS)
    meta = meta_dict(cfg, packed, max_ctx, chunk, buckets, prompt, ref_tokens)
    cfg = dict(cfg, num_hidden_layers=meta["n_layers"])  # a truncated export says so in its config
    (out / CONFIG).write_text(json.dumps(cfg, indent=1))
    (out / META).write_text(json.dumps(meta, indent=1))


def export(model, out, chunk: int, buckets, prompt=None, ref_tokens=None):
    """export_llama.py:25-54 for a q4b.LlamaQ4: packed weights, config and meta.json."""
    write(out, model.cfg, packed_state(model), model.max_ctx, chunk, buckets, prompt, ref_tokens)


def read(out):
    """(cfg, packed arrays, meta) of an export directory."""
    from safetensors.numpy import load_file
    out = pathlib.Path(out)
    meta = json.loads((out / META).read_text())
    if meta.get("format") != FORMAT:
        raise ValueError(f"{out}: not a {FORMAT} export (format {meta.get('format')!r})")
    packed = load_file(str(out / WEIGHTS))
    packed = {k: (v.reshape(()) if k.endswith("_group") else v) for k, v in packed.items()}
    return json.loads((out / CONFIG).read_text()), packed, meta


def load(out, device="cuda", max_ctx=None, max_chunk=None):
    """A LlamaQ4 from an export directory (weights used as stored: no quantisation)."""
    from .llama import LlamaQ4
    cfg, packed, meta = read(out)
    return LlamaQ4.from_packed(cfg, packed, max_ctx or meta["max_ctx"], vocab_chunk=meta["vocab"], device=device,
                               max_chunk=max_chunk or meta["chunk"])


def cache_key(cfg: dict, source: str, group: int, per_linear_group: bool, n_layers) -> str:
    """Directory name of a pack-cache entry: the config, the weight source (a checkpoint's file
    names and sizes, or a synthetic generator and its seed), the group rule and the layer count."""
    blob = json.dumps(dict(cfg=cfg, source=source, group=group, plg=per_linear_group, n_layers=n_layers,
                           format=FORMAT), sort_keys=True)
    return hashlib.sha256(blob.encode()).hexdigest()[:20]


def checkpoint_source(model_dir) -> str:
    d = pathlib.Path(model_dir)
    return "ckpt:" + ",".join(f"{f.name}:{f.stat().st_size}" for f in sorted(d.glob("*.safetensors")))


def cached(cache_dir, build, cfg: dict, source: str, group: int, max_ctx: int, *, per_linear_group=False,
           n_layers=None, chunk=128, buckets=(256, 512, 1024, 2048, 4096), device="cuda"):
    """The model for (cfg, source, group) from the pack cache, quantising with `build()` (which
    returns a LlamaQ4) and filling the cache on a miss. Returns (model, hit)."""
    d = pathlib.Path(cache_dir) / cache_key(cfg, source, group, per_linear_group, n_layers)
    if (d / META).exists() and (d / WEIGHTS).exists():
        return load(d, device=device, max_ctx=max_ctx, max_chunk=chunk), True
    model = build()
    write(d, cfg, packed_state(model), max_ctx, chunk, buckets)
    return model, False


def main(argv=None):
    import torch

    from . import SYNTHETIC, LlamaQ4, SyntheticStateDict
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--out", type=pathlib.Path, required=True)
    ap.add_argument("--model-dir", type=pathlib.Path, default=None)
    ap.add_argument("--synthetic", choices=["tiny", "3b"], default=None)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--chunk", type=int, default=128)
    ap.add_argument("--buckets", type=int, nargs="+", default=[256, 512, 1024, 2048, 4096])
    ap.add_argument("--layers", type=int, default=None)
    ap.add_argument("--group", type=int, default=128)
    a = ap.parse_args(argv)
    if bool(a.model_dir) == bool(a.synthetic):
        ap.error("give exactly one of --model-dir and --synthetic")
    max_ctx = max(a.buckets)
    if a.model_dir:
        model = LlamaQ4(a.model_dir, group=a.group, max_ctx=max_ctx, n_layers=a.layers, max_chunk=a.chunk,
                        per_linear_group=True)
    else:
        cfg = SYNTHETIC[a.synthetic]
        model = LlamaQ4(None, group=a.group, max_ctx=max_ctx, n_layers=a.layers, max_chunk=a.chunk,
                        sd=SyntheticStateDict(cfg, seed=a.seed), cfg=cfg, per_linear_group=True)
    torch.cuda.synchronize()
    export(model, a.out, a.chunk, a.buckets)
    print(json.dumps({"out": str(a.out), "entry_points": entry_names(a.chunk, a.buckets),
                      "weights_bytes": (a.out / WEIGHTS).stat().st_size}))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
