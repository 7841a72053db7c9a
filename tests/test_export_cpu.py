"""The export contract of scripts/llm/export_llama.py (entry point names, meta.json keys) and the
packed-weight file format / pack-cache keys of q4b.export, on the CPU; plus the LazySafetensors
checkpoint reader (scripts/llm/llama_q4.py:125-138)."""

import json

import numpy as np
import pytest

import golden_inputs as gi
from conftest import load_golden

REF_META_KEYS = {"n_layers", "n_kv_heads", "head_dim", "max_ctx", "vocab", "chunk", "buckets", "prompt", "ref_tokens"}


def test_entry_names_follow_the_reference():
    """export_llama.py:44-48: a prefill function per bucket >= chunk, a decode function per bucket,
    one logits-returning decode function at the smallest bucket."""
    from q4b import export
    assert export.entry_names(128, [256, 512, 1024, 2048, 4096]) == [
        "prefill_c128_l256", "decode_l256", "prefill_c128_l512", "decode_l512", "prefill_c128_l1024",
        "decode_l1024", "prefill_c128_l2048", "decode_l2048", "prefill_c128_l4096", "decode_l4096",
        "decode_logits_l256"]
    # buckets below the chunk get no prefill function (the tiny KAT model: chunk 8 fits all of them)
    assert export.entry_names(32, [16, 32, 64]) == ["decode_l16", "prefill_c32_l32", "decode_l32",
                                                    "prefill_c32_l64", "decode_l64", "decode_logits_l16"]


def test_export_round_trip(tmp_path):
    from q4b import export
    z = load_golden("model_tiny_ref")
    spec = gi.MODEL_SPECS["tiny_ref"]
    packed = {k: v for k, v in z.items() if k.startswith(("l", "embed", "ln_f")) and not k.startswith("logits")}
    export.write(tmp_path / "m", spec["cfg"], packed, spec["max_ctx"], spec["chunk"], spec["buckets"],
                 prompt=z["prompt"], ref_tokens=z["bucketed_tokens"])
    cfg, back, meta = export.read(tmp_path / "m")
    assert set(back) == set(packed)
    for k, v in packed.items():
        assert np.array_equal(np.asarray(v), back[k]) and np.asarray(v).dtype == back[k].dtype, k
    assert REF_META_KEYS <= set(meta)
    assert meta["n_layers"] == 2 and meta["vocab"] == 1000 and meta["n_kv_heads"] == 2 and meta["head_dim"] == 32
    assert meta["prompt"] == z["prompt"].tolist() and meta["ref_tokens"] == z["bucketed_tokens"].tolist()
    assert cfg == dict(spec["cfg"], num_hidden_layers=2)
    assert json.loads((tmp_path / "m" / "meta.json").read_text())["entry_points"][-1] == "decode_logits_l16"
    (tmp_path / "m" / "meta.json").write_text(json.dumps(dict(meta, format="other")))
    with pytest.raises(ValueError):
        export.read(tmp_path / "m")


def test_cache_keys():
    from q4b import export
    cfg = gi.MODEL_SPECS["tiny_ref"]["cfg"]
    k = export.cache_key(cfg, "synthetic:0", 128, True, None)
    assert k == export.cache_key(dict(cfg), "synthetic:0", 128, True, None)
    assert k != export.cache_key(cfg, "synthetic:1", 128, True, None)
    assert k != export.cache_key(cfg, "synthetic:0", 32, True, None)
    assert k != export.cache_key(cfg, "synthetic:0", 128, True, 1)
    assert k != export.cache_key(dict(cfg, hidden_size=512), "synthetic:0", 128, True, None)


def test_checkpoint_reader(tmp_path):
    """LazySafetensors: tensors of every shard by name, read on access."""
    import torch
    from safetensors.torch import save_file

    from q4b import LazySafetensors
    save_file({"model.norm.weight": torch.ones(4), "a": torch.arange(6.0).reshape(2, 3)}, str(tmp_path / "m-1.safetensors"))
    save_file({"b": torch.full((3,), 7.0)}, str(tmp_path / "m-2.safetensors"))
    sd = LazySafetensors(tmp_path)
    assert "a" in sd and "b" in sd and "c" not in sd
    assert torch.equal(sd["a"], torch.arange(6.0).reshape(2, 3)) and torch.equal(sd["b"], torch.full((3,), 7.0))
    assert export_source_changes(tmp_path)


def export_source_changes(d):
    from q4b import export
    a = export.checkpoint_source(d)
    (d / "m-3.safetensors").write_bytes(b"x")
    return a != export.checkpoint_source(d)
