"""GPU parity of the LlamaQ4 step (scripts/llm/llama_q4.py:199-239) and its kernels.

The end-to-end gate follows scripts/llm/test_tiny.py: greedy tokens identical to the reference's
(recorded in tests/golden/model_*.npz by running the reference LlamaQ4 with the schedule of
runner/llm_runner.c) and logits within 1e-3 * max(1, |ref|max) (scripts/debug/op_test.py:75)."""

import numpy as np
import pytest
import torch

import golden_inputs as gi
from oracle import q4_oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    assert torch.cuda.is_available()
    return torch.device("cuda:0")


def test_embed_lookup(dev, golden_ops):
    import q4b
    qw = torch.from_numpy(golden_ops["emb_qweight"]).to(dev)
    s = torch.from_numpy(golden_ops["emb_scales"]).to(dev)
    out = q4b.embed_lookup(torch.from_numpy(gi.EMBED_TOKENS), qw, s, 32)
    assert np.array_equal(out.cpu().numpy().view(np.uint32), golden_ops["emb_lookup"].view(np.uint32))
    emb = q4b.QEmbedding.from_packed(qw, s, 32, 256)
    lg = emb.logits(torch.from_numpy(golden_ops["emb_logits_x"]).to(dev))
    assert O.rel_err(lg.cpu().numpy(), golden_ops["emb_logits"]) <= 1e-3


def test_rmsnorm(dev, golden_ops):
    import q4b
    out = q4b.rmsnorm(torch.from_numpy(golden_ops["rms_x"]).to(dev), torch.from_numpy(golden_ops["rms_w"]).to(dev), 1e-5)
    ref = golden_ops["rms_out"]
    assert np.abs(out.cpu().numpy() - ref).max() <= 1e-5 * max(1.0, np.abs(ref).max())


@pytest.mark.parametrize("C,H,Hkv,hd,start,L", [(1, 8, 2, 32, 40, 128), (1, 24, 8, 128, 700, 1024),
                                                (3, 8, 2, 32, 5, 16), (32, 8, 2, 32, 32, 128),
                                                (17, 24, 8, 128, 300, 512), (1, 4, 4, 64, 0, 64),
                                                (2, 8, 2, 32, 60, 32), (128, 24, 8, 128, 384, 512),
                                                (13, 24, 8, 128, 100, 256), (20, 8, 8, 64, 10, 64),
                                                (9, 8, 4, 32, 3, 32), (40, 16, 2, 64, 0, 64)])
def test_attention_vs_oracle(dev, C, H, Hkv, hd, start, L):
    """Decode (split-key) and prefill forms against the reference's masked softmax over cache[:L]:
    the tiled prefill form for groups of 1-4 heads (the 3B shape's 4th prompt chunk, ragged row
    blocks, keys past the bucket), the one-row form for larger groups (16 / 2)."""
    import q4b
    rng = np.random.default_rng(C * 1000 + start)
    max_ctx = max(L, start + C) + 8
    kc = (rng.standard_normal((max_ctx, Hkv, hd)) * 0.5).astype(np.float16)
    vc = rng.standard_normal((max_ctx, Hkv, hd)).astype(np.float16)
    q = rng.standard_normal((C, H, hd)).astype(np.float32)
    pos = start + np.arange(C)
    ref = O.attention(q, kc, vc, pos, L, Hkv)
    out = q4b.attention(torch.from_numpy(q).to(dev), torch.from_numpy(kc).to(dev), torch.from_numpy(vc).to(dev),
                        start, L)
    assert np.abs(out.cpu().numpy() - ref).max() <= 1e-4 * max(1.0, np.abs(ref).max())


def _run_schedule(model, spec, prompt, schedule):
    caches = model.new_caches()
    logits = []

    def step(tokens, start, last, L):
        nxt, lg = model.step(torch.as_tensor(np.asarray(tokens, dtype=np.int32)).reshape(1, -1),
                             torch.tensor([start], dtype=torch.int32), torch.tensor([last], dtype=torch.int32),
                             caches, L)
        logits.append(lg[0].cpu().numpy())
        return int(nxt.item())

    toks, chunks, steps = O.generate(step, prompt.tolist(), spec["max_new"], spec["chunk"], spec["buckets"],
                                     schedule=schedule, max_ctx=spec["max_ctx"])
    return toks, chunks, steps, np.stack(logits), caches


def test_tiny_model_matches_reference(dev, golden_model):
    """Greedy tokens of the reference LlamaQ4 (tiny BASELINE config and the reference's own tiny KAT
    config) under both schedules, from the reference's packed weights."""
    import q4b
    name, z = golden_model
    spec = gi.MODEL_SPECS[name]
    model = q4b.LlamaQ4.from_packed(spec["cfg"], z, spec["max_ctx"], vocab_chunk=spec["vocab_chunk"],
                                    max_chunk=spec["chunk"])
    for schedule in ("bucketed", "max"):
        toks, chunks, steps, logits, caches = _run_schedule(model, spec, z["prompt"], schedule)
        assert toks == z[f"{schedule}_tokens"].tolist(), schedule
        assert chunks == z[f"{schedule}_chunk_buckets"].tolist()
        assert steps == z[f"{schedule}_step_buckets"].tolist()
        if schedule == "bucketed":
            ref = z["bucketed_logits"]
            assert np.abs(logits - ref).max() <= 1e-3 * max(1.0, np.abs(ref).max())
            k0 = caches[0].cpu().numpy()[: z["kv_l0_k"].shape[0]].astype(np.float32)
            assert np.abs(k0 - z["kv_l0_k"].astype(np.float32)).max() <= 2e-3 * max(1.0, np.abs(k0).max())


def test_tiny_model_from_state_dict(dev, golden_model):
    """The reference constructor path: HF random init (seed 0) quantised on the GPU gives the
    reference's packed weights bit for bit, then the same tokens."""
    import q4b
    from transformers import LlamaConfig, LlamaForCausalLM
    name, z = golden_model
    spec = gi.MODEL_SPECS[name]
    torch.manual_seed(spec["seed"])
    hf = LlamaForCausalLM(LlamaConfig(**spec["cfg"], attn_implementation="eager")).eval()
    sd = {k: v.clone() for k, v in hf.state_dict().items()}
    model = q4b.LlamaQ4(None, group=spec["group"], max_ctx=spec["max_ctx"], vocab_chunk=spec["vocab_chunk"], sd=sd,
                        cfg=spec["cfg"], per_linear_group=True, max_chunk=spec["chunk"])
    for i, ly in enumerate(model.layers):
        for nm in ("wqkv", "wo", "wgu", "wdown"):
            ql = getattr(ly, nm)
            assert ql.group == int(z[f"l{i}_{nm}_group"])
            assert np.array_equal(ql.qweight.cpu().numpy(), z[f"l{i}_{nm}_qweight"]), (i, nm)
            assert np.array_equal(ql.scales.cpu().numpy().view(np.uint16), z[f"l{i}_{nm}_scales"].view(np.uint16))
    assert np.array_equal(model.embed.qweight.cpu().numpy(), z["embed_qweight"])
    toks, _, _, _, _ = _run_schedule(model, spec, z["prompt"], "bucketed")
    assert toks == z["bucketed_tokens"].tolist()


def test_step_rejects_bad_positions(dev, golden_model):
    import q4b
    name, z = golden_model
    spec = gi.MODEL_SPECS[name]
    model = q4b.LlamaQ4.from_packed(spec["cfg"], z, spec["max_ctx"], vocab_chunk=spec["vocab_chunk"], max_chunk=8)
    caches = model.new_caches()
    with pytest.raises(q4b.Q4BError):  # past the cache
        model.step(torch.zeros(1, 1, dtype=torch.int32), torch.tensor([spec["max_ctx"]]), torch.tensor([0]), caches, 16)
    with pytest.raises(q4b.Q4BError):  # more rows than the model's max_chunk
        model.step(torch.zeros(1, 9, dtype=torch.int32), torch.tensor([0]), torch.tensor([0]), caches, 16)
