"""GPU tests of the native runner: the scheduler of runner/llm_runner.c with CUDA graphs.

Tokens must equal the reference's (tests/golden/model_*.npz) under both schedules, with graphs on
and off and with the per-step synchronous protocol; the JSON report keeps llm_runner.c's schema."""

import numpy as np
import pytest
import torch

import golden_inputs as gi

pytestmark = pytest.mark.gpu

KEYS = {"schedule", "chunk", "prompt_tokens", "new_tokens", "warmup_ms", "prefill_ms", "prefill_tok_s", "ttft_ms",
        "decode_ms", "decode_steps", "decode_tok_s", "chunks", "steps", "tokens"}


@pytest.mark.parametrize("graphs,sync", [(True, False), (False, False), (True, True)])
def test_runner_tokens_match_reference(golden_model, graphs, sync):
    import q4b
    name, z = golden_model
    spec = gi.MODEL_SPECS[name]
    model = q4b.LlamaQ4.from_packed(spec["cfg"], z, spec["max_ctx"], vocab_chunk=spec["vocab_chunk"],
                                    max_chunk=spec["chunk"])
    for schedule in ("bucketed", "max"):
        r = q4b.Runner(model, spec["chunk"], spec["buckets"], schedule, graphs=graphs, sync_every_step=sync)
        toks, rep = r.generate(z["prompt"].tolist(), spec["max_new"])
        assert toks == z[f"{schedule}_tokens"].tolist(), (schedule, graphs, sync)
        assert KEYS <= set(rep)
        assert rep["tokens"] == toks and rep["new_tokens"] == len(toks)
        assert [c[0] for c in rep["chunks"]] == z[f"{schedule}_chunk_buckets"].tolist()
        assert [s[0] for s in rep["steps"]] == z[f"{schedule}_step_buckets"].tolist()
        assert rep["decode_steps"] == len(toks) - 1 and rep["decode_tok_s"] > 0
        # a second generate on the same runner reuses the graphs and gives the same tokens
        toks2, _ = r.generate(z["prompt"].tolist(), spec["max_new"])
        assert toks2 == toks


@pytest.mark.parametrize("sync", [False, True])
def test_runner_stop_ids(golden_model, sync):
    """llm_runner.c:234-235: decoding ends right after a stop id is produced."""
    import q4b
    name, z = golden_model
    spec = gi.MODEL_SPECS[name]
    ref = z["bucketed_tokens"].tolist()
    model = q4b.LlamaQ4.from_packed(spec["cfg"], z, spec["max_ctx"], vocab_chunk=spec["vocab_chunk"],
                                    max_chunk=spec["chunk"])
    r = q4b.Runner(model, spec["chunk"], spec["buckets"], sync_every_step=sync)
    stop = ref[3]
    first = ref.index(stop)
    toks, rep = r.generate(z["prompt"].tolist(), spec["max_new"], stop_ids=[stop])
    assert toks == ref[: first + 1]
    assert rep["decode_steps"] == first


def test_runner_rejects_like_the_reference(golden_model):
    """llm_runner.c:168-173, 216: empty prompt, prompt + new > max_ctx, padded prompt > max_ctx."""
    import q4b
    name, z = golden_model
    spec = gi.MODEL_SPECS[name]
    model = q4b.LlamaQ4.from_packed(spec["cfg"], z, spec["max_ctx"], vocab_chunk=spec["vocab_chunk"],
                                    max_chunk=spec["chunk"])
    r = q4b.Runner(model, spec["chunk"], spec["buckets"])
    with pytest.raises(q4b.Q4BError, match="empty"):
        r.generate([], 4)
    with pytest.raises(q4b.Q4BError, match="exceeds"):
        r.generate([1] * (spec["max_ctx"] - 2), 4)
    with pytest.raises(q4b.Q4BError, match="bucket"):
        small = q4b.Runner(model, spec["chunk"], [spec["buckets"][0]])
        small.generate([1] * (spec["buckets"][0] + 1), 2)


def test_runner_whole_chunk_prefill_on_tensor_cores(golden_model):
    """A 64-row prefill chunk goes through the tcgen05 int4 GEMM (q|k|v with RoPE + KV write,
    SwiGLU, residual adds); the greedy tokens still equal the reference's (the oracle gives the
    same tokens for chunk 64 as for the golden's chunk)."""
    import q4b
    name, z = golden_model
    spec = gi.MODEL_SPECS[name]
    if name != "tiny_baseline":
        pytest.skip("needs a group-128 model with a prompt of at least 64 tokens")
    model = q4b.LlamaQ4.from_packed(spec["cfg"], z, spec["max_ctx"], vocab_chunk=spec["vocab_chunk"], max_chunk=64)
    r = q4b.Runner(model, 64, spec["buckets"], "bucketed")
    toks, rep = r.generate(z["prompt"].tolist(), spec["max_new"])
    assert toks == z["bucketed_tokens"].tolist()
    assert [c[0] for c in rep["chunks"]] == [128]
