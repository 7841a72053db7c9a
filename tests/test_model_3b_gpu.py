"""BASELINE config 4 at full depth: the benched 3B-shape path against the reference's own stream.

tests/golden/model_3b_ref.npz holds what the unmodified reference ``LlamaQ4.step``
(scripts/llm/llama_q4.py:199-239) produced on the host (tests/golden/make_golden_3b.py): the greedy
stream of the bench's request (512 prompt ids, chunk 128, KV buckets 256..4096, bucketed schedule of
runner/llm_runner.c:143-246), every step's top-2 margin, and the logits of the first 8 steps at the
top-64 ids and every 32nd id. The weights come from q4b.SyntheticStateDict(SYNTHETIC["3b"], seed=0),
whose values are integer hashing plus one fp32 multiply, so this test regenerates on the GPU exactly
the fp32 weights the reference quantised. The path under test is the bench's: tcgen05 prefill
chunks, the ring GEMV lm_head with the greedy argmax, and the persistent decode step over all 28
layers (one cooperative launch per token).

Bars (the model's own parity statement): greedy tokens identical up to the first step whose reference
margin is below 1e-3 (none is, in this fixture: all 256 must match), logits within
1e-3 * max(1, max|ref|)."""

import pathlib

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
FIX = pathlib.Path(__file__).resolve().parent / "golden" / "model_3b_ref.npz"
CHUNK, BUCKETS = 128, [256, 512, 1024, 2048, 4096]


@pytest.fixture(scope="module")
def ref():
    return dict(np.load(FIX))


@pytest.fixture(scope="module")
def model3b():
    import q4b
    dev = torch.device("cuda:0")
    cfg = q4b.SYNTHETIC["3b"]
    m = q4b.LlamaQ4(None, group=128, max_ctx=4096, vocab_chunk=32064, sd=q4b.SyntheticStateDict(cfg, seed=0, device=dev),
                    cfg=cfg, max_chunk=CHUNK, device=dev)
    torch.cuda.synchronize()
    return m


def test_weights_are_the_references(model3b):
    """Layer 0's q projection regenerated on the host and quantised by the CPU restatement of
    quantize_q4 (pinned to the reference's goldens) equals the GPU model's packed rows."""
    import q4b
    from oracle import q4_oracle as O
    sd = q4b.SyntheticStateDict(q4b.SYNTHETIC["3b"], seed=0, device="cpu")
    w = sd["model.layers.0.self_attn.q_proj.weight"].numpy()
    qw, s = O.quantize_q4(w, 128)
    got_qw = model3b.layers[0].wqkv.qweight[: w.shape[0]].cpu().numpy()
    got_s = model3b.layers[0].wqkv.scales[: w.shape[0]].cpu().numpy()
    assert np.array_equal(got_qw, qw)
    assert np.array_equal(got_s.view(np.uint16), s.view(np.uint16))


def test_greedy_stream_matches_reference(model3b, ref):
    import q4b
    runner = q4b.Runner(model3b, CHUNK, BUCKETS, "bucketed", graphs=True)
    toks, rep = runner.generate(ref["prompt"].tolist(), len(ref["tokens"]))
    assert q4b.lib().q4b_model_decode_path(model3b.native()) == 1  # the persistent decode step ran
    want = ref["tokens"].tolist()
    low = np.nonzero(ref["margin"] < 1e-3)[0]
    limit = int(low[0]) if len(low) else len(want)
    first_bad = next((i for i, (a, b) in enumerate(zip(toks, want)) if a != b), None)
    assert toks[:limit] == want[:limit], (
        f"first mismatch at step {first_bad} (reference margin {ref['margin'][first_bad]:.3g}); "
        f"bar: identical up to step {limit}")
    assert rep["chunks"] == [[int(b), rep["chunks"][i][1]] for i, b in enumerate(ref["chunk_buckets"])]
    assert q4b.lib().q4b_device_status(1) == 0


def test_logits_first_steps_match_reference(model3b, ref):
    """The first 8 steps through LlamaQ4.step on the runner's schedule: prefill chunks (the last one
    gives step 0), then single-token decode steps in bucket 1024."""
    import q4b
    caches = model3b.new_caches()
    prompt = ref["prompt"]
    nxt = None
    for s0 in range(0, len(prompt), CHUNK):
        L = next(b for b in BUCKETS if b >= s0 + CHUNK)
        nxt, lg = model3b.step(torch.from_numpy(prompt[s0:s0 + CHUNK].astype(np.int32)).reshape(1, -1),
                               torch.tensor([s0]), torch.tensor([CHUNK - 1]), caches, L)
    pos = len(prompt)
    for st in range(ref["logit_idx"].shape[0]):
        if st > 0:
            nxt, lg = model3b.step(nxt.reshape(1, 1).cpu(), torch.tensor([pos]), torch.tensor([0]), caches, 1024)
            pos += 1
        idx = ref["logit_idx"][st]
        keep = idx >= 0
        got = lg[0].cpu().numpy()[idx[keep]]
        want = ref["logit_val"][st][keep]
        tol = 1e-3 * max(1.0, float(np.abs(want).max()))
        err = float(np.abs(got - want).max())
        assert err <= tol, (st, err, tol)
        assert int(nxt) == int(ref["tokens"][st]), st
    assert q4b.lib().q4b_device_status(1) == 0
