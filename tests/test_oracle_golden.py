"""Pin the CPU oracle (oracle/q4_oracle.py) to the reference's own outputs (tests/golden/*.npz)."""

import numpy as np
import pytest

import golden_inputs as gi
from oracle import q4_oracle as O


@pytest.mark.parametrize("g", [16, 32, 128])
def test_quantize_bit_exact(golden_ops, g):
    qw, s = O.quantize_q4(gi.quant_weights(), g)
    assert np.array_equal(qw, golden_ops[f"quant_g{g}_qweight"])
    assert np.array_equal(s.view(np.uint16), golden_ops[f"quant_g{g}_scales"].view(np.uint16))


@pytest.mark.parametrize("g", [16, 32, 128])
def test_unpack_dequant_bit_exact(golden_ops, g):
    qw, s = golden_ops[f"quant_g{g}_qweight"], golden_ops[f"quant_g{g}_scales"]
    assert np.array_equal(O.unpack_q4(qw), golden_ops[f"quant_g{g}_unpack"].astype(np.int32))
    assert np.array_equal(O.dequantize_q4(qw, s, g).view(np.uint32),
                          golden_ops[f"quant_g{g}_dequant"].view(np.uint32))


def test_quantize_edge_rows(golden_ops):
    qw = golden_ops["quant_g16_qweight"]
    nib = O.unpack_q4(qw)
    assert np.all(nib[0] == 8)              # all-zero row: scale clamped, every q = 0 -> nibble 8
    assert nib.min() >= 1                   # quantize_q4 never emits nibble 0 (q = -8)
    # ties round half to even: 0.5 -> 0, 1.5 -> 2, 2.5 -> 2, -0.5 -> 0, -1.5 -> -2, -2.5 -> -2
    assert list(nib[1, :6] - 8) == [0, 2, 2, 0, -2, -2]


def test_pack_roundtrip():
    rng = np.random.default_rng(0)
    nibs = rng.integers(0, 16, (7, 64))
    assert np.array_equal(O.unpack_q4(O.pack_nibbles(nibs)), nibs)


@pytest.mark.parametrize("name", list(gi.LINEAR_CASES))
def test_linear_both_forms(golden_ops, name):
    N, K, G, Ms = gi.LINEAR_CASES[name]
    qw, s = gi.synthetic_q4(N, K, G, seed=gi.case_seed(name))
    for M in Ms:
        x = gi.linear_x(M, K, seed=gi.case_seed(name) + M).astype(np.float32)
        y = O.q4_linear(qw, s, G, x)
        assert O.rel_err(y, golden_ops[f"lin_{name}_m{M}_dequant"]) < 1e-5
        if M == 1:
            ref = golden_ops[f"lin_{name}_m{M}_fused"]
            assert O.rel_err(y, ref) < 1e-5
            assert O.rel_err(O.q4_linear_fused_f32(qw, s, G, x), ref) < 1e-5


def test_gemv_config1(golden_gemv):
    qw, s, x = gi.gemv_inputs()
    assert [gi.digest(qw), gi.digest(s), gi.digest(x)] == golden_gemv["inputs_digest"].tolist()
    y = O.q4_linear(qw, s, gi.GEMV_G, x.astype(np.float32)[None])[0]
    assert O.rel_err(y, golden_gemv["y_fused"]) < 1e-5
    assert O.rel_err(y, golden_gemv["y_dequant"]) < 1e-5


def test_embedding(golden_ops):
    qw, s = golden_ops["emb_qweight"], golden_ops["emb_scales"]
    # QEmbedding quantises each 256-row chunk on its own; rows are independent, so the chunks
    # concatenate into the table quantize_q4 makes of the whole matrix
    qw2, s2 = O.quantize_q4(gi.embed_weights(), 32)
    assert np.array_equal(qw, qw2) and np.array_equal(s.view(np.uint16), s2.view(np.uint16))
    out = O.embed_lookup(qw, s, 32, gi.EMBED_TOKENS)
    assert np.array_equal(out.view(np.uint32), golden_ops["emb_lookup"].view(np.uint32))
    assert np.all(out[-2:] == 0)  # tokens outside the vocabulary give zero rows
    lg = O.embed_logits(qw, s, 32, golden_ops["emb_logits_x"])
    assert O.rel_err(lg, golden_ops["emb_logits"]) < 1e-5


def test_rmsnorm(golden_ops):
    out = O.rms_norm(golden_ops["rms_x"], golden_ops["rms_w"], 1e-5)
    assert np.abs(out - golden_ops["rms_out"]).max() <= 1e-6 * np.abs(golden_ops["rms_out"]).max()


@pytest.mark.parametrize("name", list(gi.ROPE_CASES))
def test_rope_tables(golden_rope, name):
    cfg, max_ctx = gi.ROPE_CASES[name]
    cos, sin = O.rope_tables(cfg, max_ctx)
    if f"{name}_cos" in golden_rope:
        rc, rs = golden_rope[f"{name}_cos"], golden_rope[f"{name}_sin"]
    else:
        rows = gi.ROPE_SAMPLE_ROWS
        rc, rs = golden_rope[f"{name}_cos_rows"], golden_rope[f"{name}_sin_rows"]
        cos, sin = cos[rows], sin[rows]
    # the argument p * inv_freq is rounded to fp32 identically; cos/sin libraries may differ in ulps
    assert np.abs(cos - rc).max() < 2e-6 and np.abs(sin - rs).max() < 2e-6


def _oracle_model(z, spec):
    cfg = spec["cfg"]
    layers = []
    for i in range(cfg["num_hidden_layers"]):
        ly = {}
        for nm in ("wqkv", "wo", "wgu", "wdown"):
            ly[nm] = (z[f"l{i}_{nm}_qweight"], z[f"l{i}_{nm}_scales"], int(z[f"l{i}_{nm}_group"]))
        ly["ln_in"], ly["ln_post"] = z[f"l{i}_ln_in"], z[f"l{i}_ln_post"]
        layers.append(ly)
    embed = (z["embed_qweight"], z["embed_scales"], int(z["embed_group"]))
    return O.OracleModel(cfg, layers, embed, z["ln_f"], spec["max_ctx"])


def test_model_greedy_tokens(golden_model):
    name, z = golden_model
    spec = gi.MODEL_SPECS[name]
    m = _oracle_model(z, spec)
    assert np.array_equal(z["prompt"], gi.model_prompt(spec))
    for schedule in ("bucketed", "max"):
        caches = m.new_caches()
        logits = []

        def step(tokens, start, last, L):
            nxt, lg = m.step(tokens, start, last, caches, L)
            logits.append(lg)
            return nxt

        toks, chunks, steps = O.generate(step, z["prompt"].tolist(), spec["max_new"], spec["chunk"], spec["buckets"],
                                         schedule=schedule, max_ctx=spec["max_ctx"])
        assert toks == z[f"{schedule}_tokens"].tolist()
        assert chunks == z[f"{schedule}_chunk_buckets"].tolist()
        assert steps == z[f"{schedule}_step_buckets"].tolist()
        if schedule == "bucketed":
            ref = z["bucketed_logits"]
            assert np.abs(np.stack(logits) - ref).max() < 1e-3 * max(1.0, np.abs(ref).max())


def test_scheduler_rules():
    b = [128, 256]
    assert O.pick_bucket(b, 1, False) == 128 and O.pick_bucket(b, 129, False) == 256
    assert O.pick_bucket(b, 257, False) == -1 and O.pick_bucket(b, 1, True) == 256
    with pytest.raises(O.ScheduleError):
        O.check_request(0, 4, 32, 256)
    with pytest.raises(O.ScheduleError):
        O.check_request(250, 10, 32, 256)
    with pytest.raises(O.ScheduleError):
        O.check_request(250, 1, 32, 250)   # ceil(250 / 32) * 32 = 256 > max_ctx
    assert O.used_functions(64, 64, 32, b, False) == ([128], [128])
    assert O.used_functions(64, 64, 32, b, True) == ([256], [256])
    # a stop id ends decoding after it is emitted
    calls = []

    def step(tokens, start, last, L):
        calls.append((start, last, L))
        return 5

    toks, chunks, steps = O.generate(step, [1, 2, 3], 8, 2, b, stop_ids=(5,), max_ctx=256)
    assert toks == [5] and calls == [(0, 1, 128), (2, 0, 128)]
