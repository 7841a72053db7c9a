"""The C restatement of the reference's fused int4 GEMV (oracle/q4_cpu.c, the CPU timing leg of
bench.py) against the reference's own golden output and the numpy restatement."""

import numpy as np
import pytest

import golden_inputs as gi
from oracle import q4_cpu as C
from oracle import q4_oracle as O


def test_gemv_matches_reference_golden(golden_gemv):
    qw, s, x = gi.gemv_inputs()
    y = C.gemv(qw, s, gi.GEMV_G, x.astype(np.float32))
    assert O.rel_err(y, golden_gemv["y_fused"]) <= 1e-5
    assert O.rel_err(y, golden_gemv["y_dequant"]) <= 1e-5


@pytest.mark.parametrize("n,k,g", [(1, 64, 8), (37, 256, 16), (300, 1024, 32), (129, 3072, 128), (64, 2048, 256)])
def test_gemv_matches_numpy_restatement(n, k, g):
    qw, s = gi.synthetic_q4(n, k, g, seed=n + k)
    x = np.random.default_rng(n).standard_normal(k).astype(np.float32)
    assert O.rel_err(C.gemv(qw, s, g, x), O.q4_linear(qw, s, g, x[None])[0]) <= 1e-5


def test_decode_step_runs_on_a_small_shape():
    cfg = dict(hidden_size=256, num_hidden_layers=2, num_attention_heads=8, num_key_value_heads=2, head_dim=32,
               intermediate_size=512, vocab_size=1000, rms_norm_eps=1e-5, rope_theta=500000.0,
               max_position_embeddings=4096, tie_word_embeddings=True)
    m = C.DecodeModel(cfg, max_ctx=64)
    t = m.step(3, 10, 64)
    assert 0 <= t < 1000 and m.step(t, 11, 64) >= 0
