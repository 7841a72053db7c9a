"""Seeded inputs shared by make_golden.py (which feeds them to the reference) and the tests
(which regenerate them to feed the CUDA path). Pure numpy; never imports the reference."""

from __future__ import annotations

import hashlib
import zlib

import numpy as np

# int4 decode GEMV N=5120, K=3072, group 128, M=1
GEMV_N, GEMV_K, GEMV_G = 5120, 3072, 128

# name -> (N, K, group, batch sizes M)
LINEAR_CASES = {
    "n512_k256_g32": (512, 256, 32, (1, 8)),       # scripts/debug/llm_op_test.py:14, 33-34
    "n256_k688_g16": (256, 688, 16, (1, 3, 32)),   # tiny down_proj shape (group rule 688 -> 16)
    "n384_k3072_g128": (384, 3072, 128, (1, 4, 16, 64)),
    "n72_k136_g8": (72, 136, 8, (1, 3)),           # odd sizes
    "n1056_k256_g128": (1056, 256, 128, (1, 2, 32)),  # tiny wqkv shape
}

ROPE_SAMPLE_ROWS = np.array([0, 1, 2, 3, 17, 100, 511, 1000, 2047, 4095])

TINY_BASELINE = dict(
    hidden_size=256, num_hidden_layers=4, num_attention_heads=8, num_key_value_heads=2, head_dim=32,
    intermediate_size=688, vocab_size=1024, rms_norm_eps=1e-5, rope_theta=500000.0,
    max_position_embeddings=4096, tie_word_embeddings=True, hidden_act="silu", attention_bias=False,
    mlp_bias=False, initializer_range=0.2,
)
# the reference's own KAT config (scripts/llm/test_tiny.py:19-27)
TINY_REF = dict(
    hidden_size=256, num_hidden_layers=2, num_attention_heads=8, num_key_value_heads=2, head_dim=32,
    intermediate_size=512, vocab_size=1000, rms_norm_eps=1e-5, rope_theta=500000.0,
    rope_scaling={"rope_type": "llama3", "factor": 32.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
                  "original_max_position_embeddings": 8192},
    max_position_embeddings=131072, tie_word_embeddings=True, hidden_act="silu", attention_bias=False,
    mlp_bias=False, initializer_range=0.2,
)
LLAMA32_3B = dict(
    hidden_size=3072, num_hidden_layers=28, num_attention_heads=24, num_key_value_heads=8, head_dim=128,
    intermediate_size=8192, vocab_size=128256, rms_norm_eps=1e-5, rope_theta=500000.0,
    rope_scaling={"rope_type": "llama3", "factor": 32.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
                  "original_max_position_embeddings": 8192},
    max_position_embeddings=131072, tie_word_embeddings=True, hidden_act="silu", attention_bias=False,
    mlp_bias=False, initializer_range=0.02,
)

ROPE_CASES = {
    "tiny_baseline": (TINY_BASELINE, 256),
    "tiny_ref": (TINY_REF, 64),
    "llama32_3b": (LLAMA32_3B, 4096),
}

MODEL_SPECS = {
    # 4 layers, inter 688, vocab 1024, group 128 (688 -> 16), 64-token prompt,
    # chunk 32, buckets {128, 256}, 64 new tokens
    "tiny_baseline": dict(cfg=TINY_BASELINE, seed=0, group=128, max_ctx=256, vocab_chunk=1024, chunk=32,
                          buckets=[128, 256], n_prompt=64, max_new=64, prompt_seed=1),
    # scripts/llm/test_tiny.py: group 32, vocab chunks of 256 rows, chunk 8, bucket 32, 10 new
    "tiny_ref": dict(cfg=TINY_REF, seed=0, group=32, max_ctx=64, vocab_chunk=256, chunk=8, buckets=[16, 32, 64],
                     n_prompt=21, max_new=10, prompt_seed=2),
}


def case_seed(name: str) -> int:
    return zlib.crc32(name.encode()) & 0x7FFFFFFF


def digest(a) -> int:
    """64-bit digest of an array's bytes (checks that regenerated inputs equal the golden's)."""
    return int.from_bytes(hashlib.sha256(np.ascontiguousarray(a).tobytes()).digest()[:8], "little")


def pack_nibbles(nibs):
    nibs = np.asarray(nibs, dtype=np.int64)
    n, k = nibs.shape
    packed = (nibs.reshape(n, k // 8, 8) << (np.arange(8, dtype=np.int64) * 4)).sum(-1)
    return np.ascontiguousarray(packed.astype(np.uint32).view(np.int32))


def synthetic_q4(N, K, G, seed):
    """Uniform nibbles 0..15 packed along K and |N(0, 0.02)| fp16 scales."""
    rng = np.random.default_rng(seed)
    nibs = rng.integers(0, 16, size=(N, K), dtype=np.int64)
    scales = np.abs(rng.standard_normal((N, K // G)) * 0.02).astype(np.float16)
    return pack_nibbles(nibs), scales


def linear_x(M, K, seed):
    """x [M, K] ~ N(0, 1) rounded to fp16 (so fp16 and fp32 callers see the same values)."""
    return np.random.default_rng(seed).standard_normal((M, K)).astype(np.float16)


def gemv_inputs(seed=0):
    """BASELINE config 1 inputs: (qweight [5120, 384] int32, scales [5120, 24] fp16, x [3072] fp16)."""
    qw, s = synthetic_q4(GEMV_N, GEMV_K, GEMV_G, seed)
    x = np.random.default_rng(seed + 1).standard_normal(GEMV_K).astype(np.float16)
    return qw, s, x


def quant_weights():
    """[64, 256] fp32 weights for quantize_q4 goldens, with edge rows: an all-zero row (scale clamp
    1e-8), exact half-way ties (round half to even), tiny values and large values."""
    rng = np.random.default_rng(3)
    w = (rng.standard_normal((64, 256)) * 0.05).astype(np.float32)
    w[0] = 0.0
    # row 1: absmax 7 in every 16-group so scale == 1, then values on .5 ties
    ties = np.array([0.5, 1.5, 2.5, -0.5, -1.5, -2.5, 3.5, -3.5, 4.5, -4.5, 5.5, -5.5, 6.5, -6.5, 7.0, -7.0],
                    dtype=np.float32)
    w[1] = np.tile(ties, 16)
    w[2] = (rng.standard_normal(256) * 1e-10).astype(np.float32)
    w[3] = (rng.standard_normal(256) * 1e4).astype(np.float32)
    w[4, ::3] = 0.0
    return w


# scripts/debug/llm_op_test.py:15, 37-38 (plus two tokens outside the vocabulary)
EMBED_TOKENS = np.array([3, 300, 999, 512, 0, 767, 1000, -1], dtype=np.int64)


def embed_weights():
    """[1000, 256] fp32 table, quantised by the reference's QEmbedding with group 32 and chunks of
    256 rows (scripts/debug/llm_op_test.py:15)."""
    return (np.random.default_rng(6).standard_normal((1000, 256)) * 0.05).astype(np.float32)


def model_prompt(spec):
    rng = np.random.default_rng(spec["prompt_seed"])
    return rng.integers(0, spec["cfg"]["vocab_size"], size=spec["n_prompt"]).astype(np.int32)
