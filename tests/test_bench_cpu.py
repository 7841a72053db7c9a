"""The roofline arithmetic of bench.py on the CPU: the algorithmic bytes each bench
line divides by the measured time, and the traffic figures it reads from profiles/."""

import pathlib
import sys

ROOT = pathlib.Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "iree-adreno-genai-tuner_b200"))

import bench  # noqa: E402
import q4b  # noqa: E402


def test_decode_bytes_per_token_3b():
    """int4 weights + fp16 scales of 28 layers and the lm_head, plus KV rows 0..pos read and row pos
    written (2 x 8 KV heads x 128 x 2 bytes per layer per row)."""
    cfg = q4b.SYNTHETIC["3b"]
    weights = 1_656_483_840
    kv_row = 28 * 2 * 8 * 128 * 2
    assert bench.decode_bytes_per_token(cfg, 640) == weights + kv_row * 642
    assert bench.decode_bytes_per_token(cfg, 640, 2) == (weights + kv_row * 642) / 2


def test_gemv_config1_bytes():
    assert bench.GEMV_BYTES == 8_126_464  # qweight + scales + x + y of the 5120 x 3072 GEMV
    assert bench.linear_bytes(5120, 3072, 1) == bench.GEMV_BYTES


def test_profile_traffic_lines():
    """The traffic the bench lines report comes from the committed ncu summaries and is within a
    percent of the algorithmic bytes (no re-reads)."""
    t = bench.profile_traffic("decode_step_3b")
    assert t is not None and abs(t / bench.decode_bytes_per_token(q4b.SYNTHETIC["3b"], 640) - 1) < 0.01
    g = bench.profile_traffic("q4_gemv_mma_5120x3072")
    assert g is not None and abs(g / bench.GEMV_BYTES - 1) < 0.01
