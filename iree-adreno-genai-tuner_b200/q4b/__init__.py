"""q4b: B200-native (sm_100a) drop-in for the int4 Llama hot path of the reference's
scripts/llm/llama_q4.py (QLinear, QEmbedding, LlamaQ4) and runner/llm_runner.c (the scheduler),
computed by hand-written CUDA in libq4b.so behind the C ABI of include/q4b.h."""

from ._lib import LIB_PATH, GemmCfg, LinearCfg, Q4BError, lib
from .llama import LazySafetensors, LlamaQ4, StepFn, SyntheticStateDict, group_for, rope_tables, shard_layer
from .ops import attention, dequantize_q4, embed_lookup, gemm_f16, q4_linear, quantize_q4, rmsnorm, unpack_q4
from .qlinear import QEmbedding, QLinear
from .runner import SYNTHETIC, Runner
from .shard import shard_q4, shard_x

__all__ = ["shard_q4", "shard_x", "LIB_PATH", "GemmCfg", "LinearCfg", "gemm_f16", "Q4BError", "lib", "quantize_q4", "unpack_q4", "dequantize_q4", "q4_linear",
           "embed_lookup", "rmsnorm", "attention", "QLinear", "QEmbedding", "LlamaQ4", "StepFn", "SyntheticStateDict", "LazySafetensors",
           "group_for", "rope_tables", "shard_layer", "Runner", "SYNTHETIC"]
