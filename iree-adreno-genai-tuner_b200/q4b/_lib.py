"""ctypes binding of libq4b.so (the C ABI declared in include/q4b.h).

The library is built in-tree by ``make -C iree-adreno-genai-tuner_b200/csrc`` (or
``__graft_entry__.build()``). There is no fallback: importing an op without the library raises.
"""

from __future__ import annotations

import ctypes
import os
import pathlib

_HERE = pathlib.Path(__file__).resolve().parent
LIB_PATH = pathlib.Path(os.environ.get("Q4B_LIB", _HERE / "libq4b.so"))

c_int, c_size_t, c_void_p, c_float, c_char_p = ctypes.c_int, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_float, ctypes.c_char_p

Q4B_OK = 0
Q4B_EINVAL = -1
Q4B_ELAUNCH = -2
Q4B_ETIMEOUT = -3
Q4B_ENOMEM = -4
Q4B_EUNSUPPORTED = -5
Q4B_ECUDA = -6
Q4B_ESTATE = -7
F32, F16 = 0, 1
EPI_STORE, EPI_ACCUMULATE, EPI_SWIGLU = 0, 1, 2

_CODES = {Q4B_EINVAL: "EINVAL", Q4B_ELAUNCH: "ELAUNCH", Q4B_ETIMEOUT: "ETIMEOUT", Q4B_ENOMEM: "ENOMEM",
          Q4B_EUNSUPPORTED: "EUNSUPPORTED", Q4B_ECUDA: "ECUDA", Q4B_ESTATE: "ESTATE"}


class Q4BError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__(f"[{_CODES.get(code, code)}] {msg}")
        self.code = code


class LinearCfg(ctypes.Structure):
    _fields_ = [("kernel", c_int), ("warps", c_int), ("tiles", c_int), ("split", c_int)]


class GemmCfg(ctypes.Structure):
    _fields_ = [("kernel", c_int), ("bn", c_int), ("stages", c_int), ("split", c_int)]


class ModelCfg(ctypes.Structure):
    _fields_ = [("n_layers", c_int), ("dim", c_int), ("n_heads", c_int), ("n_kv_heads", c_int), ("head_dim", c_int),
                ("inter", c_int), ("vocab", c_int), ("rms_eps", c_float), ("max_ctx", c_int), ("max_chunk", c_int),
                ("tp_rank", c_int), ("tp_size", c_int)]


class QMat(ctypes.Structure):
    _fields_ = [("qweight", c_void_p), ("scales", c_void_p), ("n", c_int), ("k", c_int), ("group", c_int)]


class LayerWeights(ctypes.Structure):
    _fields_ = [("wqkv", QMat), ("wo", QMat), ("wgu", QMat), ("wdown", QMat), ("ln_in", c_void_p),
                ("ln_post", c_void_p), ("k_cache", c_void_p), ("v_cache", c_void_p)]


class RunnerOpts(ctypes.Structure):
    _fields_ = [("chunk", c_int), ("buckets", c_void_p), ("n_buckets", c_int), ("schedule", c_int),
                ("use_graphs", c_int), ("warmup", c_int), ("sync_every_step", c_int)]


class Report(ctypes.Structure):
    _fields_ = [("warmup_ms", ctypes.c_double), ("prefill_ms", ctypes.c_double), ("ttft_ms", ctypes.c_double),
                ("prefill_tok_s", ctypes.c_double), ("decode_ms", ctypes.c_double),
                ("decode_wall_ms", ctypes.c_double), ("decode_tok_s", ctypes.c_double), ("prompt_tokens", c_int),
                ("new_tokens", c_int), ("decode_steps", c_int)]


# name -> (restype, argtypes); must match include/q4b.h
SIGNATURES = {
    "q4b_last_error": (c_char_p, []),
    "q4b_abi_version": (c_int, []),
    "q4b_quantize_q4": (c_int, [c_void_p, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p]),
    "q4b_unpack_q4": (c_int, [c_void_p, c_int, c_int, c_void_p, c_void_p]),
    "q4b_dequantize_q4": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_void_p, c_int, c_void_p]),
    "q4b_q4_linear_workspace": (c_size_t, [c_int, c_int, c_int, c_int, c_int, c_void_p]),
    "q4b_q4_linear": (c_int, [c_void_p, c_void_p, c_int, c_void_p, c_int, c_void_p, c_int, c_int, c_int, c_int,
                              c_int, c_void_p, c_void_p, c_size_t, c_void_p]),
    "q4b_q4_linear_kernel": (c_int, [c_int, c_int, c_int, c_int, c_int, c_int, c_void_p]),
    "q4b_q4_linear_noalloc": (c_int, [c_void_p, c_void_p, c_int, c_void_p, c_int, c_void_p, c_int, c_int, c_int,
                                      c_int, c_int, c_void_p]),
    "q4b_gemm_f16_workspace": (ctypes.c_longlong, [c_int, c_int, c_int, ctypes.c_char, ctypes.c_char, c_void_p]),
    "q4b_gemm_f16_plan": (c_int, [c_int, c_int, c_int, ctypes.c_char, ctypes.c_char, c_void_p, c_void_p]),
    "q4b_gemm_f16": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, ctypes.c_char, ctypes.c_char, c_void_p,
                             c_void_p, c_size_t, c_void_p]),
    "q4b_embed_q4_lookup": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p, c_void_p]),
    "q4b_rmsnorm": (c_int, [c_void_p, c_void_p, c_float, c_int, c_int, c_void_p, c_void_p]),
    "q4b_attention_workspace": (c_size_t, [c_int, c_int, c_int, c_int, c_int]),
    "q4b_attention": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_void_p,
                              c_void_p, c_size_t, c_void_p]),
    "q4b_prefill_attn": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int,
                                 c_void_p, c_void_p]),
    "q4b_qkv_rope_kvwrite_workspace": (c_size_t, [c_int, c_int, c_int, c_int, c_int, c_int]),
    "q4b_qkv_rope_kvwrite": (c_int, [c_void_p, c_void_p, c_int, c_void_p, c_int, c_int, c_int, c_int, c_int,
                                     c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_size_t,
                                     c_void_p]),
    "q4b_silu_mul": (c_int, [c_void_p, c_int, c_int, c_void_p, c_void_p]),
    "q4b_argmax": (c_int, [c_void_p, c_int, c_void_p, c_void_p]),
    "q4b_tp_init": (c_int, [c_int, c_int, c_void_p, c_int, ctypes.POINTER(c_void_p)]),
    "q4b_tp_destroy": (None, [c_void_p]),
    "q4b_tp_allreduce_f16": (c_int, [c_void_p, c_void_p, c_size_t, c_void_p]),
    "q4b_tp_allreduce_f32": (c_int, [c_void_p, c_void_p, c_size_t, c_void_p]),
    "q4b_tp_argmax_workspace": (c_size_t, [c_void_p]),
    "q4b_tp_argmax_gather": (c_int, [c_void_p, c_void_p, c_int, c_int, c_void_p, c_void_p, c_size_t, c_void_p]),
    "q4b_model_create": (c_int, [ctypes.POINTER(ModelCfg), ctypes.POINTER(c_void_p)]),
    "q4b_model_set_layer": (c_int, [c_void_p, c_int, ctypes.POINTER(LayerWeights)]),
    "q4b_model_set_head": (c_int, [c_void_p, ctypes.POINTER(QMat), c_void_p, c_void_p, c_void_p]),
    "q4b_model_step": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p]),
    "q4b_model_destroy": (None, [c_void_p]),
    "q4b_model_decode_path": (c_int, [c_void_p]),
    "q4b_model_trace_events": (c_size_t, [c_void_p]),
    "q4b_model_set_trace": (c_int, [c_void_p, c_void_p, c_size_t]),
    "q4b_model_fail_decode": (c_int, [c_void_p]),
    "q4b_device_status": (c_int, [c_int]),
    "q4b_tp_unique_id": (c_int, [c_void_p, c_int]),
    "q4b_model_attach_tp": (c_int, [c_void_p, c_void_p, c_int]),
    "q4b_runner_create": (c_int, [c_void_p, ctypes.POINTER(RunnerOpts), ctypes.POINTER(c_void_p)]),
    "q4b_runner_generate": (c_int, [c_void_p, c_void_p, c_int, c_int, c_void_p, c_int, c_void_p,
                                    ctypes.POINTER(c_int), ctypes.POINTER(Report)]),
    "q4b_runner_report_json": (c_char_p, [c_void_p]),
    "q4b_runner_destroy": (None, [c_void_p]),
}

_lib = None


def lib():
    """Load libq4b.so once; raise if it is missing (no CPU fallback exists)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(f"libq4b.so not found at {LIB_PATH}; build it with "
                              f"`make -C iree-adreno-genai-tuner_b200/csrc` or __graft_entry__.build()")
        L = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(rc: int, what: str):
    if rc != Q4B_OK:
        raise Q4BError(rc, f"{what}: {lib().q4b_last_error().decode(errors='replace')}")
