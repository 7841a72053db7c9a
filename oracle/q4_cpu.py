"""CPU restatement of the reference's decode step with the int4 GEMVs in C (TEST AND BASELINE
INFRASTRUCTURE: checker and CPU timing leg only, never the product path).

The GEMV is oracle/q4_cpu.c (QLinear._gemv_fused, scripts/llm/llama_q4.py:74-90, OpenMP over rows);
the rest of a decode step is the numpy restatement in oracle/q4_oracle.py (RMSNorm :141-142, RoPE
:206-207/:219-220, KV write and GQA attention :208-232, SwiGLU and residuals :233-236, greedy head
:237-239). libq4cpu.so is built next to this file by `make -C oracle` (or __graft_entry__.build()).
"""

from __future__ import annotations

import ctypes
import os
import pathlib
import subprocess

import numpy as np

from . import q4_oracle as O

HERE = pathlib.Path(__file__).resolve().parent
LIB = HERE / "libq4cpu.so"
_lib = None


def build():
    subprocess.run(["make", "-C", str(HERE)], check=True, stdout=subprocess.DEVNULL)


def lib():
    global _lib
    if _lib is None:
        if not LIB.exists():
            build()
        L = ctypes.CDLL(str(LIB))
        L.q4cpu_gemv.restype = None
        L.q4cpu_gemv.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                 ctypes.c_void_p, ctypes.c_void_p]
        L.q4cpu_threads.restype = ctypes.c_int
        L.q4cpu_argmax.restype = ctypes.c_int
        L.q4cpu_argmax.argtypes = [ctypes.c_void_p, ctypes.c_int]
        _lib = L
    return _lib


def threads() -> int:
    return int(lib().q4cpu_threads())


def gemv(qweight, scales, group: int, x):
    """y [N] fp32 = the reference's fused int4 GEMV of one x row (x [K], any float dtype)."""
    qw = np.ascontiguousarray(qweight, dtype=np.int32)
    sc = np.ascontiguousarray(scales).view(np.uint16)
    xv = np.ascontiguousarray(np.asarray(x, dtype=np.float32).reshape(-1))
    n, k = qw.shape[0], qw.shape[1] * 8
    y = np.empty(n, dtype=np.float32)
    lib().q4cpu_gemv(qw.ctypes.data, sc.ctypes.data, n, k, group, xv.ctypes.data, y.ctypes.data)
    return y


class DecodeModel:
    """Packed int4 weights of a Llama-shaped model (the reference's QLinear layout: qweight [N, K/8]
    int32, fp16 scales [N, K/G]; fused q|k|v and gate|up rows), fp16 KV caches and RoPE tables, with
    one decode step in the reference's order (scripts/llm/llama_q4.py:199-239)."""

    def __init__(self, cfg: dict, max_ctx: int, seed: int = 0, group: int = 128):
        self.cfg = cfg
        D, H, Hkv = cfg["hidden_size"], cfg["num_attention_heads"], cfg["num_key_value_heads"]
        hd = cfg.get("head_dim") or D // H
        I, V, nl = cfg["intermediate_size"], cfg["vocab_size"], cfg["num_hidden_layers"]
        self.D, self.H, self.Hkv, self.hd, self.I, self.V, self.nl, self.G = D, H, Hkv, hd, I, V, nl, group
        self.eps = cfg["rms_norm_eps"]
        rng = np.random.default_rng(seed)

        def q4(n, k):  # uniform nibbles 0..15 packed 8 per word, |N(0, 0.02)| scales
            qw = rng.integers(0, 2**32, size=(n, k // 8), dtype=np.uint32).view(np.int32)
            s = (np.abs(rng.standard_normal((n, k // group), dtype=np.float32)) * 0.02).astype(np.float16)
            return qw, s

        self.layers = [dict(wqkv=q4((H + 2 * Hkv) * hd, D), wo=q4(D, H * hd), wgu=q4(2 * I, D), wdown=q4(D, I),
                            ln_in=np.ones(D, np.float32), ln_post=np.ones(D, np.float32)) for _ in range(nl)]
        self.embed = q4(V, D)
        self.ln_f = np.ones(D, np.float32)
        self.cos, self.sin = O.rope_tables(cfg, max_ctx)
        self.kc = [rng.standard_normal((max_ctx, Hkv, hd), dtype=np.float32).astype(np.float16) for _ in range(nl)]
        self.vc = [rng.standard_normal((max_ctx, Hkv, hd), dtype=np.float32).astype(np.float16) for _ in range(nl)]

    def step(self, token: int, pos: int, L: int) -> int:
        """One decode token at position pos attending over cache[:L]; returns the greedy id."""
        D, H, Hkv, hd, I, G = self.D, self.H, self.Hkv, self.hd, self.I, self.G
        qw, s = self.embed
        h = O.embed_lookup(qw, s, G, np.array([token]))[0].astype(np.float32)
        cos, sin = self.cos[pos], self.sin[pos]
        for i, ly in enumerate(self.layers):
            x = O.rms_norm(h[None], ly["ln_in"], self.eps)[0]
            qkv = gemv(*ly["wqkv"], G, x)
            q = qkv[: H * hd].reshape(H, hd)
            k = qkv[H * hd:(H + Hkv) * hd].reshape(Hkv, hd)
            v = qkv[(H + Hkv) * hd:].reshape(Hkv, hd)
            q = (q * cos + O.rotate_half(q) * sin).astype(np.float32)
            k = (k * cos + O.rotate_half(k) * sin).astype(np.float32)
            self.kc[i][pos] = k.astype(np.float16)
            self.vc[i][pos] = v.astype(np.float16)
            o = O.attention(q[None], self.kc[i], self.vc[i], np.array([pos]), L, Hkv)[0]
            h = h + gemv(*ly["wo"], G, o)
            x = O.rms_norm(h[None], ly["ln_post"], self.eps)[0]
            gu = gemv(*ly["wgu"], G, x)
            h = h + gemv(*ly["wdown"], G, (O.silu(gu[:I]) * gu[I:]).astype(np.float32))
        x = O.rms_norm(h[None], self.ln_f, self.eps)[0]
        logits = gemv(*self.embed, G, x)
        return int(lib().q4cpu_argmax(logits.ctypes.data, logits.shape[0]))
