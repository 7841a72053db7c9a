"""Drop-in LlamaQ4 (scripts/llm/llama_q4.py:145-257) whose step runs in libq4b.so.

Same constructor (model_dir, group, max_ctx, vocab_chunk, n_layers, sd, cfg), same attributes
(layers[i].wqkv / wo / wgu / wdown as QLinear, ln_in, ln_post, embed as QEmbedding, ln_f, cos, sin),
same ``step(tokens, start, last, caches, L) -> (next int32 [1], logits fp32 [1, V])`` and
``new_caches()``. Weights are quantised on the GPU (bit-exact with quantize_q4). Extra keyword
arguments: ``per_linear_group`` (use group_for(K, group) where K is not a multiple of group),
``tp_rank`` / ``tp_size`` (hold only this rank's tensor-parallel shard), ``device``.
"""

from __future__ import annotations

import ctypes
import json
import pathlib
import zlib

import torch
from torch import nn

from . import _lib
from .qlinear import QEmbedding, QLinear


def group_for(k: int, group: int) -> int:
    """`group` where K % group == 0, else the largest power of two >= 8 dividing K (688 -> 16)."""
    if k % group == 0:
        return group
    g = 8
    while k % (g * 2) == 0 and g * 2 <= group:
        g *= 2
    if k % g:
        raise ValueError(f"K={k} is not a multiple of 8")
    return g


def rope_tables(cfg: dict, max_ctx: int):
    """cos, sin [max_ctx, head_dim] fp32 from HF's LlamaRotaryEmbedding, as the reference computes
    them (scripts/llm/llama_q4.py:184-192); built once on the host at construction."""
    from transformers import LlamaConfig
    from transformers.models.llama.modeling_llama import LlamaRotaryEmbedding
    rot = LlamaRotaryEmbedding(LlamaConfig(**cfg))
    pos = torch.arange(max_ctx)[None]
    cos, sin = rot(torch.zeros(1, dtype=torch.float32), pos)
    return cos[0].float(), sin[0].float()


class LazySafetensors:
    """scripts/llm/llama_q4.py:125-138: dict-like view over HF safetensors shards, read per tensor."""

    def __init__(self, model_dir: pathlib.Path):
        from safetensors import safe_open
        self.handles = [safe_open(str(f), "pt") for f in sorted(model_dir.glob("*.safetensors"))]
        self.where = {k: h for h in self.handles for k in h.keys()}

    def __getitem__(self, k):
        return self.where[k].get_tensor(k)

    def __contains__(self, k):
        return k in self.where


_MASK32 = 0xFFFFFFFF


def _mul32(x, c: int):
    """(x * c) mod 2^32 for int64 tensors x in [0, 2^32), without any int64 product above 2^49."""
    return (x * (c & 0xFFFF) + (((x * (c >> 16)) & 0xFFFF) << 16)) & _MASK32


def hash_normal(key: int, n: int, std: float, device, chunk: int = 1 << 26):
    """n seeded values with mean 0 and standard deviation `std`, identical bit for bit on any device.

    Element i hashes the 32-bit counter (i * 0x9E3779B1 + key) with an integer avalanche mix
    (xorshift-multiply rounds, constants 0x7feb352d and 0x846ca68b); the sum of the hash's four bytes
    is an Irwin-Hall(4) variate on 0..1020 (mean 510, variance 4 (256^2 - 1) / 12), which one fp32
    multiply scales to the requested deviation. Integer arithmetic and one correctly rounded fp32
    multiply give the same bits on a CPU and a GPU, so a checker on the host regenerates exactly the
    weights a GPU run used."""
    import math
    out = torch.empty(n, dtype=torch.float32, device=device)
    scale = torch.tensor(std / math.sqrt(4 * (256 * 256 - 1) / 12.0), dtype=torch.float32, device=device)
    for s in range(0, n, chunk):
        e = min(n, s + chunk)
        x = torch.arange(s, e, dtype=torch.int64, device=device)
        x = (x * 0x9E3779B1 + (key & _MASK32)) & _MASK32
        x = x ^ (x >> 16)
        x = _mul32(x, 0x7FEB352D)
        x = x ^ (x >> 15)
        x = _mul32(x, 0x846CA68B)
        x = x ^ (x >> 16)
        b = (x & 255) + ((x >> 8) & 255) + ((x >> 16) & 255) + (x >> 24)
        out[s:e] = (b - 510).to(torch.float32) * scale
    return out


class SyntheticStateDict:
    """Seeded random-init Llama weights generated per tensor name (HF init: mean 0, deviation
    `initializer_range` for projections and the embedding, ones for the norms), so a 3B-shaped model
    never exists in fp32 all at once. The values come from hash_normal, so the same (cfg, seed) gives
    the same weights on the GPU and on the host (where the reference's own code can be run on them)."""

    def __init__(self, cfg: dict, seed: int = 0, std: float | None = None, device="cuda"):
        self.cfg, self.seed, self.device = cfg, seed, torch.device(device)
        self.std = cfg.get("initializer_range", 0.02) if std is None else std

    def _shape(self, k):
        c = self.cfg
        D, H, Hkv = c["hidden_size"], c["num_attention_heads"], c["num_key_value_heads"]
        hd = c.get("head_dim") or D // H
        I, V = c["intermediate_size"], c["vocab_size"]
        if k == "model.embed_tokens.weight":
            return (V, D)
        if k.endswith("norm.weight") or k.endswith("layernorm.weight"):
            return (D,)
        tail = {"self_attn.q_proj.weight": (H * hd, D), "self_attn.k_proj.weight": (Hkv * hd, D),
                "self_attn.v_proj.weight": (Hkv * hd, D), "self_attn.o_proj.weight": (D, H * hd),
                "mlp.gate_proj.weight": (I, D), "mlp.up_proj.weight": (I, D), "mlp.down_proj.weight": (D, I)}
        for t, shp in tail.items():
            if k.endswith(t):
                return shp
        raise KeyError(k)

    def __getitem__(self, k):
        shp = self._shape(k)
        if len(shp) == 1:
            return torch.ones(shp, device=self.device)
        key = (zlib.crc32(k.encode()) ^ (self.seed * 0x85EBCA6B)) & _MASK32
        return hash_normal(key, shp[0] * shp[1], self.std, self.device).reshape(shp)

    def __contains__(self, k):
        try:
            self._shape(k)
            return True
        except KeyError:
            return False


def shard_layer(cfg: dict, get, rank: int = 0, world: int = 1):
    """Tensor-parallel shard of one layer's fp32 weights (scripts/llm/llama_q4.py:149-153 fused row
    orders kept per rank). get(name) returns the full HF tensor "model.layers.i.<name>".
      wqkv  rows q heads [rH/t, (r+1)H/t) | k heads [rHkv/t, ..) | v heads [rHkv/t, ..)  (column split)
      wgu   rows gate [rI/t, (r+1)I/t) | up [rI/t, (r+1)I/t)                            (column split)
      wo    columns of this rank's q heads; wdown columns [rI/t, (r+1)I/t)                (row split:
            the partial outputs are summed across ranks)
    Pure torch on whatever device get() returns."""
    D, H, Hkv = cfg["hidden_size"], cfg["num_attention_heads"], cfg["num_key_value_heads"]
    hd = cfg.get("head_dim") or D // H
    I = cfg["intermediate_size"]
    r, t = rank, world
    if H % t or Hkv % t or I % t:
        raise ValueError(f"heads {H}, KV heads {Hkv} and intermediate {I} must divide by {t}")

    def rows(w, n):
        return w[r * n:(r + 1) * n]

    wqkv = torch.cat([rows(get("self_attn.q_proj.weight"), H // t * hd), rows(get("self_attn.k_proj.weight"),
                      Hkv // t * hd), rows(get("self_attn.v_proj.weight"), Hkv // t * hd)], 0)
    wo = get("self_attn.o_proj.weight")[:, r * (H // t) * hd:(r + 1) * (H // t) * hd].contiguous()
    wgu = torch.cat([rows(get("mlp.gate_proj.weight"), I // t), rows(get("mlp.up_proj.weight"), I // t)], 0)
    wdown = get("mlp.down_proj.weight")[:, r * (I // t):(r + 1) * (I // t)].contiguous()
    return dict(wqkv=wqkv, wo=wo, wgu=wgu, wdown=wdown)


class Layer(nn.Module):
    """scripts/llm/llama_q4.py:145-155 (fused q|k|v and gate|up), optionally one TP shard."""

    def __init__(self, cfg, sd, i, group, per_linear_group=False, tp_rank=0, tp_size=1, device="cuda"):
        super().__init__()
        p = f"model.layers.{i}."

        def g(k):
            return group_for(k, group) if per_linear_group else group

        def get(name):
            return sd[p + name].to(device)

        w = shard_layer(cfg, get, tp_rank, tp_size)
        for name in ("wqkv", "wo", "wgu", "wdown"):
            if w[name].shape[1] % g(w[name].shape[1]):
                raise ValueError(f"{name}: shard K={w[name].shape[1]} is not a multiple of its group")
            setattr(self, name, QLinear(w[name], g(w[name].shape[1])))
        self.ln_in = nn.Parameter(get("input_layernorm.weight").float().contiguous(), requires_grad=False)
        self.ln_post = nn.Parameter(get("post_attention_layernorm.weight").float().contiguous(), requires_grad=False)


class LlamaQ4(nn.Module):
    """scripts/llm/llama_q4.py:158-243 on B200."""

    def __init__(self, model_dir=None, group=32, max_ctx=4096, vocab_chunk=32064, n_layers=None, sd=None, cfg=None,
                 *, per_linear_group=False, tp_rank=0, tp_size=1, device="cuda", max_chunk=128, _skip_init=False):
        super().__init__()
        if _skip_init:
            return
        model_dir = pathlib.Path(model_dir) if model_dir else None
        cfg = cfg or json.loads((model_dir / "config.json").read_text())
        if sd is None:
            sd = LazySafetensors(model_dir)
        self._setup_cfg(cfg, n_layers, max_ctx, group, vocab_chunk, tp_rank, tp_size, device, max_chunk)
        emb = sd["model.embed_tokens.weight"].to(self.device)
        ge = group_for(self.dim, group) if per_linear_group else group
        self.embed = QEmbedding(emb, ge, vocab_chunk, device=self.device)
        del emb
        if not cfg.get("tie_word_embeddings", False):
            raise NotImplementedError("untied lm_head")
        self.layers = nn.ModuleList(Layer(cfg, sd, i, group, per_linear_group, tp_rank, tp_size, self.device)
                                    for i in range(self.n_layers))
        self.ln_f = nn.Parameter(sd["model.norm.weight"].to(self.device).float().contiguous(), requires_grad=False)
        self._setup_rope()

    def _setup_cfg(self, cfg, n_layers, max_ctx, group, vocab_chunk, tp_rank, tp_size, device, max_chunk):
        self.cfg = cfg
        self.n_layers = n_layers or cfg["num_hidden_layers"]
        self.dim = cfg["hidden_size"]
        self.n_heads = cfg["num_attention_heads"]
        self.n_kv = cfg["num_key_value_heads"]
        self.head_dim = cfg.get("head_dim") or self.dim // self.n_heads
        self.inter = cfg["intermediate_size"]
        self.eps = cfg["rms_norm_eps"]
        self.vocab = cfg["vocab_size"]
        self.max_ctx = max_ctx
        self.group = group
        self.vocab_chunk = vocab_chunk
        self.tp_rank, self.tp_size = tp_rank, tp_size
        self.device = torch.device(device)
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.max_chunk = max_chunk
        self._handle = None
        self._bound = None

    def _setup_rope(self):
        cos, sin = rope_tables(self.cfg, self.max_ctx)
        self.register_buffer("cos", cos.to(self.device).contiguous(), persistent=False)
        self.register_buffer("sin", sin.to(self.device).contiguous(), persistent=False)

    @classmethod
    def from_packed(cls, cfg: dict, packed: dict, max_ctx: int, vocab_chunk: int = 32064, device="cuda",
                    max_chunk=128):
        """Build from already-quantised weights (the layout of the reference's QLinear attributes):
        packed[f"l{i}_{name}_qweight"/"_scales"/"_group"], "l{i}_ln_in", "l{i}_ln_post",
        "embed_qweight", "embed_scales", "embed_group", "ln_f"."""
        self = cls(_skip_init=True)
        self._setup_cfg(cfg, None, max_ctx, int(packed["embed_group"]), vocab_chunk, 0, 1, device, max_chunk)
        t = lambda a: torch.as_tensor(a).to(self.device)  # noqa: E731
        self.embed = QEmbedding.from_packed(t(packed["embed_qweight"]), t(packed["embed_scales"]),
                                            int(packed["embed_group"]), vocab_chunk)
        layers = []
        for i in range(self.n_layers):
            ly = nn.Module()
            for nm in ("wqkv", "wo", "wgu", "wdown"):
                setattr(ly, nm, QLinear.from_packed(t(packed[f"l{i}_{nm}_qweight"]), t(packed[f"l{i}_{nm}_scales"]),
                                                    int(packed[f"l{i}_{nm}_group"])))
            ly.ln_in = nn.Parameter(t(packed[f"l{i}_ln_in"]).float().contiguous(), requires_grad=False)
            ly.ln_post = nn.Parameter(t(packed[f"l{i}_ln_post"]).float().contiguous(), requires_grad=False)
            layers.append(ly)
        self.layers = nn.ModuleList(layers)
        self.ln_f = nn.Parameter(t(packed["ln_f"]).float().contiguous(), requires_grad=False)
        self._setup_rope()
        return self

    # ---- the native model object ------------------------------------------------------------

    @staticmethod
    def _qmat(ql):
        return _lib.QMat(ql.qweight.data_ptr(), ql.scales.data_ptr(), ql.qweight.shape[0], ql.qweight.shape[1] * 8,
                         ql.group)

    def native(self):
        """The q4b_model handle (created on first use on this model's device)."""
        if self._handle is None:
            L = _lib.lib()
            c = _lib.ModelCfg(self.n_layers, self.dim, self.n_heads, self.n_kv, self.head_dim, self.inter, self.vocab,
                              self.eps, self.max_ctx, self.max_chunk, self.tp_rank, self.tp_size)
            h = ctypes.c_void_p()
            with torch.cuda.device(self.device):
                _lib.check(L.q4b_model_create(ctypes.byref(c), ctypes.byref(h)), "model_create")
            self._handle = h
            head = self._qmat(self.embed)
            _lib.check(L.q4b_model_set_head(h, ctypes.byref(head), self.ln_f.data_ptr(), self.cos.data_ptr(),
                                            self.sin.data_ptr()), "model_set_head")
        return self._handle

    def decode_trace(self, on: bool = True):
        """Turn the persistent decode step's phase trace on (returns the int64 device buffer the
        steps fill: [CTAs, 15 * n_layers + 4] %globaltimer stamps, layout of q4b_model_set_trace) or
        off (returns None)."""
        L = _lib.lib()
        h = self.native()
        if not on:
            _lib.check(L.q4b_model_set_trace(h, None, 0), "model_set_trace")
            self._trace = None
            return None
        with torch.cuda.device(self.device):
            n = int(L.q4b_model_trace_events(h))
        stride = 15 * self.n_layers + 4
        buf = torch.zeros(n // stride, stride, dtype=torch.int64, device=self.device)
        _lib.check(L.q4b_model_set_trace(h, buf.data_ptr(), n), "model_set_trace")
        self._trace = buf  # held while the native model may write it
        return buf

    def attach_tp(self, dist_mod=None):
        """Join this model's NCCL communicator (tp_size ranks, one process per GPU): rank 0 makes
        the id and torch.distributed broadcasts it. Collective: every rank calls it."""
        import torch.distributed as dist
        dist_mod = dist_mod or dist
        L = _lib.lib()
        h = self.native()
        uid = (ctypes.c_ubyte * 128)()
        if self.tp_rank == 0:
            _lib.check(L.q4b_tp_unique_id(uid, 128), "tp_unique_id")
        obj = [bytes(uid)]
        dist_mod.broadcast_object_list(obj, src=0)
        uid = (ctypes.c_ubyte * 128).from_buffer_copy(obj[0])
        with torch.cuda.device(self.device):
            _lib.check(L.q4b_model_attach_tp(h, uid, 128), "model_attach_tp")

    def bind_caches(self, caches):
        """Point the native layers at these cache tensors (k0, v0, k1, v1, ...)."""
        key = tuple(c.data_ptr() for c in caches)
        if self._bound == key:
            return
        if len(caches) != 2 * self.n_layers:
            raise ValueError(f"need {2 * self.n_layers} caches")
        L = _lib.lib()
        h = self.native()
        for i, ly in enumerate(self.layers):
            kc, vc = caches[2 * i], caches[2 * i + 1]
            for c in (kc, vc):
                if not (c.is_cuda and c.dtype == torch.float16 and c.is_contiguous()
                        and tuple(c.shape) == (self.max_ctx, self.n_kv // self.tp_size, self.head_dim)):
                    raise ValueError("caches must be contiguous fp16 CUDA tensors [max_ctx, n_kv/tp, head_dim]")
            w = _lib.LayerWeights(self._qmat(ly.wqkv), self._qmat(ly.wo), self._qmat(ly.wgu), self._qmat(ly.wdown),
                                  ly.ln_in.data_ptr(), ly.ln_post.data_ptr(), kc.data_ptr(), vc.data_ptr())
            _lib.check(L.q4b_model_set_layer(h, i, ctypes.byref(w)), "model_set_layer")
        self._bound = key

    def new_caches(self):
        """scripts/llm/llama_q4.py:241-243 (on the GPU; this rank's KV heads under TP)."""
        return [torch.zeros(self.max_ctx, self.n_kv // self.tp_size, self.head_dim, dtype=torch.float16,
                            device=self.device) for _ in range(2 * self.n_layers)]

    def step(self, tokens, start, last, caches, L):
        """scripts/llm/llama_q4.py:199-239: tokens [1, C] int32, start [1], last [1]; writes KV for
        positions start..start+C-1 into `caches`, attends over cache[:L]; returns (next [1] int32,
        logits [1, V] fp32), both on the GPU."""
        toks = torch.as_tensor(tokens).reshape(-1).to(device=self.device, dtype=torch.int32).contiguous()
        s, l = int(torch.as_tensor(start).reshape(-1)[0]), int(torch.as_tensor(last).reshape(-1)[0])
        self.bind_caches(caches)
        nxt = torch.empty(1, dtype=torch.int32, device=self.device)
        logits = torch.empty(1, self.vocab // self.tp_size, dtype=torch.float32, device=self.device)
        with torch.cuda.device(self.device):
            st = torch.cuda.current_stream().cuda_stream
            _lib.check(_lib.lib().q4b_model_step(self.native(), toks.data_ptr(), toks.numel(), s, l, int(L),
                                                 nxt.data_ptr(), logits.data_ptr(), st), "model_step")
        return nxt, logits

    def __del__(self):
        h = getattr(self, "_handle", None)
        if h is not None:
            try:
                _lib.lib().q4b_model_destroy(h)
            except Exception:
                pass


class StepFn(nn.Module):
    """scripts/llm/llama_q4.py:246-257: fixed-bucket wrapper returning the next id (or logits)."""

    def __init__(self, model, L, return_logits=False):
        super().__init__()
        self.model = model
        self.L = L
        self.return_logits = return_logits

    def forward(self, tokens, start, last, *caches):
        nxt, logits = self.model.step(tokens, start, last, caches, self.L)
        return logits if self.return_logits else nxt

