"""numpy restatement of the reference's int4 Llama path (TEST INFRASTRUCTURE: checker only).

Every function cites the reference lines it restates (paths relative to the reference project).
Arithmetic follows the reference: fp32 values, fp16 group scales, fp16 KV cache storage. Where the
reference leaves the summation order to PyTorch, this file accumulates in float64, which is closer
to the exact result than either reference form; parity tests use the reference's tolerance
(max|d| / max|ref| <= 1e-3) for such outputs and bit equality for integer work.
"""

from __future__ import annotations

import math

import numpy as np

F32 = np.float32


# --------------------------------------------------------------------------------------------
# int4 packing (scripts/llm/llama_q4.py:25-51)
# --------------------------------------------------------------------------------------------

def quantize_q4(w, group: int):
    """scripts/llm/llama_q4.py:25-38. w [N, K] float -> (qweight [N, K/8] int32, scales [N, K/G] fp16).

    scale = max(absmax(group), 1e-8) / 7 in fp32; q = clamp(round_half_even(w / scale), -8, 7) + 8;
    nibble b (bits 4b..4b+3) of word j holds k = 8j + b; the word is stored as two's-complement int32.
    """
    w = np.asarray(w, dtype=F32)
    n, k = w.shape
    if k % group or group % 8:
        raise AssertionError((n, k, group))
    wg = w.reshape(n, k // group, group)
    scale = np.maximum(np.abs(wg).max(-1, keepdims=True), F32(1e-8)) / F32(7.0)
    q = np.clip(np.rint(wg / scale), -8, 7).astype(np.int64) + 8
    q = q.reshape(n, k // 8, 8)
    packed = (q << (np.arange(8, dtype=np.int64) * 4)).sum(-1)
    packed = packed.astype(np.uint32).view(np.int32)
    return np.ascontiguousarray(packed), np.ascontiguousarray(scale.reshape(n, k // group).astype(np.float16))


def unpack_q4(qweight):
    """scripts/llm/llama_q4.py:41-45. [N, K/8] int32 -> [N, K] int32 nibbles in [0, 15]
    (arithmetic shift of the int32 word, then mask)."""
    qweight = np.asarray(qweight, dtype=np.int32)
    nibs = (qweight[..., None] >> (4 * np.arange(8, dtype=np.int32))) & 15
    return nibs.reshape(qweight.shape[0], -1).astype(np.int32)


def dequantize_q4(qweight, scales, group: int):
    """scripts/llm/llama_q4.py:48-51. W[n, k] = (nib - 8) * float(scales[n, k // G]) in fp32 (exact)."""
    q = unpack_q4(qweight).astype(F32) - F32(8)
    n, k = q.shape
    s = np.asarray(scales, dtype=np.float16).astype(F32)
    return (q.reshape(n, k // group, group) * s[..., None]).reshape(n, k)


def pack_nibbles(nibs):
    """Inverse of unpack_q4 for arbitrary nibbles 0..15 (used to build synthetic weights with the
    full nibble range, which quantize_q4 itself never emits for 0)."""
    nibs = np.asarray(nibs, dtype=np.int64)
    n, k = nibs.shape
    packed = (nibs.reshape(n, k // 8, 8) << (np.arange(8, dtype=np.int64) * 4)).sum(-1)
    return np.ascontiguousarray(packed.astype(np.uint32).view(np.int32))


# --------------------------------------------------------------------------------------------
# quantised linear (scripts/llm/llama_q4.py:60-90)
# --------------------------------------------------------------------------------------------

def q4_linear(qweight, scales, group: int, x):
    """scripts/llm/llama_q4.py:69-72 and :74-90. y[m, n] = sum_k x[m, k] * W[n, k] with W from
    dequantize_q4. Both reference forms (fused GEMV and dequant + F.linear) compute this sum; they
    differ only in fp32 summation order. Accumulates in float64, returns float32 [M, N]."""
    W = dequantize_q4(qweight, scales, group).astype(np.float64)
    x = np.asarray(x, dtype=F32).astype(np.float64)
    return (x @ W.T).astype(F32)


def q4_linear_fused_f32(qweight, scales, group: int, x):
    """scripts/llm/llama_q4.py:74-90, term by term in fp32 (M = 1): each term is
    x[g, 8w+b] * (((q >> 4b) & 15) - 8) * s[n, g]; the terms are summed over b, then over (g, w)."""
    qweight = np.asarray(qweight, dtype=np.int32)
    n, kw = qweight.shape
    k = kw * 8
    kg, wpg = k // group, group // 8
    q = qweight.reshape(n, kg, wpg)
    x4 = np.asarray(x, dtype=F32).reshape(kg, wpg, 8)
    s = np.asarray(scales, dtype=np.float16).astype(F32)[:, :, None]
    acc = None
    for b in range(8):
        term = x4[:, :, b] * ((((q >> (4 * b)) & 15).astype(F32) - F32(8.0)) * s)
        acc = term if acc is None else acc + term
    return acc.sum(axis=(1, 2), dtype=F32).reshape(1, n)


def rel_err(out, ref):
    """max|out - ref| / max|ref| (the metric of gemm/harness/vk_gemm_bench.c:411-422); NaN -> inf."""
    out = np.asarray(out, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    d = np.abs(out - ref)
    if not np.all(np.isfinite(d)):
        return math.inf
    return float(d.max() / max(np.abs(ref).max(), 1e-6)) if d.size else 0.0


def op_tol(ref):
    """scripts/debug/op_test.py:75: absolute tolerance 1e-3 * max(1, |ref|max)."""
    ref = np.asarray(ref, dtype=np.float64)
    return 1e-3 * max(1.0, float(np.abs(ref).max()) if ref.size else 1.0)


# --------------------------------------------------------------------------------------------
# tied int4 embedding / lm_head (scripts/llm/llama_q4.py:93-122)
# --------------------------------------------------------------------------------------------

def embed_lookup(qweight, scales, group: int, tokens):
    """scripts/llm/llama_q4.py:106-119 over the concatenation of the vocab chunks: row `t` of the
    dequantised table for 0 <= t < vocab, a zero row otherwise (no chunk claims the token)."""
    tokens = np.asarray(tokens, dtype=np.int64)
    vocab, dim = qweight.shape[0], qweight.shape[1] * 8
    out = np.zeros((tokens.shape[0], dim), dtype=F32)
    valid = (tokens >= 0) & (tokens < vocab)
    if valid.any():
        rows = tokens[valid]
        out[valid] = dequantize_q4(qweight[rows], scales[rows], group)
    return out


def embed_logits(qweight, scales, group: int, x):
    """scripts/llm/llama_q4.py:121-122: concatenation of the chunk QLinears = one q4_linear over the
    whole [vocab, dim] table (chunking splits rows; quantisation groups run along K)."""
    return q4_linear(qweight, scales, group, x)


# --------------------------------------------------------------------------------------------
# norm, rope, attention (scripts/llm/llama_q4.py:141-142, 184-239)
# --------------------------------------------------------------------------------------------

def rms_norm(x, w, eps):
    """scripts/llm/llama_q4.py:141-142: x * rsqrt(mean(x^2, -1) + eps) * w (fp32)."""
    x = np.asarray(x, dtype=F32)
    ms = (x.astype(np.float64) ** 2).mean(-1, keepdims=True)
    return (x * (F32(1.0) / np.sqrt(ms + eps)).astype(F32) * np.asarray(w, dtype=F32)).astype(F32)


def rope_inv_freq(cfg: dict):
    """Inverse frequencies of HF's LlamaRotaryEmbedding, which the reference uses for its tables
    (scripts/llm/llama_q4.py:184-192). Third-party algorithm (transformers, not pinned by the
    reference; this container has 5.5.0): default RoPE inv_freq = 1 / theta^(2i/d), and for
    rope_type "llama3" the published Llama 3.1 frequency smoothing (wavelengths above
    original_ctx / low_freq_factor are divided by `factor`, those below original_ctx /
    high_freq_factor are kept, the band between is interpolated linearly in 1/wavelength)."""
    hd = cfg.get("head_dim") or cfg["hidden_size"] // cfg["num_attention_heads"]
    rs = cfg.get("rope_scaling") or cfg.get("rope_parameters") or {}
    theta = cfg.get("rope_theta", rs.get("rope_theta", 10000.0))
    # theta ** e correctly rounded to fp32 (torch's fp32 pow agrees with it on these inputs;
    # numpy's fp32 pow differs by an ulp on some), then the fp32 reciprocal
    e = np.arange(0, hd, 2, dtype=np.int64).astype(F32) / F32(hd)
    inv = (F32(1.0) / (np.float64(theta) ** e.astype(np.float64)).astype(F32)).astype(F32)
    if rs.get("rope_type", rs.get("type", "default")) == "llama3":
        factor = rs["factor"]
        lo, hi = rs["low_freq_factor"], rs["high_freq_factor"]
        old = rs["original_max_position_embeddings"]
        lo_wl, hi_wl = old / lo, old / hi
        wavelen = (F32(2 * math.pi) / inv).astype(F32)
        inv_l = np.where(wavelen > lo_wl, inv / F32(factor), inv).astype(F32)
        smooth = ((F32(old) / wavelen - F32(lo)) / F32(hi - lo)).astype(F32)
        smoothed = ((F32(1) - smooth) * inv_l / F32(factor) + smooth * inv_l).astype(F32)
        medium = ~(wavelen < hi_wl) & ~(wavelen > lo_wl)
        inv = np.where(medium, smoothed, inv_l).astype(F32)
    return inv


def rope_tables(cfg: dict, max_ctx: int):
    """scripts/llm/llama_q4.py:184-192: cos, sin [max_ctx, head_dim] fp32 with
    freqs[p, i] = inv_freq[i] * p (fp32) and emb = cat(freqs, freqs)."""
    inv = rope_inv_freq(cfg)
    pos = np.arange(max_ctx, dtype=np.int64).astype(F32)
    freqs = (pos[:, None] * inv[None, :]).astype(F32)
    emb = np.concatenate([freqs, freqs], -1)
    return np.cos(emb).astype(F32), np.sin(emb).astype(F32)


def rotate_half(x):
    """scripts/llm/llama_q4.py:195-197: cat(-x[..., h:], x[..., :h])."""
    h = x.shape[-1] // 2
    return np.concatenate([-x[..., h:], x[..., :h]], -1)


def silu(x):
    x = np.asarray(x, dtype=np.float64)
    return (x / (1.0 + np.exp(-x))).astype(F32)


def attention(q, k_cache, v_cache, pos, L, n_kv):
    """scripts/llm/llama_q4.py:208-232: GQA over cache[:L] (fp16 storage read as fp32) with the
    causal mask key_pos <= pos (masked scores -1e30), softmax, p @ V. q [C, H, hd] fp32 ->
    o [C, H*hd] fp32. Query head h uses KV head h // (H / n_kv)."""
    C, H, hd = q.shape
    g = H // n_kv
    K = k_cache[:L].astype(np.float64)  # [L, kv, hd]
    V = v_cache[:L].astype(np.float64)
    key_pos = np.arange(L)
    mask = key_pos[None, :] <= np.asarray(pos)[:, None]  # [C, L]
    out = np.zeros((C, H, hd), dtype=np.float64)
    scale = 1.0 / math.sqrt(hd)
    for h in range(H):
        kv = h // g
        s = (q[:, h, :].astype(np.float64) @ K[:, kv, :].T) * scale  # [C, L]
        s = np.where(mask, s, -1e30)
        s = s - s.max(-1, keepdims=True)
        p = np.exp(s)
        p /= p.sum(-1, keepdims=True)
        out[:, h, :] = p @ V[:, kv, :]
    return out.reshape(C, H * hd).astype(F32)


# --------------------------------------------------------------------------------------------
# the model step (scripts/llm/llama_q4.py:145-243)
# --------------------------------------------------------------------------------------------

def group_for(k: int, group: int = 128) -> int:
    """Per-linear group rule used by the tiny BASELINE config: `group` where K % group == 0, else
    the largest power of two >= 8 dividing K (688 -> 16). Identity for every 3B projection."""
    if k % group == 0:
        return group
    g = 8
    while k % (g * 2) == 0 and g * 2 <= group:
        g *= 2
    if k % g:
        raise ValueError(f"K={k} is not a multiple of 8")
    return g


class OracleModel:
    """Packed weights of LlamaQ4 (scripts/llm/llama_q4.py:145-182) held as numpy arrays.

    layers[i] = dict(wqkv=(qw, s, G), wo=..., wgu=..., wdown=..., ln_in, ln_post) with the
    reference's fused row orders (q | k | v and gate | up, :149-152); embed = (qw, s, G)."""

    def __init__(self, cfg: dict, layers, embed, ln_f, max_ctx: int):
        self.cfg = cfg
        self.layers = layers
        self.embed = embed
        self.ln_f = np.asarray(ln_f, dtype=F32)
        self.max_ctx = max_ctx
        self.dim = cfg["hidden_size"]
        self.n_heads = cfg["num_attention_heads"]
        self.n_kv = cfg["num_key_value_heads"]
        self.head_dim = cfg.get("head_dim") or self.dim // self.n_heads
        self.inter = cfg["intermediate_size"]
        self.eps = cfg["rms_norm_eps"]
        self.cos, self.sin = rope_tables(cfg, max_ctx)

    @classmethod
    def from_state_dict(cls, cfg: dict, sd, max_ctx: int, group: int = 128):
        """Quantise an HF-named fp32 state dict like Layer / LlamaQ4.__init__
        (scripts/llm/llama_q4.py:145-182), with the per-linear group rule of group_for()."""
        def ql(w):
            w = np.asarray(w, dtype=F32)
            g = group_for(w.shape[1], group)
            qw, s = quantize_q4(w, g)
            return qw, s, g
        layers = []
        for i in range(cfg["num_hidden_layers"]):
            p = f"model.layers.{i}."
            layers.append(dict(
                wqkv=ql(np.concatenate([sd[p + "self_attn.q_proj.weight"], sd[p + "self_attn.k_proj.weight"],
                                        sd[p + "self_attn.v_proj.weight"]], 0)),
                wo=ql(sd[p + "self_attn.o_proj.weight"]),
                wgu=ql(np.concatenate([sd[p + "mlp.gate_proj.weight"], sd[p + "mlp.up_proj.weight"]], 0)),
                wdown=ql(sd[p + "mlp.down_proj.weight"]),
                ln_in=np.asarray(sd[p + "input_layernorm.weight"], dtype=F32),
                ln_post=np.asarray(sd[p + "post_attention_layernorm.weight"], dtype=F32)))
        return cls(cfg, layers, ql(sd["model.embed_tokens.weight"]), sd["model.norm.weight"], max_ctx)

    def new_caches(self):
        """scripts/llm/llama_q4.py:241-243: 2 * n_layers zeroed fp16 [max_ctx, n_kv, head_dim]."""
        return [np.zeros((self.max_ctx, self.n_kv, self.head_dim), dtype=np.float16)
                for _ in range(2 * len(self.layers))]

    def step(self, tokens, start: int, last: int, caches, L: int):
        """scripts/llm/llama_q4.py:199-239. tokens [C] ints; writes KV rows start..start+C-1 in
        place (fp16), attends over cache[:L] with the causal mask, returns (next id, logits [V])."""
        tokens = np.asarray(tokens, dtype=np.int64).reshape(-1)
        C = tokens.shape[0]
        pos = start + np.arange(C)
        H, Hkv, hd = self.n_heads, self.n_kv, self.head_dim
        qw, s, g = self.embed
        h = embed_lookup(qw, s, g, tokens)
        cos = self.cos[pos][:, None, :]
        sin = self.sin[pos][:, None, :]
        for i, ly in enumerate(self.layers):
            kc, vc = caches[2 * i], caches[2 * i + 1]
            x = rms_norm(h, ly["ln_in"], self.eps)
            qkv = q4_linear(*ly["wqkv"][:2], ly["wqkv"][2], x)
            q = qkv[:, : H * hd].reshape(C, H, hd)
            k = qkv[:, H * hd: (H + Hkv) * hd].reshape(C, Hkv, hd)
            v = qkv[:, (H + Hkv) * hd:].reshape(C, Hkv, hd)
            q = (q * cos + rotate_half(q) * sin).astype(F32)
            k = (k * cos + rotate_half(k) * sin).astype(F32)
            kc[pos] = k.astype(np.float16)
            vc[pos] = v.astype(np.float16)
            o = attention(q, kc, vc, pos, L, Hkv)
            h = (h + q4_linear(*ly["wo"][:2], ly["wo"][2], o)).astype(F32)
            x = rms_norm(h, ly["ln_post"], self.eps)
            gu = q4_linear(*ly["wgu"][:2], ly["wgu"][2], x)
            a = (silu(gu[:, : self.inter]) * gu[:, self.inter:]).astype(F32)
            h = (h + q4_linear(*ly["wdown"][:2], ly["wdown"][2], a)).astype(F32)
        x = rms_norm(h[[last]], self.ln_f, self.eps)
        logits = embed_logits(qw, s, g, x)[0]
        return int(np.argmax(logits)), logits


# --------------------------------------------------------------------------------------------
# scheduler (runner/llm_runner.c:143-246, scripts/llm/run_host.py:40-54)
# --------------------------------------------------------------------------------------------

class ScheduleError(ValueError):
    """Raised where runner/llm_runner.c returns OUT_OF_RANGE / INVALID_ARGUMENT."""


def pick_bucket(buckets, needed: int, use_max: bool) -> int:
    """runner/llm_runner.c:143-149: the largest bucket under --schedule max, else the smallest
    bucket >= needed, else -1."""
    if use_max:
        return buckets[-1]
    for b in buckets:
        if b >= needed:
            return b
    return -1


def check_request(n_prompt: int, max_new: int, chunk: int, max_ctx: int):
    """runner/llm_runner.c:168-173."""
    if n_prompt == 0:
        raise ScheduleError("empty prompt")
    if n_prompt + max_new > max_ctx or -(-n_prompt // chunk) * chunk > max_ctx:
        raise ScheduleError(f"prompt {n_prompt} + new {max_new} exceeds max_ctx {max_ctx}")


def used_functions(n_prompt, max_new, chunk, buckets, use_max):
    """runner/llm_runner.c:181-189: (prefill buckets, decode buckets) the schedule will call."""
    pre = sorted({pick_bucket(buckets, s + chunk, use_max) for s in range(0, n_prompt, chunk)})
    dec = sorted({pick_bucket(buckets, p + 1, use_max) for p in range(n_prompt, n_prompt + max_new - 1)})
    return pre, dec


def generate(step, prompt, max_new: int, chunk: int, buckets, schedule="bucketed", stop_ids=(),
             max_ctx: int = 4096):
    """runner/llm_runner.c:205-246. `step(tokens[C], start, last, L) -> next id`.

    Prefill: chunks at start = 0, C, 2C, ... zero-padded to C, L = pick_bucket(start + C),
    last = n - 1 within the chunk. Decode: while fewer than max_new tokens (the prefill token
    counts): stop if the last token is a stop id; L = pick_bucket(pos + 1) (stop when none);
    step(next, pos, 0). Returns (tokens, prefill_buckets, decode_buckets)."""
    use_max = schedule == "max"
    n = len(prompt)
    check_request(n, max_new, chunk, max_ctx)
    nxt, chunks = None, []
    for s in range(0, n, chunk):
        m = min(chunk, n - s)
        buf = np.zeros(chunk, dtype=np.int64)
        buf[:m] = prompt[s: s + m]
        L = pick_bucket(buckets, s + chunk, use_max)
        if L < 0:
            raise ScheduleError(f"no bucket >= {s + chunk}")
        nxt = step(buf, s, m - 1, L)
        chunks.append(L)
    out, steps, pos = [nxt], [], n
    while len(out) < max_new:
        if nxt in stop_ids:
            break
        L = pick_bucket(buckets, pos + 1, use_max)
        if L < 0:
            break
        nxt = step(np.array([nxt]), pos, 0, L)
        steps.append(L)
        out.append(nxt)
        pos += 1
    return out, chunks, steps


# --------------------------------------------------------------------------------------------
# fp16 GEMM shape -> result interface (gemm/shapes.py:14-66)
# --------------------------------------------------------------------------------------------

GEMM_TOL = 5e-3  # gemm/shapes.py:53


def gemm_make_data(M, N, K, la="N", lb="N", seed=0):
    """gemm/shapes.py:56-66: A, B ~ U(-1, 1) rounded to fp16 (logical [M, K] and [K, N]);
    Cref = A.f32 @ B.f32 (here in float64 then rounded to fp32). Returns (A_stored, B_stored, Cref)
    with the stored layouts of the BLAS letters (T = stored transposed)."""
    rng = np.random.default_rng(seed)
    a = rng.uniform(-1, 1, (M, K)).astype(np.float16)
    b = rng.uniform(-1, 1, (K, N)).astype(np.float16)
    c = (a.astype(np.float64) @ b.astype(np.float64)).astype(F32)
    a_st = a if la == "N" else np.ascontiguousarray(a.T)
    b_st = b if lb == "N" else np.ascontiguousarray(b.T)
    return a_st, b_st, c
