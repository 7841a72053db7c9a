"""torch-tensor wrappers over the C ABI. Every op runs on CUDA tensors on the current stream and
calls libq4b.so; there is no CPU implementation here."""

from __future__ import annotations

import torch

from ._lib import EPI_ACCUMULATE, EPI_STORE, EPI_SWIGLU, F16, F32, GemmCfg, LinearCfg, Q4B_EINVAL as _lib_EINVAL, Q4BError, check, lib

_DT = {torch.float32: F32, torch.float16: F16}


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _need_cuda(*ts):
    for t in ts:
        if not t.is_cuda:
            raise ValueError("q4b ops take CUDA tensors (there is no CPU path)")
        if not t.is_contiguous():
            raise ValueError("q4b ops take contiguous tensors")


def quantize_q4(w: torch.Tensor, group: int):
    """scripts/llm/llama_q4.py:25-38 on the GPU, bit-exact: w [N, K] -> (qweight int32 [N, K/8],
    scales fp16 [N, K/G]). CPU inputs are copied to the current CUDA device first."""
    w = w.detach()
    if not w.is_cuda:
        w = w.to("cuda")
    w = w.float().contiguous()
    n, k = w.shape
    qw = torch.empty(n, k // 8, dtype=torch.int32, device=w.device)
    sc = torch.empty(n, k // group if group else 0, dtype=torch.float16, device=w.device)
    check(lib().q4b_quantize_q4(w.data_ptr(), n, k, group, qw.data_ptr(), sc.data_ptr(), _stream()), "quantize_q4")
    return qw, sc


def unpack_q4(qweight: torch.Tensor):
    """scripts/llm/llama_q4.py:41-45: [N, K/8] int32 -> [N, K] nibbles (uint8 here; the reference
    returns int64 of the same values)."""
    _need_cuda(qweight)
    n, kw = qweight.shape
    out = torch.empty(n, kw * 8, dtype=torch.uint8, device=qweight.device)
    check(lib().q4b_unpack_q4(qweight.data_ptr(), n, kw * 8, out.data_ptr(), _stream()), "unpack_q4")
    return out


def dequantize_q4(qweight: torch.Tensor, scales: torch.Tensor, group: int, dtype=torch.float32):
    """scripts/llm/llama_q4.py:48-51 (exact in fp32)."""
    _need_cuda(qweight, scales)
    n, kw = qweight.shape
    out = torch.empty(n, kw * 8, dtype=dtype, device=qweight.device)
    check(lib().q4b_dequantize_q4(qweight.data_ptr(), scales.data_ptr(), n, kw * 8, group, out.data_ptr(),
                                  _DT[dtype], _stream()), "dequantize_q4")
    return out


class _Workspace:
    """Split-K workspace per (device, stream): zero-filled at allocation; every call leaves its
    counters at zero, and calls on one stream are ordered, so one buffer serves them all."""

    def __init__(self):
        self.bufs = {}

    def get(self, nbytes: int, device: torch.device):
        if nbytes == 0:
            return None
        key = (device.index, torch.cuda.current_stream(device).cuda_stream)
        buf = self.bufs.get(key)
        if buf is None or buf.numel() < nbytes:
            buf = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
            self.bufs[key] = buf
        return buf


WORKSPACE = _Workspace()


def _cfg(cfg):
    if cfg is None:
        return None
    if isinstance(cfg, LinearCfg):
        return cfg
    return LinearCfg(**cfg)


def gemm_f16(a: torch.Tensor, b: torch.Tensor, la: str = "N", lb: str = "N", *, out=None, cfg=None):
    """C = op(A) @ op(B) in fp16 with fp32 accumulation (gemm/shapes.py:1-6, 56-66).

    ``a`` and ``b`` are the STORED fp16 matrices: la "N" -> a is [M, K], "T" -> a is [K, M];
    lb "N" -> b is [K, N], "T" -> b is [N, K] (a torch Linear weight). Returns C [M, N] fp16."""
    _need_cuda(a, b)
    if a.dtype != torch.float16 or b.dtype != torch.float16:
        raise ValueError("gemm_f16 takes fp16 A and B")
    if la not in ("N", "T") or lb not in ("N", "T"):
        raise ValueError("layouts are 'N' or 'T'")
    if a.dim() != 2 or b.dim() != 2 or not a.is_contiguous() or not b.is_contiguous():
        raise ValueError("A and B must be contiguous 2-D tensors")
    m, k = a.shape if la == "N" else (a.shape[1], a.shape[0])
    kb, n = b.shape if lb == "N" else (b.shape[1], b.shape[0])
    if k != kb:
        raise ValueError(f"op(A) has K={k}, op(B) has K={kb}")
    if out is None:
        out = torch.empty(m, n, dtype=torch.float16, device=a.device)
    elif tuple(out.shape) != (m, n) or out.dtype != torch.float16 or not out.is_contiguous():
        raise ValueError(f"out must be a contiguous fp16 [{m}, {n}] tensor")
    c = None if cfg is None else (cfg if isinstance(cfg, GemmCfg) else GemmCfg(**cfg))
    cp = None if c is None else ctypes_byref(c)
    L = lib()
    wsb = L.q4b_gemm_f16_workspace(m, n, k, la.encode(), lb.encode(), cp)
    if wsb < 0:
        raise Q4BError(_lib_EINVAL, "gemm_f16: " + L.q4b_last_error().decode(errors="replace"))
    ws = WORKSPACE.get(wsb, a.device)
    check(L.q4b_gemm_f16(a.data_ptr(), b.data_ptr(), out.data_ptr(), m, n, k, la.encode(), lb.encode(), cp,
                         0 if ws is None else ws.data_ptr(), 0 if ws is None else ws.numel(), _stream()),
          "gemm_f16")
    return out


def q4_linear(x: torch.Tensor, qweight: torch.Tensor, scales: torch.Tensor, group: int, *, out=None,
              epilogue: str = "store", out_dtype=None, cfg=None):
    """QLinear.forward (scripts/llm/llama_q4.py:69-90) as one CUDA call.

    x [M, K] fp16 or fp32 -> y [M, N] (``epilogue="swiglu"``: [M, N/2] = silu(gate) * up with
    gate rows first, ``"accumulate"``: out += x W^T). The output dtype defaults to x's dtype."""
    _need_cuda(x, qweight, scales)
    if x.dim() != 2:
        raise ValueError("x must be [M, K]")
    m, k = x.shape
    n = qweight.shape[0]
    if qweight.shape[1] * 8 != k:
        raise ValueError(f"x has K={k}, qweight has K={qweight.shape[1] * 8}")
    epi = {"store": EPI_STORE, "accumulate": EPI_ACCUMULATE, "swiglu": EPI_SWIGLU}[epilogue]
    n_out = n // 2 if epi == EPI_SWIGLU else n
    if out is None:
        if epi == EPI_ACCUMULATE:
            raise ValueError("accumulate needs out=")
        out = torch.empty(m, n_out, dtype=out_dtype or x.dtype, device=x.device)
    else:
        _need_cuda(out)
        if tuple(out.shape) != (m, n_out):
            raise ValueError(f"out must be [{m}, {n_out}]")
    c = _cfg(cfg)
    cp = None if c is None else ctypes_byref(c)
    L = lib()
    wsb = L.q4b_q4_linear_workspace(m, n, k, group, epi, cp)
    ws = WORKSPACE.get(wsb, x.device)
    check(L.q4b_q4_linear(qweight.data_ptr(), scales.data_ptr(), group, x.data_ptr(), _DT[x.dtype], out.data_ptr(),
                          _DT[out.dtype], m, n, k, epi, cp, 0 if ws is None else ws.data_ptr(),
                          0 if ws is None else ws.numel(), _stream()), "q4_linear")
    return out


def ctypes_byref(c):
    import ctypes
    return ctypes.byref(c)


def embed_lookup(tokens: torch.Tensor, qweight: torch.Tensor, scales: torch.Tensor, group: int):
    """QEmbedding.lookup (scripts/llm/llama_q4.py:106-119): [C] ids -> [C, dim] fp32 rows (zeros
    for ids outside the vocabulary)."""
    _need_cuda(qweight, scales)
    toks = tokens.reshape(-1).to(device=qweight.device, dtype=torch.int32).contiguous()
    vocab, dim = qweight.shape[0], qweight.shape[1] * 8
    out = torch.empty(toks.numel(), dim, dtype=torch.float32, device=qweight.device)
    check(lib().q4b_embed_q4_lookup(toks.data_ptr(), toks.numel(), qweight.data_ptr(), scales.data_ptr(), vocab, dim,
                                    group, out.data_ptr(), _stream()), "embed_q4_lookup")
    return out


def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float):
    """rms_norm (scripts/llm/llama_q4.py:141-142) on fp32 [rows, dim]."""
    _need_cuda(x, weight)
    x2 = x.reshape(-1, x.shape[-1]).float().contiguous()
    out = torch.empty_like(x2)
    check(lib().q4b_rmsnorm(x2.data_ptr(), weight.float().contiguous().data_ptr(), eps, x2.shape[0], x2.shape[1],
                            out.data_ptr(), _stream()), "rmsnorm")
    return out.reshape(x.shape)


_ATTN_WS = {}


def attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, start, L: int):
    """Bucketed GQA attention (scripts/llm/llama_q4.py:208-232): q [C, H, hd] fp32 (RoPE applied),
    caches fp16 [max_ctx, Hkv, hd], rows at positions start + c -> out [C, H * hd] fp32."""
    _need_cuda(q, k_cache, v_cache)
    C, H, hd = q.shape
    Hkv = k_cache.shape[1]
    st = torch.as_tensor([int(start)], dtype=torch.int32).to(q.device) if not torch.is_tensor(start) or \
        not start.is_cuda else start.to(torch.int32)
    out = torch.empty(C, H * hd, dtype=torch.float32, device=q.device)
    need = lib().q4b_attention_workspace(C, H, Hkv, hd, L)
    ws = None
    if need:
        key = (q.device.index, torch.cuda.current_stream().cuda_stream)
        ws = _ATTN_WS.get(key)
        if ws is None or ws.numel() < need:
            ws = torch.zeros(need, dtype=torch.uint8, device=q.device)
            _ATTN_WS[key] = ws
    check(lib().q4b_attention(q.float().contiguous().data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), st.data_ptr(),
                              C, H, Hkv, hd, L, out.data_ptr(), 0 if ws is None else ws.data_ptr(),
                              0 if ws is None else ws.numel(), _stream()), "attention")
    return out
