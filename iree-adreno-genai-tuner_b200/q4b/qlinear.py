"""Drop-in QLinear / QEmbedding (scripts/llm/llama_q4.py:60-122) backed by libq4b.so."""

from __future__ import annotations

import torch
from torch import nn

from . import ops


class QLinear(nn.Module):
    """scripts/llm/llama_q4.py:60-90: same constructor (w [N, K], group), same attributes
    (qweight [N, K/8] int32, scales [N, K/G] fp16, group, n, k) and packing, quantised on the GPU
    bit-exactly. forward(x [M, K]) returns x @ dequantize(W)^T with fp32 accumulation in one CUDA
    call (the reference's fused GEMV and dequant + linear forms compute the same sum). fp32 x gives
    fp32 y like the reference; fp16 x gives fp16 y unless out_dtype says otherwise."""

    def __init__(self, w: torch.Tensor, group: int, *, device=None):
        super().__init__()
        if w.dim() != 2:
            raise ValueError("w must be [N, K]")
        if w.shape[1] % group or group % 8:
            raise AssertionError((*w.shape, group))  # the reference asserts the same
        if device is not None:
            w = w.to(device)
        qweight, scales = ops.quantize_q4(w, group)
        self.qweight = nn.Parameter(qweight, requires_grad=False)
        self.scales = nn.Parameter(scales, requires_grad=False)
        self.group = group
        self.n, self.k = w.shape

    @classmethod
    def from_packed(cls, qweight: torch.Tensor, scales: torch.Tensor, group: int):
        """Wrap already-packed weights (e.g. the reference's QLinear.qweight / .scales)."""
        self = cls.__new__(cls)
        nn.Module.__init__(self)
        self.qweight = nn.Parameter(qweight.to("cuda").contiguous(), requires_grad=False)
        self.scales = nn.Parameter(scales.to("cuda").to(torch.float16).contiguous(), requires_grad=False)
        self.group = group
        self.n, self.k = qweight.shape[0], qweight.shape[1] * 8
        return self

    def forward(self, x: torch.Tensor, *, out_dtype=None, epilogue: str = "store", out=None, cfg=None):
        squeeze = x.dim() == 1
        x2 = x.reshape(1, -1) if squeeze else x
        y = ops.q4_linear(x2.contiguous(), self.qweight, self.scales, self.group, out=out, epilogue=epilogue,
                          out_dtype=out_dtype, cfg=cfg)
        return y.reshape(-1) if squeeze else y


class QEmbedding(nn.Module):
    """scripts/llm/llama_q4.py:93-122: tied int4 embedding / lm_head. The reference keeps vocab
    chunks of `chunk_rows` rows (a phone buffer-size limit); rows are independent, so here the
    chunks are views of one contiguous [vocab, dim/8] table and `logits` is one GEMV."""

    def __init__(self, w: torch.Tensor, group: int, chunk_rows: int, *, device=None):
        super().__init__()
        self.vocab, self.dim = w.shape
        self.chunk_rows = chunk_rows
        self.group = group
        parts = [ops.quantize_q4(w[i: i + chunk_rows].to(device or "cuda"), group)
                 for i in range(0, self.vocab, chunk_rows)]
        self.qweight = nn.Parameter(torch.cat([p[0] for p in parts]), requires_grad=False)
        self.scales = nn.Parameter(torch.cat([p[1] for p in parts]), requires_grad=False)

    @classmethod
    def from_packed(cls, qweight, scales, group, chunk_rows):
        self = cls.__new__(cls)
        nn.Module.__init__(self)
        self.vocab, self.dim = qweight.shape[0], qweight.shape[1] * 8
        self.chunk_rows, self.group = chunk_rows, group
        self.qweight = nn.Parameter(qweight.to("cuda").contiguous(), requires_grad=False)
        self.scales = nn.Parameter(scales.to("cuda").to(torch.float16).contiguous(), requires_grad=False)
        return self

    @property
    def chunks(self):
        """QLinear views of the vocab chunks (scripts/llm/llama_q4.py:102-104)."""
        out = []
        for i in range(0, self.vocab, self.chunk_rows):
            out.append(QLinear.from_packed(self.qweight[i: i + self.chunk_rows], self.scales[i: i + self.chunk_rows],
                                           self.group))
        return out

    def lookup(self, tokens: torch.Tensor) -> torch.Tensor:
        return ops.embed_lookup(tokens, self.qweight, self.scales, self.group)

    def logits(self, x: torch.Tensor) -> torch.Tensor:
        return ops.q4_linear(x.contiguous(), self.qweight, self.scales, self.group, out_dtype=torch.float32)
