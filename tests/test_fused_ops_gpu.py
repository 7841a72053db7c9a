"""GPU parity of the single-op entry points (the model's fused pieces as calls of their own,
scripts/llm/llama_q4.py:204-239) against the oracle, and of the standalone tensor-parallel
collectives on a one-rank communicator (the multi-rank forms run in tests/test_tp_gpu.py)."""

import ctypes

import numpy as np
import pytest
import torch

from oracle import q4_oracle as O

pytestmark = pytest.mark.gpu
TOL = 1e-3


@pytest.fixture(scope="module")
def L():
    import q4b
    return q4b.lib()


def _st():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("m", [1, 5, 40])
def test_qkv_rope_kvwrite(L, m):
    """q|k|v projection, RoPE on q and k at positions start + r, k and v written into the fp16
    caches in place (llama_q4.py:204-223)."""
    import q4b
    from q4b import ops
    dev = torch.device("cuda:0")
    D, H, Hkv, hd, G, max_ctx, start = 1024, 8, 2, 128, 128, 256, 37
    cfg = dict(hidden_size=D, num_attention_heads=H, num_key_value_heads=Hkv, head_dim=hd, rope_theta=500000.0,
               max_position_embeddings=4096)
    rng = np.random.default_rng(m)
    w = (rng.standard_normal(((H + 2 * Hkv) * hd, D)) * 0.05).astype(np.float32)
    qw, s = O.quantize_q4(w, G)
    x = rng.standard_normal((m, D)).astype(np.float32)
    cos, sin = O.rope_tables(cfg, max_ctx)
    full = O.q4_linear(qw, s, G, x)  # [m, N]
    pos = start + np.arange(m)
    q = full[:, : H * hd].reshape(m, H, hd)
    k = full[:, H * hd:(H + Hkv) * hd].reshape(m, Hkv, hd)
    v = full[:, (H + Hkv) * hd:].reshape(m, Hkv, hd)
    c, sn = cos[pos][:, None, :], sin[pos][:, None, :]
    q_ref = q * c + O.rotate_half(q) * sn
    k_ref = k * c + O.rotate_half(k) * sn
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)  # noqa: E731
    qw_t, s_t, x_t = t(qw), t(s), t(x)
    cos_t, sin_t = t(cos), t(sin)
    st = torch.tensor([start], dtype=torch.int32, device=dev)
    q_out = torch.full((m, H, hd), float("nan"), device=dev)
    kc = torch.zeros(max_ctx, Hkv, hd, dtype=torch.float16, device=dev)
    vc = torch.zeros(max_ctx, Hkv, hd, dtype=torch.float16, device=dev)
    need = L.q4b_qkv_rope_kvwrite_workspace(m, D, H, Hkv, hd, G)
    ws = ops.WORKSPACE.get(need, dev)
    rc = L.q4b_qkv_rope_kvwrite(qw_t.data_ptr(), s_t.data_ptr(), G, x_t.data_ptr(), m, D, H, Hkv, hd,
                                cos_t.data_ptr(), sin_t.data_ptr(), st.data_ptr(), q_out.data_ptr(), kc.data_ptr(),
                                vc.data_ptr(), 0 if ws is None else ws.data_ptr(), 0 if ws is None else ws.numel(),
                                _st())
    assert rc == 0, L.q4b_last_error()
    torch.cuda.synchronize()
    assert O.rel_err(q_out.cpu().numpy(), q_ref) <= TOL
    assert O.rel_err(kc[start:start + m].float().cpu().numpy(), k_ref) <= TOL
    assert O.rel_err(vc[start:start + m].float().cpu().numpy(), v) <= TOL
    assert not kc[:start].any() and not kc[start + m:].any()  # only rows start.. were written
    assert q4b.lib().q4b_device_status(1) == 0


def test_silu_mul(L):
    dev = torch.device("cuda:0")
    rng = np.random.default_rng(1)
    gu = rng.standard_normal((7, 2 * 688)).astype(np.float32) * 3
    out = torch.empty(7, 688, device=dev)
    gu_t = torch.from_numpy(gu).to(dev)
    rc = L.q4b_silu_mul(gu_t.data_ptr(), 7, 688, out.data_ptr(), _st())
    assert rc == 0
    torch.cuda.synchronize()
    ref = O.silu(gu[:, :688]) * gu[:, 688:]
    assert np.allclose(out.cpu().numpy(), ref, rtol=1e-5, atol=1e-6)


def test_argmax_first_max(L):
    dev = torch.device("cuda:0")
    for n in (1, 1000, 128256):
        v = torch.randn(n, device=dev)
        idx = torch.empty(1, dtype=torch.int32, device=dev)
        assert L.q4b_argmax(v.data_ptr(), n, idx.data_ptr(), _st()) == 0
        assert int(idx) == int(torch.argmax(v))
    v = torch.zeros(5000, device=dev)
    v[[17, 300, 4999]] = 3.0  # ties: the first index wins (torch.argmax)
    idx = torch.empty(1, dtype=torch.int32, device=dev)
    L.q4b_argmax(v.data_ptr(), 5000, idx.data_ptr(), _st())
    assert int(idx) == 17


@pytest.mark.parametrize("rows,L_", [(1, 64), (8, 128), (37, 256)])
def test_prefill_attn_matches_oracle(L, rows, L_):
    dev = torch.device("cuda:0")
    H, Hkv, hd, max_ctx, start = 8, 2, 64, 256, 20
    rng = np.random.default_rng(rows)
    q = rng.standard_normal((rows, H, hd)).astype(np.float32)
    kc = rng.standard_normal((max_ctx, Hkv, hd)).astype(np.float16)
    vc = rng.standard_normal((max_ctx, Hkv, hd)).astype(np.float16)
    pos = start + np.arange(rows)
    ref = O.attention(q, kc, vc, pos, L_, Hkv)
    out = torch.empty(rows, H * hd, device=dev)
    st = torch.tensor([start], dtype=torch.int32, device=dev)
    q_t, kc_t, vc_t = (torch.from_numpy(a).to(dev) for a in (q, kc, vc))  # held until the kernel ran
    rc = L.q4b_prefill_attn(q_t.data_ptr(), kc_t.data_ptr(), vc_t.data_ptr(), st.data_ptr(), rows, H, Hkv, hd, L_,
                            out.data_ptr(), _st())
    assert rc == 0, L.q4b_last_error()
    torch.cuda.synchronize()
    assert O.rel_err(out.cpu().numpy(), ref) <= TOL


def test_tp_collectives_one_rank(L):
    """A one-rank communicator: the all-reduce is the identity, the gathered argmax is the local one
    shifted by the shard's first vocabulary row."""
    from q4b import _lib
    dev = torch.device("cuda:0")
    uid = (ctypes.c_ubyte * 128)()
    _lib.check(L.q4b_tp_unique_id(uid, 128), "tp_unique_id")
    tp = ctypes.c_void_p()
    _lib.check(L.q4b_tp_init(0, 1, uid, 128, ctypes.byref(tp)), "tp_init")
    try:
        a = torch.randn(1000, device=dev)
        b = a.clone()
        _lib.check(L.q4b_tp_allreduce_f32(tp, b.data_ptr(), 1000, _st()), "allreduce")
        h = a.half()
        h2 = h.clone()
        _lib.check(L.q4b_tp_allreduce_f16(tp, h2.data_ptr(), 1000, _st()), "allreduce f16")
        logits = torch.randn(32064, device=dev)
        ws = torch.zeros(L.q4b_tp_argmax_workspace(tp) // 8, dtype=torch.int64, device=dev)
        tok = torch.empty(1, dtype=torch.int32, device=dev)
        _lib.check(L.q4b_tp_argmax_gather(tp, logits.data_ptr(), 32064, 64128, tok.data_ptr(), ws.data_ptr(),
                                          ws.numel() * 8, _st()), "argmax_gather")
        torch.cuda.synchronize()
        assert torch.equal(a, b) and torch.equal(h, h2)
        assert int(tok) == 64128 + int(torch.argmax(logits))
    finally:
        L.q4b_tp_destroy(tp)
