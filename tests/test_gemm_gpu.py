"""fp16 GEMM (q4b_gemm_f16) against Cref = A.f32 @ B.f32 with the harness tolerance
max|C - Cref| / max|Cref| <= 5e-3 (gemm/shapes.py:53-66, gemm/harness/vk_gemm_bench.c:411-425).

Small problems are checked against the CPU oracle (oracle.gemm_make_data); problems too large for a
quick float64 product use a torch fp32 matmul on the GPU (TF32 off) as the reference."""

import numpy as np
import pytest
import torch

from oracle import q4_oracle as O

pytestmark = pytest.mark.gpu
TOL = O.GEMM_TOL

# the reference tuner's eight problems (gemm/shapes.py:41-50): M, N, K, layout
REF_SHAPES = [(1024, 1024, 1024, "NN"), (128, 3072, 3072, "NT"), (4096, 64, 1024, "TN"), (16, 4096, 4096, "NT"),
              (256, 256, 8192, "TT"), (2048, 2048, 32, "NN"), (1, 4096, 4096, "NT"), (768, 768, 768, "TN")]
# the B200 sweep: M in {1, 128, 2048} x the 3B projection shapes, row-major A [M,K], B [K,N]
SWEEP_NK = [(5120, 3072), (3072, 3072), (16384, 3072), (3072, 8192)]


def _rel(c, ref):
    return float((c.float() - ref).abs().max() / ref.abs().max())


def _run_oracle_case(M, N, K, layout, seed, cfg=None):
    import q4b
    la, lb = layout
    a, b, c = O.gemm_make_data(M, N, K, la, lb, seed=seed)
    dev = torch.device("cuda:0")
    out = q4b.gemm_f16(torch.from_numpy(a).to(dev), torch.from_numpy(b).to(dev), la, lb, cfg=cfg)
    torch.cuda.synchronize()
    return _rel(out.cpu(), torch.from_numpy(c))


def _device_ref(M, N, K, la, lb, seed):
    g = torch.Generator(device="cuda:0")
    g.manual_seed(seed)
    a = (torch.rand(M, K, device="cuda:0", generator=g) * 2 - 1).half()
    b = (torch.rand(K, N, device="cuda:0", generator=g) * 2 - 1).half()
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    ref = a.float() @ b.float()
    torch.backends.cuda.matmul.allow_tf32 = prev
    a_st = a if la == "N" else a.t().contiguous()
    b_st = b if lb == "N" else b.t().contiguous()
    return a_st, b_st, ref


@pytest.mark.parametrize("M,N,K,layout", REF_SHAPES, ids=[f"{m}x{n}x{k}{l}" for m, n, k, l in REF_SHAPES])
def test_reference_tuner_shapes(M, N, K, layout):
    if M * N * K > 2**31:
        import q4b
        a, b, ref = _device_ref(M, N, K, layout[0], layout[1], seed=M + N + K)
        out = q4b.gemm_f16(a, b, layout[0], layout[1])
        torch.cuda.synchronize()
        assert _rel(out, ref) <= TOL
    else:
        assert _run_oracle_case(M, N, K, layout, seed=M + N + K) <= TOL


@pytest.mark.parametrize("M", [1, 128, 2048])
@pytest.mark.parametrize("N,K", SWEEP_NK, ids=[f"{n}x{k}" for n, k in SWEEP_NK])
def test_sweep_shapes(M, N, K):
    import q4b
    a, b, ref = _device_ref(M, N, K, "N", "N", seed=M * 7 + N + K)
    out = q4b.gemm_f16(a, b, "N", "N")
    torch.cuda.synchronize()
    assert _rel(out, ref) <= TOL


# ragged sizes, every layout: tails in M / N / K, K below one 64-wide step, row pitches TMA cannot
# describe (kernel 2 takes those)
RAGGED = [(100, 200, 136), (1, 64, 32), (130, 72, 200), (37, 100, 64), (257, 264, 8), (3, 5, 7), (64, 64, 4104)]


@pytest.mark.parametrize("layout", ["NN", "NT", "TN", "TT"])
@pytest.mark.parametrize("M,N,K", RAGGED, ids=[f"{m}x{n}x{k}" for m, n, k in RAGGED])
def test_ragged(M, N, K, layout):
    assert _run_oracle_case(M, N, K, layout, seed=M + 3 * N + 5 * K) <= TOL


# the schedule space of the tcgen05 kernel (the gemm/fuzz.py pattern: every legal schedule computes
# the same product)
CFGS = [dict(kernel=2), dict(kernel=1, bn=64), dict(kernel=1, bn=128), dict(kernel=1, bn=256),
        dict(kernel=1, bn=64, stages=2), dict(kernel=1, bn=256, stages=2), dict(kernel=1, bn=128, split=3),
        dict(kernel=1, bn=64, split=16), dict(kernel=1, bn=256, split=2, stages=3), dict(kernel=1, bn=128, stages=5),
        dict(kernel=3), dict(kernel=3, bn=64), dict(kernel=3, bn=256), dict(kernel=3, bn=128, stages=3)]


@pytest.mark.parametrize("cfg", CFGS, ids=[str(c) for c in CFGS])
@pytest.mark.parametrize("layout", ["NN", "TT"])
def test_schedule_space(cfg, layout):
    for (M, N, K) in [(256, 384, 1024), (200, 520, 1088)]:
        assert _run_oracle_case(M, N, K, layout, seed=M + N, cfg=cfg) <= TOL, (M, N, K)


def test_split_k_is_deterministic():
    import q4b
    a, b, _ = _device_ref(128, 3072, 8192, "N", "N", seed=3)
    cfg = dict(kernel=1, bn=128, split=8)
    c1 = q4b.gemm_f16(a, b, cfg=cfg)
    c2 = q4b.gemm_f16(a, b, cfg=cfg)
    torch.cuda.synchronize()
    assert torch.equal(c1, c2)


# kernel 3 (stream-K): runs of units that cover whole tiles in the middle and part-tiles at both ends
# (4096 x 4096 x 128: ~7 units of 2-step tiles per CTA), every tile split over several CTAs (the
# M = 128 projection), and long K (8192)
SK_SHAPES = [(4096, 4096, 128), (128, 5120, 3072), (2048, 3072, 8192), (136, 200, 4160)]


@pytest.mark.parametrize("M,N,K", SK_SHAPES, ids=[f"{m}x{n}x{k}" for m, n, k in SK_SHAPES])
def test_stream_k(M, N, K):
    import q4b
    a, b, ref = _device_ref(M, N, K, "N", "N", seed=M + 11 * N + K)
    c1 = q4b.gemm_f16(a, b, cfg=dict(kernel=3))
    c2 = q4b.gemm_f16(a, b, cfg=dict(kernel=3))
    torch.cuda.synchronize()
    assert _rel(c1, ref) <= TOL
    assert torch.equal(c1, c2)  # the part-tiles are added in k order: deterministic


def test_rejects_bad_config():
    import q4b
    a = torch.zeros(128, 128, dtype=torch.float16, device="cuda:0")
    with pytest.raises(q4b.Q4BError):
        q4b.gemm_f16(a, a, cfg=dict(kernel=1, bn=96))
    with pytest.raises(q4b.Q4BError):
        q4b.gemm_f16(a, a, cfg=dict(kernel=1, stages=1))
    with pytest.raises(q4b.Q4BError):
        q4b.gemm_f16(a, a, cfg=dict(kernel=1, split=3))  # K = 128 has two 64-wide steps
    with pytest.raises(q4b.Q4BError):
        q4b.gemm_f16(a, a, cfg=dict(kernel=3, split=2))  # kernel 3 balances k itself


def test_no_timeouts():
    from q4b import _lib
    assert _lib.lib().q4b_device_status(1) == 0
