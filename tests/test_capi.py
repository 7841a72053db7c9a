"""CPU-side checks of the C ABI: the library loads, exports every symbol include/q4b.h declares,
and rejects bad arguments on the host before any launch (no GPU needed)."""

import ctypes
import pathlib
import re

import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]


def header_symbols():
    text = (ROOT / "include" / "q4b.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(q4b_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def L():
    from q4b import _lib
    return _lib.lib()


def test_header_symbols_exported(L):
    syms = header_symbols()
    assert len(syms) >= 7
    missing = [s for s in syms if not hasattr(L, s)]
    assert not missing, missing


def test_bindings_cover_header():
    from q4b import _lib
    assert set(header_symbols()) == set(_lib.SIGNATURES)


def test_abi_version(L):
    assert L.q4b_abi_version() == 1


def test_linear_rejects_bad_args_on_host(L):
    from q4b import _lib
    p = ctypes.c_void_p(16)  # never dereferenced: validation fails first
    # null pointers
    assert L.q4b_q4_linear(None, p, 128, p, 0, p, 0, 1, 16, 128, 0, None, None, 0, None) == _lib.Q4B_EINVAL
    assert b"null" in L.q4b_last_error()
    # K not a multiple of the group
    assert L.q4b_q4_linear(p, p, 128, p, 0, p, 0, 1, 16, 200, 0, None, None, 0, None) == _lib.Q4B_EINVAL
    assert b"group" in L.q4b_last_error()
    # bad dtype, bad epilogue, odd rows for SwiGLU
    assert L.q4b_q4_linear(p, p, 128, p, 7, p, 0, 1, 16, 128, 0, None, None, 0, None) == _lib.Q4B_EINVAL
    assert L.q4b_q4_linear(p, p, 128, p, 0, p, 0, 1, 16, 128, 9, None, None, 0, None) == _lib.Q4B_EINVAL
    assert L.q4b_q4_linear(p, p, 128, p, 0, p, 0, 1, 15, 128, 2, None, None, 0, None) == _lib.Q4B_EINVAL
    # tensor-core kernel forced on a group it cannot handle
    cfg = _lib.LinearCfg(kernel=1)
    assert L.q4b_q4_linear(p, p, 32, p, 0, p, 0, 1, 16, 128, 0, ctypes.byref(cfg), None, 0,
                           None) == _lib.Q4B_EUNSUPPORTED
    # split that cannot be covered by warps * tiles
    cfg = _lib.LinearCfg(kernel=1, warps=1, tiles=1, split=2)
    assert L.q4b_q4_linear(p, p, 128, p, 0, p, 0, 1, 16, 3072, 0, ctypes.byref(cfg), None, 0,
                           None) == _lib.Q4B_EINVAL


def test_pack_rejects_bad_args_on_host(L):
    from q4b import _lib
    p = ctypes.c_void_p(16)
    assert L.q4b_quantize_q4(p, 4, 100, 32, p, p, None) == _lib.Q4B_EINVAL
    assert L.q4b_quantize_q4(p, 4, 96, 12, p, p, None) == _lib.Q4B_EINVAL
    assert L.q4b_unpack_q4(p, 4, 12, p, None) == _lib.Q4B_EINVAL
    assert L.q4b_dequantize_q4(p, p, 4, 128, 128, p, 5, None) == _lib.Q4B_EINVAL


def test_linear_workspace_plan(L):
    # decode 5120 x 3072, group 128, M = 1: all of K in one CTA of the register GEMV, no workspace
    assert L.q4b_q4_linear_workspace(1, 5120, 3072, 128, 0, None) == 0
    # the lm_head (197 MB of weights): the ring GEMV (kernel 6); row pairs cut between CTAs meet in
    # the workspace (counters + one 32-float partial per (row pair, 1024-k stage))
    assert L.q4b_q4_linear_workspace(1, 128256, 3072, 128, 0, None) == 65536 + 4008 * 3 * 32 * 4
    # 16 rows of x over K = 8192 do not fit one CTA's shared memory: split-K partials + counters
    ws = L.q4b_q4_linear_workspace(16, 3072, 8192, 128, 0, None)
    assert ws > 65536 and ws % 256 == 0
    # a non-128 group uses the SIMT kernel, which needs no workspace
    assert L.q4b_q4_linear_workspace(1, 256, 688, 16, 0, None) == 0
    # a configuration without split needs none
    from q4b import _lib
    cfg = _lib.LinearCfg(kernel=1, warps=8, tiles=3, split=1)
    assert L.q4b_q4_linear_workspace(1, 5120, 3072, 128, 0, ctypes.byref(cfg)) == 0


def test_prefill_gemm_plan(L):
    """Kernel 5 (prefill, M > 32) plans: every configuration form plans without a fault, and the
    default for the 3B prefill shapes picks the wide tile and a split that fills one wave."""
    from q4b import _lib
    KB = 65536  # the split-K counters
    x2 = lambda m, k: ((m * k * 2 + 255) // 256) * 256  # noqa: E731  (x hi + x lo)

    def ws(m, n, k, epi=0, **cfg):
        c = _lib.LinearCfg(**cfg) if cfg else None
        return L.q4b_q4_linear_workspace(m, n, k, 128, epi, ctypes.byref(c) if c else None)

    for cfg in (dict(kernel=5), dict(kernel=5, tiles=4), dict(kernel=5, tiles=8), dict(kernel=5, split=3),
                dict(kernel=5, tiles=4, split=5), dict(kernel=5, tiles=8, split=1)):
        for m, n, k in ((128, 5120, 3072), (64, 384, 3072), (33, 3072, 8192), (128, 16384, 3072)):
            assert ws(m, n, k, **cfg) >= KB, (cfg, m, n, k)
    # 3B o projection at a 128-row chunk: 24 tiles of 128 rows x 6 splits = 144 CTAs
    assert ws(128, 3072, 3072) == KB + 2 * x2(128, 3072) + 6 * 24 * 128 * 128 * 4
    # gate|up (16384 rows): 128 wide tiles already fill a wave, no split
    assert ws(128, 16384, 3072, epi=2) == KB + 2 * x2(128, 3072)


def test_small_m_gemv_plan_splits_k(L):
    """9..32 rows: the GEMV splits K so a CTA stages at most 8 k-tiles of x (8 splits of the 64
    tiles of K = 8192 at 16 rows); up to 8 rows K stays whole (no workspace)."""
    counters = 65536
    assert L.q4b_q4_linear_workspace(4, 3072, 8192, 128, 0, None) == 0
    ws = L.q4b_q4_linear_workspace(16, 3072, 8192, 128, 0, None)
    assert ws == counters + 8 * 16 * (3072 // 16) * 16 * 4
    ws = L.q4b_q4_linear_workspace(16, 5120, 3072, 128, 0, None)  # 24 tiles: 3 splits
    assert ws == counters + 3 * 16 * (5120 // 16) * 16 * 4


def test_linear_kernel_choice(L):
    """The planner's kernel for the reference's shapes: the ring GEMV for decode rows over large
    weights (the lm_head), the register GEMV for the layer projections and 9..32 rows, tcgen05 for
    prefill chunks, SIMT for groups that are not a multiple of 128; a fixed configuration is
    honoured."""
    from q4b import _lib
    F32, F16 = 0, 1
    assert L.q4b_q4_linear_kernel(1, 128256, 3072, 128, 0, F16, None) == 6
    assert L.q4b_q4_linear_kernel(1, 64128, 3072, 128, 0, F32, None) == 6
    assert L.q4b_q4_linear_kernel(1, 5120, 3072, 128, 0, F16, None) == 1
    assert L.q4b_q4_linear_kernel(8, 3072, 8192, 128, 1, F32, None) == 1
    assert L.q4b_q4_linear_kernel(4, 16384, 3072, 128, 2, F32, None) == 1
    assert L.q4b_q4_linear_kernel(1, 256, 256, 128, 0, F32, None) == 1  # K % 1024
    assert L.q4b_q4_linear_kernel(16, 3072, 8192, 128, 0, F32, None) == 1
    assert L.q4b_q4_linear_kernel(128, 5120, 3072, 128, 0, F32, None) == 5
    assert L.q4b_q4_linear_kernel(1, 256, 688, 16, 0, F32, None) == 2
    cfg = _lib.LinearCfg(kernel=6, tiles=1)
    assert L.q4b_q4_linear_kernel(1, 5120, 3072, 128, 0, F16, ctypes.byref(cfg)) == 6
    bad = _lib.LinearCfg(kernel=6, tiles=4)
    assert L.q4b_q4_linear_kernel(1, 5120, 3072, 128, 0, F16, ctypes.byref(bad)) == _lib.Q4B_EINVAL
    assert L.q4b_q4_linear_kernel(0, 5120, 3072, 128, 0, F16, None) == _lib.Q4B_EINVAL


def test_no_cpu_fallback_without_gpu():
    """The product ops refuse CPU tensors instead of computing on the host."""
    import torch

    from q4b import ops
    with pytest.raises(ValueError, match="CUDA"):
        ops.unpack_q4(torch.zeros(4, 4, dtype=torch.int32))
