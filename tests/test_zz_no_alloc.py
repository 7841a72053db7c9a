"""The allocation-free entry point q4b_q4_linear_noalloc, for callers that cannot allocate device
memory (a plain C FFI host without a CUDA allocator, a plugin inside a framework that owns the
memory pool, a fixed memory budget). Called through the C ABI with ctypes; its output must match
q4b_q4_linear with a caller-provided workspace on two calls in a row (the static scratch keeps
the last call's contents, so the second call checks that it starts clean).

Kept in its own file, named to be collected last."""

import ctypes

import numpy as np
import pytest
import torch

import golden_inputs as gi
from oracle import q4_oracle as O

pytestmark = pytest.mark.gpu
TOL = 1e-3

# (N, K, group, M, x dtype): split-K shapes that use the scratch, plus a no-split shape
CASES = [(5120, 3072, 128, 1, torch.float16), (3072, 8192, 128, 4, torch.float32),
         (384, 3072, 128, 16, torch.float32), (256, 688, 16, 3, torch.float32)]


@pytest.mark.parametrize("N,K,G,M,xdt", CASES)
def test_noalloc_matches_workspace_entry_point(N, K, G, M, xdt):
    from q4b import _lib, ops
    L = _lib.lib()
    dev = torch.device("cuda:0")
    qw, s = gi.synthetic_q4(N, K, G, seed=N + K + M)
    qwt, st = torch.from_numpy(qw).to(dev), torch.from_numpy(s).to(dev)
    dt = _lib.F32 if xdt == torch.float32 else _lib.F16
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):
        x = torch.randn(M, K, device=dev, generator=torch.Generator(device=dev).manual_seed(call)).to(xdt)
        ref = ops.q4_linear(x, qwt, st, G, out_dtype=torch.float32)
        y = torch.full((M, N), float("nan"), device=dev)
        rc = L.q4b_q4_linear_noalloc(qwt.data_ptr(), st.data_ptr(), G, x.data_ptr(), dt, y.data_ptr(), _lib.F32, M, N,
                                     K, _lib.EPI_STORE, stream)
        assert rc == 0, L.q4b_last_error()
        torch.cuda.synchronize()
        assert O.rel_err(y.cpu().numpy(), ref.cpu().numpy()) <= TOL, call
        # and against the CPU oracle
        assert O.rel_err(y.cpu().numpy(), O.q4_linear(qw, s, G, x.float().cpu().numpy())) <= TOL, call


def test_noalloc_rejects_sizes_beyond_the_static_scratch():
    """Real (allocated) buffers, so nothing can read a bad address even if a future plan accepted
    the shape: 1024 rows of x over K = 4096 need 16 MiB of converted activations, over 8 MiB."""
    from q4b import _lib
    L = _lib.lib()
    dev = torch.device("cuda:0")
    M, N, K = 1024, 64, 4096
    qw = torch.zeros(N, K // 8, dtype=torch.int32, device=dev)
    s = torch.ones(N, K // 128, dtype=torch.float16, device=dev)
    x = torch.zeros(M, K, device=dev)
    y = torch.zeros(M, N, device=dev)
    rc = L.q4b_q4_linear_noalloc(qw.data_ptr(), s.data_ptr(), 128, x.data_ptr(), _lib.F32, y.data_ptr(), _lib.F32,
                                 M, N, K, _lib.EPI_STORE, None)
    assert rc == _lib.Q4B_EINVAL
    assert b"static scratch" in L.q4b_last_error()
    torch.cuda.synchronize()
