"""The standalone tensor-parallel collectives of the C ABI (q4b_tp_*: NCCL loaded by libq4b.so,
one process per GPU) for callers outside the model: rank 0 makes the communicator id and
torch.distributed broadcasts it. The calls take device tensors and the current stream, so they can
be captured in CUDA graphs."""

from __future__ import annotations

import ctypes

import torch

from . import _lib


class TpComm:
    def __init__(self, rank: int, world: int, dist_mod=None):
        import torch.distributed as dist
        dist_mod = dist_mod or dist
        L = _lib.lib()
        uid = (ctypes.c_ubyte * 128)()
        if rank == 0:
            _lib.check(L.q4b_tp_unique_id(uid, 128), "tp_unique_id")
        obj = [bytes(uid)]
        dist_mod.broadcast_object_list(obj, src=0)
        uid = (ctypes.c_ubyte * 128).from_buffer_copy(obj[0])
        self._h = ctypes.c_void_p()
        _lib.check(L.q4b_tp_init(rank, world, uid, 128, ctypes.byref(self._h)), "tp_init")
        self.rank, self.world = rank, world

    def allreduce(self, t: torch.Tensor):
        """In-place sum over the ranks of an fp32 or fp16 CUDA tensor, on the current stream."""
        if not t.is_cuda or not t.is_contiguous():
            raise ValueError("allreduce needs a contiguous CUDA tensor")
        L = _lib.lib()
        st = ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)
        if t.dtype == torch.float32:
            _lib.check(L.q4b_tp_allreduce_f32(self._h, t.data_ptr(), t.numel(), st), "tp_allreduce_f32")
        elif t.dtype == torch.float16:
            _lib.check(L.q4b_tp_allreduce_f16(self._h, t.data_ptr(), t.numel(), st), "tp_allreduce_f16")
        else:
            raise ValueError(f"allreduce takes fp32 or fp16, not {t.dtype}")

    def close(self):
        if self._h:
            _lib.lib().q4b_tp_destroy(self._h)
            self._h = ctypes.c_void_p()
