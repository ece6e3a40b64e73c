"""Tensor-parallel communicator of the decode step (mslim_cuda_tp_* in
include/mslim_cuda.h): every rank's partial-sum slots and ready counters,
mapped into every rank through CUDA IPC, and the fused
all-reduce + residual + RMSNorm that reads them over NVLink.

Host side only: allocation, the handle exchange (over the torch.distributed
group the ranks already share) and the views torch GEMMs write into.  One rank
per GPU; the ranks' kernels wait for one another, so a group must never put two
ranks on one GPU."""
from __future__ import annotations

import ctypes

from . import _lib
from .attention import _ptr, _stream, check

MAX_WORLD = 8


class _DeviceArray:
    """A raw device allocation seen by torch through __cuda_array_interface__."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (ptr, False),
                                         "version": 3, "strides": None}


class TpComm:
    def __init__(self, world: int, rank: int, max_rows: int, hidden: int, group=None):
        import torch
        import torch.distributed as dist
        if not 1 <= world <= MAX_WORLD or not 0 <= rank < world:
            raise ValueError("tensor-parallel world of 1..8 ranks")
        if hidden % 8:
            raise ValueError("hidden size must be a multiple of 8")
        L = _lib.lib()
        self.torch, self.world, self.rank, self.max_rows, self.hidden = torch, world, rank, max_rows, hidden
        self._own = []
        self._opened = []

        def alloc(nbytes):
            p = ctypes.c_void_p()
            check(L.mslim_cuda_tp_alloc(nbytes, ctypes.byref(p)))
            self._own.append(p.value)
            return p.value

        data = alloc(2 * max_rows * hidden * 2)
        flags = alloc(max_rows * MAX_WORLD * 4)
        epoch = alloc(max_rows * 4)

        def handle(ptr):
            h = ctypes.create_string_buffer(64)
            check(L.mslim_cuda_ipc_handle(ptr, h))
            return h.raw

        mine = (handle(data), handle(flags))
        every = [None] * world
        if world > 1:
            dist.all_gather_object(every, mine, group=group)
        else:
            every = [mine]
        c = _lib.TpComm()
        c.world, c.rank, c.max_rows, c.hidden = world, rank, max_rows, hidden
        for r in range(world):
            if r == rank:
                c.data[r], c.flags[r] = data, flags
                continue
            ptrs = []
            for h in every[r]:
                p = ctypes.c_void_p()
                check(L.mslim_cuda_ipc_open(ctypes.create_string_buffer(h, 64), ctypes.byref(p)))
                self._opened.append(p.value)
                ptrs.append(p.value)
            c.data[r], c.flags[r] = ptrs
        c.epoch = epoch
        self.c = c
        self._data = data
        self.calls = 0   # slot of the next call = calls & 1

    def slot(self, slot: int, rows: int):
        """bf16 view [rows][hidden] of this rank's partial-sum slot."""
        t = self.torch
        base = self._data + slot * self.max_rows * self.hidden * 2
        return t.as_tensor(_DeviceArray(base, (rows, self.hidden), "<i2"), device="cuda").view(t.bfloat16)

    def next_slot(self) -> int:
        s = self.calls & 1
        self.calls += 1
        return s

    def allreduce_rmsnorm(self, slot: int, x, w, y, rows: int, eps: float, stream=None) -> None:
        check(_lib.lib().mslim_cuda_tp_allreduce_rmsnorm(ctypes.byref(self.c), slot, _ptr(x), _ptr(w), _ptr(y),
                                                         rows, eps, _stream(stream)))

    def close(self):
        """Unmaps the peers and frees this rank's regions (after a barrier:
        no peer may still read them)."""
        L = _lib.lib()
        for p in self._opened:
            L.mslim_cuda_ipc_close(p)
        for p in self._own:
            L.mslim_cuda_tp_free(p)
        self._opened, self._own = [], []
