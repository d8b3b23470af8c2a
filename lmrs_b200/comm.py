"""Tensor-parallel all-reduce for the row-parallel projections (include/lmrs_comm.h).

``PeerAllReduce`` owns one receive buffer per rank, shares it with the other
ranks of a torch.distributed group through CUDA IPC handles (exchanged with
``all_gather_object``: torch.distributed is only the plumbing), and sums a
bf16/fp16 tensor across the group with the one-shot packet kernel.  Each call
is a single kernel, capturable in a CUDA graph.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from .ops import DTypeMismatch, ShapeMismatch, _require_cuda

_DT = {torch.bfloat16: _lib.DTYPE_BF16, torch.float16: _lib.DTYPE_F16}


class PeerAllReduce:
    """Sum of a tensor over a process group (one GPU per rank, one node)."""

    def __init__(self, max_elems: int, group=None):
        import torch.distributed as dist
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.max_elems = max_elems + (max_elems & 1)
        lib = self.lib = _lib.load()
        nbytes = lib.lmrs_allreduce_buffer_bytes(self.world, self.max_elems)
        if nbytes == 0:
            raise ShapeMismatch(f"world size {self.world} not supported (1..8)")
        own = ctypes.c_void_p()
        _lib.check("lmrs_comm_alloc", lib.lmrs_comm_alloc(ctypes.byref(own), nbytes))
        self.own = own
        h = ctypes.create_string_buffer(64)
        _lib.check("lmrs_ipc_get_handle", lib.lmrs_ipc_get_handle(own, h, 64))
        handles = [None] * self.world
        dist.all_gather_object(handles, h.raw, group=group)
        self.opened = []
        ptrs = []
        for r, hb in enumerate(handles):
            if r == self.rank:
                ptrs.append(own.value)
                continue
            p = ctypes.c_void_p()
            _lib.check("lmrs_ipc_open",
                       lib.lmrs_ipc_open(ctypes.create_string_buffer(hb, 64), ctypes.byref(p)))
            self.opened.append(p)
            ptrs.append(p.value)
        self.bases = (ctypes.c_void_p * self.world)(*ptrs)
        dist.barrier(group=group)  # every rank has mapped every buffer

    def __call__(self, t: torch.Tensor) -> torch.Tensor:
        """In-place sum over the group; returns t."""
        _require_cuda(t, "all-reduce input")
        if t.dtype not in _DT:
            raise DTypeMismatch(f"all-reduce takes bf16 or f16, got {t.dtype}")
        n = t.numel()
        if n % 2 or n > self.max_elems:
            raise ShapeMismatch(f"all-reduce of {n} elements (even, <= {self.max_elems})")
        _lib.check("lmrs_allreduce_sum", self.lib.lmrs_allreduce_sum(
            ctypes.c_void_p(t.data_ptr()), ctypes.c_void_p(t.data_ptr()), n, _DT[t.dtype],
            self.rank, self.world, self.bases, self.max_elems,
            ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)))
        return t

    def close(self):
        for p in self.opened:
            self.lib.lmrs_ipc_close(p)
        self.opened = []
        if self.own is not None:
            self.lib.lmrs_comm_free(self.own)
            self.own = None
