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

    def _norm_args(self, partial, residual, weight):
        for t, n in ((partial, "partial sums"), (residual, "residual"), (weight, "norm weight")):
            _require_cuda(t, "all-reduce + norm " + n)
        if residual.dtype not in _DT or partial.dtype != residual.dtype or weight.dtype != residual.dtype:
            raise DTypeMismatch("all-reduce + norm takes bf16 or f16 partial / residual / weight "
                                "of one dtype")
        rows, H = residual.reshape(-1, residual.shape[-1]).shape
        if partial.numel() != rows * H or weight.numel() != H:
            raise ShapeMismatch("all-reduce + norm: partial, residual [rows, H] and weight [H]")
        return rows, H

    def rmsnorm(self, partial: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor,
                eps: float, out: torch.Tensor = None) -> torch.Tensor:
        """residual += sum over the group of partial (in place); returns
        rmsnorm(residual) * weight: one kernel for the all-reduce of a
        row-parallel projection and the norm after it."""
        rows, H = self._norm_args(partial, residual, weight)
        if out is None:
            out = torch.empty_like(residual)
        _lib.check("lmrs_allreduce_rmsnorm", self.lib.lmrs_allreduce_rmsnorm(
            ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(residual.data_ptr()),
            ctypes.c_void_p(partial.data_ptr()), ctypes.c_void_p(weight.data_ptr()), rows, H,
            float(eps), _DT[residual.dtype], self.rank, self.world, self.bases, self.max_elems,
            ctypes.c_void_p(torch.cuda.current_stream(residual.device).cuda_stream)))
        return out

    def rmsnorm_fp8(self, partial: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor,
                    eps: float, q_out: torch.Tensor = None, scale_out: torch.Tensor = None):
        """As rmsnorm, returning the e4m3 bytes and per-row scales of the output."""
        rows, H = self._norm_args(partial, residual, weight)
        dev = residual.device
        if q_out is None:
            q_out = torch.empty((rows, H), dtype=torch.uint8, device=dev)
        if scale_out is None:
            scale_out = torch.empty((rows,), dtype=torch.float32, device=dev)
        _lib.check("lmrs_allreduce_rmsnorm_fp8", self.lib.lmrs_allreduce_rmsnorm_fp8(
            ctypes.c_void_p(q_out.data_ptr()), ctypes.c_void_p(scale_out.data_ptr()),
            ctypes.c_void_p(residual.data_ptr()), ctypes.c_void_p(partial.data_ptr()),
            ctypes.c_void_p(weight.data_ptr()), rows, H, float(eps), _DT[residual.dtype],
            self.rank, self.world, self.bases, self.max_elems,
            ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)))
        return q_out, scale_out

    def close(self):
        for p in self.opened:
            self.lib.lmrs_ipc_close(p)
        self.opened = []
        if self.own is not None:
            self.lib.lmrs_comm_free(self.own)
            self.own = None
