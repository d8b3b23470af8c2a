"""Tensor parallelism for the quantized projections (one process per GPU).

The reference runs a single GPU (crates/engine/src/generation.rs:209-211) and
ships only an orphaned CUDA-IPC all-reduce (kernels/comm/custom_all_reduce.cuh:372);
this module is the B200 layout the task asks for:

* column-parallel (q, k, v, gate, up): split the output features N — AWQ
  ``qweight``/``qzeros`` by whole packed words, ``scales`` to match; FP8 ``wq``
  rows and ``w_scale`` entries.  No communication.
* row-parallel (o, down): split the input features K — AWQ by whole
  quantisation groups (K/world must be a multiple of the group size); FP8
  ``wq`` column slices (per-channel ``w_scale`` is unaffected).  Each rank's
  partial output is summed with one all-reduce (NCCL over NVLink/NVSwitch on
  the GPU; any torch.distributed backend works, gloo is used for CPU tests).
  The bias is added once, after the reduction.

The per-rank compute is any object with ``forward(x)`` (normally a
``QuantLinearOp``), so the sharding and reduction logic is testable on CPU.
"""
from __future__ import annotations

from typing import Callable, Optional

import torch

from .ops import AWQ_PACK_FACTOR, AwqConfig, LinearConfig, QuantLinearOp


def _split(n: int, world: int, rank: int, align: int = 1):
    if n % (world * align):
        raise ValueError(f"{n} is not divisible by world ({world}) x alignment ({align})")
    per = n // world
    return rank * per, (rank + 1) * per


# --------------------------------------------------------------- AWQ shards
def shard_awq_column(qweight, qzeros, scales, rank: int, world: int):
    """Output-feature shard: columns [rank*N/world, (rank+1)*N/world)."""
    words = qweight.shape[1]
    a, b = _split(words, world, rank)
    return (qweight[:, a:b].contiguous(), qzeros[:, a:b].contiguous(),
            scales[:, a * AWQ_PACK_FACTOR:b * AWQ_PACK_FACTOR].contiguous())


def shard_awq_row(qweight, qzeros, scales, rank: int, world: int, group: int):
    """Input-feature shard: rows [rank*K/world, ...) in whole quantisation groups."""
    K = qweight.shape[0]
    a, b = _split(K, world, rank, group)
    return (qweight[a:b].contiguous(), qzeros[a // group:b // group].contiguous(),
            scales[a // group:b // group].contiguous())


# --------------------------------------------------------------- FP8 shards
def shard_fp8_column(weight_q, weight_scale, rank: int, world: int):
    a, b = _split(weight_q.shape[0], world, rank)
    return weight_q[a:b].contiguous(), weight_scale[a:b].contiguous()


def shard_fp8_row(weight_q, weight_scale, rank: int, world: int, align: int = 16):
    a, b = _split(weight_q.shape[1], world, rank, align)
    return weight_q[:, a:b].contiguous(), weight_scale


def shard_bias_column(bias, rank, world):
    if bias is None:
        return None
    a, b = _split(bias.shape[0], world, rank)
    return bias[a:b].contiguous()


# --------------------------------------------------------------- layers
class ColumnParallel:
    """y_local = x @ W[:, shard]; outputs stay sharded along N (no communication)."""

    def __init__(self, local):
        self.local = local

    def forward(self, x):
        return self.local.forward(x)

    __call__ = forward


class RowParallel:
    """y = all_reduce_sum(x_local @ W[shard, :]) (+ bias once, after the sum)."""

    def __init__(self, local, bias: Optional[torch.Tensor] = None, group=None,
                 all_reduce: Optional[Callable] = None):
        self.local = local
        self.bias = bias
        self.group = group
        self._all_reduce = all_reduce

    def reduce(self, y):
        if self._all_reduce is not None:
            self._all_reduce(y)
        elif torch.distributed.is_initialized() and torch.distributed.get_world_size(self.group) > 1:
            torch.distributed.all_reduce(y, op=torch.distributed.ReduceOp.SUM, group=self.group)
        return y

    def forward(self, x_local):
        y = self.reduce(self.local.forward(x_local))
        if self.bias is not None:
            y = y + self.bias
        return y

    __call__ = forward


def awq_column_parallel(config: LinearConfig, qweight, qzeros, scales, rank, world,
                        bias=None, awq: AwqConfig = AwqConfig()) -> ColumnParallel:
    qw, qz, sc = shard_awq_column(qweight, qzeros, scales, rank, world)
    cfg = LinearConfig(config.in_features, config.out_features // world, bias is not None)
    return ColumnParallel(QuantLinearOp.awq(cfg, qw, qz, sc, shard_bias_column(bias, rank, world), awq))


def awq_row_parallel(config: LinearConfig, qweight, qzeros, scales, rank, world, bias=None,
                     awq: AwqConfig = AwqConfig(), group=None) -> RowParallel:
    qw, qz, sc = shard_awq_row(qweight, qzeros, scales, rank, world, awq.group_size)
    cfg = LinearConfig(config.in_features // world, config.out_features, False)
    return RowParallel(QuantLinearOp.awq(cfg, qw, qz, sc, None, awq), bias, group)


def fp8_column_parallel(config: LinearConfig, weight_q, weight_scale, rank, world,
                        bias=None) -> ColumnParallel:
    wq, sw = shard_fp8_column(weight_q, weight_scale, rank, world)
    cfg = LinearConfig(config.in_features, config.out_features // world, bias is not None)
    return ColumnParallel(QuantLinearOp.fp8(cfg, wq, sw, shard_bias_column(bias, rank, world)))


def fp8_row_parallel(config: LinearConfig, weight_q, weight_scale, rank, world, bias=None,
                     group=None) -> RowParallel:
    wq, sw = shard_fp8_row(weight_q, weight_scale, rank, world)
    cfg = LinearConfig(config.in_features // world, config.out_features, False)
    return RowParallel(QuantLinearOp.fp8(cfg, wq, sw, None), bias, group)
