"""Host wrappers of the decode-step kernels (include/lmrs_decode.h) and of the
persistent FP8 decode-layer kernel (include/lmrs_layer.h).

Argument checking and dtype dispatch mirror ``ops.py``: tensors must be CUDA,
contiguous and of the documented dtype, outputs are allocated on the input's
device unless given, and every call goes through the C-ABI (no torch fallback).
"""
from __future__ import annotations

from typing import Optional

import torch

from . import _lib
from .ops import DTypeMismatch, ShapeMismatch, _ptr, _require_cuda, _stream

_DT = {torch.bfloat16: _lib.DTYPE_BF16, torch.float16: _lib.DTYPE_F16}


def _code(t: torch.Tensor) -> int:
    if t.dtype not in _DT:
        raise DTypeMismatch(f"expected bf16 or f16, got {t.dtype}")
    return _DT[t.dtype]


def rmsnorm(residual: torch.Tensor, weight: torch.Tensor, eps: float,
            delta: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None):
    """residual (+)= delta (in place), returns rmsnorm(residual) * weight."""
    _require_cuda(residual, "residual")
    rows, H = residual.reshape(-1, residual.shape[-1]).shape
    if out is None:
        out = torch.empty_like(residual)
    _lib.check("lmrs_rmsnorm", _lib.load().lmrs_rmsnorm(
        _ptr(out), _ptr(residual), _ptr(delta), _ptr(weight), rows, H, float(eps),
        _code(residual), _stream(residual)))
    return out


def rmsnorm_fp8(residual: torch.Tensor, weight: torch.Tensor, eps: float,
                delta: Optional[torch.Tensor] = None, q_out=None, scale_out=None):
    """residual (+)= delta, returns (e4m3 bytes, per-row fp32 scales) of the
    normalised rows, as fp8_quant_rows(rmsnorm(...)) would."""
    _require_cuda(residual, "residual")
    rows, H = residual.reshape(-1, residual.shape[-1]).shape
    if q_out is None:
        q_out = torch.empty((rows, H), dtype=torch.uint8, device=residual.device)
    if scale_out is None:
        scale_out = torch.empty((rows,), dtype=torch.float32, device=residual.device)
    _lib.check("lmrs_rmsnorm_fp8", _lib.load().lmrs_rmsnorm_fp8(
        _ptr(q_out), _ptr(scale_out), _ptr(residual), _ptr(delta), _ptr(weight), rows, H,
        float(eps), _code(residual), _stream(residual)))
    return q_out, scale_out


def silu_mul(gate_up: torch.Tensor, out: Optional[torch.Tensor] = None):
    """silu(gate) * up for a merged [rows, 2 * inter] projection output."""
    _require_cuda(gate_up, "gate_up")
    rows, two_i = gate_up.shape
    if two_i % 2:
        raise ShapeMismatch("gate_up last dim must be even")
    if out is None:
        out = torch.empty((rows, two_i // 2), dtype=gate_up.dtype, device=gate_up.device)
    _lib.check("lmrs_silu_mul", _lib.load().lmrs_silu_mul(
        _ptr(out), _ptr(gate_up), rows, two_i // 2, _code(gate_up), _stream(gate_up)))
    return out


def silu_mul_fp8(gate_up: torch.Tensor, q_out=None, scale_out=None):
    _require_cuda(gate_up, "gate_up")
    rows, two_i = gate_up.shape
    inter = two_i // 2
    if q_out is None:
        q_out = torch.empty((rows, inter), dtype=torch.uint8, device=gate_up.device)
    if scale_out is None:
        scale_out = torch.empty((rows,), dtype=torch.float32, device=gate_up.device)
    _lib.check("lmrs_silu_mul_fp8", _lib.load().lmrs_silu_mul_fp8(
        _ptr(q_out), _ptr(scale_out), _ptr(gate_up), rows, inter, _code(gate_up),
        _stream(gate_up)))
    return q_out, scale_out


def rope_kv_write(qkv: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                  key_cache: torch.Tensor, value_cache: torch.Tensor,
                  block_tables: torch.Tensor, positions: torch.Tensor, num_heads: int,
                  num_kv_heads: int, head_size: int, q_out: Optional[torch.Tensor] = None):
    """RoPE of q and k (cos/sin: head_size/2 entries for the step's position);
    returns q [num_seqs, num_heads, head_size], writes k and v into the paged
    cache [blocks, num_kv_heads, block_size, head_size] at positions."""
    _require_cuda(qkv, "qkv")
    seqs = qkv.shape[0]
    if q_out is None:
        q_out = torch.empty((seqs, num_heads, head_size), dtype=qkv.dtype, device=qkv.device)
    block_size = key_cache.shape[2]
    _lib.check("lmrs_rope_kv_write", _lib.load().lmrs_rope_kv_write(
        _ptr(q_out), _ptr(key_cache), _ptr(value_cache), _ptr(qkv), _ptr(cos), _ptr(sin),
        _ptr(block_tables), _ptr(positions), seqs, num_heads, num_kv_heads, head_size,
        block_size, block_tables.shape[1], _code(qkv), _stream(qkv)))
    return q_out


class AttentionWorkspace:
    """Grow-only split-context scratch for paged_attention_decode.  Zero-filled
    when (re)allocated: it holds the per-(sequence, KV head) arrival counters of
    the workspace merge, which every call leaves at zero again."""

    def __init__(self):
        self.buf = None

    def get(self, nbytes: int, device):
        if nbytes == 0:
            return None
        if self.buf is None or self.buf.numel() < nbytes or self.buf.device != device:
            self.buf = torch.zeros(nbytes, dtype=torch.uint8, device=device)
        return self.buf


def paged_attention_decode(query: torch.Tensor, key_cache: torch.Tensor,
                           value_cache: torch.Tensor, block_tables: torch.Tensor,
                           context_lens: torch.Tensor, max_context: int, scale: float,
                           kv_head_map: int = 1, workspace: Optional[AttentionWorkspace] = None,
                           out: Optional[torch.Tensor] = None):
    """query [seqs, heads, 128] against the paged cache; kv_head_map 1 = grouped
    heads (h / G), 0 = h % num_kv_heads (the reference's paged kernel)."""
    _require_cuda(query, "query")
    seqs, heads, d = query.shape
    num_kv_heads, block_size = key_cache.shape[1], key_cache.shape[2]
    lib = _lib.load()
    need = lib.lmrs_paged_attention_workspace_bytes(seqs, heads, num_kv_heads, max_context)
    ws = (workspace or AttentionWorkspace()).get(need, query.device)
    if out is None:
        out = torch.empty_like(query)
    _lib.check("lmrs_paged_attention_decode", lib.lmrs_paged_attention_decode(
        _ptr(out), _ptr(query), _ptr(key_cache), _ptr(value_cache), _ptr(block_tables),
        _ptr(context_lens), seqs, heads, num_kv_heads, d, block_size, block_tables.shape[1],
        int(max_context), float(scale), int(kv_head_map), _code(query), _ptr(ws), need,
        _stream(query)))
    return out


def paged_attention_decode_fp8(query: torch.Tensor, key_cache: torch.Tensor,
                               value_cache: torch.Tensor, block_tables: torch.Tensor,
                               context_lens: torch.Tensor, max_context: int, scale: float,
                               kv_head_map: int = 1,
                               workspace: Optional[AttentionWorkspace] = None):
    """paged_attention_decode, then the per-row e4m3 quantisation of its output
    rows [seqs, heads * 128] (the input of an FP8 o projection): returns (e4m3
    bytes, per-row fp32 scales, out).  One kernel when the cache has one KV head."""
    _require_cuda(query, "query")
    seqs, heads, d = query.shape
    num_kv_heads, block_size = key_cache.shape[1], key_cache.shape[2]
    lib = _lib.load()
    need = lib.lmrs_paged_attention_workspace_bytes(seqs, heads, num_kv_heads, max_context)
    ws = (workspace or AttentionWorkspace()).get(need, query.device)
    out = torch.empty_like(query)
    q = torch.empty((seqs, heads * d), dtype=torch.uint8, device=query.device)
    sc = torch.empty((seqs,), dtype=torch.float32, device=query.device)
    _lib.check("lmrs_paged_attention_decode_fp8", lib.lmrs_paged_attention_decode_fp8(
        _ptr(q), _ptr(sc), _ptr(out), _ptr(query), _ptr(key_cache), _ptr(value_cache),
        _ptr(block_tables), _ptr(context_lens), seqs, heads, num_kv_heads, d, block_size,
        block_tables.shape[1], int(max_context), float(scale), int(kv_head_map), _code(query),
        _ptr(ws), need, _stream(query)))
    return q, sc, out


def rope_paged_attention_decode(qkv: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                                key_cache: torch.Tensor, value_cache: torch.Tensor,
                                block_tables: torch.Tensor, context_lens: torch.Tensor,
                                max_context: int, num_heads: int, num_kv_heads: int,
                                scale: float, kv_head_map: int = 1,
                                workspace: Optional[AttentionWorkspace] = None,
                                fp8: bool = False):
    """rope_kv_write (positions = context_lens - 1) then paged_attention_decode in
    one kernel: qkv [seqs, (num_heads + 2 num_kv_heads) * 128] is the merged
    projection output.  Returns out [seqs, num_heads, 128]; with fp8=True
    (e4m3 bytes [seqs, num_heads * 128], per-row scales, out), as
    paged_attention_decode_fp8."""
    _require_cuda(qkv, "qkv")
    seqs, d = qkv.shape[0], 128
    block_size = key_cache.shape[2]
    lib = _lib.load()
    need = lib.lmrs_paged_attention_workspace_bytes(seqs, num_heads, num_kv_heads, max_context)
    ws = (workspace or AttentionWorkspace()).get(need, qkv.device)
    out = torch.empty((seqs, num_heads, d), dtype=qkv.dtype, device=qkv.device)
    q = sc = None
    if fp8:
        q = torch.empty((seqs, num_heads * d), dtype=torch.uint8, device=qkv.device)
        sc = torch.empty((seqs,), dtype=torch.float32, device=qkv.device)
    _lib.check("lmrs_rope_paged_attention_decode", lib.lmrs_rope_paged_attention_decode(
        _ptr(out), _ptr(q), _ptr(sc), _ptr(qkv), _ptr(cos), _ptr(sin), _ptr(key_cache),
        _ptr(value_cache), _ptr(block_tables), _ptr(context_lens), seqs, num_heads, num_kv_heads,
        d, block_size, block_tables.shape[1], int(max_context), float(scale), int(kv_head_map),
        _code(qkv), _ptr(ws), need, _stream(qkv)))
    return (q, sc, out) if fp8 else out


class Fp8DecodeLayer:
    """Host side of the persistent FP8 decode-layer kernel (include/lmrs_layer.h):
    the shapes, a prepared workspace, and one ``run`` per layer and step.

    Every tensor is bf16 except the e4m3 weights (uint8 [N, K]) and their fp32
    scales; the KV cache is [blocks, num_kv_heads, block_size, 128].  The
    workspace belongs to this object: calls that overlap on the GPU need
    separate objects."""

    def __init__(self, num_seqs: int, hidden: int, num_heads: int, num_kv_heads: int,
                 intermediate: int, block_size: int, max_blocks_per_seq: int, max_context: int,
                 eps: float, scale: float, device, head_size: int = 128):
        import ctypes
        self.shape = _lib.Fp8LayerShape(num_seqs, hidden, num_heads, num_kv_heads, head_size,
                                        intermediate, block_size, max_blocks_per_seq,
                                        max_context, float(eps), float(scale))
        self._sp = ctypes.byref(self.shape)
        lib = self.lib = _lib.load()
        self.nbytes = lib.lmrs_fp8_decode_layer_workspace_bytes(self._sp)
        if self.nbytes == 0:
            raise ShapeMismatch(f"decode-layer kernel: unsupported shapes {num_seqs} tokens, "
                                f"hidden {hidden}, heads {num_heads}/{num_kv_heads}, "
                                f"intermediate {intermediate}")
        self.num_seqs, self.hidden = num_seqs, hidden
        self.ws = torch.empty(self.nbytes, dtype=torch.uint8, device=device)
        if self.ws.data_ptr() % 256:
            raise ShapeMismatch("decode-layer workspace is not 256-byte aligned")
        self.prepare()

    def prepare(self):
        """(Re)initialise the workspace: barrier words and the unit schedule
        (synchronises the current stream; not inside a CUDA-graph capture)."""
        _lib.check("lmrs_fp8_decode_layer_prepare", self.lib.lmrs_fp8_decode_layer_prepare(
            self._sp, _ptr(self.ws), self.nbytes, _stream(self.ws)))

    @staticmethod
    def layer(qkv, o, gate_up, down, input_norm, post_norm, key_cache, value_cache):
        """lmrs_fp8_layer_t of one layer: qkv/o/gate_up/down are (e4m3 weight,
        fp32 scale) pairs.  The tensors must outlive every run that uses it."""
        for t in (*qkv, *o, *gate_up, *down, input_norm, post_norm, key_cache, value_cache):
            _require_cuda(t, "decode-layer tensor")
        lay = _lib.Fp8Layer(*[t.data_ptr() for t in (*qkv, *o, *gate_up, *down, input_norm,
                                                      post_norm, key_cache, value_cache)])
        lay._keep = (qkv, o, gate_up, down, input_norm, post_norm, key_cache, value_cache)
        return lay

    def run(self, layer, residual: torch.Tensor, delta_out: torch.Tensor,
            block_tables: torch.Tensor, context_lens: torch.Tensor, cos: torch.Tensor,
            sin: torch.Tensor, delta_in: Optional[torch.Tensor] = None, flags: int = 0,
            rank: int = 0, world: int = 1, bases=None, max_elems: int = 0):
        """One layer in place on residual [num_seqs, hidden]; the down projection's
        output goes to delta_out (or, with LAYER_PUSH_DELTA, to the ranks)."""
        import ctypes
        for t, n in ((residual, "residual"), (delta_out, "delta_out")):
            _require_cuda(t, n)
            if t.dtype != torch.bfloat16 or t.shape != (self.num_seqs, self.hidden):
                raise ShapeMismatch(f"{n}: bf16 [{self.num_seqs}, {self.hidden}]")
        _lib.check("lmrs_fp8_decode_layer", self.lib.lmrs_fp8_decode_layer(
            ctypes.byref(layer), self._sp, _ptr(residual), _ptr(delta_in), _ptr(delta_out),
            int(flags), _ptr(block_tables), _ptr(context_lens), _ptr(cos), _ptr(sin), int(rank),
            int(world), bases, int(max_elems), _ptr(self.ws), self.nbytes, _stream(residual)))
        return residual
