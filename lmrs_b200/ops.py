"""Operator layer of the quantized linear — the host side above the C-ABI.

Mirrors the reference's linear operator stack so a caller of one finds the
other:

* ``LinearConfig``                  <- crates/ops/src/linear/linear.rs:5-12
* ``QuantLinearOp`` (new/forward/...) <- ``LinearOp`` crates/ops/src/linear/linear.rs:15-46,
  with ``validate_shape`` (:48-66) extended to the AWQ and FP8 tensor sets
* ``awq_linear`` / ``fp8_linear``    <- ``kernels::linear`` crates/kernels/src/tensor_ops.rs:225-246:
  contiguity + dtype checks (:453-468), rows = numel / in_features, output
  allocated (uninitialised) on the input's device and stream, one C-ABI call.
* errors: ``ShapeMismatch`` / ``DTypeMismatch`` / ``NonContiguous`` mirror the
  reference's ``TensorError`` variants; a nonzero C-ABI status raises
  ``LmrsError``.

Tensors are torch CUDA tensors (torch is the device-memory / stream plumbing
here, playing the role of the reference's cudarc ``CudaBuf``); all arithmetic
runs in ``liblmrs_quant.so``.  There is no CPU path: CPU tensors are rejected.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Optional

import torch

from . import _lib

AWQ_PACK_FACTOR = 8  # int4 values per int32 word


class TensorError(ValueError):
    pass


class ShapeMismatch(TensorError):
    pass


class DTypeMismatch(TensorError):
    pass


class NonContiguous(TensorError):
    pass


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(t: torch.Tensor):
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def _require_cuda(t: torch.Tensor, what: str):
    if not t.is_cuda:
        raise TensorError(f"{what}: tensor must live on a CUDA device (no CPU path)")
    if not t.is_contiguous():
        raise NonContiguous(f"{what}: tensor must be contiguous")


def _require_dtype(t: torch.Tensor, dtype: torch.dtype, what: str):
    if t.dtype != dtype:
        raise DTypeMismatch(f"{what}: expected {dtype}, got {t.dtype}")


# ---------------------------------------------------------------- kernels layer
def awq_unpack(packed: torch.Tensor, cols: Optional[int] = None) -> torch.Tensor:
    """int32 [R, C/8] AWQ-packed -> int8 [R, C] in natural column order."""
    _require_cuda(packed, "awq_unpack")
    _require_dtype(packed, torch.int32, "awq_unpack")
    rows, words = packed.shape
    cols = words * AWQ_PACK_FACTOR if cols is None else cols
    out = torch.empty((rows, cols), dtype=torch.int8, device=packed.device)
    _lib.check("lmrs_awq_unpack", _lib.load().lmrs_awq_unpack(
        _ptr(out), _ptr(packed), rows, cols, _stream(packed)))
    return out


# activation dtypes of the AWQ linear -> KernelDType code (crates/kernels/src/raw.rs:9-13)
AWQ_ACT_DTYPES = {torch.bfloat16: _lib.DTYPE_BF16, torch.float16: _lib.DTYPE_F16}


def awq_dequant(qweight, qzeros, scales, group_size: int,
                dtype: torch.dtype = torch.float16) -> torch.Tensor:
    """[K, N] = dtype_rne((q - z) * s) (fp16 or bf16; scales fp16), bit-exact."""
    for t, n in ((qweight, "qweight"), (qzeros, "qzeros"), (scales, "scales")):
        _require_cuda(t, "awq_dequant " + n)
    if dtype not in AWQ_ACT_DTYPES:
        raise DTypeMismatch(f"awq_dequant: dtype must be fp16 or bf16, got {dtype}")
    K, words = qweight.shape
    N = words * AWQ_PACK_FACTOR
    out = torch.empty((K, N), dtype=dtype, device=qweight.device)
    _lib.check("lmrs_awq_dequant_dtype", _lib.load().lmrs_awq_dequant_dtype(
        _ptr(out), _ptr(qweight), _ptr(qzeros), _ptr(scales), K, N, group_size,
        AWQ_ACT_DTYPES[dtype], _stream(qweight)))
    return out


def awq_linear(x: torch.Tensor, qweight: torch.Tensor, qzeros: torch.Tensor,
               scales: torch.Tensor, bias: Optional[torch.Tensor], group_size: int,
               out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """y[..., N] = x[..., K] @ dequant(AWQ) (+ bias); x, y and bias share one
    dtype, bf16 (the reference model's) or fp16; scales fp16."""
    _require_cuda(x, "awq_linear")
    if x.dtype not in AWQ_ACT_DTYPES:
        raise DTypeMismatch(f"awq_linear input: expected bf16 or fp16, got {x.dtype}")
    for t, n in ((qweight, "qweight"), (qzeros, "qzeros")):
        _require_cuda(t, "awq_linear " + n)
        _require_dtype(t, torch.int32, "awq_linear " + n)
    _require_cuda(scales, "awq_linear scales")
    _require_dtype(scales, torch.float16, "awq_linear scales")
    if x.dim() < 1:
        raise ShapeMismatch("linear input needs rank >= 1")
    K = x.shape[-1]
    if qweight.shape[0] != K:
        raise ShapeMismatch("linear input and weight dimensions mismatch")
    N = qweight.shape[1] * AWQ_PACK_FACTOR
    rows = x.numel() // K if K else 0
    if out is None:
        out = torch.empty((*x.shape[:-1], N), dtype=x.dtype, device=x.device)
    _require_dtype(out, x.dtype, "awq_linear output")
    if bias is not None:
        _require_cuda(bias, "awq_linear bias")
        _require_dtype(bias, x.dtype, "awq_linear bias")
    L = _lib.load()
    ws_bytes = L.lmrs_awq_linear_workspace_bytes(rows, K, N, group_size)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=x.device) if ws_bytes else None
    _lib.check("lmrs_awq_linear", L.lmrs_awq_linear(
        _ptr(out), _ptr(x), _ptr(qweight), _ptr(qzeros), _ptr(scales), _ptr(bias),
        rows, K, N, group_size, AWQ_ACT_DTYPES[x.dtype], _ptr(ws), ws_bytes, _stream(x)))
    return out


def fp8_quant_rows(x: torch.Tensor):
    """Per-row e4m3: returns (q uint8 [R, K], scale fp32 [R])."""
    _require_cuda(x, "fp8_quant_rows")
    code = {torch.bfloat16: _lib.DTYPE_BF16, torch.float16: _lib.DTYPE_F16,
            torch.float32: _lib.DTYPE_F32}.get(x.dtype)
    if code is None:
        raise DTypeMismatch(f"fp8_quant_rows: expected bf16/f16/f32, got {x.dtype}")
    K = x.shape[-1]
    rows = x.numel() // K if K else 0
    q = torch.empty((*x.shape[:-1], K), dtype=torch.uint8, device=x.device)
    s = torch.empty(x.shape[:-1], dtype=torch.float32, device=x.device)
    _lib.check("lmrs_fp8_quant_rows", _lib.load().lmrs_fp8_quant_rows(
        _ptr(q), _ptr(s), _ptr(x), rows, K, code, _stream(x)))
    return q, s


class Workspace:
    """Grow-only device scratch buffer, owned by the caller (the C-ABI never allocates)."""

    def __init__(self):
        self.buf: Optional[torch.Tensor] = None

    def get(self, nbytes: int, device) -> Optional[torch.Tensor]:
        if nbytes == 0:
            return None
        if self.buf is None or self.buf.numel() < nbytes or self.buf.device != torch.device(device):
            self.buf = torch.empty(nbytes, dtype=torch.uint8, device=device)
        return self.buf


def fp8_linear(x: torch.Tensor, weight_q: torch.Tensor, weight_scale: torch.Tensor,
               bias: Optional[torch.Tensor] = None, workspace: Optional[Workspace] = None,
               out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """y bf16 [..., N] = per-token-e4m3(x bf16 [..., K]) @ weight_q^T, scaled."""
    _require_cuda(x, "fp8_linear")
    _require_dtype(x, torch.bfloat16, "fp8_linear input")
    _require_cuda(weight_q, "fp8_linear weight")
    _require_dtype(weight_q, torch.uint8, "fp8_linear weight (e4m3 bytes)")
    _require_cuda(weight_scale, "fp8_linear weight_scale")
    _require_dtype(weight_scale, torch.float32, "fp8_linear weight_scale")
    K = x.shape[-1]
    N, Kw = weight_q.shape
    if Kw != K:
        raise ShapeMismatch("linear input and weight dimensions mismatch")
    if bias is not None:
        _require_cuda(bias, "fp8_linear bias")
        _require_dtype(bias, torch.bfloat16, "fp8_linear bias")
    rows = x.numel() // K if K else 0
    if out is None:
        out = torch.empty((*x.shape[:-1], N), dtype=torch.bfloat16, device=x.device)
    L = _lib.load()
    ws_bytes = L.lmrs_fp8_linear_workspace_bytes(rows, K, N)
    ws = (workspace or Workspace()).get(ws_bytes, x.device)
    _lib.check("lmrs_fp8_linear", L.lmrs_fp8_linear(
        _ptr(out), _ptr(x), _ptr(weight_q), _ptr(weight_scale), _ptr(bias), rows, K, N,
        _ptr(ws), ws_bytes, _stream(x)))
    return out


def fp8_linear_prequant(xq: torch.Tensor, x_scale: torch.Tensor, weight_q: torch.Tensor,
                        weight_scale: torch.Tensor, bias: Optional[torch.Tensor] = None,
                        out: Optional[torch.Tensor] = None) -> torch.Tensor:
    _require_cuda(xq, "fp8_linear_prequant")
    _require_dtype(xq, torch.uint8, "fp8_linear_prequant input (e4m3 bytes)")
    K = xq.shape[-1]
    N = weight_q.shape[0]
    rows = xq.numel() // K if K else 0
    if out is None:
        out = torch.empty((*xq.shape[:-1], N), dtype=torch.bfloat16, device=xq.device)
    _lib.check("lmrs_fp8_linear_prequant", _lib.load().lmrs_fp8_linear_prequant(
        _ptr(out), _ptr(xq), _ptr(x_scale), _ptr(weight_q), _ptr(weight_scale), _ptr(bias),
        rows, K, N, _stream(xq)))
    return out


# ------------------------------------------------------------------ ops layer
@dataclass(frozen=True)
class LinearConfig:
    """Linear projection configuration (crates/ops/src/linear/linear.rs:5-12)."""
    in_features: int
    out_features: int
    bias: bool = False


@dataclass(frozen=True)
class AwqConfig:
    """AutoAWQ-style quantisation config (the reference reads none; new)."""
    group_size: int = 128
    bits: int = 4


class QuantLinearOp:
    """Quantized linear projection over the final input dimension.

    Sits beside the reference's ``LinearOp`` (crates/ops/src/linear/linear.rs:15-46)
    with the same surface: ``new``-style validated constructors, ``from_parts``,
    ``forward``, ``weight``, ``bias``.  ``kind`` is ``"awq"`` or ``"fp8"``.
    """

    def __init__(self, kind: str, config: LinearConfig, tensors: dict,
                 bias: Optional[torch.Tensor], awq: Optional[AwqConfig] = None):
        self.kind = kind
        self.config = config
        self.tensors = tensors
        self._bias = bias
        self.awq_config = awq
        self._ws = Workspace()

    # -- constructors (validated, like LinearOp::new)
    @classmethod
    def awq(cls, config: LinearConfig, qweight, qzeros, scales, bias=None,
            awq: AwqConfig = AwqConfig()) -> "QuantLinearOp":
        validate_awq_shape(config, awq, qweight, qzeros, scales, bias)
        return cls("awq", config, dict(qweight=qweight, qzeros=qzeros, scales=scales), bias, awq)

    @classmethod
    def fp8(cls, config: LinearConfig, weight_q, weight_scale, bias=None) -> "QuantLinearOp":
        validate_fp8_shape(config, weight_q, weight_scale, bias)
        return cls("fp8", config, dict(weight_q=weight_q, weight_scale=weight_scale), bias)

    @classmethod
    def from_parts(cls, kind: str, tensors: dict, bias=None, awq: Optional[AwqConfig] = None):
        """Wraps existing tensors without validation (LinearOp::from_parts)."""
        if kind == "awq":
            K, w = tensors["qweight"].shape
            cfg = LinearConfig(K, w * AWQ_PACK_FACTOR, bias is not None)
        else:
            N, K = tensors["weight_q"].shape
            cfg = LinearConfig(K, N, bias is not None)
        return cls(kind, cfg, tensors, bias, awq or (AwqConfig() if kind == "awq" else None))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        t = self.tensors
        if self.kind == "awq":
            return awq_linear(x, t["qweight"], t["qzeros"], t["scales"], self._bias,
                              self.awq_config.group_size)
        return fp8_linear(x, t["weight_q"], t["weight_scale"], self._bias, self._ws)

    __call__ = forward

    def forward_prequant(self, xq: torch.Tensor, x_scale: torch.Tensor) -> torch.Tensor:
        """FP8 only: the activations already quantised per token (e4m3 bytes and
        fp32 scales, e.g. by a fused norm or activation kernel)."""
        if self.kind != "fp8":
            raise DTypeMismatch("forward_prequant applies to FP8 W8A8 projections")
        t = self.tensors
        return fp8_linear_prequant(xq, x_scale, t["weight_q"], t["weight_scale"], self._bias)

    def weight(self) -> dict:
        return self.tensors

    def bias(self) -> Optional[torch.Tensor]:
        return self._bias


def validate_awq_shape(config: LinearConfig, awq: AwqConfig, qweight, qzeros, scales, bias):
    K, N, g = config.in_features, config.out_features, awq.group_size
    if awq.bits != 4:
        raise ShapeMismatch(f"awq: only 4-bit weights are supported, got {awq.bits}")
    if N % AWQ_PACK_FACTOR or g <= 0 or K % g:
        raise ShapeMismatch(f"awq: out_features % 8 and in_features % group_size must be 0 "
                            f"(K={K}, N={N}, group={g})")
    want = {"qweight": (K, N // 8), "qzeros": (K // g, N // 8), "scales": (K // g, N)}
    for name, t in (("qweight", qweight), ("qzeros", qzeros), ("scales", scales)):
        if tuple(t.shape) != want[name]:
            raise ShapeMismatch(f"awq {name} must have shape {list(want[name])}, got {list(t.shape)}")
    if bias is not None and tuple(bias.shape) != (N,):
        raise ShapeMismatch(f"linear bias must have shape [{N}], got {list(bias.shape)}")


def validate_fp8_shape(config: LinearConfig, weight_q, weight_scale, bias):
    N, K = config.out_features, config.in_features
    if tuple(weight_q.shape) != (N, K):
        raise ShapeMismatch(f"linear weight must have shape [{N}, {K}], got {list(weight_q.shape)}")
    if tuple(weight_scale.shape) != (N,):
        raise ShapeMismatch(f"fp8 weight_scale must have shape [{N}], got {list(weight_scale.shape)}")
    if bias is not None and tuple(bias.shape) != (N,):
        raise ShapeMismatch(f"linear bias must have shape [{N}], got {list(bias.shape)}")


def quantize_fp8_weight(w_bf16: torch.Tensor):
    """Load-time per-output-channel e4m3 quantisation of a bf16 [N, K] weight."""
    return fp8_quant_rows(w_bf16.contiguous())
