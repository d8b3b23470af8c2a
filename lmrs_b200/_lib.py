"""ctypes binding of the C-ABI in ``include/lmrs_quant.h``, ``include/lmrs_decode.h``,
``include/lmrs_comm.h`` and ``include/lmrs_layer.h``.

This is the Python counterpart of the reference's raw FFI declarations
(crates/kernels/src/tensor_ops.rs:8-22, crates/kernels/src/raw.rs:53-147): one
foreign declaration per exported symbol, no logic.  Loading fails loudly: there
is no CPU fallback anywhere in the package.
"""
from __future__ import annotations

import ctypes
import pathlib

PKG = pathlib.Path(__file__).resolve().parent
LIB_PATH = PKG / "liblmrs_quant.so"

# status codes (lmrs_quant.h)
LMRS_OK = 0
LMRS_ERR_SHAPE = 1
LMRS_ERR_DTYPE = 2
LMRS_ERR_ALIGN = 3
LMRS_ERR_GROUP = 4
LMRS_ERR_WORKSPACE = 5
LMRS_ERR_CUDA = 6
LMRS_ERR_DEVICE = 7
LMRS_ERR_NULL = 8
LMRS_ERR_TIMEOUT = 9
LMRS_ERR_TOO_LARGE = 10
FP8_NOALLOC_SCRATCH_BYTES = 4 * 1024 * 1024

# KernelDType (crates/kernels/src/raw.rs:9-13)
DTYPE_BF16 = 0
DTYPE_F16 = 1
DTYPE_F32 = 2

P = ctypes.c_void_p
I = ctypes.c_int
SZ = ctypes.c_size_t

F = ctypes.c_float

# name -> (restype, argtypes); mirrors include/lmrs_{quant,decode,comm,layer}.h exactly
SIGNATURES = {
    "lmrs_version": (I, []),
    "lmrs_status_string": (ctypes.c_char_p, [I]),
    "lmrs_last_cuda_error": (I, []),
    "lmrs_read_device_error": (I, [ctypes.POINTER(I)]),
    "lmrs_set_tuning": (I, [ctypes.c_char_p, I]),
    "lmrs_awq_unpack": (I, [P, P, I, I, P]),
    "lmrs_awq_dequant": (I, [P, P, P, P, I, I, I, P]),
    "lmrs_awq_dequant_dtype": (I, [P, P, P, P, I, I, I, I, P]),
    "lmrs_awq_linear_workspace_bytes": (SZ, [I, I, I, I]),
    "lmrs_awq_linear": (I, [P, P, P, P, P, P, I, I, I, I, I, P, SZ, P]),
    "lmrs_fp8_quant_rows": (I, [P, P, P, I, I, I, P]),
    "lmrs_fp8_linear_workspace_bytes": (SZ, [I, I, I]),
    "lmrs_fp8_linear": (I, [P, P, P, P, P, I, I, I, P, SZ, P]),
    "lmrs_fp8_linear_prequant": (I, [P, P, P, P, P, P, I, I, I, P]),
    "lmrs_fp8_linear_noalloc": (I, [P, P, P, P, P, I, I, I, P]),
    # lmrs_decode.h
    "lmrs_rmsnorm": (I, [P, P, P, P, I, I, F, I, P]),
    "lmrs_rmsnorm_fp8": (I, [P, P, P, P, P, I, I, F, I, P]),
    "lmrs_silu_mul": (I, [P, P, I, I, I, P]),
    "lmrs_silu_mul_fp8": (I, [P, P, P, I, I, I, P]),
    "lmrs_rope_kv_write": (I, [P, P, P, P, P, P, P, P, I, I, I, I, I, I, I, P]),
    "lmrs_paged_attention_workspace_bytes": (SZ, [I, I, I, I]),
    "lmrs_paged_attention_decode": (I, [P, P, P, P, P, P, I, I, I, I, I, I, I, F, I, I, P, SZ, P]),
    "lmrs_paged_attention_decode_fp8": (I, [P, P, P, P, P, P, P, P, I, I, I, I, I, I, I, F, I, I, P, SZ, P]),
    "lmrs_rope_paged_attention_decode": (I, [P, P, P, P, P, P, P, P, P, P, I, I, I, I, I, I, I, F, I, I,
                                              P, SZ, P]),
    # lmrs_comm.h
    "lmrs_allreduce_buffer_bytes": (SZ, [I, SZ]),
    "lmrs_comm_alloc": (I, [ctypes.POINTER(P), SZ]),
    "lmrs_comm_free": (I, [P]),
    "lmrs_ipc_get_handle": (I, [P, P, SZ]),
    "lmrs_ipc_open": (I, [P, ctypes.POINTER(P)]),
    "lmrs_ipc_close": (I, [P]),
    "lmrs_allreduce_sum": (I, [P, P, SZ, I, I, I, P, SZ, P]),
    "lmrs_allreduce_rmsnorm": (I, [P, P, P, P, I, I, F, I, I, I, P, SZ, P]),
    "lmrs_allreduce_rmsnorm_fp8": (I, [P, P, P, P, P, I, I, F, I, I, I, P, SZ, P]),
    # lmrs_layer.h (struct arguments by pointer: Fp8Layer, Fp8LayerShape below)
    "lmrs_fp8_decode_layer_workspace_bytes": (SZ, [P]),
    "lmrs_fp8_decode_layer_prepare": (I, [P, P, SZ, P]),
    "lmrs_fp8_decode_layer": (I, [P, P, P, P, P, I, P, P, P, P, I, I, P, SZ, P, SZ, P]),
}

# lmrs_layer.h
LAYER_RECV_DELTA = 1
LAYER_PUSH_DELTA = 2


class Fp8Layer(ctypes.Structure):
    """lmrs_fp8_layer_t: one layer's device pointers."""
    _fields_ = [(n, P) for n in (
        "qkv_weight", "qkv_scale", "o_weight", "o_scale", "gate_up_weight", "gate_up_scale",
        "down_weight", "down_scale", "input_norm", "post_norm", "key_cache", "value_cache")]


class Fp8LayerShape(ctypes.Structure):
    """lmrs_fp8_layer_shape_t."""
    _fields_ = [(n, I) for n in (
        "num_seqs", "hidden", "num_heads", "num_kv_heads", "head_size", "intermediate",
        "block_size", "max_blocks_per_seq", "max_context")] + [("eps", F), ("scale", F)]


class LmrsError(RuntimeError):
    """A nonzero status from the C-ABI."""

    def __init__(self, fn: str, status: int, detail: str = ""):
        self.status = status
        super().__init__(f"{fn}: {status_string(status)} (status {status}){detail}")


_LIB = None


def load() -> ctypes.CDLL:
    """Load the in-tree library; raise ImportError if it has not been built."""
    global _LIB
    if _LIB is not None:
        return _LIB
    if not LIB_PATH.exists():
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python -m lmrs_b200.build` "
            "(the quantized linears have no CPU fallback)")
    lib = ctypes.CDLL(str(LIB_PATH))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _LIB = lib
    return lib


def status_string(status: int) -> str:
    return load().lmrs_status_string(int(status)).decode()


def check(fn: str, status: int) -> None:
    if status != LMRS_OK:
        detail = ""
        if status == LMRS_ERR_CUDA:
            detail = f"; cuda error {load().lmrs_last_cuda_error()}"
        raise LmrsError(fn, status, detail)


def read_device_error() -> int:
    v = I(0)
    check("lmrs_read_device_error", load().lmrs_read_device_error(ctypes.byref(v)))
    return v.value


def set_tuning(key: str, value: int) -> None:
    check("lmrs_set_tuning", load().lmrs_set_tuning(key.encode(), int(value)))
