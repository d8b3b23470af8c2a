"""The C-ABI library on a machine without a GPU: it loads, exports exactly the
symbols the headers in include/ declare, and rejects bad
arguments with the documented status codes before touching the device (no
compute is launched)."""
import ctypes
import pathlib
import re

import pytest

from lmrs_b200 import _lib

ROOT = pathlib.Path(__file__).resolve().parent.parent
HEADERS = sorted((ROOT / "include").glob("*.h"))


def header_symbols():
    text = "".join(h.read_text() for h in HEADERS)
    return set(re.findall(r"LMRS_API\s+[\w\s\*]*?\b(lmrs_\w+)\s*\(", text))


def test_library_loads_and_exports_header():
    lib = _lib.load()
    syms = header_symbols()
    assert len(syms) >= 12
    for s in syms:
        assert hasattr(lib, s), s
    assert set(_lib.SIGNATURES) == syms
    assert lib.lmrs_version() >= 1


def test_status_strings():
    for code in range(10):
        assert _lib.status_string(code)
    assert "sm_100" in _lib.status_string(_lib.LMRS_ERR_DEVICE)


FAKE = ctypes.c_void_p(0x10000)  # 16-byte aligned, never dereferenced


def test_awq_validation_codes():
    lib = _lib.load()
    f = lib.lmrs_awq_linear
    # act dtype must be bf16 (0) or fp16 (1); f32 (2) and unknown codes are rejected
    assert f(FAKE, FAKE, FAKE, FAKE, FAKE, None, 4, 256, 64, 128, 2, None, 0, None) == _lib.LMRS_ERR_DTYPE
    assert f(FAKE, FAKE, FAKE, FAKE, FAKE, None, 4, 256, 64, 128, 7, None, 0, None) == _lib.LMRS_ERR_DTYPE
    # N % 32, for both activation types
    for act in (0, 1):
        assert f(FAKE, FAKE, FAKE, FAKE, FAKE, None, 4, 256, 40, 128, act, None, 0,
                 None) == _lib.LMRS_ERR_SHAPE
    # the bf16 dequant rejects f32 output and the same shape errors
    d = lib.lmrs_awq_dequant_dtype
    assert d(FAKE, FAKE, FAKE, FAKE, 256, 64, 128, 2, None) == _lib.LMRS_ERR_DTYPE
    assert d(FAKE, FAKE, FAKE, FAKE, 256, 60, 128, 0, None) == _lib.LMRS_ERR_SHAPE
    assert d(FAKE, FAKE, FAKE, FAKE, 200, 64, 128, 0, None) == _lib.LMRS_ERR_GROUP
    # group must divide K and be a multiple of 64
    assert f(FAKE, FAKE, FAKE, FAKE, FAKE, None, 4, 256, 64, 96, 1, None, 0, None) == _lib.LMRS_ERR_GROUP
    assert f(FAKE, FAKE, FAKE, FAKE, FAKE, None, 4, 192, 64, 128, 1, None, 0, None) == _lib.LMRS_ERR_GROUP
    # NULL and misaligned pointers
    assert f(None, FAKE, FAKE, FAKE, FAKE, None, 4, 256, 64, 128, 1, None, 0, None) == _lib.LMRS_ERR_NULL
    assert f(ctypes.c_void_p(0x10002), FAKE, FAKE, FAKE, FAKE, None, 4, 256, 64, 128, 1, None, 0,
             None) == _lib.LMRS_ERR_ALIGN
    # M == 0 is a successful no-op
    assert f(FAKE, FAKE, FAKE, FAKE, FAKE, None, 0, 256, 64, 128, 1, None, 0, None) == _lib.LMRS_OK
    assert lib.lmrs_awq_linear_workspace_bytes(16, 4096, 14336, 128) == 0


def test_awq_pack_validation_codes():
    lib = _lib.load()
    assert lib.lmrs_awq_unpack(FAKE, FAKE, 4, 12, None) == _lib.LMRS_ERR_SHAPE
    assert lib.lmrs_awq_unpack(FAKE, FAKE, 0, 16, None) == _lib.LMRS_OK
    assert lib.lmrs_awq_dequant(FAKE, FAKE, FAKE, FAKE, 100, 64, 64, None) == _lib.LMRS_ERR_GROUP
    assert lib.lmrs_awq_dequant(FAKE, FAKE, FAKE, FAKE, 128, 60, 64, None) == _lib.LMRS_ERR_SHAPE


def test_fp8_validation_codes():
    lib = _lib.load()
    need = lib.lmrs_fp8_linear_workspace_bytes(4, 256, 64)
    assert need >= 4 * 256 + 4 * 4 and need % 256 == 0
    f = lib.lmrs_fp8_linear
    assert f(FAKE, FAKE, FAKE, FAKE, None, 4, 250, 64, FAKE, need, None) == _lib.LMRS_ERR_SHAPE
    assert f(FAKE, FAKE, FAKE, FAKE, None, 4, 256, 64, FAKE, need - 1, None) == _lib.LMRS_ERR_WORKSPACE
    assert f(FAKE, FAKE, FAKE, FAKE, None, 4, 256, 64, None, need, None) == _lib.LMRS_ERR_WORKSPACE
    assert f(FAKE, FAKE, FAKE, FAKE, None, 0, 256, 64, None, 0, None) == _lib.LMRS_OK
    assert lib.lmrs_fp8_quant_rows(FAKE, FAKE, FAKE, 4, 256, 7, None) == _lib.LMRS_ERR_DTYPE
    assert lib.lmrs_fp8_quant_rows(FAKE, FAKE, FAKE, 4, 24, 0, None) == _lib.LMRS_ERR_SHAPE


def test_valid_call_without_gpu_fails_cleanly():
    """Arguments that pass validation reach the device check, which reports a
    CUDA error (no device here) instead of launching or crashing."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("has a GPU")
    lib = _lib.load()
    rc = lib.lmrs_awq_linear(FAKE, FAKE, FAKE, FAKE, FAKE, None, 4, 256, 64, 128, 1, None, 0, None)
    assert rc in (_lib.LMRS_ERR_CUDA, _lib.LMRS_ERR_DEVICE)


def test_tuning_keys():
    assert _lib.load().lmrs_set_tuning(b"no_such_key", 1) == _lib.LMRS_ERR_SHAPE
    _lib.set_tuning("awq_gemv_max_m", 16)


def test_decode_layer_validation_codes():
    """lmrs_fp8_decode_layer checks shapes, flags and pointers before the device."""
    import torch
    lib = _lib.load()
    f = lib.lmrs_fp8_decode_layer
    ptr = 0x10000
    lay = _lib.Fp8Layer(*[ptr + 256 * i for i in range(12)])

    def shape(**kw):
        base = dict(num_seqs=2, hidden=1024, num_heads=8, num_kv_heads=1, head_size=128,
                    intermediate=768, block_size=16, max_blocks_per_seq=8, max_context=128)
        base.update(kw)
        return _lib.Fp8LayerShape(*base.values(), 1e-5, 0.088)

    def call(sh, layer=lay, flags=0, world=1, bufs=None, delta_out=FAKE, ws=FAKE):
        return f(ctypes.byref(layer) if layer is not None else None, ctypes.byref(sh), FAKE, None,
                 delta_out, flags, FAKE, FAKE, FAKE, FAKE, 0, world, bufs, 1 << 20, ws, 1 << 30, None)

    assert call(shape(), layer=None) == _lib.LMRS_ERR_NULL
    for bad in (dict(num_seqs=9), dict(num_seqs=0), dict(head_size=64), dict(num_heads=12),
                dict(num_heads=16, num_kv_heads=1), dict(hidden=1000), dict(intermediate=100),
                dict(block_size=0), dict(max_context=0), dict(num_seqs=8, intermediate=16384)):
        assert call(shape(**bad)) == _lib.LMRS_ERR_SHAPE, bad
    assert call(shape(), flags=_lib.LAYER_PUSH_DELTA) == _lib.LMRS_ERR_SHAPE  # flags need world > 1
    assert call(shape(), flags=4, world=2) == _lib.LMRS_ERR_SHAPE
    assert call(shape(), delta_out=None) == _lib.LMRS_ERR_NULL
    assert call(shape(), ws=None) == _lib.LMRS_ERR_NULL
    assert call(shape(), world=2) == _lib.LMRS_ERR_NULL  # no all-reduce buffers
    assert call(shape(), delta_out=ctypes.c_void_p(0x10008)) == _lib.LMRS_ERR_ALIGN
    if not torch.cuda.is_available():
        assert call(shape()) in (_lib.LMRS_ERR_CUDA, _lib.LMRS_ERR_DEVICE)
        assert lib.lmrs_fp8_decode_layer_workspace_bytes(ctypes.byref(shape())) == 0
