"""CPU oracle for the quantized-linear hot path (TEST INFRASTRUCTURE ONLY).

Two independent restatements of the same arithmetic:

* ``np_*`` functions: numpy, vectorised, used to cross-check the C oracle and
  to build golden fixtures;
* ``c_*`` functions: ctypes wrappers over ``oracle/liblmrs_oracle.so`` (built by
  ``oracle/Makefile`` from ``oracle/lmrs_oracle.c``), fast enough for the
  full-size parity inputs and used as the timed CPU baseline.

The dense-linear arithmetic follows the reference's ``linear_kernel``
(kernels/ffi/tensor_ffi.cu:229-257): fp32 accumulator seeded with the bias,
``acc += x * w`` over k in order (contracted to one FMA by nvcc), one rounding
to the I/O dtype.  The AWQ and FP8 formats are not in the reference; they follow
the task's config text (see ``lmrs_oracle.c``'s header).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline /
reference legs import this module.  The ``lmrs_b200`` package never does.
"""
from __future__ import annotations

import ctypes
import os
import pathlib

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
AWQ_ORDER = np.array([0, 2, 4, 6, 1, 3, 5, 7], dtype=np.int64)
AWQ_INV = np.argsort(AWQ_ORDER)  # column -> nibble: [0,4,1,5,2,6,3,7]
E4M3_MAX = 448.0


# ----------------------------------------------------------------- generators
def awq_inputs(M, K, N, group=128, seed=0, with_bias=False, act="f16"):
    """Seeded AWQ inputs with the config-0 distributions.

    Draw order (recorded convention): q, then z, then s, then x (then bias).
    q, z ~ U{0..15}; s ~ U[0.001, 0.02] as fp16; x ~ N(0, 1) in the activation
    type: fp16 (act="f16"), or bf16 bit patterns as uint16 (act="bf16", the
    same draws rounded to bf16 instead).
    """
    rng = np.random.default_rng(seed)
    q = rng.integers(0, 16, size=(K, N), dtype=np.int64).astype(np.int8)
    z = rng.integers(0, 16, size=(K // group, N), dtype=np.int64).astype(np.int8)
    s = rng.uniform(0.001, 0.02, size=(K // group, N)).astype(np.float16)
    xd = rng.standard_normal((M, K))
    bd = rng.standard_normal(N) if with_bias else None
    if act == "bf16":
        x = f32_to_bf16_bits(xd.astype(np.float32))
        bias = None if bd is None else f32_to_bf16_bits(bd.astype(np.float32))
    else:
        x = xd.astype(np.float16)
        bias = None if bd is None else bd.astype(np.float16)
    return dict(q=q, z=z, qweight=np_awq_pack(q), qzeros=np_awq_pack(z), scales=s,
                x=x, bias=bias, M=M, K=K, N=N, group=group, act=act)


def fp8_inputs(M, K, N, seed=0, with_bias=False):
    """Seeded FP8 inputs with the config-2 distributions (draw order: W, then X).

    W ~ N(0, 0.02) as bf16 [N, K]; X ~ N(0, 1) as bf16 [M, K].  bf16 values are
    held as uint16 bit patterns (numpy has no bf16).
    """
    rng = np.random.default_rng(seed)
    w = f32_to_bf16_bits(rng.normal(0.0, 0.02, size=(N, K)).astype(np.float32))
    x = f32_to_bf16_bits(rng.standard_normal((M, K)).astype(np.float32))
    bias = (f32_to_bf16_bits(rng.standard_normal(N).astype(np.float32))
            if with_bias else None)
    return dict(w_bf16=w, x_bf16=x, bias_bf16=bias, M=M, K=K, N=N)


# --------------------------------------------------------------- bf16 helpers
def f32_to_bf16_bits(a):
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    return np.where(nan, ((u >> 16) | 0x40).astype(np.uint16), r)


def bf16_bits_to_f32(b):
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


# ----------------------------------------------------------------- numpy AWQ
def np_awq_pack(q):
    """int4 values [R, C] (column order natural) -> int32 [R, C/8], AWQ order."""
    q = np.asarray(q).astype(np.uint32) & 0xF
    R, C = q.shape
    q = q.reshape(R, C // 8, 8)[:, :, AWQ_ORDER]  # nibble i holds column ORDER[i]
    shifts = (4 * np.arange(8, dtype=np.uint32))
    return (q << shifts).sum(axis=2, dtype=np.uint64).astype(np.uint32).view(np.int32)


def np_awq_unpack(packed):
    p = np.asarray(packed).view(np.uint32)
    R, W = p.shape
    nib = (p[:, :, None] >> (4 * np.arange(8, dtype=np.uint32))) & 0xF  # [R, W, nibble]
    return nib[:, :, AWQ_INV].reshape(R, W * 8).astype(np.int8)


def np_awq_dequant(qweight, qzeros, scales, group, act="f16"):
    """[K, N] = T_rne(float32(q - z) * float32(s)); the fp32 product is exact.
    act="f16": fp16 array; act="bf16": bf16 bit patterns (uint16)."""
    q = np_awq_unpack(qweight).astype(np.int32)
    z = np_awq_unpack(qzeros).astype(np.int32)
    zk = np.repeat(z, group, axis=0)
    sk = np.repeat(np.asarray(scales, dtype=np.float16).astype(np.float32), group, axis=0)
    p = (q - zk).astype(np.float32) * sk
    return f32_to_bf16_bits(p) if act == "bf16" else p.astype(np.float16)


def np_linear_f64(x, w_kn, bias=None):
    """Float64 dense product x[M,K] @ w[K,N] (+bias): a rounding-free yardstick."""
    y = np.asarray(x, np.float64) @ np.asarray(w_kn, np.float64)
    if bias is not None:
        y = y + np.asarray(bias, np.float64)
    return y


# ----------------------------------------------------------------- numpy e4m3
def np_e4m3_to_f32(v):
    v = np.asarray(v, dtype=np.uint8).astype(np.int32)
    sign = np.where(v >> 7, -1.0, 1.0)
    exp = (v >> 3) & 0xF
    man = v & 7
    mag = np.where(exp == 0, man * 2.0 ** -9, (8 + man) * np.exp2(exp.astype(np.float64) - 10))
    out = (sign * mag).astype(np.float32)
    return np.where((exp == 15) & (man == 7), np.float32(np.nan), out)


_E4M3_POS = np_e4m3_to_f32(np.arange(0x7F, dtype=np.uint8)).astype(np.float64)  # 0x00..0x7e


def np_e4m3_from_f32(f):
    """RNE to the nearest e4m3 value, finite values saturated to +-448, NaN -> 0x7f."""
    f = np.asarray(f, dtype=np.float32)
    a = np.abs(f.astype(np.float64))
    a_sat = np.minimum(a, E4M3_MAX)
    idx = np.searchsorted(_E4M3_POS, a_sat, side="left")  # first value >= a
    idx = np.clip(idx, 0, len(_E4M3_POS) - 1)
    lo = np.clip(idx - 1, 0, None)
    hi_v, lo_v = _E4M3_POS[idx], _E4M3_POS[lo]
    pick_hi = (hi_v - a_sat < a_sat - lo_v) | ((hi_v - a_sat == a_sat - lo_v) & (idx % 2 == 0))
    code = np.where(hi_v == a_sat, idx, np.where(pick_hi, idx, lo)).astype(np.uint8)
    code = np.where(np.signbit(f), code | 0x80, code).astype(np.uint8)
    return np.where(np.isnan(f), np.uint8(0x7F), code).astype(np.uint8)


def np_fp8_quant_rows(x_f32):
    """Per-row e4m3 quantisation: s = absmax/448 (fp32), q = e4m3(x / s); s == 0 -> q = 0."""
    x = np.asarray(x_f32, dtype=np.float32)
    amax = np.abs(x).max(axis=1).astype(np.float32)
    s = (amax / np.float32(E4M3_MAX)).astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        q = np_e4m3_from_f32((x / s[:, None]).astype(np.float32))
    q[s == 0] = 0
    return q, s


def np_fp8_linear_f64(xq, sx, wq, sw, bias_f32=None):
    xf = np_e4m3_to_f32(xq).astype(np.float64)
    wf = np_e4m3_to_f32(wq).astype(np.float64)
    y = (xf @ wf.T) * np.asarray(sx, np.float64)[:, None] * np.asarray(sw, np.float64)[None, :]
    if bias_f32 is not None:
        y = y + np.asarray(bias_f32, np.float64)
    return y


# ------------------------------------------------------------------- C oracle
_LIB = None


def lib():
    """Load (building on first use if gcc is available) the C oracle."""
    global _LIB
    if _LIB is not None:
        return _LIB
    so = HERE / "liblmrs_oracle.so"
    if not so.exists() or so.stat().st_mtime < (HERE / "lmrs_oracle.c").stat().st_mtime:
        import subprocess
        subprocess.run(["make", "-s", "-C", str(HERE), "all"], check=True)
    L = ctypes.CDLL(str(so))
    P, I = ctypes.c_void_p, ctypes.c_int
    L.oracle_awq_pack.argtypes = [P, I, I, P]
    L.oracle_awq_unpack.argtypes = [P, I, I, P]
    L.oracle_awq_dequant.argtypes = [P, P, P, I, I, I, P, I]
    L.oracle_awq_dequant_dt.argtypes = [P, P, P, I, I, I, I, P, I]
    L.oracle_awq_linear.argtypes = [P, P, P, P, P, I, I, I, I, P, I]
    L.oracle_awq_linear.restype = I
    L.oracle_awq_linear_dt.argtypes = [P, P, P, P, P, I, I, I, I, I, P, I]
    L.oracle_awq_linear_dt.restype = I
    L.oracle_linear_kn.argtypes = [P, P, P, I, I, I, I, P, I]
    L.oracle_linear_kn.restype = I
    L.oracle_linear_nk.argtypes = [P, P, P, I, I, I, I, P, I]
    L.oracle_fp8_quant_rows.argtypes = [P, I, I, I, P, P, I]
    L.oracle_fp8_linear_prequant.argtypes = [P, P, P, P, P, I, I, I, P, I]
    L.oracle_e4m3_from_float.argtypes = [ctypes.c_float]
    L.oracle_e4m3_from_float.restype = ctypes.c_uint8
    L.oracle_e4m3_to_float.argtypes = [ctypes.c_uint8]
    L.oracle_e4m3_to_float.restype = ctypes.c_float
    L.oracle_float_to_half.argtypes = [ctypes.c_float]
    L.oracle_float_to_half.restype = ctypes.c_uint16
    L.oracle_float_to_bf16.argtypes = [ctypes.c_float]
    L.oracle_float_to_bf16.restype = ctypes.c_uint16
    L.oracle_max_threads.restype = I
    _LIB = L
    return L


def _p(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _nt(nthreads):
    return int(nthreads) if nthreads else int(os.cpu_count() or 1)


def c_awq_pack(q):
    q = np.ascontiguousarray(q, dtype=np.int8)
    R, C = q.shape
    out = np.empty((R, C // 8), dtype=np.int32)
    lib().oracle_awq_pack(_p(q), R, C, _p(out))
    return out


def c_awq_unpack(packed, cols):
    packed = np.ascontiguousarray(packed, dtype=np.int32)
    R = packed.shape[0]
    out = np.empty((R, cols), dtype=np.int8)
    lib().oracle_awq_unpack(_p(packed), R, cols, _p(out))
    return out


_ACT = {"f16": (1, np.float16), "bf16": (0, np.uint16)}  # dtype code, numpy storage


def c_awq_dequant(qweight, qzeros, scales, K, N, group, nthreads=0, act="f16"):
    """[K, N] dequantised weights: fp16 (act="f16") or bf16 bits as uint16 (act="bf16")."""
    code, st = _ACT[act]
    out = np.empty((K, N), dtype=st)
    lib().oracle_awq_dequant_dt(_p(np.ascontiguousarray(qweight, np.int32)),
                                _p(np.ascontiguousarray(qzeros, np.int32)),
                                _p(np.ascontiguousarray(scales, np.float16)),
                                K, N, group, code, _p(out), _nt(nthreads))
    return out


def c_awq_linear(x, qweight, qzeros, scales, bias, M, K, N, group, nthreads=0, act="f16"):
    """[M, N] in the activation type (fp16, or bf16 bits as uint16): bit-exact
    restatement of dequant + the reference's linear in that type."""
    code, st = _ACT[act]
    y = np.empty((M, N), dtype=st)
    b = None if bias is None else np.ascontiguousarray(bias, st)
    rc = lib().oracle_awq_linear_dt(_p(np.ascontiguousarray(x, st)),
                                    _p(np.ascontiguousarray(qweight, np.int32)),
                                    _p(np.ascontiguousarray(qzeros, np.int32)),
                                    _p(np.ascontiguousarray(scales, np.float16)),
                                    _p(b), M, K, N, group, code, _p(y), _nt(nthreads))
    if rc:
        raise MemoryError("oracle_awq_linear_dt: allocation failed")
    return y


def as_f32(a, act="f16"):
    """Values of an activation-type array (fp16, or bf16 bits) as float32."""
    return bf16_bits_to_f32(a) if act == "bf16" else np.asarray(a, np.float32)


def c_linear_nk(x, w_nk, bias, dtype_code, nthreads=0):
    """Restatement of linear_fwd(out, x, w[N,K], bias, ...) for dtype 0/1/2."""
    M, K = x.shape
    N = w_nk.shape[0]
    y = np.empty((M, N), dtype=x.dtype)
    lib().oracle_linear_nk(_p(np.ascontiguousarray(x)), _p(np.ascontiguousarray(w_nk)),
                           _p(None if bias is None else np.ascontiguousarray(bias)),
                           M, K, N, dtype_code, _p(y), _nt(nthreads))
    return y


def c_fp8_quant_rows(x, dtype_code, nthreads=0):
    x = np.ascontiguousarray(x)
    R, K = x.shape
    q = np.empty((R, K), dtype=np.uint8)
    s = np.empty(R, dtype=np.float32)
    lib().oracle_fp8_quant_rows(_p(x), R, K, dtype_code, _p(q), _p(s), _nt(nthreads))
    return q, s


def c_fp8_linear_prequant(xq, sx, wq, sw, bias_bf16=None, nthreads=0):
    M, K = xq.shape
    N = wq.shape[0]
    y = np.empty((M, N), dtype=np.uint16)
    lib().oracle_fp8_linear_prequant(
        _p(np.ascontiguousarray(xq, np.uint8)), _p(np.ascontiguousarray(sx, np.float32)),
        _p(np.ascontiguousarray(wq, np.uint8)), _p(np.ascontiguousarray(sw, np.float32)),
        _p(None if bias_bf16 is None else np.ascontiguousarray(bias_bf16, np.uint16)),
        M, K, N, _p(y), _nt(nthreads))
    return y


def c_fp8_linear(x_bf16, wq, sw, bias_bf16=None, nthreads=0):
    """Full W8A8 linear: per-token quant of bf16 x, then the scaled GEMM (bf16 bits out)."""
    xq, sx = c_fp8_quant_rows(x_bf16, 0, nthreads)
    return c_fp8_linear_prequant(xq, sx, wq, sw, bias_bf16, nthreads), xq, sx


def max_rel_err(y, y_ref):
    """The task's metric: max|y - y_ref| / max|y_ref|."""
    y = np.asarray(y, np.float64)
    y_ref = np.asarray(y_ref, np.float64)
    den = np.abs(y_ref).max()
    return float(np.abs(y - y_ref).max() / (den if den > 0 else 1.0))
