"""The CPU oracle, pinned against the golden fixtures (no GPU needed).

The reference holds no vectors for this path, so the pins are: AWQ known-answer
words written from the format text, float64-then-fp16 dequant, torch's
float8_e4m3fn encoder, and (on the GPU, tests/test_awq_gpu.py) the reference's
own linear_fwd kernel.  Two restatements (numpy, C) must also agree bit for bit.
"""
import pathlib

import numpy as np
import pytest

from oracle import oracle as O

GOLD = pathlib.Path(__file__).resolve().parent / "golden"


@pytest.fixture(scope="module")
def kat():
    return np.load(GOLD / "awq_kat.npz")


def test_awq_unpack_known_answers(kat):
    words, expect = kat["words"], kat["unpacked"]
    assert np.array_equal(O.np_awq_unpack(words), expect)
    assert np.array_equal(O.c_awq_unpack(words, words.shape[1] * 8), expect)
    assert np.array_equal(O.np_awq_pack(expect), words)
    assert np.array_equal(O.c_awq_pack(expect), words)


def test_awq_pack_roundtrip_random():
    rng = np.random.default_rng(5)
    q = rng.integers(0, 16, size=(37, 96)).astype(np.int8)
    p = O.c_awq_pack(q)
    assert np.array_equal(p, O.np_awq_pack(q))
    assert np.array_equal(O.c_awq_unpack(p, 96), q)


def test_awq_dequant_golden(kat):
    g = int(kat["group"])
    K, N = kat["q"].shape
    w_np = O.np_awq_dequant(kat["qweight"], kat["qzeros"], kat["scales"], g)
    w_c = O.c_awq_dequant(kat["qweight"], kat["qzeros"], kat["scales"], K, N, g)
    assert np.array_equal(w_np.view(np.uint16), kat["w"].view(np.uint16))
    assert np.array_equal(w_c.view(np.uint16), kat["w"].view(np.uint16))


def test_awq_linear_golden(kat):
    g = int(kat["group"])
    K, N = kat["q"].shape
    M = kat["x"].shape[0]
    y = O.c_awq_linear(kat["x"], kat["qweight"], kat["qzeros"], kat["scales"], None, M, K, N, g)
    assert O.max_rel_err(y, kat["y64"]) < 1e-3


def test_linear_kn_matches_nk():
    """The [K,N] and [N,K] restatements of linear_fwd agree bit for bit."""
    rng = np.random.default_rng(3)
    x = rng.standard_normal((3, 64)).astype(np.float16)
    w = (rng.standard_normal((64, 40)) * 0.1).astype(np.float16)
    b = rng.standard_normal(40).astype(np.float16)
    y_nk = O.c_linear_nk(x, np.ascontiguousarray(w.T), b, 1)
    y_kn = np.empty((3, 40), np.float16)
    O.lib().oracle_linear_kn(O._p(x), O._p(w), O._p(b), 3, 64, 40, 1, O._p(y_kn), 1)
    assert np.array_equal(y_nk.view(np.uint16), y_kn.view(np.uint16))


def test_e4m3_encoder_golden():
    e = np.load(GOLD / "e4m3.npz")
    vals, codes = e["values"], e["codes"]
    assert np.array_equal(O.np_e4m3_from_f32(vals), codes)
    L = O.lib()
    c = np.fromiter((L.oracle_e4m3_from_float(float(v)) for v in vals), dtype=np.uint8)
    assert np.array_equal(c, codes)


def test_e4m3_saturates():
    L = O.lib()
    for v, want in ((480.0, 0x7E), (1e9, 0x7E), (-1e9, 0xFE), (float("inf"), 0x7E)):
        assert L.oracle_e4m3_from_float(v) == want
        assert O.np_e4m3_from_f32(np.float32(v)) == want
    assert L.oracle_e4m3_from_float(float("nan")) == 0x7F


def test_e4m3_decoder_golden():
    e = np.load(GOLD / "e4m3.npz")
    dec = e["decoded"]
    mine = O.np_e4m3_to_f32(np.arange(256, dtype=np.uint8))
    nan = np.isnan(dec)
    assert np.array_equal(np.isnan(mine), nan)
    assert np.array_equal(mine[~nan], dec[~nan])
    L = O.lib()
    c = np.array([L.oracle_e4m3_to_float(i) for i in range(256)], dtype=np.float32)
    assert np.array_equal(c[~nan], dec[~nan])


def test_fp8_quant_golden():
    f = np.load(GOLD / "fp8_quant.npz")
    q, s = O.c_fp8_quant_rows(f["x_bf16"], 0)
    assert np.array_equal(s.view(np.uint32), f["s"].view(np.uint32))
    assert np.array_equal(q, f["q"])
    q2, s2 = O.np_fp8_quant_rows(O.bf16_bits_to_f32(f["x_bf16"]))
    assert np.array_equal(q2, f["q"]) and np.array_equal(s2, f["s"])


def test_fp8_linear_oracle_vs_f64():
    f = O.fp8_inputs(5, 512, 96, seed=11, with_bias=True)
    wq, sw = O.c_fp8_quant_rows(f["w_bf16"], 0)
    y, xq, sx = O.c_fp8_linear(f["x_bf16"], wq, sw, f["bias_bf16"])
    y64 = O.np_fp8_linear_f64(xq, sx, wq, sw, O.bf16_bits_to_f32(f["bias_bf16"]))
    assert O.max_rel_err(O.bf16_bits_to_f32(y), y64) < 8e-3


def test_half_and_bf16_rounding_vs_numpy():
    rng = np.random.default_rng(0)
    v = np.concatenate([rng.standard_normal(20000).astype(np.float32) * 1000,
                        np.array([65504.0, 65519.0, 65520.0, 1e-8, 6e-8, -3e-5], np.float32)])
    L = O.lib()
    h = np.array([L.oracle_float_to_half(float(x)) for x in v], dtype=np.uint16)
    assert np.array_equal(h, v.astype(np.float16).view(np.uint16))
    b = np.array([L.oracle_float_to_bf16(float(x)) for x in v], dtype=np.uint16)
    assert np.array_equal(b, O.f32_to_bf16_bits(v))
