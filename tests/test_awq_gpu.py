"""AWQ W4A16 parity on the B200: the CUDA path through the C-ABI vs the oracle.

Bars (the task's north star): unpack and dequantised fp16 weights bit-exact;
linear outputs within max relative error 1e-2 (max|y - y_ref| / max|y_ref|)
with fp32 accumulation.  The CUDA linear accumulates in a different order than
the sequential oracle, so outputs agree to fp16 rounding, not bit for bit; the
tests hold them to a tighter 2e-3 as well, to catch layout bugs early.
"""
import numpy as np
import pytest

from conftest import bits16, ref_linear, to_dev
from oracle import oracle as O

pytestmark = pytest.mark.gpu

TOL = 1e-2
TIGHT = 2e-3        # what a correct fp32-accumulating kernel reaches here


def _awq_dev(d, dev):
    import torch
    return (to_dev(d["qweight"], dev), to_dev(d["qzeros"], dev),
            to_dev(d["scales"], dev), to_dev(d["x"], dev),
            None if d["bias"] is None else to_dev(d["bias"], dev))


@pytest.mark.parametrize("rows,cols", [(1, 8), (3, 40), (128, 4096), (4096, 512)])
def test_unpack_bit_exact(cuda, rows, cols):
    import lmrs_b200 as L
    rng = np.random.default_rng(rows * 7 + cols)
    q = rng.integers(0, 16, size=(rows, cols)).astype(np.int8)
    packed = O.c_awq_pack(q)
    out = L.awq_unpack(to_dev(packed, cuda)).cpu().numpy()
    assert np.array_equal(out, q)
    assert np.array_equal(out, O.c_awq_unpack(packed, cols))


@pytest.mark.parametrize("K,N,g", [(128, 8, 128), (256, 40, 64), (4096, 4096, 128),
                                   (512, 14336, 128)])
def test_dequant_bit_exact(cuda, K, N, g):
    import lmrs_b200 as L
    d = O.awq_inputs(1, K, N, g, seed=K + N)
    qw, qz, sc, _, _ = _awq_dev(d, cuda)
    w = L.awq_dequant(qw, qz, sc, g)
    ref = O.c_awq_dequant(d["qweight"], d["qzeros"], d["scales"], K, N, g)
    assert np.array_equal(bits16(w), ref.view(np.uint16))


def test_dequant_extremes(cuda):
    """q = z (exact zero), q = 0 / z = 15, q = 15 / z = 0, largest and smallest scales."""
    import lmrs_b200 as L
    K, N, g = 128, 64, 128
    q = np.zeros((K, N), np.int8)
    z = np.zeros((1, N), np.int8)
    q[:, 0:8] = 7; z[:, 0:8] = 7          # q == z -> 0
    q[:, 8:16] = 0; z[:, 8:16] = 15       # -15 * s
    q[:, 16:24] = 15; z[:, 16:24] = 0     # +15 * s
    q[:, 24:] = np.arange(K)[:, None] % 16
    z[:, 24:] = np.arange(N - 24) % 16
    s = np.full((1, N), 0.02, np.float16)
    s[:, 32:] = np.float16(0.001)
    s[:, 40:48] = np.float16(65504.0)      # overflow to inf when |q - z| >= 2
    s[:, 48:56] = np.float16(6e-8)         # subnormal products
    qw, qz = O.np_awq_pack(q), O.np_awq_pack(z)
    w = L.awq_dequant(to_dev(qw, cuda), to_dev(qz, cuda), to_dev(s, cuda), g)
    ref = O.c_awq_dequant(qw, qz, s, K, N, g)
    assert np.array_equal(bits16(w), ref.view(np.uint16))
    assert np.array_equal(ref, O.np_awq_dequant(qw, qz, s, g))


@pytest.mark.parametrize("M", [1, 2, 7, 8, 9, 16])
@pytest.mark.parametrize("bias", [False, True])
def test_linear_gemv_small(cuda, M, bias):
    """Default dispatch, and the register-fed GEMV with the TMEM-staged kernel
    switched off (it takes 9..16 tokens by default)."""
    import lmrs_b200 as L
    K, N, g = 1024, 512, 128
    d = O.awq_inputs(M, K, N, g, seed=M, with_bias=bias)
    qw, qz, sc, x, b = _awq_dev(d, cuda)
    ref = O.c_awq_linear(d["x"], d["qweight"], d["qzeros"], d["scales"], d["bias"], M, K, N, g)
    for tmem_max in (32, 0):
        try:
            L.set_tuning("awq_tmem_max_m", tmem_max)
            y = L.awq_linear(x, qw, qz, sc, b, g)
        finally:
            L.set_tuning("awq_tmem_max_m", 32)
        err = O.max_rel_err(y.cpu().numpy(), ref)
        assert err < TIGHT, (tmem_max, err)


@pytest.mark.parametrize("M", [17, 100, 128, 129, 300, 512])
@pytest.mark.parametrize("bias", [False, True])
def test_linear_gemm_small(cuda, M, bias):
    import lmrs_b200 as L
    K, N, g = 512, 768, 128
    d = O.awq_inputs(M, K, N, g, seed=1000 + M, with_bias=bias)
    qw, qz, sc, x, b = _awq_dev(d, cuda)
    y = L.awq_linear(x, qw, qz, sc, b, g)
    ref = O.c_awq_linear(d["x"], d["qweight"], d["qzeros"], d["scales"], d["bias"], M, K, N, g)
    err = O.max_rel_err(y.cpu().numpy(), ref)
    assert err < TIGHT, err


@pytest.mark.parametrize("N", [32, 96, 160, 288])
def test_linear_ragged_n(cuda, N):
    """N not a multiple of the 128/256-column tiles (AWQ needs N % 32 == 0 here)."""
    import lmrs_b200 as L
    K, g = 256, 64
    for M in (4, 40, 200):
        d = O.awq_inputs(M, K, N, g, seed=N + M, with_bias=True)
        qw, qz, sc, x, b = _awq_dev(d, cuda)
        y = L.awq_linear(x, qw, qz, sc, b, g)
        ref = O.c_awq_linear(d["x"], d["qweight"], d["qzeros"], d["scales"], d["bias"], M, K, N, g)
        assert O.max_rel_err(y.cpu().numpy(), ref) < TIGHT


def test_config0_vs_reference_linear_fwd(cuda, ref_ffi):
    """Config 0 (M=8, K=N=4096, g=128): pins the oracle against the reference's
    own linear_fwd on the dequantised weights (bit-exact: same fp32 FMA chain),
    then holds the CUDA path to both."""
    import torch
    import lmrs_b200 as L
    M, K, N, g = 8, 4096, 4096, 128
    d = O.awq_inputs(M, K, N, g, seed=0)
    qw, qz, sc, x, _ = _awq_dev(d, cuda)
    w_kn = L.awq_dequant(qw, qz, sc, g)
    w_nk = w_kn.t().contiguous()
    y_ref = ref_linear(ref_ffi, x, w_nk, None, 1)
    y_oracle = O.c_awq_linear(d["x"], d["qweight"], d["qzeros"], d["scales"], None, M, K, N, g)
    assert np.array_equal(bits16(y_ref), y_oracle.view(np.uint16)), "oracle != reference linear_fwd"
    y = L.awq_linear(x, qw, qz, sc, None, g)
    assert O.max_rel_err(y.cpu().numpy(), y_oracle) < TIGHT


@pytest.mark.slow
@pytest.mark.parametrize("M", [1, 16, 128, 1024, 4096])
def test_config1_full_size(cuda, ref_ffi, M):
    """Config 1 shape (K=4096, N=14336, g=128) at every M of the sweep against the
    reference's linear_fwd on the dequantised weights, over all M x N outputs.
    M=4096 is the bench line's dominant kernel, where each persistent CTA of the
    prefill GEMM walks several 128-channel x 256-token tiles."""
    import lmrs_b200 as L
    K, N, g = 4096, 14336, 128
    d = O.awq_inputs(M, K, N, g, seed=0)
    qw, qz, sc, x, _ = _awq_dev(d, cuda)
    w_nk = L.awq_dequant(qw, qz, sc, g).t().contiguous()
    y_ref = ref_linear(ref_ffi, x, w_nk, None, 1)
    y = L.awq_linear(x, qw, qz, sc, None, g)
    err = O.max_rel_err(y.cpu().numpy(), y_ref.cpu().numpy())
    assert err < TOL and err < TIGHT, err


def test_linear_4096_rows_properties(cuda):
    """M=4096 (largest config-1 sweep point): linearity in x and agreement of
    row blocks with the GEMV path, size-independent checks that need no CPU oracle."""
    import torch
    import lmrs_b200 as L
    M, K, N, g = 4096, 4096, 14336, 128
    d = O.awq_inputs(8, K, N, g, seed=0)
    qw, qz, sc, _, _ = _awq_dev(d, cuda)
    torch.manual_seed(0)
    x = torch.randn(M, K, device=cuda).half()
    y = L.awq_linear(x, qw, qz, sc, None, g).float()
    # rows computed through the decode GEMV must match rows of the big GEMM
    for r0 in (0, 1234, 4088):
        yr = L.awq_linear(x[r0:r0 + 8].contiguous(), qw, qz, sc, None, g).float()
        e = (yr - y[r0:r0 + 8]).abs().max().item() / y[r0:r0 + 8].abs().max().item()
        assert e < TIGHT, (r0, e)
    # linearity: f(2x) == 2 f(x) up to rounding
    y2 = L.awq_linear((x * 2), qw, qz, sc, None, g).float()
    assert ((y2 - 2 * y).abs().max() / (2 * y).abs().max()).item() < TIGHT
    assert torch.isfinite(y).all()


def test_status_codes(cuda):
    import torch
    import lmrs_b200 as L
    from lmrs_b200 import _lib
    d = O.awq_inputs(2, 256, 64, 128, seed=3)
    qw, qz, sc, x, _ = _awq_dev(d, cuda)
    with pytest.raises(L.LmrsError) as e:
        L.awq_linear(x, qw, qz, sc, None, 96)      # group not a multiple of 64 / not dividing K
    assert e.value.status == _lib.LMRS_ERR_GROUP
    y = torch.empty(2, 64, dtype=torch.float16, device=cuda)
    lib = _lib.load()
    rc = lib.lmrs_awq_linear(y.data_ptr() + 2, x.data_ptr(), qw.data_ptr(), qz.data_ptr(),
                             sc.data_ptr(), None, 2, 256, 64, 128, 1, None, 0,
                             torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.LMRS_ERR_ALIGN
    rc = lib.lmrs_awq_linear(y.data_ptr(), x.data_ptr(), qw.data_ptr(), qz.data_ptr(),
                             sc.data_ptr(), None, 2, 256, 64, 128, 2, None, 0,
                             torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.LMRS_ERR_DTYPE   # f32 activations are not an AWQ type
    # M == 0 is a no-op
    rc = lib.lmrs_awq_linear(y.data_ptr(), x.data_ptr(), qw.data_ptr(), qz.data_ptr(),
                             sc.data_ptr(), None, 0, 256, 64, 128, 1, None, 0,
                             torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    assert L.read_device_error() == 0


@pytest.mark.parametrize("knob,value,Ms", [("awq_gemm_pair", 1, (129, 300, 512)),
                                           ("awq_gemv_max_m", 8, (9, 12, 16)),
                                           ("awq_swap_max_m", 128, (65, 100, 128)),
                                           ("gemm_bn", 0, (100, 300, 512)),
                                           ("gemm_bn", 224, (100, 300, 512)),
                                           ("awq_gemv4", 0, (1, 3, 4)),
                                           ("gemv_box_rows", 64, (1, 4, 8, 16)),
                                           ("awq_gemv_cluster", 2, (1, 5, 16)),
                                           ("awq_gemv_cluster", 8, (1, 5, 16)),
                                           ("awq_gemv_slots", 8, (5, 16)),
                                           ("awq_gemv4_slots", 8, (1, 4)),
                                           ("awq_tmem_max_m", 0, (17, 24, 32)),
                                           ("awq_gemm_tmem", 0, (100, 300, 512)),
                                           ("pdl", 0, (1, 8, 20, 40, 300))])
def test_opt_in_paths(cuda, knob, value, Ms):
    """Kernels and launch shapes the default dispatch does not pick for these M
    (CTA-pair GEMM, the shared-memory-staged GEMM, swap-AB below 17 or from 17
    to 32 tokens (where the TMEM-staged kernel is the default) or above 64, the general GEMV for
    M <= 4, 64-row boxes, other cluster sizes and ring depths, launches without
    programmatic dependent launch) stay correct and deterministic when selected."""
    import torch
    import lmrs_b200 as L
    from lmrs_b200 import _lib
    defaults = {"awq_gemm_pair": 0, "awq_gemv_max_m": 16, "awq_swap_max_m": 64, "gemm_bn": 256,
                "awq_gemv4": 1, "gemv_box_rows": 128, "awq_gemv_cluster": 0, "awq_gemv_slots": 4,
                "awq_gemv4_slots": 4, "awq_tmem_max_m": 32, "awq_gemm_tmem": 1, "pdl": 1}
    K, N, g = 1024, 1280, 128
    # the smem-staged GEMM's own knobs are only reached with the TMEM GEMM off
    also_off = knob in ("awq_gemm_pair", "gemm_bn")
    gemv_knob = knob in ("awq_gemv_cluster", "awq_gemv_slots", "gemv_box_rows", "awq_gemv4",
                         "awq_gemv4_slots")
    try:
        L.set_tuning("awq_i8_max_m", 0)   # 1-2 tokens: the fp16 GEMVs these knobs steer
        if gemv_knob:
            L.set_tuning("awq_tmem_max_m", 0)  # 5..16 tokens go to the TMEM kernel by default
        L.set_tuning(knob, value)
        if also_off:
            L.set_tuning("awq_gemm_tmem", 0)
        for M in Ms:
            d = O.awq_inputs(M, K, N, g, seed=M + 7, with_bias=True)
            qw, qz, sc, x, b = _awq_dev(d, cuda)
            y = L.awq_linear(x, qw, qz, sc, b, g)
            ref = O.c_awq_linear(d["x"], d["qweight"], d["qzeros"], d["scales"], d["bias"], M, K, N, g)
            assert O.max_rel_err(y.cpu().numpy(), ref) < TIGHT, (knob, M)
            for _ in range(3):
                assert torch.equal(L.awq_linear(x, qw, qz, sc, b, g), y), (knob, M, "nondeterministic")
    finally:
        L.set_tuning(knob, defaults[knob])
        L.set_tuning("awq_gemm_tmem", 1)
        L.set_tuning("awq_i8_max_m", 1)
        L.set_tuning("awq_tmem_max_m", 32)
    assert L.read_device_error() == 0


def _awq_case(dev, M, K, N, g, seed, bias=True):
    import lmrs_b200 as L
    d = O.awq_inputs(M, K, N, g, seed=seed, with_bias=bias)
    qw, qz, sc, x, b = _awq_dev(d, dev)
    y = L.awq_linear(x, qw, qz, sc, b, g)
    ref = O.c_awq_linear(d["x"], d["qweight"], d["qzeros"], d["scales"], d["bias"], M, K, N, g)
    return O.max_rel_err(y.cpu().numpy(), ref), (x, qw, qz, sc, b, y)


@pytest.mark.parametrize("M", [1, 3, 4, 5, 8, 15, 16, 17, 31, 32])
@pytest.mark.parametrize("K,N,g", [(1024, 1280, 128), (2048, 1312, 64), (4096, 512, 128),
                                   (3072, 768, 256)])
def test_tmem_linear(cuda, M, K, N, g):
    """AWQ linear with the weights dequantised into tensor memory (tcgen05 with
    the A operand in TMEM), forced on for every M up to 32: both token-tile
    widths (16/32), N not a multiple of the 256-channel strip, groups of 64,
    128 and 256 rows, and deterministic across calls."""
    import torch
    import lmrs_b200 as L
    try:
        L.set_tuning("awq_tmem_min_m", 1)
        err, (x, qw, qz, sc, b, y) = _awq_case(cuda, M, K, N, g, 300 + M + N)
        for _ in range(2):
            assert torch.equal(L.awq_linear(x, qw, qz, sc, b, g), y)
    finally:
        L.set_tuning("awq_tmem_min_m", 9)
        L.set_tuning("awq_tmem_max_m", 32)
    assert err < TIGHT, err
    assert L.read_device_error() == 0


@pytest.mark.parametrize("C", [1, 2, 4, 8])
@pytest.mark.parametrize("M", [1, 12])
def test_tmem_linear_clusters(cuda, C, M):
    """Every split-K cluster size, with 17 boxes of 64 rows that do not divide
    evenly over the cluster."""
    import lmrs_b200 as L
    try:
        L.set_tuning("awq_tmem_min_m", 1)
        L.set_tuning("awq_tmem_cluster", C)
        err, _ = _awq_case(cuda, M, 17 * 64, 768, 64, 41 + C, bias=False)
    finally:
        L.set_tuning("awq_tmem_min_m", 9)
        L.set_tuning("awq_tmem_cluster", 0)
    assert err < TIGHT, err


@pytest.mark.parametrize("bt", [128, 192, 256])
@pytest.mark.parametrize("M,K,N,g", [(65, 1024, 1280, 128), (128, 2048, 1312, 64), (200, 1024, 768, 128),
                                     (513, 3072, 640, 256), (1000, 1024, 2048, 128)])
def test_gemm_tmem_opt_in(cuda, bt, M, K, N, g):
    """Prefill GEMM with the dequantised weights as the TMEM A operand (the
    default above 64 tokens): ragged token and channel tiles, groups of
    64/128/256 rows, every token-tile width, deterministic across calls."""
    import torch
    import lmrs_b200 as L
    try:
        L.set_tuning("awq_gemm_tmem_bt", bt)
        L.set_tuning("awq_swap_deep_k", 0)  # deep-K shapes up to 128 tokens go to swap-AB by default
        err, (x, qw, qz, sc, b, y) = _awq_case(cuda, M, K, N, g, 900 + M + bt)
        assert torch.equal(L.awq_linear(x, qw, qz, sc, b, g), y)
    finally:
        L.set_tuning("awq_gemm_tmem_bt", 256)
        L.set_tuning("awq_swap_deep_k", 5)
    assert err < TIGHT, err
    assert L.read_device_error() == 0


@pytest.mark.parametrize("M", [65, 96, 128])
@pytest.mark.parametrize("K,N", [(4096, 3072), (6144, 4096)])
def test_default_dispatch_deep_k_band(cuda, M, K, N):
    """Default dispatch in the 1.25 <= K/N < 2 band at 65-128 tokens, where the
    split-K swap-AB kernel is picked over the prefill GEMM (4K >= 5N), against
    the C oracle."""
    import torch
    import lmrs_b200 as L
    err, (x, qw, qz, sc, b, y) = _awq_case(cuda, M, K, N, 128, 77 + M + N)
    assert err < TIGHT, err
    assert torch.equal(L.awq_linear(x, qw, qz, sc, b, 128), y)
    assert L.read_device_error() == 0


# ------------------------------------------------------------ bf16 activations
# The reference model runs bf16 end to end (KernelDType::Bf16 = 0,
# crates/kernels/src/raw.rs:9-13), so lmrs_awq_linear takes bf16 x / y / bias as
# well; scales stay fp16.  The dequantised weight is bf16_rne((q - z) * s), one
# rounding of the exact product.  bf16 keeps 8 significant bits, so one output
# ulp is 2^-8 = 3.9e-3 of the element: the bf16 linears are held to 8e-3 (the
# bound the FP8 tests use for their bf16 outputs) and to the north star's 1e-2.
TIGHT_BF16 = 8e-3


def _bf16_dev(a, dev):
    import torch
    return to_dev(np.asarray(a, np.uint16), dev, torch.bfloat16)


def _awq_case_bf16(dev, M, K, N, g, seed, bias=True):
    import lmrs_b200 as L
    d = O.awq_inputs(M, K, N, g, seed=seed, with_bias=bias, act="bf16")
    qw, qz, sc = to_dev(d["qweight"], dev), to_dev(d["qzeros"], dev), to_dev(d["scales"], dev)
    x = _bf16_dev(d["x"], dev)
    b = None if d["bias"] is None else _bf16_dev(d["bias"], dev)
    y = L.awq_linear(x, qw, qz, sc, b, g)
    assert y.dtype == x.dtype
    ref = O.c_awq_linear(d["x"], d["qweight"], d["qzeros"], d["scales"], d["bias"], M, K, N, g,
                         act="bf16")
    err = O.max_rel_err(O.bf16_bits_to_f32(bits16(y)), O.bf16_bits_to_f32(ref))
    return err, (x, qw, qz, sc, b, y)


@pytest.mark.parametrize("K,N,g", [(128, 8, 128), (256, 40, 64), (4096, 4096, 128),
                                   (512, 14336, 128)])
def test_dequant_bf16_bit_exact(cuda, K, N, g):
    import torch
    import lmrs_b200 as L
    d = O.awq_inputs(1, K, N, g, seed=K + N + 1)
    w = L.awq_dequant(to_dev(d["qweight"], cuda), to_dev(d["qzeros"], cuda),
                      to_dev(d["scales"], cuda), g, dtype=torch.bfloat16)
    ref = O.c_awq_dequant(d["qweight"], d["qzeros"], d["scales"], K, N, g, act="bf16")
    assert np.array_equal(bits16(w), ref)
    assert np.array_equal(ref, O.np_awq_dequant(d["qweight"], d["qzeros"], d["scales"], g,
                                                act="bf16"))


def test_dequant_bf16_extremes(cuda):
    """The fp16 extremes of test_dequant_extremes in bf16: q == z, +-15 * s, the
    largest fp16 scale (finite in bf16: 15 x 65504 does not overflow), fp16
    subnormal scales, and every fp16 scale whose bf16 rounding carries into the
    next binade (the s_hi + s_lo split at its edge)."""
    import torch
    import lmrs_b200 as L
    K, N, g = 128, 96, 128
    q = np.zeros((K, N), np.int8)
    z = np.zeros((1, N), np.int8)
    q[:, 0:8] = 7; z[:, 0:8] = 7
    q[:, 8:16] = 0; z[:, 8:16] = 15
    q[:, 16:24] = 15; z[:, 16:24] = 0
    q[:, 24:] = np.arange(K)[:, None] % 16
    z[:, 24:] = np.arange(N - 24) % 16
    s = np.full((1, N), 0.02, np.float16)
    s[:, 32:] = np.float16(0.001)
    s[:, 40:48] = np.float16(65504.0)
    s[:, 48:56] = np.float16(6e-8)
    s[:, 56:64] = np.float16(1.0) - np.float16(2.0 ** -11)          # rounds up to 1.0 in bf16
    s[:, 64:72] = (np.arange(8) + 1017).astype(np.float16) / 1024    # near-ties of the split
    s[:, 72:80] = np.float16(-0.0137)                                # negative scales
    s[:, 80:96] = np.random.default_rng(5).uniform(1e-4, 4.0, (1, 16)).astype(np.float16)
    qw, qz = O.np_awq_pack(q), O.np_awq_pack(z)
    w = L.awq_dequant(to_dev(qw, cuda), to_dev(qz, cuda), to_dev(s, cuda), g, dtype=torch.bfloat16)
    ref = O.c_awq_dequant(qw, qz, s, K, N, g, act="bf16")
    assert np.array_equal(bits16(w), ref)


def test_config0_bf16_vs_reference_linear_fwd(cuda, ref_ffi):
    """Config 0 shapes in bf16: the oracle equals the reference's own linear_fwd
    (dtype 0 = bf16) on the bf16-dequantised weights bit for bit, and the CUDA
    path is within TIGHT_BF16 of both."""
    import torch
    import lmrs_b200 as L
    M, K, N, g = 8, 4096, 4096, 128
    d = O.awq_inputs(M, K, N, g, seed=0, act="bf16")
    qw, qz, sc = to_dev(d["qweight"], cuda), to_dev(d["qzeros"], cuda), to_dev(d["scales"], cuda)
    x = _bf16_dev(d["x"], cuda)
    w_nk = L.awq_dequant(qw, qz, sc, g, dtype=torch.bfloat16).t().contiguous()
    y_ref = ref_linear(ref_ffi, x, w_nk, None, 0)
    y_oracle = O.c_awq_linear(d["x"], d["qweight"], d["qzeros"], d["scales"], None, M, K, N, g,
                              act="bf16")
    assert np.array_equal(bits16(y_ref), y_oracle), "oracle != reference linear_fwd (bf16)"
    y = L.awq_linear(x, qw, qz, sc, None, g)
    err = O.max_rel_err(O.bf16_bits_to_f32(bits16(y)), O.bf16_bits_to_f32(y_oracle))
    assert err < TIGHT_BF16, err


# (M, K, N, g): default dispatch through every regime — integer GEMV (1), the
# 2-4 token GEMV (3), the general GEMV (5..8 on deep K), the TMEM-staged kernel
# (5..8 wide, 9..32), swap-AB (33..64 and deep-K up to 128), the prefill GEMM
# (shallow K above 64, and above 128) with ragged token and channel tiles
BF16_CASES = [(1, 1024, 1280, 128), (2, 2048, 768, 64), (3, 1024, 1280, 128),
              (4, 4096, 512, 128), (7, 4096, 512, 128), (8, 1024, 2048, 128),
              (12, 1024, 1280, 128), (16, 2048, 1312, 64), (31, 1024, 768, 256),
              (40, 1024, 1280, 128), (64, 2048, 512, 128), (96, 4096, 3072, 128),
              (100, 1024, 1280, 128), (200, 1024, 768, 128), (513, 3072, 640, 256)]


@pytest.mark.parametrize("M,K,N,g", BF16_CASES)
def test_linear_bf16_default_dispatch(cuda, M, K, N, g):
    import torch
    import lmrs_b200 as L
    err, (x, qw, qz, sc, b, y) = _awq_case_bf16(cuda, M, K, N, g, 4000 + M + N)
    assert err < TIGHT_BF16 and err < TOL, err
    assert torch.equal(L.awq_linear(x, qw, qz, sc, b, g), y), "nondeterministic"
    assert L.read_device_error() == 0


@pytest.mark.parametrize("knob,value,Ms", [("awq_gemm_pair", 1, (129, 300)),
                                           ("awq_gemm_tmem", 0, (100, 300)),
                                           ("gemm_bn", 224, (100, 300)),
                                           ("awq_gemv4", 0, (1, 3)),
                                           ("awq_i8_max_m", 2, (1, 2)),
                                           ("awq_i8_max_m", 0, (1, 2)),
                                           ("awq_tmem_max_m", 0, (9, 16, 24)),
                                           ("awq_swap_max_m", 128, (65, 128)),
                                           ("awq_gemm_tmem_bt", 128, (65, 200)),
                                           ("awq_gemm_tmem_bt", 192, (65, 200)),
                                           ("gemv_box_rows", 64, (1, 4, 8))])
def test_linear_bf16_opt_in_paths(cuda, knob, value, Ms):
    """Every kernel variant the knobs reach, in bf16, against the C oracle."""
    import lmrs_b200 as L
    defaults = {"awq_gemm_pair": 0, "awq_gemm_tmem": 1, "gemm_bn": 256, "awq_gemv4": 1,
                "awq_i8_max_m": 1, "awq_tmem_max_m": 32, "awq_swap_max_m": 64,
                "awq_gemm_tmem_bt": 256, "gemv_box_rows": 128}
    K, N, g = 1024, 1280, 128
    try:
        if knob in ("awq_gemm_pair", "gemm_bn"):
            L.set_tuning("awq_gemm_tmem", 0)
        if knob in ("awq_gemv4", "gemv_box_rows"):
            L.set_tuning("awq_i8_max_m", 0)
            L.set_tuning("awq_tmem_max_m", 0)
        if knob == "awq_gemm_tmem_bt":
            L.set_tuning("awq_swap_deep_k", 0)
        L.set_tuning(knob, value)
        for M in Ms:
            err, _ = _awq_case_bf16(cuda, M, K, N, g, 5000 + M + len(knob))
            assert err < TIGHT_BF16, (knob, value, M, err)
    finally:
        for k, v in defaults.items():
            L.set_tuning(k, v)
        L.set_tuning("awq_swap_deep_k", 5)
    assert L.read_device_error() == 0


def test_linear_bf16_large_values(cuda):
    """bf16 has fp32's range: activations far outside fp16's (1e6 .. 1e-20) stay
    finite and accurate on every regime's path (the integer GEMV rescales each
    box by a power of two chosen from its maximum)."""
    import torch
    import lmrs_b200 as L
    K, N, g = 1024, 512, 128
    d = O.awq_inputs(40, K, N, g, seed=77, act="bf16")
    xf = O.bf16_bits_to_f32(d["x"]).copy()
    xf[:, :512] *= 1e6
    xf[1::2, 512:] *= 1e-20
    xb = O.f32_to_bf16_bits(xf)
    qw, qz, sc = to_dev(d["qweight"], cuda), to_dev(d["qzeros"], cuda), to_dev(d["scales"], cuda)
    for M in (1, 2, 4, 8, 16, 40):
        y = L.awq_linear(_bf16_dev(xb[:M], cuda), qw, qz, sc, None, g)
        ref = O.c_awq_linear(xb[:M], d["qweight"], d["qzeros"], d["scales"], None, M, K, N, g,
                             act="bf16")
        yf, rf = O.bf16_bits_to_f32(bits16(y)), O.bf16_bits_to_f32(ref)
        assert np.isfinite(yf).all()
        assert O.max_rel_err(yf, rf) < TIGHT_BF16, M


@pytest.mark.parametrize("act", ["f16", "bf16"])
@pytest.mark.parametrize("M,K,N,g", [(129, 1024, 768, 128), (256, 2048, 512, 64),
                                     (300, 3072, 1280, 256), (1000, 1024, 2048, 128),
                                     (2100, 4096, 1024, 128)])
def test_gemm_pair(cuda, act, M, K, N, g):
    """The CTA-pair prefill GEMM (cta_group::2, 256 channels x 256 tokens per
    pair, weights dequantised into each CTA's TMEM): ragged token tiles, groups
    of 64/128/256 rows, several tiles per pair, both activation types,
    deterministic across calls."""
    import torch
    import lmrs_b200 as L
    try:
        L.set_tuning("awq_gemm_tmem_pair", 1)
        if act == "bf16":
            err, (x, qw, qz, sc, b, y) = _awq_case_bf16(cuda, M, K, N, g, 7000 + M)
            tol = TIGHT_BF16
        else:
            err, (x, qw, qz, sc, b, y) = _awq_case(cuda, M, K, N, g, 7000 + M)
            tol = TIGHT
        assert torch.equal(L.awq_linear(x, qw, qz, sc, b, g), y), "nondeterministic"
    finally:
        L.set_tuning("awq_gemm_tmem_pair", 0)
    assert err < tol, err
    assert L.read_device_error() == 0


@pytest.mark.slow
def test_gemm_pair_config1_vs_reference(cuda, ref_ffi):
    """Config 1 (K=4096, N=14336) at M=4096 on the CTA-pair GEMM against the
    reference's linear_fwd on the dequantised weights, every output."""
    import lmrs_b200 as L
    M, K, N, g = 4096, 4096, 14336, 128
    d = O.awq_inputs(M, K, N, g, seed=0)
    qw, qz, sc, x, _ = _awq_dev(d, cuda)
    w_nk = L.awq_dequant(qw, qz, sc, g).t().contiguous()
    y_ref = ref_linear(ref_ffi, x, w_nk, None, 1)
    try:
        L.set_tuning("awq_gemm_tmem_pair", 1)
        y = L.awq_linear(x, qw, qz, sc, None, g)
    finally:
        L.set_tuning("awq_gemm_tmem_pair", 0)
    err = O.max_rel_err(y.cpu().numpy(), y_ref.cpu().numpy())
    assert err < TIGHT, err
    assert L.read_device_error() == 0
