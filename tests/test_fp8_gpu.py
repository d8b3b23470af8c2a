"""FP8 e4m3 W8A8 parity on the B200: C-ABI path vs the oracle.

Quantisation (bytes and fp32 scales) must be bit-exact; linear outputs within
the north star's max relative error 1e-2 (held to 1e-2 and, for layout bugs,
to a tighter bound: bf16 output rounding is the only expected difference).
"""
import numpy as np
import pytest

from conftest import bf16_dev, bits16, ref_linear, to_dev
from oracle import oracle as O

pytestmark = pytest.mark.gpu

TOL = 1e-2
TIGHT = 8e-3  # one bf16 ulp relative is 2^-8 = 3.9e-3 of the element itself


def _dev_fp8(f, dev, bias):
    import torch
    x = bf16_dev(f["x_bf16"], dev)
    w = bf16_dev(f["w_bf16"], dev)
    b = bf16_dev(f["bias_bf16"], dev) if bias else None
    return x, w, b


@pytest.mark.parametrize("dtype", ["bf16", "f16", "f32"])
@pytest.mark.parametrize("rows,K", [(1, 16), (5, 4096), (64, 14336), (3, 48)])
def test_quant_rows_bit_exact(cuda, dtype, rows, K):
    import torch
    import lmrs_b200 as L
    rng = np.random.default_rng(rows + K)
    x32 = (rng.standard_normal((rows, K)) * rng.uniform(0.01, 100, size=(rows, 1))).astype(np.float32)
    x32[0, :] = 0.0                      # all-zero row -> scale 0, q 0
    if rows > 2:
        x32[1, K // 2] = 1e4             # one outlier
        x32[2, :] = np.float32(1e-30)    # tiny values
    if dtype == "bf16":
        bits = O.f32_to_bf16_bits(x32)
        xd, code, src = bf16_dev(bits, cuda), 0, bits
    elif dtype == "f16":
        h = x32.astype(np.float16)
        xd, code, src = to_dev(h, cuda), 1, h
    else:
        xd, code, src = to_dev(x32, cuda), 2, x32
    q, s = L.fp8_quant_rows(xd)
    q_ref, s_ref = O.c_fp8_quant_rows(src, code)
    assert np.array_equal(s.cpu().numpy().view(np.uint32), s_ref.view(np.uint32))
    assert np.array_equal(q.cpu().numpy(), q_ref)


def test_e4m3_encoder_vs_torch(cuda):
    """The e4m3 bytes our quantiser writes equal torch's float8_e4m3fn cast of x/s."""
    import torch
    import lmrs_b200 as L
    torch.manual_seed(0)
    x = (torch.randn(32, 4096, device=cuda) * 3).bfloat16()
    q, s = L.fp8_quant_rows(x)
    t = (x.float() / s[:, None]).to(torch.float8_e4m3fn).view(torch.uint8)
    assert torch.equal(q, t)


@pytest.mark.parametrize("M", [1, 3, 8, 9, 16, 17, 32])
@pytest.mark.parametrize("bias", [False, True])
def test_linear_gemv_small(cuda, M, bias):
    import lmrs_b200 as L
    K, N = 1024, 640
    f = O.fp8_inputs(M, K, N, seed=M, with_bias=bias)
    x, w, b = _dev_fp8(f, cuda, bias)
    wq, sw = L.quantize_fp8_weight(w)
    y = L.fp8_linear(x, wq, sw, b)
    wq_ref, sw_ref = O.c_fp8_quant_rows(f["w_bf16"], 0)
    assert np.array_equal(wq.cpu().numpy(), wq_ref)
    y_ref, _, _ = O.c_fp8_linear(f["x_bf16"], wq_ref, sw_ref, f["bias_bf16"])
    err = O.max_rel_err(O.bf16_bits_to_f32(bits16(y)), O.bf16_bits_to_f32(y_ref))
    assert err < TIGHT, err


@pytest.mark.parametrize("M", [33, 128, 200, 512])
@pytest.mark.parametrize("bias", [False, True])
def test_linear_gemm_small(cuda, M, bias):
    import lmrs_b200 as L
    K, N = 1024, 768
    f = O.fp8_inputs(M, K, N, seed=100 + M, with_bias=bias)
    x, w, b = _dev_fp8(f, cuda, bias)
    wq, sw = L.quantize_fp8_weight(w)
    y = L.fp8_linear(x, wq, sw, b)
    wq_ref, sw_ref = O.c_fp8_quant_rows(f["w_bf16"], 0)
    y_ref, _, _ = O.c_fp8_linear(f["x_bf16"], wq_ref, sw_ref, f["bias_bf16"])
    err = O.max_rel_err(O.bf16_bits_to_f32(bits16(y)), O.bf16_bits_to_f32(y_ref))
    assert err < TIGHT, err


@pytest.mark.parametrize("K,N", [(4096, 4096), (4096, 28672), (14336, 4096)])
@pytest.mark.parametrize("M", [1, 32, 512, 8192])
def test_config2_shapes_vs_reference(cuda, ref_ffi, K, N, M):
    """Config 2, every (K, N) at every M of the sweep (M=8192 is the FP8 GEMM's
    headline point): CUDA W8A8 vs the reference's linear_fwd (f32 variant) run on
    the dequantised operands xq*s_x and wq*s_w, over all M x N outputs."""
    import torch
    import lmrs_b200 as L
    f = O.fp8_inputs(M, K, N, seed=0)
    x, w, _ = _dev_fp8(f, cuda, False)
    wq, sw = L.quantize_fp8_weight(w)
    y = L.fp8_linear(x, wq, sw)
    xq, sx = L.fp8_quant_rows(x)
    xf = (xq.view(torch.float8_e4m3fn).float() * sx[:, None]).contiguous()
    wf = (wq.view(torch.float8_e4m3fn).float() * sw[:, None]).contiguous()
    y_ref = ref_linear(ref_ffi, xf, wf, None, 2)
    err = O.max_rel_err(y.float().cpu().numpy(), y_ref.cpu().numpy())
    assert err < TOL and err < TIGHT, err


def test_config2_large_m_properties(cuda):
    """M=8192 (largest config-2 point): rows through the GEMV path agree with the
    GEMM's rows; scaling one token scales only its output row."""
    import torch
    import lmrs_b200 as L
    K, N, M = 4096, 4096, 8192
    f = O.fp8_inputs(1, K, N, seed=0)
    _, w, _ = _dev_fp8(f, cuda, False)
    wq, sw = L.quantize_fp8_weight(w)
    torch.manual_seed(1)
    x = torch.randn(M, K, device=cuda).bfloat16()
    y = L.fp8_linear(x, wq, sw).float()
    for r0 in (0, 4000, 8160):
        yr = L.fp8_linear(x[r0:r0 + 32].contiguous(), wq, sw).float()
        e = ((yr - y[r0:r0 + 32]).abs().max() / y[r0:r0 + 32].abs().max()).item()
        assert e < TIGHT, (r0, e)
    x2 = x.clone()
    x2[7] *= 4  # a power of two: quantised bytes unchanged, scale x4
    y2 = L.fp8_linear(x2, wq, sw).float()
    assert torch.equal(y2[:7], y[:7]) and torch.equal(y2[8:16], y[8:16])
    assert ((y2[7] - 4 * y[7]).abs().max() / (4 * y[7]).abs().max()).item() < TIGHT


def test_prequant_matches_full(cuda):
    import torch
    import lmrs_b200 as L
    torch.manual_seed(2)
    x = torch.randn(48, 2048, device=cuda).bfloat16()
    w = (torch.randn(1024, 2048, device=cuda) * 0.02).bfloat16()
    wq, sw = L.quantize_fp8_weight(w)
    xq, sx = L.fp8_quant_rows(x)
    assert torch.equal(L.fp8_linear(x, wq, sw), L.fp8_linear_prequant(xq, sx, wq, sw))


def test_workspace_and_status(cuda):
    import torch
    import lmrs_b200 as L
    from lmrs_b200 import _lib
    lib = _lib.load()
    M, K, N = 4, 256, 64
    x = torch.randn(M, K, device=cuda).bfloat16()
    wq = torch.zeros(N, K, dtype=torch.uint8, device=cuda)
    sw = torch.ones(N, device=cuda)
    y = torch.empty(M, N, dtype=torch.bfloat16, device=cuda)
    need = lib.lmrs_fp8_linear_workspace_bytes(M, K, N)
    ws = torch.empty(need, dtype=torch.uint8, device=cuda)
    s = torch.cuda.current_stream().cuda_stream
    assert lib.lmrs_fp8_linear(y.data_ptr(), x.data_ptr(), wq.data_ptr(), sw.data_ptr(), None,
                               M, K, N, ws.data_ptr(), need - 1, s) == _lib.LMRS_ERR_WORKSPACE
    assert lib.lmrs_fp8_linear(y.data_ptr(), x.data_ptr(), wq.data_ptr(), sw.data_ptr(), None,
                               M, K + 8, N, ws.data_ptr(), need, s) == _lib.LMRS_ERR_SHAPE
    assert lib.lmrs_fp8_linear(y.data_ptr(), x.data_ptr(), wq.data_ptr(), sw.data_ptr(), None,
                               M, K, N, ws.data_ptr(), need, s) == 0
    torch.cuda.synchronize()
    assert torch.count_nonzero(y.float()) == 0
    assert L.read_device_error() == 0


@pytest.mark.parametrize("bn", [256, 224])
def test_gemm_tile_widths(cuda, bn):
    """Both tcgen05 tile widths (the dispatcher picks per shape) against the oracle."""
    import lmrs_b200 as L
    K, N, M = 1024, 1000, 300  # N % 8 == 0 but not a multiple of either tile width
    f = O.fp8_inputs(M, K, N, seed=bn, with_bias=True)
    x, w, b = _dev_fp8(f, cuda, True)
    try:
        L.set_tuning("gemm_bn", bn)
        wq, sw = L.quantize_fp8_weight(w)
        y = L.fp8_linear(x, wq, sw, b)
    finally:
        L.set_tuning("gemm_bn", 256)
    wq_ref, sw_ref = O.c_fp8_quant_rows(f["w_bf16"], 0)
    y_ref, _, _ = O.c_fp8_linear(f["x_bf16"], wq_ref, sw_ref, f["bias_bf16"])
    err = O.max_rel_err(O.bf16_bits_to_f32(bits16(y)), O.bf16_bits_to_f32(y_ref))
    assert err < TIGHT, err


@pytest.mark.parametrize("ksub", [1, 2])
@pytest.mark.parametrize("M,K,N", [(1100, 1024, 1000), (300, 4224, 768)])
def test_gemm_cta_pair(cuda, ksub, M, K, N):
    """The CTA-pair (cta_group::2, 256 x 256) FP8 GEMM, both K-stage depths: bit for
    bit the one-SM kernel's output (same K order per output), and the oracle at the
    tile bound; ragged M (CTA 1's rows partly or wholly past M), N and K."""
    import torch
    import lmrs_b200 as L
    f = O.fp8_inputs(M, K, N, seed=ksub * 7 + M, with_bias=True)
    x, w, b = _dev_fp8(f, cuda, True)
    wq, sw = L.quantize_fp8_weight(w)
    xq, sx = L.fp8_quant_rows(x)
    try:
        L.set_tuning("fp8_gemm_pair", 0)
        L.set_tuning("fp8_gemm_bn128", 0)
        one = L.fp8_linear_prequant(xq, sx, wq, sw, b)
        L.set_tuning("fp8_gemm_pair", 1)
        L.set_tuning("fp8_gemm_pair_ksub", ksub)
        L.set_tuning("fp8_gemm_pair_min_m", 1)
        pair = L.fp8_linear_prequant(xq, sx, wq, sw, b)
        torch.cuda.synchronize()
    finally:
        L.set_tuning("fp8_gemm_bn128", 1)
        L.set_tuning("fp8_gemm_pair", 1)
        L.set_tuning("fp8_gemm_pair_ksub", 2)
        L.set_tuning("fp8_gemm_pair_min_m", 256)
    assert L.read_device_error() == 0
    assert torch.equal(pair, one)
    wq_ref, sw_ref = O.c_fp8_quant_rows(f["w_bf16"], 0)
    y_ref, _, _ = O.c_fp8_linear(f["x_bf16"], wq_ref, sw_ref, f["bias_bf16"])
    err = O.max_rel_err(O.bf16_bits_to_f32(bits16(pair)), O.bf16_bits_to_f32(y_ref))
    assert err < TIGHT, err


def _fp8_case(dev, M, K, N, seed, bias):
    import lmrs_b200 as L
    f = O.fp8_inputs(M, K, N, seed=seed, with_bias=bias)
    x, w, b = _dev_fp8(f, dev, bias)
    wq, sw = L.quantize_fp8_weight(w)
    y = L.fp8_linear(x, wq, sw, b)
    wq_ref, sw_ref = O.c_fp8_quant_rows(f["w_bf16"], 0)
    y_ref, _, _ = O.c_fp8_linear(f["x_bf16"], wq_ref, sw_ref, f["bias_bf16"])
    return O.max_rel_err(O.bf16_bits_to_f32(bits16(y)), O.bf16_bits_to_f32(y_ref))


@pytest.mark.parametrize("M", [9, 16, 17, 31, 32, 33, 48, 64])
@pytest.mark.parametrize("K,N", [(1024, 640), (1040, 1000), (2176, 1001)])
@pytest.mark.parametrize("bias", [False, True])
def test_linear_swap_ab(cuda, M, K, N, bias):
    """9..64 tokens: the swap-AB tcgen05 kernel (weights as the MMA's 128-row
    operand); ragged K (not a multiple of 128), ragged N (not a multiple of the
    128-channel strip, odd N: single-channel stores)."""
    err = _fp8_case(cuda, M, K, N, 1000 + M + K + N, bias)
    assert err < TIGHT, err


@pytest.mark.parametrize("C", [1, 2, 4, 8])
@pytest.mark.parametrize("M", [12, 40])
def test_linear_swap_ab_clusters(cuda, C, M):
    """Every split-K cluster size of the swap-AB kernel, including K ranges that
    do not divide evenly (17 K units over C CTAs)."""
    import lmrs_b200 as L
    try:
        L.set_tuning("fp8_swap_cluster", C)
        err = _fp8_case(cuda, M, 17 * 128, 384, 77 + C, True)
    finally:
        L.set_tuning("fp8_swap_cluster", 0)
    assert err < TIGHT, err


@pytest.mark.parametrize("M", [9, 20, 32])
def test_linear_gemv_wide_opt_in(cuda, M):
    """The register-fed GEMV for 9..32 tokens (off by default since the swap-AB
    kernel took that range) stays correct when selected."""
    import lmrs_b200 as L
    try:
        L.set_tuning("fp8_gemv_max_m", 32)
        err = _fp8_case(cuda, M, 1024, 640, 5 + M, True)
    finally:
        L.set_tuning("fp8_gemv_max_m", 8)
    assert err < TIGHT, err
