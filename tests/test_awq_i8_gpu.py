"""AWQ decode GEMV on the integer tensor path (awq_i8.cuh), 1-2 tokens: the
packed bytes as u8 MMA operands, activations as three exact s8 limbs per
box.  Parity with the oracle's fp32-accumulated linear at the tight bar of the
other AWQ tests, over strip and box raggedness, every cluster size and ring
depth, activations with a wide dynamic range, and NaN propagation."""
import numpy as np
import pytest

from oracle import oracle as O
from test_awq_gpu import TIGHT, _awq_case, _awq_dev

pytestmark = pytest.mark.gpu


def _tuned(knobs):
    import lmrs_b200 as L
    defaults = {"awq_i8_max_m": 1, "awq_i8_slots": 5, "awq_i8_ctas_per_sm": 2, "awq_i8_cluster": 0,
                "awq_i8_box_rows": 128}

    class _Ctx:
        def __enter__(self):
            for k, v in knobs.items():
                L.set_tuning(k, v)

        def __exit__(self, *exc):
            for k in knobs:
                L.set_tuning(k, defaults[k])
    return _Ctx()


@pytest.mark.parametrize("M", [1, 2])
@pytest.mark.parametrize("K,N,g", [(1024, 1280, 128), (2048, 1312, 64), (4096, 512, 128),
                                   (3072, 768, 256), (4096, 14336, 128), (14336, 4096, 128)])
def test_i8_linear(cuda, M, K, N, g):
    """1 token (the default) and 2 tokens (opt-in): ragged 256-column strips
    (1312), 64-row boxes (group 64), groups spanning two boxes (256), the
    config-1 shape and its down projection; deterministic across calls."""
    import torch
    import lmrs_b200 as L
    with _tuned({"awq_i8_max_m": 2}):
        err, (x, qw, qz, sc, b, y) = _awq_case(cuda, M, K, N, g, 500 + M + N)
        assert err < TIGHT, err
        for _ in range(2):
            assert torch.equal(L.awq_linear(x, qw, qz, sc, b, g), y)
    assert L.read_device_error() == 0


@pytest.mark.parametrize("C", [1, 2, 3, 5, 7, 8])
@pytest.mark.parametrize("M", [1, 2])
def test_i8_clusters(cuda, C, M):
    """Every split-K cluster size, 17 boxes of 64 rows that do not divide evenly
    over the cluster, and owner column ranges of uneven width (C = 3, 5, 7)."""
    import lmrs_b200 as L
    with _tuned({"awq_i8_cluster": C, "awq_i8_max_m": 2}):
        err, _ = _awq_case(cuda, M, 17 * 64, 768, 64, 61 + C + M, bias=False)
    assert err < TIGHT, err
    assert L.read_device_error() == 0


@pytest.mark.parametrize("S,rows", [(2, 128), (3, 128), (12, 128), (5, 64), (12, 64)])
def test_i8_ring_depths(cuda, S, rows):
    """Ring depths up to what fits in shared memory, and 64-row boxes for
    128-row groups (two boxes per group, each with its own limb scale)."""
    import lmrs_b200 as L
    with _tuned({"awq_i8_slots": S, "awq_i8_cluster": 2, "awq_i8_box_rows": rows,
                 "awq_i8_max_m": 2}):
        for M in (1, 2):
            err, _ = _awq_case(cuda, M, 40 * 128, 1024, 128, 71 + S + M)
            assert err < TIGHT, (S, M, err)
    assert L.read_device_error() == 0


def test_i8_activation_range(cuda):
    """Activations spanning the fp16 range inside one box (an outlier next to
    subnormals), exact powers of two at the box maximum, an all-zero box and an
    all-zero token: the limb split keeps them to fp32-accumulation accuracy."""
    import torch
    import lmrs_b200 as L
    M, K, N, g = 2, 2048, 1024, 128
    d = O.awq_inputs(M, K, N, g, seed=5, with_bias=True)
    x = d["x"].astype(np.float32)
    x[0, 5] = 60000.0
    x[0, 6:20] = 3e-7
    x[0, 128:256] = 0.0
    x[0, 256:384] = np.where(np.arange(128) % 2, 2.0 ** -14, -1.0)
    x[0, 384] = 0.5
    x[1, :] = 0.0
    d["x"] = x.astype(np.float16)
    qw, qz, sc, xd, b = _awq_dev(d, cuda)
    with _tuned({"awq_i8_max_m": 2}):
        y = L.awq_linear(xd, qw, qz, sc, b, g)
        assert torch.equal(L.awq_linear(xd, qw, qz, sc, b, g), y)
    ref = O.c_awq_linear(d["x"], d["qweight"], d["qzeros"], d["scales"], d["bias"], M, K, N, g)
    out = y.cpu().numpy()
    assert O.max_rel_err(out[:1], ref[:1]) < TIGHT
    # a zero token gives exactly the bias
    assert np.array_equal(out[1].view(np.uint16), d["bias"].view(np.uint16))
    # the same box limits through the 1-token kernel
    y1 = L.awq_linear(xd[:1], qw, qz, sc, b, g)
    assert O.max_rel_err(y1.cpu().numpy(), ref[:1]) < TIGHT
    assert L.read_device_error() == 0


def test_i8_nan_propagates(cuda):
    """A NaN activation poisons its own token's outputs and no other token's."""
    import lmrs_b200 as L
    M, K, N, g = 2, 1024, 512, 128
    d = O.awq_inputs(M, K, N, g, seed=9, with_bias=False)
    d["x"][1, 300] = np.float16(np.nan)
    qw, qz, sc, xd, b = _awq_dev(d, cuda)
    with _tuned({"awq_i8_max_m": 2}):
        out = L.awq_linear(xd, qw, qz, sc, b, g).cpu().numpy().astype(np.float32)
    assert np.isnan(out[1]).all()
    assert np.isnan(L.awq_linear(xd[1:], qw, qz, sc, b, g).cpu().numpy().astype(np.float32)).all()
    ref = O.c_awq_linear(d["x"][:1], d["qweight"], d["qzeros"], d["scales"], None, 1, K, N, g)
    assert O.max_rel_err(out[:1].astype(np.float16), ref) < TIGHT
    assert L.read_device_error() == 0


def test_i8_off_matches_fp16_gemv(cuda):
    """With the integer path switched off, 1-2 tokens take the fp16 GEMV; both
    agree with the oracle."""
    import lmrs_b200 as L
    with _tuned({"awq_i8_max_m": 0}):
        for M in (1, 2):
            err, _ = _awq_case(cuda, M, 2048, 1280, 128, 81 + M)
            assert err < TIGHT, (M, err)
    assert L.read_device_error() == 0
