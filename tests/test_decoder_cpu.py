"""Decode harness bookkeeping (no GPU): projection shapes per tensor-parallel
rank, AWQ group alignment of the row-parallel splits, and the byte counts the
decode roofline divides by (configs 3 and 4)."""
import pytest

from lmrs_b200 import decoder as D


def test_config3_bytes():
    c = D.LLAMA3_8B_AWQ
    params = sum(K * N for K, N in c.projections()) * c.layers
    assert params == 6_979_321_856
    assert abs(c.linear_bytes() / 1e9 - 3.63) < 0.01
    assert abs(D.QuantDecoder.kv_bytes(c, 1, 2048) / 1e6 - 268.4) < 0.1


def test_config4_bytes_and_fit():
    c = D.LLAMA3_70B_FP8
    assert abs(c.linear_bytes() / 1e9 - 68.45) < 0.05  # 68.45e9 e4m3 params + fp32 scales
    assert abs(D.QuantDecoder.kv_bytes(c, 32, 4096) / 1e9 - 42.9) < 0.1
    assert abs(D.QuantDecoder.kv_bytes(c, 256, 4096) / 1e9 - 343.6) < 0.1
    for tp in (1, 2, 4, 8):
        assert c.linear_bytes(tp) * tp == pytest.approx(c.linear_bytes(), rel=1e-3)  # row-split scales repeat


@pytest.mark.parametrize("cfg", [D.LLAMA3_8B_AWQ, D.LLAMA3_70B_FP8])
@pytest.mark.parametrize("tp", [1, 2, 4, 8])
def test_tp_shards(cfg, tp):
    qkv, o, gu, down = cfg.projections(tp)
    d = cfg.head_dim
    assert qkv == (cfg.hidden, (cfg.heads // tp + 2 * cfg.kv_heads // tp) * d)
    assert o == (cfg.heads * d // tp, cfg.hidden) and down == (cfg.intermediate // tp, cfg.hidden)
    assert gu == (cfg.hidden, 2 * cfg.intermediate // tp)
    for K, N in (qkv, o, gu, down):
        assert N % 32 == 0                       # AWQ / FP8 output alignment
        if cfg.quant == "awq":
            assert K % cfg.group == 0            # row-parallel K split stays group-aligned
