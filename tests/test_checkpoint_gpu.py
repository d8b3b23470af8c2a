"""Quantized checkpoint round trip on the B200: a decoder saved with
checkpoint.save_decoder (one file or shards) and loaded back with
QuantDecoder.from_checkpoint computes bit-identical logits, and a
tensor-parallel rank loaded from the checkpoint holds exactly its slices."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("quant", ["awq", "fp8"])
@pytest.mark.parametrize("shards", [1, 3])
def test_decoder_round_trip(cuda, tmp_path, quant, shards):
    from lmrs_b200 import checkpoint as C
    from lmrs_b200.decoder import DecoderConfig, QuantDecoder
    cfg = DecoderConfig(2, 512, 4, 2, 128, 1024, 2048, quant, group=128)
    a = QuantDecoder(cfg, batch=3, ctx=64, device=cuda, seed=5)
    C.save_decoder(a, str(tmp_path), shards=shards)
    b = QuantDecoder.from_checkpoint(str(tmp_path), batch=3, ctx=64, device=cuda, seed=5)
    assert b.cfg == cfg
    for la, lb in zip(a.layers, b.layers):
        for key in ("qkv", "o", "gate_up", "down"):
            for n, t in la[key].tensors.items():
                assert torch.equal(t, lb[key].tensors[n]), (key, n)
    b.load_state(dict(a.state()))  # same KV cache and tokens (weights already equal)
    assert torch.equal(a.logits(), b.logits())


def test_tp_rank_from_checkpoint(cuda, tmp_path):
    """Rank 1 of 2 loaded on one GPU: its merged qkv is its heads' q, k, v
    columns of the full decoder's, and its o holds its K rows (whole groups)."""
    from lmrs_b200 import checkpoint as C
    from lmrs_b200.decoder import DecoderConfig, QuantDecoder
    cfg = DecoderConfig(1, 512, 4, 2, 128, 1024, 2048, "awq", group=128)
    a = QuantDecoder(cfg, batch=2, ctx=32, device=cuda, seed=2)
    C.save_decoder(a, str(tmp_path))
    _, w1 = C.load_decoder_weights(str(tmp_path), rank=1, world=2, device=cuda)
    r1 = {"qkv": w1["layers"][0]["qkv"], "o": w1["layers"][0]["o"]}
    d = cfg.head_dim
    qw = a.layers[0]["qkv"].tensors["qweight"]
    hq, hkv = cfg.heads // 2, cfg.kv_heads // 2
    q = qw[:, (hq * d) // 8:(2 * hq * d) // 8]
    k0 = cfg.heads * d // 8
    k = qw[:, k0 + (hkv * d) // 8:k0 + (2 * hkv * d) // 8]
    v0 = k0 + cfg.kv_heads * d // 8
    v = qw[:, v0 + (hkv * d) // 8:v0 + (2 * hkv * d) // 8]
    assert torch.equal(r1["qkv"]["qweight"], torch.cat([q, k, v], 1))
    o = a.layers[0]["o"].tensors
    assert torch.equal(r1["o"]["qweight"], o["qweight"][hq * d:])
    assert torch.equal(r1["o"]["scales"], o["scales"][hq * d // 128:])
