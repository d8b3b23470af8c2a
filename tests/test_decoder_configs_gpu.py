"""Decoder layers at the task's full config-3 and config-4 shapes (two layers
each, full width), against fp64 / fp32 forwards.

* Config 3, Llama-3-8B AWQ W4A16: hidden 4096, 32 q / 8 KV heads, head_dim 128,
  intermediate 14336, vocab 128256, bf16 embeddings and norms (so bf16
  activations), context 2048, batch 1 / 16 / 64.  Its projections are the
  merged qkv 4096 -> 6144, o 4096 -> 4096, merged gate/up 4096 -> 28672 and
  down 14336 -> 4096.
* Config 4, Llama-3-70B FP8 W8A8: hidden 8192, 64 q / 8 KV heads, intermediate
  28672, vocab 128256, context 4096, batch 1 / 32: qkv 8192 -> 10240, o 8192 ->
  8192, gate/up 8192 -> 57344, down 28672 -> 8192.

The decoder block is the reference's qwen3 block with use_qk_norm = false
(crates/model/src/layers/block.rs:118-130; config mapping
crates/model/src/models/qwen3.rs:35-67).  Every projection is held to the north
star's max relative error 1e-2 on the activations the step fed it
(teacher-forced), and the whole step's logits to an fp32 forward of the same
weights and cache."""
import pytest
import torch

from lmrs_b200 import decoder as D
from test_decoder_gpu import _reference_logits, teacher_forced_errors

pytestmark = pytest.mark.gpu

SHAPE3 = dict(hidden=4096, heads=32, kv_heads=8, head_dim=128, intermediate=14336, vocab=128256)
SHAPE4 = dict(hidden=8192, heads=64, kv_heads=8, head_dim=128, intermediate=28672, vocab=128256)
TOL = 1e-2   # north-star bound per projection


def _decoder(cuda, quant, shape, batch, ctx, seed):
    cfg = D.DecoderConfig(layers=2, quant=quant, **shape)
    return D.QuantDecoder(cfg, batch=batch, ctx=ctx, device=cuda, seed=seed)


@pytest.mark.parametrize("batch", [1, 16, 64])
def test_config3_layers_teacher_forced(cuda, batch, monkeypatch):
    dec = _decoder(cuda, "awq", SHAPE3, batch, 2048, seed=11)
    assert dec.act == torch.bfloat16
    errs = teacher_forced_errors(dec, monkeypatch)
    assert len(errs) == 8
    shapes = {s[1][1] for s in errs}
    assert shapes == {4096, 14336}, shapes          # K of qkv/o/gate_up, and of down
    for kind, shape, err in errs:
        assert err < TOL, (kind, shape, err)
    del dec
    torch.cuda.empty_cache()


@pytest.mark.parametrize("batch", [1, 32])
def test_config4_layers_teacher_forced(cuda, batch, monkeypatch):
    dec = _decoder(cuda, "fp8", SHAPE4, batch, 4096, seed=12)
    errs = teacher_forced_errors(dec, monkeypatch)
    assert len(errs) == 8
    for kind, shape, err in errs:
        assert err < TOL, (kind, shape, err)
    del dec
    torch.cuda.empty_cache()


@pytest.mark.parametrize("quant,shape,batch,ctx,tol", [
    ("awq", SHAPE3, 1, 2048, 4e-2), ("awq", SHAPE3, 64, 2048, 4e-2),
    ("fp8", SHAPE4, 1, 4096, 1.5e-1), ("fp8", SHAPE4, 32, 4096, 1.5e-1)])
def test_config_step_matches_fp32(cuda, quant, shape, batch, ctx, tol):
    """Whole two-layer step at full width vs an fp32 forward: bf16 rounding of
    the activations between ops (AWQ); for FP8 also the per-token e4m3 round
    trip of bf16 vs fp32 activations (see test_decoder_gpu)."""
    dec = _decoder(cuda, quant, shape, batch, ctx, seed=13)
    ref = _reference_logits(dec)
    got = dec.logits().float()
    err = ((got - ref).abs().max() / ref.abs().max()).item()
    assert err < tol, err
    del dec, ref, got
    torch.cuda.empty_cache()
