"""Quantized checkpoint loading on the host (lmrs_b200/checkpoint.py): the
safetensors layout pinned against the `safetensors` package in both
directions, sharded indexes, quantization_config parsing, and the
tensor-parallel slicing of AWQ and FP8 projections (the rank shards must
reassemble to the tensor-parallelism-1 weights)."""
import json
import os

import numpy as np
import pytest
import torch

from lmrs_b200 import checkpoint as C


def _tensors():
    g = torch.Generator().manual_seed(0)
    return {
        "a.f16": torch.randn(3, 5, generator=g).half(),
        "a.bf16": torch.randn(4, 7, generator=g).bfloat16(),
        "b.f32": torch.randn(6, generator=g),
        "c.i32": torch.randint(-2 ** 31, 2 ** 31 - 1, (2, 3, 4), dtype=torch.int32, generator=g),
        "d.u8": torch.randint(0, 256, (9,), dtype=torch.uint8, generator=g),
        "e.f8": torch.randint(0, 256, (4, 8), dtype=torch.uint8, generator=g).view(torch.float8_e4m3fn),
        "f.i64": torch.arange(5, dtype=torch.int64),
        "g.scalar": torch.tensor(2.5, dtype=torch.float32),
    }


def _same(a, b):
    if a.dtype != b.dtype or a.shape != b.shape:
        return False
    return torch.equal(a.reshape(-1).view(torch.uint8), b.reshape(-1).view(torch.uint8))


def test_write_read_against_safetensors_package(tmp_path):
    from safetensors.torch import load_file, save_file
    t = _tensors()
    ours = str(tmp_path / "ours.safetensors")
    C.save_safetensors(ours, t, {"format": "pt"})
    theirs = load_file(ours)
    assert set(theirs) == set(t)
    for k in t:
        assert _same(theirs[k], t[k]), k
    ref = str(tmp_path / "ref.safetensors")
    save_file(t, ref, metadata={"format": "pt"})
    f = C.SafetensorsFile(ref)
    assert f.metadata == {"format": "pt"}
    for k in t:
        assert _same(f.get(k), t[k]), k
    # row / column slices come from the memory map
    assert torch.equal(f.get("a.f16", slice(1, 3), slice(2, 5)), t["a.f16"][1:3, 2:5])


def test_header_validation(tmp_path):
    p = str(tmp_path / "x.safetensors")
    C.save_safetensors(p, {"w": torch.zeros(4, 4)})
    raw = bytearray(open(p, "rb").read())
    n = int.from_bytes(raw[:8], "little")
    hdr = json.loads(raw[8:8 + n])
    hdr["w"]["data_offsets"] = [0, 60]          # does not hold F32[4, 4]
    hj = json.dumps(hdr).encode()
    bad = str(tmp_path / "bad.safetensors")
    with open(bad, "wb") as f:
        f.write(len(hj).to_bytes(8, "little") + hj + bytes(raw[8 + n:]))
    with pytest.raises(C.CheckpointError):
        C.SafetensorsFile(bad)
    with pytest.raises(C.CheckpointError):
        C.Checkpoint(str(tmp_path / "nowhere"))


def test_sharded_index(tmp_path):
    t = _tensors()
    C.save_sharded(str(tmp_path), t, shards=3, config={"x": 1})
    idx = json.load(open(tmp_path / "model.safetensors.index.json"))
    assert len(set(idx["weight_map"].values())) == 3
    ck = C.Checkpoint(str(tmp_path))
    assert ck.config == {"x": 1}
    for k in t:
        assert _same(ck.get(k), t[k]), k


@pytest.mark.parametrize("qc,ok", [
    ({"quant_method": "awq", "bits": 4, "group_size": 128, "zero_point": True, "version": "gemm"}, "awq"),
    ({"quant_method": "AWQ", "w_bit": 4, "q_group_size": 64}, "awq"),
    ({"quant_method": "awq", "bits": 8, "group_size": 128}, None),
    ({"quant_method": "awq", "bits": 4, "group_size": 100}, None),
    ({"quant_method": "awq", "bits": 4, "group_size": 128, "version": "gemv"}, None),
    ({"quant_method": "awq", "bits": 4, "group_size": 128, "zero_point": False}, None),
    ({"quant_method": "fp8", "activation_scheme": "dynamic"}, "fp8"),
    ({"quant_method": "fp8"}, "fp8"),
    ({"quant_method": "fp8", "activation_scheme": "static"}, None),
    ({"quant_method": "fp8", "activation_scheme": "dynamic", "weight_block_size": [128, 128]},
     None),
    ({"quant_method": "gptq", "bits": 4}, None),
])
def test_quant_spec(qc, ok):
    if ok is None:
        with pytest.raises(C.CheckpointError):
            C.quant_spec({"quantization_config": qc})
    else:
        assert C.quant_spec({"quantization_config": qc}).method == ok
    with pytest.raises(C.CheckpointError):
        C.quant_spec({})


def _cfg(quant):
    from lmrs_b200.decoder import DecoderConfig
    return DecoderConfig(2, 512, 4, 2, 128, 1024, 2048, quant, group=128)


def _awq(K, N, g, gen):
    return dict(qweight=torch.randint(-2 ** 31, 2 ** 31 - 1, (K, N // 8), dtype=torch.int32, generator=gen),
                qzeros=torch.randint(-2 ** 31, 2 ** 31 - 1, (K // g, N // 8), dtype=torch.int32, generator=gen),
                scales=(torch.rand(K // g, N, generator=gen) * 0.02).half())


def _fp8(K, N, gen, per_tensor=False):
    w = torch.randint(0, 0x7E, (N, K), dtype=torch.uint8, generator=gen).view(torch.float8_e4m3fn)
    s = torch.tensor(0.01) if per_tensor else torch.rand(N, 1, generator=gen) * 0.01
    return dict(weight=w, weight_scale=s)


def _write_model(path, cfg, per_tensor=False):
    gen = torch.Generator().manual_seed(1)
    act = cfg.act_dtype
    d, H, I = cfg.head_dim, cfg.hidden, cfg.intermediate
    shapes = {"q": (H, cfg.heads * d), "k": (H, cfg.kv_heads * d), "v": (H, cfg.kv_heads * d),
              "o": (cfg.heads * d, H), "gate": (H, I), "up": (H, I), "down": (I, H)}
    t = {"model.embed_tokens.weight": torch.randn(cfg.vocab, H, generator=gen).to(act),
         "model.norm.weight": torch.randn(H, generator=gen).to(act),
         "lm_head.weight": torch.randn(cfg.vocab, H, generator=gen).to(act)}
    for i in range(cfg.layers):
        t[f"model.layers.{i}.input_layernorm.weight"] = torch.randn(H, generator=gen).to(act)
        t[f"model.layers.{i}.post_attention_layernorm.weight"] = torch.randn(H, generator=gen).to(act)
        for p, (K, N) in shapes.items():
            base = (f"model.layers.{i}.self_attn.{p}_proj" if p in "qkvo"
                    else f"model.layers.{i}.mlp.{p}_proj")
            parts = _awq(K, N, cfg.group, gen) if cfg.quant == "awq" else _fp8(K, N, gen, per_tensor)
            for k, v in parts.items():
                t[f"{base}.{k}"] = v
    C.save_sharded(str(path), t, shards=2, config=C.hf_config(cfg))
    return t


@pytest.mark.parametrize("quant", ["awq", "fp8"])
def test_decoder_weights_and_tp_shards(tmp_path, quant):
    cfg = _cfg(quant)
    t = _write_model(tmp_path, cfg)
    c1, full = C.load_decoder_weights(str(tmp_path))
    assert c1 == cfg
    d = cfg.head_dim
    # rank-1 merged projections equal the checkpoint tensors concatenated
    L0 = full["layers"][0]
    if quant == "awq":
        for k in ("qweight", "qzeros", "scales"):
            ref = torch.cat([t[f"model.layers.0.self_attn.{p}_proj.{k}"] for p in "qkv"], 1)
            assert torch.equal(L0["qkv"][k], ref)
    else:
        ref = torch.cat([t[f"model.layers.0.self_attn.{p}_proj.weight"] for p in "qkv"], 0)
        assert torch.equal(L0["qkv"]["weight_q"], ref.view(torch.uint8))
        assert L0["qkv"]["weight_scale"].shape == (cfg.heads * d + 2 * cfg.kv_heads * d,)
    # two ranks reassemble to the full weights
    shards = [C.load_decoder_weights(str(tmp_path), rank=r, world=2)[1] for r in range(2)]
    from lmrs_b200.decoder import assemble_awq_tp
    st = [dict(s_, tokens=torch.zeros(1), kv=torch.zeros(1, 1, 1, 1)) for s_ in shards]
    asm = assemble_awq_tp(st, cfg)
    assert torch.equal(asm["lm_head"], full["lm_head"])
    for li, (a, b) in enumerate(zip(asm["layers"], full["layers"])):
        for key in ("qkv", "o", "gate_up", "down"):
            for n in b[key]:
                if quant == "fp8" and key in ("o", "down"):
                    # row-parallel FP8: each rank holds K columns of [N, K], all N scales
                    parts = [s_["layers"][li][key][n] for s_ in shards]
                    ref = torch.cat(parts, 1) if n == "weight_q" else parts[0]
                    assert all(torch.equal(p, parts[0]) for p in parts) or n == "weight_q"
                    assert torch.equal(ref, b[key][n]), (key, n)
                else:
                    assert torch.equal(a[key][n], b[key][n]), (key, n)


def test_fp8_per_tensor_scale(tmp_path):
    cfg = _cfg("fp8")
    _write_model(tmp_path, cfg, per_tensor=True)
    _, w = C.load_decoder_weights(str(tmp_path), rank=1, world=2)
    s = w["layers"][0]["o"]["weight_scale"]
    assert s.shape == (cfg.hidden,) and torch.all(s == s[0])


def test_awq_split_must_keep_groups(tmp_path):
    from lmrs_b200.decoder import DecoderConfig
    cfg = DecoderConfig(1, 512, 4, 2, 128, 768, 2048, "awq", group=256)
    _write_model(tmp_path, cfg)
    C.load_decoder_weights(str(tmp_path), rank=0, world=1)
    with pytest.raises(C.CheckpointError):   # down: 768 / 2 = 384 rows cut a 256-row group
        C.load_decoder_weights(str(tmp_path), rank=0, world=2)


def test_rejects_qk_norm_tensors(tmp_path):
    """A Qwen3 checkpoint carries per-head q/k norms (use_qk_norm); the decoder
    does not implement them, so loading must fail instead of giving wrong
    attention outputs."""
    cfg = _cfg("awq")
    t = _write_model(tmp_path / "a", cfg)
    t["model.layers.0.self_attn.q_norm.weight"] = torch.ones(cfg.head_dim).half()
    t["model.layers.0.self_attn.k_norm.weight"] = torch.ones(cfg.head_dim).half()
    C.save_sharded(str(tmp_path / "b"), t, shards=1, config=C.hf_config(cfg))
    with pytest.raises(C.CheckpointError, match="q_norm|k_norm"):
        C.load_decoder_weights(str(tmp_path / "b"))


@pytest.mark.parametrize("extra", [{"use_qk_norm": True},
                                   {"rope_scaling": {"rope_type": "llama3", "factor": 8.0}}])
def test_rejects_unimplemented_config(tmp_path, extra):
    cfg = _cfg("fp8")
    t = _write_model(tmp_path, cfg)
    hf = dict(C.hf_config(cfg), **extra)
    C.save_sharded(str(tmp_path / "c"), t, shards=1, config=hf)
    with pytest.raises(C.CheckpointError):
        C.load_decoder_weights(str(tmp_path / "c"))


def test_fp8_input_scale_warns(tmp_path):
    cfg = _cfg("fp8")
    t = _write_model(tmp_path, cfg)
    t["model.layers.0.self_attn.q_proj.input_scale"] = torch.tensor(0.5)
    C.save_sharded(str(tmp_path / "d"), t, shards=1, config=C.hf_config(cfg))
    with pytest.warns(UserWarning, match="input_scale"):
        C.load_decoder_weights(str(tmp_path / "d"))
