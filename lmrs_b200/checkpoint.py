"""Quantized checkpoint loading (and saving) for the decoder of ``decoder.py``.

The reference loads one BF16 ``model.safetensors`` (crates/model/src/loader/
safetensors.rs:267-283, the dtype check at :274; tensors are fetched by name
through WeightBuilder::get at :112) and reads hyper-parameters from
``config.json`` (crates/model/src/config/hparams.rs).  This module extends
that path to the quantized formats this package runs:

* AWQ W4A16 as written by AutoAWQ's GEMM packing: per projection ``qweight``
  int32 [K, N/8], ``qzeros`` int32 [K/g, N/8] (nibble i of word j is column
  8j + ORDER[i], ORDER = {0,2,4,6,1,3,5,7}) and ``scales`` fp16 [K/g, N];
  ``quantization_config = {"quant_method": "awq", "bits": 4, "group_size": g,
  "zero_point": true, "version": "gemm"}``.
* FP8 W8A8: ``weight`` F8_E4M3 [N, K] with ``weight_scale`` fp32 per output
  channel ([N] or [N, 1]) or per tensor ([] or [1], expanded to [N]);
  ``quantization_config = {"quant_method": "fp8", "activation_scheme":
  "dynamic"}``.  Activations are always quantized per token at run time: a
  static scheme and block-wise weight scales (``weight_block_size``) are
  rejected, and a stray ``input_scale`` tensor is ignored with a warning.
* Single-file or sharded checkpoints (``model.safetensors.index.json`` with a
  ``weight_map`` from tensor name to file), read through memory maps so a
  tensor-parallel rank only copies its own slices.

Tensor names follow the Llama / Qwen3 layout the decoder implements
(``model.layers.{i}.self_attn.{q,k,v,o}_proj``, ``model.layers.{i}.mlp.
{gate,up,down}_proj``, ``model.embed_tokens``, ``model.norm``, ``lm_head``,
``input_layernorm`` / ``post_attention_layernorm``).  q/k/v and gate/up are
merged into the decoder's column-parallel projections; o and down are split
along K (AWQ by whole quantization groups).

This is host-side plumbing (file format, naming, sharding); every byte it
returns is consumed by the CUDA kernels unchanged.
"""
from __future__ import annotations

import json
import os
import struct
import warnings
from dataclasses import dataclass
from typing import Dict, Iterable, List, Optional, Tuple

import numpy as np
import torch

# ----------------------------------------------------------------- safetensors

# safetensors dtype tag -> (numpy storage dtype, torch dtype of the tensor)
_DTYPES = {
    "BOOL": (np.bool_, torch.bool),
    "U8": (np.uint8, torch.uint8),
    "I8": (np.int8, torch.int8),
    "I16": (np.int16, torch.int16),
    "U16": (np.uint16, torch.uint16),
    "I32": (np.int32, torch.int32),
    "U32": (np.uint32, torch.uint32),
    "I64": (np.int64, torch.int64),
    "U64": (np.uint64, torch.uint64),
    "F16": (np.float16, torch.float16),
    "BF16": (np.uint16, torch.bfloat16),
    "F32": (np.float32, torch.float32),
    "F64": (np.float64, torch.float64),
    "F8_E4M3": (np.uint8, torch.float8_e4m3fn),
    "F8_E5M2": (np.uint8, torch.float8_e5m2),
}
_TAG = {tdt: tag for tag, (_, tdt) in _DTYPES.items()}
_MAX_HEADER = 100 << 20


class CheckpointError(ValueError):
    """Malformed or unsupported checkpoint."""


class SafetensorsFile:
    """One .safetensors file: the JSON header plus a read-only memory map of
    the data section.  ``get`` returns a CPU torch tensor (a copy of the
    requested slice only)."""

    def __init__(self, path: str):
        self.path = path
        with open(path, "rb") as f:
            raw = f.read(8)
            if len(raw) != 8:
                raise CheckpointError(f"{path}: truncated header length")
            (n,) = struct.unpack("<Q", raw)
            if n > _MAX_HEADER:
                raise CheckpointError(f"{path}: header of {n} bytes")
            header = json.loads(f.read(n))
        self.metadata = header.pop("__metadata__", {}) or {}
        self.entries: Dict[str, dict] = header
        self.data_start = 8 + n
        size = os.path.getsize(path)
        for name, e in self.entries.items():
            if e["dtype"] not in _DTYPES:
                raise CheckpointError(f"{path}: {name}: unsupported dtype {e['dtype']}")
            b, end = e["data_offsets"]
            want = int(np.prod(e["shape"], dtype=np.int64)) * np.dtype(_DTYPES[e["dtype"]][0]).itemsize
            if end - b != want or self.data_start + end > size:
                raise CheckpointError(f"{path}: {name}: data_offsets {b}..{end} do not hold "
                                      f"{e['dtype']}{e['shape']}")
        self._mm = None

    def names(self) -> List[str]:
        return list(self.entries)

    def dtype(self, name: str) -> str:
        return self.entries[name]["dtype"]

    def shape(self, name: str) -> Tuple[int, ...]:
        return tuple(self.entries[name]["shape"])

    def _map(self):
        if self._mm is None:
            self._mm = np.memmap(self.path, dtype=np.uint8, mode="r")
        return self._mm

    def array(self, name: str) -> np.ndarray:
        """Read-only numpy view of a tensor's storage (bf16/fp8 as integers)."""
        e = self.entries[name]
        npdt = _DTYPES[e["dtype"]][0]
        b, end = e["data_offsets"]
        buf = self._map()[self.data_start + b: self.data_start + end]
        return buf.view(npdt).reshape(e["shape"])

    def get(self, name: str, rows: Optional[slice] = None, cols: Optional[slice] = None) -> torch.Tensor:
        a = self.array(name)
        if rows is not None:
            a = a[rows]
        if cols is not None:
            a = a[:, cols]
        t = torch.from_numpy(np.array(a, copy=True, order="C"))  # keeps 0-d shapes
        tdt = _DTYPES[self.dtype(name)][1]
        return t.view(tdt) if t.dtype != tdt else t


def save_safetensors(path: str, tensors: Dict[str, torch.Tensor],
                     metadata: Optional[Dict[str, str]] = None) -> None:
    """Write ``tensors`` (any device; stored contiguous, little-endian) in the
    safetensors layout: u64 header length, JSON header padded with spaces to
    a multiple of 8 bytes, then the data in header order."""
    header: dict = {}
    if metadata:
        header["__metadata__"] = {str(k): str(v) for k, v in metadata.items()}
    blobs = []
    off = 0
    for name, t in tensors.items():
        if t.dtype not in _TAG:
            raise CheckpointError(f"{name}: dtype {t.dtype} has no safetensors tag")
        c = t.detach().to("cpu").contiguous()
        raw = c.reshape(-1).view(torch.uint8).numpy().tobytes() if c.numel() else b""
        header[name] = {"dtype": _TAG[t.dtype], "shape": list(c.shape),
                        "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    hj = json.dumps(header, separators=(",", ":")).encode()
    hj += b" " * ((8 - len(hj) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hj)))
        f.write(hj)
        for raw in blobs:
            f.write(raw)


class Checkpoint:
    """A checkpoint directory: ``model.safetensors``, or shards listed by
    ``model.safetensors.index.json`` (``weight_map``: tensor name -> file)."""

    def __init__(self, path: str):
        self.path = path
        index = os.path.join(path, "model.safetensors.index.json")
        single = os.path.join(path, "model.safetensors")
        self.files: Dict[str, SafetensorsFile] = {}
        self.where: Dict[str, str] = {}
        if os.path.exists(index):
            with open(index) as f:
                wm = json.load(f).get("weight_map")
            if not isinstance(wm, dict) or not wm:
                raise CheckpointError(f"{index}: no weight_map")
            for name, fname in wm.items():
                if fname not in self.files:
                    self.files[fname] = SafetensorsFile(os.path.join(path, fname))
                if name not in self.files[fname].entries:
                    raise CheckpointError(f"{index}: {name} is not in {fname}")
                self.where[name] = fname
        elif os.path.exists(single):
            self.files["model.safetensors"] = SafetensorsFile(single)
            self.where = {n: "model.safetensors" for n in self.files["model.safetensors"].names()}
        else:
            raise CheckpointError(f"{path}: neither model.safetensors nor its index")
        cfg = os.path.join(path, "config.json")
        self.config: dict = {}
        if os.path.exists(cfg):
            with open(cfg) as f:
                self.config = json.load(f)

    def has(self, name: str) -> bool:
        return name in self.where

    def names(self) -> List[str]:
        return list(self.where)

    def file(self, name: str) -> SafetensorsFile:
        if name not in self.where:
            raise CheckpointError(f"{self.path}: missing tensor {name}")
        return self.files[self.where[name]]

    def get(self, name: str, rows=None, cols=None) -> torch.Tensor:
        return self.file(name).get(name, rows, cols)

    def shape(self, name: str):
        return self.file(name).shape(name)

    def dtype(self, name: str) -> str:
        return self.file(name).dtype(name)


def save_sharded(path: str, tensors: Dict[str, torch.Tensor], shards: int,
                 config: Optional[dict] = None) -> None:
    """Write ``tensors`` as ``shards`` files plus the index (one file, no index,
    when shards == 1) and ``config.json`` when given."""
    os.makedirs(path, exist_ok=True)
    names = list(tensors)
    if shards <= 1:
        save_safetensors(os.path.join(path, "model.safetensors"), tensors)
    else:
        per = (len(names) + shards - 1) // shards
        wm = {}
        for i in range(shards):
            part = names[i * per:(i + 1) * per]
            fname = f"model-{i + 1:05d}-of-{shards:05d}.safetensors"
            save_safetensors(os.path.join(path, fname), {n: tensors[n] for n in part})
            wm.update({n: fname for n in part})
        total = sum(t.numel() * t.element_size() for t in tensors.values())
        with open(os.path.join(path, "model.safetensors.index.json"), "w") as f:
            json.dump({"metadata": {"total_size": total}, "weight_map": wm}, f, indent=1)
    if config is not None:
        with open(os.path.join(path, "config.json"), "w") as f:
            json.dump(config, f, indent=1)


# ----------------------------------------------------------- quantization spec

@dataclass(frozen=True)
class QuantSpec:
    method: str             # "awq" or "fp8"
    group: int = 128        # AWQ group size (rows of K per scale / zero)
    activation_scheme: str = "dynamic"


def quant_spec(config: dict) -> QuantSpec:
    """``quantization_config`` of a config.json (the ModelConfig raw map)."""
    qc = config.get("quantization_config")
    if not isinstance(qc, dict):
        raise CheckpointError("config.json has no quantization_config")
    method = str(qc.get("quant_method", "")).lower()
    if method == "awq":
        bits = int(qc.get("bits", qc.get("w_bit", 4)))
        group = int(qc.get("group_size", qc.get("q_group_size", 128)))
        version = str(qc.get("version", "gemm")).lower()
        zp = qc.get("zero_point", True)
        if bits != 4:
            raise CheckpointError(f"AWQ with {bits} bits: only 4-bit weights are supported")
        if version != "gemm":
            raise CheckpointError(f"AWQ version {version!r}: only the GEMM packing is supported")
        if not zp:
            raise CheckpointError("AWQ without zero points is not supported")
        if group <= 0 or group % 64:
            raise CheckpointError(f"AWQ group size {group}: must be a positive multiple of 64")
        return QuantSpec("awq", group=group)
    if method == "fp8":
        if qc.get("weight_block_size") is not None:
            raise CheckpointError(
                f"FP8 with weight_block_size {qc['weight_block_size']}: only per-channel or "
                "per-tensor weight scales are supported, not block-wise scales")
        scheme = str(qc.get("activation_scheme", "dynamic")).lower()
        if scheme != "dynamic":
            raise CheckpointError(
                f"FP8 activation_scheme {scheme!r}: activations are quantized per token at run "
                "time ('dynamic'); static input scales are not supported")
        return QuantSpec("fp8", activation_scheme=scheme)
    raise CheckpointError(f"quant_method {method!r}: expected 'awq' or 'fp8'")


def decoder_config(config: dict):
    """DecoderConfig from the hyper-parameters of a Llama / Qwen3 config.json."""
    from .decoder import DecoderConfig
    spec = quant_spec(config)
    # The decoder is the reference's qwen3 block with use_qk_norm = false and
    # plain RoPE (crates/model/src/models/qwen3.rs:35-67); a checkpoint that
    # needs per-head q/k norms or scaled RoPE would load and give wrong outputs.
    if config.get("use_qk_norm"):
        raise CheckpointError("use_qk_norm: per-head q/k RMSNorm is not implemented")
    if config.get("rope_scaling") is not None:
        raise CheckpointError(f"rope_scaling {config['rope_scaling']!r}: only plain RoPE "
                              "(rope_theta) is implemented")
    H = int(config["hidden_size"])
    heads = int(config["num_attention_heads"])
    # activations follow the checkpoint's torch_dtype: fp16 for an AWQ model
    # saved in fp16, bf16 otherwise (the FP8 linear always takes bf16)
    f16 = str(config.get("torch_dtype", "")).lower() in ("float16", "fp16", "half")
    return DecoderConfig(
        layers=int(config["num_hidden_layers"]), hidden=H, heads=heads,
        kv_heads=int(config.get("num_key_value_heads", heads)),
        head_dim=int(config.get("head_dim") or H // heads),
        intermediate=int(config["intermediate_size"]), vocab=int(config["vocab_size"]),
        quant=spec.method, group=spec.group,
        rope_theta=float(config.get("rope_theta", 10000.0)),
        eps=float(config.get("rms_norm_eps", 1e-6)),
        act="f16" if (f16 and spec.method == "awq") else "bf16")


# ------------------------------------------------------------ decoder weights

_ATTN = "model.layers.{i}.self_attn.{p}_proj"
_MLP = "model.layers.{i}.mlp.{p}_proj"


def _proj_names(i: int) -> Dict[str, str]:
    d = {p: _ATTN.format(i=i, p=p) for p in ("q", "k", "v", "o")}
    d.update({p: _MLP.format(i=i, p=p) for p in ("gate", "up", "down")})
    return d


def _load_awq(ck: Checkpoint, base: str, group: int, ncols: Optional[Tuple[int, int]] = None,
              krows: Optional[Tuple[int, int]] = None) -> Dict[str, torch.Tensor]:
    """One AWQ projection, optionally restricted to output columns [c0, c1)
    (multiples of 8) or input rows [k0, k1) (multiples of the group)."""
    for t, dt in (("qweight", "I32"), ("qzeros", "I32"), ("scales", "F16")):
        if ck.dtype(f"{base}.{t}") != dt:
            raise CheckpointError(f"{base}.{t}: dtype {ck.dtype(f'{base}.{t}')}, expected {dt}")
    if ck.has(f"{base}.bias"):
        raise CheckpointError(f"{base}.bias: projection biases are not part of this decoder")
    K, W = ck.shape(f"{base}.qweight")
    if ck.shape(f"{base}.qzeros") != (K // group, W) or ck.shape(f"{base}.scales") != (K // group, 8 * W):
        raise CheckpointError(f"{base}: qzeros/scales shapes do not match qweight [{K}, {W}] "
                              f"with group {group}")
    wc = sc = rw = rg = None
    if ncols is not None:
        c0, c1 = ncols
        if c0 % 8 or c1 % 8:
            raise CheckpointError(f"{base}: column split {c0}:{c1} is not a multiple of 8")
        wc, sc = slice(c0 // 8, c1 // 8), slice(c0, c1)
    if krows is not None:
        k0, k1 = krows
        if k0 % group or k1 % group:
            raise CheckpointError(f"{base}: row split {k0}:{k1} cuts a quantization group")
        rw, rg = slice(k0, k1), slice(k0 // group, k1 // group)
    return dict(qweight=ck.get(f"{base}.qweight", rw, wc),
                qzeros=ck.get(f"{base}.qzeros", rg, wc),
                scales=ck.get(f"{base}.scales", rg, sc))


def _load_fp8(ck: Checkpoint, base: str, nrows: Optional[Tuple[int, int]] = None,
              kcols: Optional[Tuple[int, int]] = None) -> Dict[str, torch.Tensor]:
    """One FP8 projection (e4m3 bytes [N, K] as uint8 + fp32 scale [N]),
    optionally restricted to output rows [n0, n1) or input columns [k0, k1)."""
    if ck.dtype(f"{base}.weight") != "F8_E4M3":
        raise CheckpointError(f"{base}.weight: dtype {ck.dtype(f'{base}.weight')}, expected F8_E4M3")
    if ck.has(f"{base}.bias"):
        raise CheckpointError(f"{base}.bias: projection biases are not part of this decoder")
    if ck.has(f"{base}.input_scale"):
        warnings.warn(f"{base}.input_scale is ignored: activations are quantized per token "
                      "at run time", stacklevel=2)
    N, K = ck.shape(f"{base}.weight")
    rs = slice(*nrows) if nrows is not None else None
    cs = slice(*kcols) if kcols is not None else None
    wq = ck.get(f"{base}.weight", rs, cs).view(torch.uint8)
    sshape = ck.shape(f"{base}.weight_scale")
    s = ck.get(f"{base}.weight_scale").to(torch.float32).reshape(-1)
    if s.numel() == 1:
        s = s.expand(N).contiguous()          # per-tensor scale
    elif s.numel() != N:
        raise CheckpointError(f"{base}.weight_scale: shape {sshape}, expected [] or [{N}]")
    if rs is not None:
        s = s[rs].contiguous()
    return dict(weight_q=wq.contiguous(), weight_scale=s)


def _cat(parts: List[Dict[str, torch.Tensor]], kind: str) -> Dict[str, torch.Tensor]:
    """Merge column-parallel projections (AWQ: along N = dim 1; FP8: rows)."""
    dim = 1 if kind == "awq" else 0
    return {k: torch.cat([p[k] for p in parts], dim) for k in parts[0]}


def load_decoder_weights(path_or_ck, rank: int = 0, world: int = 1, device="cpu") -> Tuple[object, dict]:
    """(DecoderConfig, weights) of one tensor-parallel rank from a checkpoint.

    ``weights`` has the layout of QuantDecoder.state() without the KV cache and
    tokens: embed, final_norm, lm_head (this rank's vocabulary rows) and per
    layer in_norm, post_norm and the quantized tensors of qkv (q/k/v merged,
    this rank's heads), o (this rank's K rows), gate_up, down."""
    ck = path_or_ck if isinstance(path_or_ck, Checkpoint) else Checkpoint(path_or_ck)
    cfg = decoder_config(ck.config)
    spec = quant_spec(ck.config)
    qk = [n for n in ck.names() if n.endswith((".q_norm.weight", ".k_norm.weight"))]
    if qk:
        raise CheckpointError(f"{qk[0]}: per-head q/k RMSNorm (Qwen3 use_qk_norm) is not "
                              "implemented by this decoder")
    R, r = world, rank
    if cfg.heads % R or cfg.kv_heads % R or cfg.intermediate % R or cfg.vocab % R:
        raise CheckpointError(f"tensor parallelism {R} does not divide heads / kv heads / "
                              "intermediate / vocab")
    act = cfg.act_dtype
    d, hq, hkv, I = cfg.head_dim, cfg.heads // R, cfg.kv_heads // R, cfg.intermediate // R
    dev = torch.device(device)

    def dense(name, rows=None):
        t = ck.get(name, rows)
        if not t.is_floating_point():
            raise CheckpointError(f"{name}: dtype {ck.dtype(name)} is not a float type")
        return t.to(act).to(dev)

    def put(d_):
        return {k: v.to(dev) for k, v in d_.items()}

    vl = cfg.vocab // R
    head_name = "lm_head.weight" if ck.has("lm_head.weight") else "model.embed_tokens.weight"
    out = dict(embed=dense("model.embed_tokens.weight"),
               final_norm=dense("model.norm.weight"),
               lm_head=dense(head_name, slice(r * vl, (r + 1) * vl)), layers=[])
    for i in range(cfg.layers):
        n = _proj_names(i)
        cols = {"q": (r * hq * d, (r + 1) * hq * d), "k": (r * hkv * d, (r + 1) * hkv * d),
                "v": (r * hkv * d, (r + 1) * hkv * d), "gate": (r * I, (r + 1) * I),
                "up": (r * I, (r + 1) * I)}
        rows = {"o": (r * hq * d, (r + 1) * hq * d), "down": (r * I, (r + 1) * I)}
        if spec.method == "awq":
            lin = {p: _load_awq(ck, n[p], spec.group, ncols=cols[p]) for p in cols}
            lin.update({p: _load_awq(ck, n[p], spec.group, krows=rows[p]) for p in rows})
        else:
            lin = {p: _load_fp8(ck, n[p], nrows=cols[p]) for p in cols}
            lin.update({p: _load_fp8(ck, n[p], kcols=rows[p]) for p in rows})
        out["layers"].append(dict(
            in_norm=dense(f"model.layers.{i}.input_layernorm.weight"),
            post_norm=dense(f"model.layers.{i}.post_attention_layernorm.weight"),
            qkv=put(_cat([lin["q"], lin["k"], lin["v"]], spec.method)),
            o=put(lin["o"]), gate_up=put(_cat([lin["gate"], lin["up"]], spec.method)),
            down=put(lin["down"])))
    return cfg, out


def _split_cols(t: Dict[str, torch.Tensor], widths: Iterable[int], kind: str):
    """Inverse of _cat for one rank-1 merged projection."""
    widths = list(widths)
    out = [dict() for _ in widths]
    for k, v in t.items():
        if kind == "awq":
            per = 8 if k in ("qweight", "qzeros") else 1
            parts = torch.split(v, [w // per for w in widths], dim=1)
        else:
            parts = torch.split(v, widths, dim=0)
        for o, p in zip(out, parts):
            o[k] = p
    return out


def decoder_tensors(dec) -> Dict[str, torch.Tensor]:
    """A tensor-parallelism-1 QuantDecoder's weights under checkpoint names
    (q/k/v and gate/up split back out of the merged projections)."""
    if dec.world != 1:
        raise CheckpointError("saving needs the tensor-parallelism-1 decoder (assemble ranks first)")
    cfg = dec.cfg
    d = cfg.head_dim
    kind = cfg.quant
    t: Dict[str, torch.Tensor] = {"model.embed_tokens.weight": dec.embed,
                                  "model.norm.weight": dec.final_norm, "lm_head.weight": dec.lm_head}
    for i, L in enumerate(dec.layers):
        n = _proj_names(i)
        t[f"model.layers.{i}.input_layernorm.weight"] = L["in_norm"]
        t[f"model.layers.{i}.post_attention_layernorm.weight"] = L["post_norm"]
        q, k, v = _split_cols(L["qkv"].tensors, [cfg.heads * d, cfg.kv_heads * d, cfg.kv_heads * d], kind)
        g, u = _split_cols(L["gate_up"].tensors, [cfg.intermediate, cfg.intermediate], kind)
        for p, tens in (("q", q), ("k", k), ("v", v), ("gate", g), ("up", u),
                        ("o", L["o"].tensors), ("down", L["down"].tensors)):
            if kind == "awq":
                for key in ("qweight", "qzeros", "scales"):
                    t[f"{n[p]}.{key}"] = tens[key]
            else:
                t[f"{n[p]}.weight"] = tens["weight_q"].view(torch.float8_e4m3fn)
                t[f"{n[p]}.weight_scale"] = tens["weight_scale"]
    return t


def hf_config(cfg) -> dict:
    """config.json for a DecoderConfig (Llama architecture + quantization_config)."""
    qc = ({"quant_method": "awq", "bits": 4, "group_size": cfg.group, "zero_point": True,
           "version": "gemm"} if cfg.quant == "awq"
          else {"quant_method": "fp8", "activation_scheme": "dynamic"})
    return {"architectures": ["LlamaForCausalLM"], "model_type": "llama",
            "num_hidden_layers": cfg.layers, "hidden_size": cfg.hidden,
            "num_attention_heads": cfg.heads, "num_key_value_heads": cfg.kv_heads,
            "head_dim": cfg.head_dim, "intermediate_size": cfg.intermediate,
            "vocab_size": cfg.vocab, "rope_theta": cfg.rope_theta, "rms_norm_eps": cfg.eps,
            "torch_dtype": "float16" if cfg.act == "f16" else "bfloat16",
            "tie_word_embeddings": False, "quantization_config": qc}


def save_decoder(dec, path: str, shards: int = 1) -> None:
    """Write a tensor-parallelism-1 QuantDecoder as a (sharded) checkpoint."""
    save_sharded(path, decoder_tensors(dec), shards, hf_config(dec.cfg))
