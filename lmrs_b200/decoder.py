"""Decode-step harness for the quantized linears (BASELINE configs 3 and 4).

A Llama-shaped decoder (the reference's qwen3 block with use_qk_norm = false,
crates/model/src/layers/block.rs:118-130) whose q/k/v/o/gate/up/down
projections run on lmrs_b200's AWQ W4A16 or FP8 W8A8 linears.
- q/k/v and gate/up are each merged into one column-parallel projection (one
  launch instead of three or two).
- o and down are row-parallel and are followed by a sum all-reduce when
  tensor parallelism is on.

The support ops (residual add + RMSNorm, RoPE + KV write, paged GQA decode
attention, SiLU * up) run on this package's decode kernels (decode_ops.py,
include/lmrs_decode.h), with the FP8 per-token quantisation folded into the
norm and activation kernels; fused=False runs them in plain torch instead (for
comparison).  The LM head is a plain bf16/fp16 matmul.  Weights are random
(seeded), the KV cache is pre-filled
with random values to the configured context, and one decode step feeds one
token per sequence at position ctx - 1 (the step is replayed unchanged, which
keeps it CUDA-graph friendly).
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional

import torch
import torch.nn.functional as F

from . import decode_ops as DO
from . import ops


@dataclass(frozen=True)
class DecoderConfig:
    layers: int
    hidden: int
    heads: int
    kv_heads: int
    head_dim: int
    intermediate: int
    vocab: int
    quant: str            # "awq" (W4A16) or "fp8" (W8A8)
    group: int = 128
    rope_theta: float = 500000.0
    eps: float = 1e-5
    # activation / embedding / norm / KV dtype: "bf16" (the reference model's,
    # crates/model/src/loader/safetensors.rs:274) or "f16" (AWQ only; the FP8
    # linear takes bf16)
    act: str = "bf16"

    def __post_init__(self):
        if self.act not in ("bf16", "f16") or (self.quant == "fp8" and self.act != "bf16"):
            raise ValueError(f"activation dtype {self.act!r} with {self.quant}: AWQ takes bf16 "
                             "or f16, FP8 bf16")

    @property
    def act_dtype(self) -> torch.dtype:
        return torch.bfloat16 if self.act == "bf16" else torch.float16

    def projections(self, world: int = 1):
        """(K, N) of one rank's qkv, o, gate_up, down projections."""
        d, H = self.head_dim, self.hidden
        hq, hkv, inter = self.heads // world, self.kv_heads // world, self.intermediate // world
        return [(H, (hq + 2 * hkv) * d), (hq * d, H), (H, 2 * inter), (inter, H)]

    def linear_bytes(self, world: int = 1) -> int:
        """One rank's quantized projection bytes over all layers (AWQ: packed
        weights + zeros + fp16 scales; FP8: e4m3 weights + fp32 channel scales)."""
        n = 0
        for K, N in self.projections(world):
            if self.quant == "awq":
                g = self.group
                n += K * N // 2 + (K // g) * (N // 8) * 4 + (K // g) * N * 2
            else:
                n += N * K + 4 * N
        return n * self.layers


LLAMA3_8B_AWQ = DecoderConfig(32, 4096, 32, 8, 128, 14336, 128256, "awq")
LLAMA3_70B_FP8 = DecoderConfig(80, 8192, 64, 8, 128, 28672, 128256, "fp8")


def _awq_random(K: int, N: int, group: int, gen: torch.Generator, device) -> dict:
    """Random AWQ tensors with the config-0 distributions: uniform nibbles for q
    and z (uniform 32-bit words), scales U[0.001, 0.02] fp16."""
    qw = torch.randint(-2 ** 31, 2 ** 31 - 1, (K, N // 8), dtype=torch.int32, generator=gen,
                       device=device)
    qz = torch.randint(-2 ** 31, 2 ** 31 - 1, (K // group, N // 8), dtype=torch.int32,
                       generator=gen, device=device)
    sc = (torch.rand((K // group, N), generator=gen, device=device) * 0.019 + 0.001).half()
    return dict(qweight=qw, qzeros=qz, scales=sc)


def _fp8_random(K: int, N: int, gen: torch.Generator, device) -> dict:
    """W ~ N(0, 0.02) bf16 [N, K], quantised per output channel to e4m3 (on the GPU)."""
    w = (torch.randn((N, K), generator=gen, device=device) * 0.02).bfloat16()
    wq, sw = ops.quantize_fp8_weight(w)
    del w
    return dict(weight_q=wq, weight_scale=sw)


class QuantDecoder:
    """One tensor-parallel rank of the decoder (world = 1 for a single GPU)."""

    def __init__(self, cfg: DecoderConfig, batch: int, ctx: int, device, rank: int = 0,
                 world: int = 1, seed: int = 0, group=None, fused: bool = True,
                 allreduce: str = "peer", weights: Optional[dict] = None):
        """Random (seeded) weights, or `weights` in the layout of state() without
        the KV cache and tokens (e.g. checkpoint.load_decoder_weights for this
        rank); the KV cache and token ids are random either way."""
        if cfg.heads % world or cfg.intermediate % world or cfg.kv_heads % world:
            raise ValueError(f"tensor parallelism {world} does not divide heads / kv heads / intermediate")
        if cfg.vocab % world:
            raise ValueError(f"vocab {cfg.vocab} not divisible by {world}")
        self.cfg, self.batch, self.ctx = cfg, batch, ctx
        self.fused = fused
        # row-parallel sums: the package's one-shot NVLink all-reduce ("peer") up to
        # PEER_MAX_ELEMS elements, NCCL above that or when allreduce == "nccl";
        # with the peer all-reduce the sum is fused into the norm that follows it
        # (lmrs_allreduce_rmsnorm[_fp8]) unless fuse_allreduce is False
        self.allreduce_kind = allreduce
        self.fuse_allreduce = True
        # RoPE + KV write inside the attention kernel (lmrs_rope_paged_attention_decode)
        self.fuse_rope = True
        # FP8: each layer as one persistent kernel (lmrs_fp8_decode_layer) instead of
        # the per-op kernels; set_batch turns it on where the shapes allow it
        self.layer_kernel = False
        self._lk = None
        self.par = None
        self.device = torch.device(device)
        self.rank, self.world, self.pg = rank, world, group
        self.hq, self.hkv = cfg.heads // world, cfg.kv_heads // world
        self.inter = cfg.intermediate // world
        self.vocab_local = cfg.vocab // world
        self.act = cfg.act_dtype
        d, H = cfg.head_dim, cfg.hidden
        # shard-local weights from a per-rank stream; replicated tensors (embedding,
        # norms) from one stream shared by all ranks
        gen = torch.Generator(device=self.device).manual_seed(seed * 1000 + rank)
        rep = torch.Generator(device=self.device).manual_seed(seed * 1000 + 999)

        def lin(K, N, given=None):
            if given is not None:
                if cfg.quant == "awq":
                    return ops.QuantLinearOp.awq(ops.LinearConfig(K, N), given["qweight"],
                                                 given["qzeros"], given["scales"], None,
                                                 ops.AwqConfig(cfg.group))
                return ops.QuantLinearOp.fp8(ops.LinearConfig(K, N), given["weight_q"],
                                             given["weight_scale"])
            if cfg.quant == "awq":
                t = _awq_random(K, N, cfg.group, gen, self.device)
                return ops.QuantLinearOp.awq(ops.LinearConfig(K, N), t["qweight"], t["qzeros"],
                                             t["scales"], None, ops.AwqConfig(cfg.group))
            t = _fp8_random(K, N, gen, self.device)
            return ops.QuantLinearOp.fp8(ops.LinearConfig(K, N), t["weight_q"], t["weight_scale"])

        shapes = cfg.projections(world)
        self.layers = []
        if weights is not None:
            dev = self.device
            self.embed = weights["embed"].to(dev, self.act)
            self.final_norm = weights["final_norm"].to(dev, self.act)
            self.lm_head = weights["lm_head"].to(dev, self.act)
            if len(weights["layers"]) != cfg.layers:
                raise ValueError(f"{len(weights['layers'])} layers given, config has {cfg.layers}")
            for W in weights["layers"]:
                self.layers.append(dict(
                    in_norm=W["in_norm"].to(dev, self.act), post_norm=W["post_norm"].to(dev, self.act),
                    **{k: lin(*shp, {n: t.to(dev) for n, t in W[k].items()})
                       for k, shp in zip(("qkv", "o", "gate_up", "down"), shapes)}))
        else:
            self.embed = (torch.randn((cfg.vocab, H), generator=rep, device=self.device) * 0.02).to(self.act)
            for _ in range(cfg.layers):
                self.layers.append(dict(
                    in_norm=(1.0 + 0.02 * torch.randn(H, generator=rep, device=self.device)).to(self.act),
                    post_norm=(1.0 + 0.02 * torch.randn(H, generator=rep, device=self.device)).to(self.act),
                    qkv=lin(*shapes[0]),        # column-parallel, q/k/v merged
                    o=lin(*shapes[1]),          # row-parallel
                    gate_up=lin(*shapes[2]),    # column-parallel, gate/up merged
                    down=lin(*shapes[3]),       # row-parallel
                ))
            self.final_norm = (1.0 + 0.02 * torch.randn(H, generator=rep, device=self.device)).to(self.act)
            self.lm_head = (torch.randn((self.vocab_local, H), generator=gen, device=self.device)
                            * 0.02).to(self.act)
        pos = ctx - 1
        inv = 1.0 / (cfg.rope_theta ** (torch.arange(0, d, 2, device=self.device, dtype=torch.float32) / d))
        ang = pos * inv
        self.cos = torch.cat([ang.cos(), ang.cos()]).to(self.act)
        self.sin = torch.cat([ang.sin(), ang.sin()]).to(self.act)
        self.kv = None
        self.set_batch(batch, seed)

    @classmethod
    def from_checkpoint(cls, path: str, batch: int, ctx: int, device, rank: int = 0,
                        world: int = 1, **kw) -> "QuantDecoder":
        """This rank's decoder from a quantized (AWQ or FP8) safetensors
        checkpoint directory (checkpoint.load_decoder_weights)."""
        from .checkpoint import load_decoder_weights
        cfg, weights = load_decoder_weights(path, rank, world, device)
        return cls(cfg, batch, ctx, device, rank=rank, world=world, weights=weights, **kw)

    # ---------------------------------------------------------------- state
    def state(self) -> dict:
        """Every tensor of this rank (weights, KV cache, token ids), by reference."""
        return dict(embed=self.embed, final_norm=self.final_norm, lm_head=self.lm_head,
                    tokens=self.tokens, kv=self.kv,
                    layers=[dict(in_norm=L["in_norm"], post_norm=L["post_norm"],
                                 **{k: dict(L[k].tensors) for k in ("qkv", "o", "gate_up", "down")})
                            for L in self.layers])

    def load_state(self, st: dict) -> None:
        """Copy a state() of the same shapes into this decoder (in place)."""
        own = self.state()
        for key in ("embed", "final_norm", "lm_head", "tokens", "kv"):
            own[key].copy_(st[key])
        for mine, theirs in zip(own["layers"], st["layers"]):
            for key in ("in_norm", "post_norm"):
                mine[key].copy_(theirs[key])
            for key in ("qkv", "o", "gate_up", "down"):
                for name, t in mine[key].items():
                    t.copy_(theirs[key][name])

    @staticmethod
    def kv_bytes(cfg: DecoderConfig, batch: int, ctx: int, world: int = 1) -> int:
        """Bytes of one rank's KV cache ([layers, 2, batch, kv_heads / world, ctx, head_dim])."""
        return cfg.layers * 2 * batch * (cfg.kv_heads // world) * ctx * cfg.head_dim * 2

    def set_batch(self, batch: int, seed: int = 0):
        """(Re)allocate the KV cache, pre-filled with random values to ctx, and
        draw random token ids for `batch` sequences; the weights are kept."""
        cfg = self.cfg
        self.kv = None
        torch.cuda.empty_cache()
        self.batch = batch
        gen = torch.Generator(device=self.device).manual_seed(seed * 1000 + self.rank + 7)
        kv_shape = (cfg.layers, 2, batch, self.hkv, self.ctx, cfg.head_dim)
        self.kv = torch.empty(kv_shape, dtype=self.act, device=self.device)
        for li in range(cfg.layers):  # per layer, in the activation dtype: no fp32 temporaries
            self.kv[li].normal_(0.0, 0.5, generator=gen)
        # every rank draws the same ids (replicated embedding)
        tg = torch.Generator(device=self.device).manual_seed(seed * 1000 + 11)
        self.tokens = torch.randint(0, cfg.vocab, (batch,), generator=tg, device=self.device)
        # the per-layer cache [batch, kv_heads, ctx, d] read as a paged cache with one
        # block of ctx positions per sequence (block table row b = [b])
        self.block_tables = torch.arange(batch, dtype=torch.int32, device=self.device).view(batch, 1)
        self.positions = torch.full((batch,), self.ctx - 1, dtype=torch.int32, device=self.device)
        self.context_lens = torch.full((batch,), self.ctx, dtype=torch.int32, device=self.device)
        self.attn_ws = DO.AttentionWorkspace()
        self._lk = None
        n = batch * cfg.hidden
        if self.world > 1 and self.allreduce_kind == "peer" and n <= self.PEER_MAX_ELEMS:
            if self.par is None or self.par.max_elems < n:
                from .comm import PeerAllReduce
                self.close()
                self.par = PeerAllReduce(n, group=self.pg)

    # ---------------------------------------------------------------- pieces
    def _rms(self, x, w):
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.cfg.eps)).to(self.act) * w

    def _rope(self, x):  # x [B, heads, d] — rotate-half, as the reference's pos_embed kernel
        half = x.shape[-1] // 2
        rot = torch.cat([-x[..., half:], x[..., :half]], dim=-1)
        return x * self.cos + rot * self.sin

    PEER_MAX_ELEMS = 1 << 22
    # lmrs_allreduce_sum's defaults for its two-stage form (reduce-scatter +
    # all-gather); the fused all-reduce + norm is one-shot only
    TWO_STAGE_MIN_WORLD, TWO_STAGE_MIN_ELEMS = 4, 131072

    def _all_reduce(self, y):
        if self.world > 1:
            if self.par is not None and y.numel() <= self.par.max_elems:
                self.par(y)
            else:
                torch.distributed.all_reduce(y, group=self.pg)
        return y

    def _fused_ar(self, partial) -> bool:
        # the fused kernel's cluster barriers cost more than the saved launch on
        # one short row (world 1, graph-timed: H 4096 x 1 row 4.67 us against 4.29
        # for all-reduce + norm; H 8192: 5.25 against 5.92; 64 rows of 4096: 6.10
        # against 6.73); large messages at 4+ ranks take the two-stage all-reduce
        # (about 2n packets per rank instead of world x n) and a separate norm
        rows, H = partial.shape[0], partial.shape[-1]
        two_stage = (self.world >= self.TWO_STAGE_MIN_WORLD
                     and partial.numel() >= self.TWO_STAGE_MIN_ELEMS)
        return (self.fuse_allreduce and self.world > 1 and self.par is not None
                and partial.numel() <= self.par.max_elems and (H >= 8192 or rows >= 16)
                and not two_stage)

    def _norm(self, h, w, delta, fp8: bool):
        """residual h += delta, then the norm (FP8: its e4m3 bytes and scales).
        delta is a row-parallel projection's per-rank partial sum (None for the
        first layer): summed over the ranks in the norm's own kernel when the
        peer all-reduce is up, else all-reduced first."""
        eps = self.cfg.eps
        if delta is not None and self._fused_ar(delta):
            return self.par.rmsnorm_fp8(delta, h, w, eps) if fp8 else self.par.rmsnorm(delta, h, w, eps)
        if delta is not None:
            delta = self._all_reduce(delta)
        return DO.rmsnorm_fp8(h, w, eps, delta) if fp8 else DO.rmsnorm(h, w, eps, delta)

    def close(self):
        """Release the all-reduce buffers' IPC mappings (before the process group goes)."""
        if self.par is not None:
            self.par.close()
            self.par = None

    def layer_kernel_ok(self) -> bool:
        """Whether lmrs_fp8_decode_layer can run this decoder: FP8, 1..8 tokens,
        the kernel's shape rules, and (tensor parallel) the peer all-reduce."""
        cfg = self.cfg
        if cfg.quant != "fp8" or not 1 <= self.batch <= 8 or cfg.head_dim != 128:
            return False
        if self.world > 1 and (self.par is None or self.batch * cfg.hidden > self.par.max_elems):
            return False
        shp = DO._lib.Fp8LayerShape(self.batch, cfg.hidden, self.hq, self.hkv, cfg.head_dim,
                                    self.inter, self.ctx, 1, self.ctx, cfg.eps, 1.0)
        import ctypes
        return DO._lib.load().lmrs_fp8_decode_layer_workspace_bytes(ctypes.byref(shp)) > 0

    def _layer_setup(self):
        if self._lk is None:
            cfg, d = self.cfg, self.cfg.head_dim
            lk = DO.Fp8DecodeLayer(self.batch, cfg.hidden, self.hq, self.hkv, self.inter,
                                   block_size=self.ctx, max_blocks_per_seq=1, max_context=self.ctx,
                                   eps=cfg.eps, scale=1.0 / math.sqrt(d), device=self.device)
            structs = []
            for li, L in enumerate(self.layers):
                w = [(L[k].tensors["weight_q"], L[k].tensors["weight_scale"])
                     for k in ("qkv", "o", "gate_up", "down")]
                structs.append(lk.layer(*w, L["in_norm"], L["post_norm"], self.kv[li, 0],
                                        self.kv[li, 1]))
            delta = torch.empty((self.batch, cfg.hidden), dtype=self.act, device=self.device)
            self._lk = (lk, structs, delta)
        return self._lk

    def _logits_layer_kernel(self, tokens: Optional[torch.Tensor] = None) -> torch.Tensor:
        """The FP8 step with one persistent kernel per layer (lmrs_fp8_decode_layer):
        norms, projections, RoPE + KV write, attention, SiLU and, tensor parallel,
        the all-reduces inside it; the last layer's down output goes through the
        final norm's all-reduce as in the per-op step."""
        lk, structs, delta = self._layer_setup()
        tok = self.tokens if tokens is None else tokens
        h = self.embed[tok]                                    # [B, H], residual stream
        half = self.cfg.head_dim // 2
        cos, sin = self.cos[:half], self.sin[:half]
        tp = self.world > 1
        bases = self.par.bases if tp else None
        max_elems = self.par.max_elems if tp else 0
        n = len(structs)
        for li, lay in enumerate(structs):
            flags = 0
            if tp:
                flags = ((DO._lib.LAYER_RECV_DELTA if li > 0 else 0)
                         | (DO._lib.LAYER_PUSH_DELTA if li < n - 1 else 0))
            lk.run(lay, h, delta, self.block_tables, self.context_lens, cos, sin,
                   delta_in=delta if (not tp and li > 0) else None, flags=flags,
                   rank=self.rank, world=self.world, bases=bases, max_elems=max_elems)
        r = self._norm(h, self.final_norm, delta, False)
        return r @ self.lm_head.t()                            # [B, vocab / world]

    def step(self, tokens: Optional[torch.Tensor] = None) -> torch.Tensor:
        """One decode step: returns the next token of every sequence."""
        return self._argmax(self.logits(tokens))

    def logits(self, tokens: Optional[torch.Tensor] = None) -> torch.Tensor:
        """One decode step up to this rank's vocabulary shard of the logits."""
        return self._logits_fused(tokens) if self.fused else self._logits_torch(tokens)

    def _logits_fused(self, tokens: Optional[torch.Tensor] = None) -> torch.Tensor:
        """The step on this package's kernels: fused residual add + RMSNorm (with
        the per-token e4m3 quantisation folded in for FP8), RoPE + KV write,
        paged GQA decode attention, SiLU * up, and the quantized projections."""
        if self.layer_kernel:
            return self._logits_layer_kernel(tokens)
        cfg, d, B = self.cfg, self.cfg.head_dim, self.batch
        tok = self.tokens if tokens is None else tokens
        fp8 = cfg.quant == "fp8"
        h = self.embed[tok]                                    # [B, H], residual stream
        half = d // 2
        cos, sin = self.cos[:half], self.sin[:half]
        scale = 1.0 / math.sqrt(d)
        delta = None
        for li, L in enumerate(self.layers):
            kc, vc = self.kv[li, 0], self.kv[li, 1]            # [B, hkv, ctx, d]
            if fp8:
                qkv = L["qkv"].forward_prequant(*self._norm(h, L["in_norm"], delta, True))
            else:
                qkv = L["qkv"].forward(self._norm(h, L["in_norm"], delta, False))
            if self.fuse_rope:  # RoPE + KV write inside the attention kernel
                att = DO.rope_paged_attention_decode(
                    qkv, cos, sin, kc, vc, self.block_tables, self.context_lens, self.ctx,
                    self.hq, self.hkv, scale, kv_head_map=1, workspace=self.attn_ws, fp8=fp8)
            else:
                q = DO.rope_kv_write(qkv, cos, sin, kc, vc, self.block_tables, self.positions,
                                     self.hq, self.hkv, d)
                att = (DO.paged_attention_decode_fp8 if fp8 else DO.paged_attention_decode)(
                    q, kc, vc, self.block_tables, self.context_lens, self.ctx, scale,
                    kv_head_map=1, workspace=self.attn_ws)
            if fp8:  # the o projection's e4m3 input straight from the attention
                aq, asc, _ = att
                o = L["o"].forward_prequant(aq, asc)      # this rank's partial sum
            else:
                o = L["o"].forward(att.view(B, self.hq * d))  # this rank's partial sum
            if fp8:
                xq, sx = self._norm(h, L["post_norm"], o, True)
                mq, ms = DO.silu_mul_fp8(L["gate_up"].forward_prequant(xq, sx))
                delta = L["down"].forward_prequant(mq, ms)
            else:
                gu = L["gate_up"].forward(self._norm(h, L["post_norm"], o, False))
                delta = L["down"].forward(DO.silu_mul(gu))
        r = self._norm(h, self.final_norm, delta, False)
        return r @ self.lm_head.t()                            # [B, vocab / world]

    def _logits_torch(self, tokens: Optional[torch.Tensor] = None) -> torch.Tensor:
        """The same step with the support ops in plain torch (comparison path)."""
        cfg, d, B = self.cfg, self.cfg.head_dim, self.batch
        tok = self.tokens if tokens is None else tokens
        h = self.embed[tok]                                    # [B, H]
        pos = self.ctx - 1
        for li, L in enumerate(self.layers):
            r = self._rms(h, L["in_norm"])
            qkv = L["qkv"].forward(r)                          # [B, (hq + 2 hkv) d]
            q = qkv[:, : self.hq * d].view(B, self.hq, d)
            k = qkv[:, self.hq * d: (self.hq + self.hkv) * d].view(B, self.hkv, d)
            v = qkv[:, (self.hq + self.hkv) * d:].view(B, self.hkv, d)
            q, k = self._rope(q), self._rope(k)
            kc, vc = self.kv[li, 0], self.kv[li, 1]            # [B, hkv, ctx, d]
            kc[:, :, pos] = k
            vc[:, :, pos] = v
            a = F.scaled_dot_product_attention(q.unsqueeze(2), kc, vc, enable_gqa=True)
            a = a.reshape(B, self.hq * d).contiguous()
            h = h + self._all_reduce(L["o"].forward(a))
            r = self._rms(h, L["post_norm"])
            gu = L["gate_up"].forward(r)
            m = (F.silu(gu[:, : self.inter]) * gu[:, self.inter:]).contiguous()
            h = h + self._all_reduce(L["down"].forward(m))
        h = self._rms(h, self.final_norm)
        return h @ self.lm_head.t()                            # [B, vocab / world]

    def _argmax(self, logits):
        val, idx = logits.float().max(dim=-1)
        if self.world > 1:
            vals = [torch.empty_like(val) for _ in range(self.world)]
            idxs = [torch.empty_like(idx) for _ in range(self.world)]
            torch.distributed.all_gather(vals, val, group=self.pg)
            torch.distributed.all_gather(idxs, idx, group=self.pg)
            allv, alli = torch.stack(vals), torch.stack(idxs)   # [world, B]
            best = allv.argmax(dim=0)
            idx = alli.gather(0, best.unsqueeze(0)).squeeze(0) + best * self.vocab_local
        return idx

    def linears_only(self):
        """The step's quantized projections alone (same shapes and order), for the
        linear-layer share of the step time."""
        cfg, d, B = self.cfg, self.cfg.head_dim, self.batch
        x = torch.zeros(B, cfg.hidden, dtype=self.act, device=self.device)
        a = torch.zeros(B, self.hq * d, dtype=self.act, device=self.device)
        m = torch.zeros(B, self.inter, dtype=self.act, device=self.device)
        for L in self.layers:
            L["qkv"].forward(x)
            L["o"].forward(a)
            L["gate_up"].forward(x)
            L["down"].forward(m)

    def own_launches_per_step(self) -> int:
        """Kernels of this package one fused decode step launches: per layer the
        norm, qkv projection, RoPE + KV write (inside the attention unless
        fuse_rope is off), attention, o projection (FP8: its per-token
        quantisation is a second kernel), norm, gate/up, SiLU * up and
        down, plus one all-reduce after o and after down when tensor parallel
        unless it is fused into the norm that follows it; then the final norm
        (the embedding gather and the LM head are torch)."""
        fused_ar = self.world > 1 and self._fused_ar(
            torch.empty((self.batch, self.cfg.hidden), device="meta"))
        if self.layer_kernel:  # one kernel per layer, then the final norm (+ its all-reduce)
            return self.cfg.layers + 1 + (1 if self.world > 1 and not fused_ar else 0)
        # FP8: the o projection's input quantisation is its own kernel unless the
        # attention emits it (one KV head on this rank)
        fp8_quant = 1 if self.cfg.quant == "fp8" and self.hkv != 1 else 0
        rope = 0 if self.fuse_rope else 1
        per = 8 + rope + fp8_quant + (2 if self.world > 1 and not fused_ar else 0)
        return per * self.cfg.layers + 1

    def weight_bytes(self) -> int:
        n = 0
        for L in self.layers:
            for key in ("qkv", "o", "gate_up", "down"):
                for t in L[key].tensors.values():
                    n += t.numel() * t.element_size()
        return n


def assemble_awq_tp(states: list, cfg: DecoderConfig) -> dict:
    """The tensor-parallelism-1 state equivalent to per-rank AWQ states (rank
    order): column-parallel projections concatenate their q/k/v (gate/up)
    column blocks rank by rank, row-parallel ones concatenate their K rows
    (whole quantisation groups, so the packing stays exact), the LM head and
    the KV cache concatenate over vocabulary / KV heads."""
    R, d = len(states), cfg.head_dim
    hq, hkv, inter = cfg.heads // R, cfg.kv_heads // R, cfg.intermediate // R

    def cols(t, name, widths):
        # split a column-parallel tensor of one rank into its blocks (in columns of
        # the output; qweight / qzeros hold 8 columns per word)
        per = 8 if name in ("qweight", "qzeros") else 1
        if name in ("weight_q", "weight_scale"):          # FP8 [N, K] / [N]: rows
            return list(torch.split(t, widths, dim=0))
        return list(torch.split(t, [w // per for w in widths], dim=1))

    def merge_col(parts_per_rank, name, widths):
        blocks = [cols(t, name, widths) for t in parts_per_rank]
        out = [blocks[r][j] for j in range(len(widths)) for r in range(R)]
        dim = 0 if name in ("weight_q", "weight_scale") else 1
        return torch.cat(out, dim=dim)

    full = dict(embed=states[0]["embed"], final_norm=states[0]["final_norm"],
                tokens=states[0]["tokens"],
                lm_head=torch.cat([s_["lm_head"] for s_ in states], 0),
                kv=torch.cat([s_["kv"] for s_ in states], 3), layers=[])
    for li in range(cfg.layers):
        ls = [s_["layers"][li] for s_ in states]
        lay = dict(in_norm=ls[0]["in_norm"], post_norm=ls[0]["post_norm"])
        lay["qkv"] = {n: merge_col([l_["qkv"][n] for l_ in ls], n, [hq * d, hkv * d, hkv * d])
                      for n in ls[0]["qkv"]}
        lay["gate_up"] = {n: merge_col([l_["gate_up"][n] for l_ in ls], n, [inter, inter])
                          for n in ls[0]["gate_up"]}
        for key in ("o", "down"):
            lay[key] = {n: torch.cat([l_[key][n] for l_ in ls], 0) for n in ls[0][key]}
        full["layers"].append(lay)
    return full


def graph_step(dec: QuantDecoder, fn=None, warmup: int = 3):
    """Capture one decode step (or `fn`) into a CUDA graph after eager warm-ups."""
    fn = fn or dec.step
    s = torch.cuda.Stream(dec.device)
    s.wait_stream(torch.cuda.current_stream(dec.device))
    with torch.cuda.stream(s):
        for _ in range(warmup):
            fn()
    torch.cuda.current_stream(dec.device).wait_stream(s)
    torch.cuda.synchronize(dec.device)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = fn()
    return g, out
