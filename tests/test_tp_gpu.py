"""Tensor-parallel decode step on 2 GPUs (NCCL): the TP=2 AWQ decoder (column-
parallel merged q/k/v and gate/up, row-parallel o and down with a sum
all-reduce, vocab-parallel LM head) against a TP=1 decoder assembled from the
two ranks' shards; FP8 against an fp32 forward on the assembled dequantised
weights (the row-parallel layers quantise each rank's K slice with its own
per-token scale, so TP=2 and TP=1 FP8 differ by design).  Skipped with fewer
than two GPUs."""
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu

TINY = dict(layers=2, hidden=512, heads=4, kv_heads=2, head_dim=128, intermediate=1024, vocab=1000)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, quant, batch, out_path):
    import datetime
    import torch.distributed as dist
    from lmrs_b200 import decoder as D
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    try:
        cfg = D.DecoderConfig(quant=quant, **TINY)
        dec = D.QuantDecoder(cfg, batch=batch, ctx=64, device=dev, rank=rank, world=world, seed=5,
                             group=dist.group.WORLD)
        logits = dec.logits()
        parts = [torch.empty_like(logits) for _ in range(world)]
        dist.all_gather(parts, logits)
        nxt = dec.step()  # exercises the (value, index) all-gather argmax
        state = {k: v for k, v in dec.state().items()}
        cpu = _to_cpu(state)
        dec.close()
        states = [None] * world
        dist.all_gather_object(states, cpu)
        if rank == 0:
            torch.save(dict(logits=torch.cat(parts, 1).cpu(), next=nxt.cpu(), states=states), out_path)
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _to_cpu(x):
    if isinstance(x, torch.Tensor):
        return x.detach().cpu()
    if isinstance(x, dict):
        return {k: _to_cpu(v) for k, v in x.items()}
    if isinstance(x, list):
        return [_to_cpu(v) for v in x]
    return x


@pytest.mark.parametrize("quant,batch", [("awq", 1), ("awq", 16), ("fp8", 1), ("fp8", 40)])
def test_tp2_matches_tp1(tmp_path, quant, batch):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    from lmrs_b200 import decoder as D
    out = str(tmp_path / "tp.pt")
    mp.start_processes(_worker, args=(2, _free_port(), quant, batch, out), nprocs=2, join=True,
                       start_method="spawn")
    res = torch.load(out, weights_only=False)
    cfg = D.DecoderConfig(quant=quant, **TINY)
    full = D.assemble_awq_tp(res["states"], cfg)
    dev = torch.device("cuda", 0)
    got = res["logits"].to(dev).float()
    if quant == "awq":
        dec1 = D.QuantDecoder(cfg, batch=batch, ctx=64, device=dev, seed=1)
        dec1.load_state(_to_dev(full, dev))
        ref = dec1.logits().float()
        tol = 2e-2
    else:
        # FP8 row-parallel shards carry per-rank channel scales: no single TP=1 FP8
        # weight holds them, so the reference is fp32 on the dequantised shards
        from test_decoder_gpu import _reference_logits
        dec1 = D.QuantDecoder(cfg, batch=batch, ctx=64, device=dev, seed=1)
        for key in ("embed", "final_norm", "lm_head", "tokens", "kv"):
            dec1.state()[key].copy_(full[key])
        dense = []
        for li in range(cfg.layers):
            mine = dec1.layers[li]
            mine["in_norm"].copy_(full["layers"][li]["in_norm"])
            mine["post_norm"].copy_(full["layers"][li]["post_norm"])
            dense.append(_dense_tp([s_["layers"][li] for s_ in res["states"]], cfg, dev))
        ref = _reference_logits(dec1, fake_quant=False, dense=dense).float()
        tol = 1.5e-1
    err = ((got - ref).abs().max() / ref.abs().max()).item()
    assert err < tol, err
    assert torch.equal(res["next"].to(dev), got.argmax(-1))


def _dense_tp(layer_states, cfg, dev):
    """fp32 [K, N] TP=1 projections from per-rank FP8 shards."""
    R, d = len(layer_states), cfg.head_dim
    hq, hkv, inter = cfg.heads // R, cfg.kv_heads // R, cfg.intermediate // R

    def dq(t):
        return (t["weight_q"].to(dev).view(torch.float8_e4m3fn).float()
                * t["weight_scale"].to(dev)[:, None]).t()          # [K, N]

    def merge(key, widths):
        blocks = [torch.split(dq(ls[key]), widths, dim=1) for ls in layer_states]
        return torch.cat([blocks[r][j] for j in range(len(widths)) for r in range(R)], 1)

    return dict(qkv=merge("qkv", [hq * d, hkv * d, hkv * d]),
                gate_up=merge("gate_up", [inter, inter]),
                o=torch.cat([dq(ls["o"]) for ls in layer_states], 0),
                down=torch.cat([dq(ls["down"]) for ls in layer_states], 0))


def _to_dev(x, dev):
    if isinstance(x, torch.Tensor):
        return x.to(dev)
    if isinstance(x, dict):
        return {k: _to_dev(v, dev) for k, v in x.items()}
    if isinstance(x, list):
        return [_to_dev(v, dev) for v in x]
    return x
