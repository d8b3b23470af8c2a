"""Tensor-parallel sharding and reduction on CPU: world_size-2 gloo process groups.

The per-rank compute is a test double backed by the CPU oracle (tests only);
what is under test is the host logic of lmrs_b200.tp — how AWQ / FP8 tensors
are cut (whole packed words, whole quantisation groups, per-channel scales),
the all-reduce of row-parallel partials, the bias added once — and that a rank
that never arrives turns into an error on the other rank instead of a hang.
"""
import os
import socket
import traceback

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from lmrs_b200 import tp
from lmrs_b200.ops import AwqConfig, LinearConfig
from oracle import oracle as O


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


class OracleAwq:
    """Test double: AWQ linear on CPU through the oracle, fp32 output."""

    def __init__(self, qw, qz, sc, group):
        self.qw, self.qz, self.sc, self.g = qw.numpy(), qz.numpy(), sc.numpy(), group

    def forward(self, x):
        x = x.numpy()
        w = O.c_awq_dequant(self.qw, self.qz, self.sc, self.qw.shape[0], self.qw.shape[1] * 8, self.g)
        return torch.from_numpy((x.astype(np.float64) @ w.astype(np.float64)).astype(np.float32))


class OracleFp8:
    def __init__(self, wq, sw):
        self.wq, self.sw = wq.numpy(), sw.numpy()

    def forward(self, x_bf16_bits):
        xq, sx = O.c_fp8_quant_rows(x_bf16_bits.numpy(), 0)
        return torch.from_numpy(O.np_fp8_linear_f64(xq, sx, self.wq, self.sw).astype(np.float32))


def _worker(rank, world, port, fn, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        import datetime
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=10))
        out = fn(rank, world)
        q.put((rank, "ok", out))
    except Exception as e:  # noqa: BLE001
        q.put((rank, "err", f"{type(e).__name__}: {e}\n{traceback.format_exc()}"))
    finally:
        if dist.is_initialized():
            try:
                dist.destroy_process_group()
            except Exception:  # noqa: BLE001
                pass


def _run(fn, world=2, timeout=120):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, fn, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, status, out = q.get(timeout=timeout)
        res[r] = (status, out)
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    return res


# ------------------------------------------------------------ rank bodies
def _awq_case():
    d = O.awq_inputs(3, 512, 256, 128, seed=21, with_bias=True)
    return d


def _awq_column_body(rank, world):
    d = _awq_case()
    qw, qz, sc = (torch.from_numpy(d[k]) for k in ("qweight", "qzeros", "scales"))
    lqw, lqz, lsc = tp.shard_awq_column(qw, qz, sc, rank, world)
    y_local = tp.ColumnParallel(OracleAwq(lqw, lqz, lsc, 128)).forward(torch.from_numpy(d["x"]))
    parts = [torch.empty_like(y_local) for _ in range(world)]
    dist.all_gather(parts, y_local)
    return torch.cat(parts, dim=1).numpy()


def _awq_row_body(rank, world):
    d = _awq_case()
    qw, qz, sc = (torch.from_numpy(d[k]) for k in ("qweight", "qzeros", "scales"))
    lqw, lqz, lsc = tp.shard_awq_row(qw, qz, sc, rank, world, 128)
    K = d["K"] // world
    x_local = torch.from_numpy(np.ascontiguousarray(d["x"][:, rank * K:(rank + 1) * K]))
    bias = torch.from_numpy(d["bias"].astype(np.float32))
    layer = tp.RowParallel(OracleAwq(lqw, lqz, lsc, 128), bias=bias)
    return layer.forward(x_local).numpy()


def _fp8_row_body(rank, world):
    f = O.fp8_inputs(2, 256, 64, seed=5)
    wq, sw = O.c_fp8_quant_rows(f["w_bf16"], 0)
    lwq, lsw = tp.shard_fp8_row(torch.from_numpy(wq), torch.from_numpy(sw), rank, world)
    K = 256 // world
    x_local = torch.from_numpy(np.ascontiguousarray(f["x_bf16"][:, rank * K:(rank + 1) * K]))
    return tp.RowParallel(OracleFp8(lwq, lsw)).forward(x_local).numpy()


def _silent_rank_body(rank, world):
    """Rank 1 skips the collective; rank 0 must get an error, not hang."""
    y = torch.ones(4)
    if rank == 1:
        import time
        time.sleep(15)
        return "skipped"
    dist.all_reduce(y)
    return y.numpy()


# ------------------------------------------------------------------ tests
def test_awq_column_parallel_matches_full():
    d = _awq_case()
    res = _run(_awq_column_body)
    w = O.np_awq_dequant(d["qweight"], d["qzeros"], d["scales"], 128)
    full = d["x"].astype(np.float64) @ w.astype(np.float64)
    for r in (0, 1):
        status, out = res[r]
        assert status == "ok", out
        assert np.allclose(out, full, rtol=1e-5, atol=1e-4)


def test_awq_row_parallel_matches_full():
    d = _awq_case()
    res = _run(_awq_row_body)
    w = O.np_awq_dequant(d["qweight"], d["qzeros"], d["scales"], 128)
    full = d["x"].astype(np.float64) @ w.astype(np.float64) + d["bias"].astype(np.float64)
    for r in (0, 1):
        status, out = res[r]
        assert status == "ok", out
        assert np.allclose(out, full, rtol=1e-5, atol=1e-3)


def test_fp8_row_parallel_uses_local_token_scales():
    """Row-parallel FP8 quantises each rank's K-slice with its own per-token scale,
    so TP results equal the oracle run with the same sharding (not TP=1)."""
    res = _run(_fp8_row_body)
    f = O.fp8_inputs(2, 256, 64, seed=5)
    wq, sw = O.c_fp8_quant_rows(f["w_bf16"], 0)
    ref = 0
    for r in range(2):
        xs = np.ascontiguousarray(f["x_bf16"][:, r * 128:(r + 1) * 128])
        xq, sx = O.c_fp8_quant_rows(xs, 0)
        ref = ref + O.np_fp8_linear_f64(xq, sx, np.ascontiguousarray(wq[:, r * 128:(r + 1) * 128]), sw)
    for r in (0, 1):
        status, out = res[r]
        assert status == "ok", out
        assert np.allclose(out, ref, rtol=1e-5, atol=1e-4)


def test_shard_shapes_and_validation():
    d = O.awq_inputs(1, 1024, 512, 128, seed=2)
    qw, qz, sc = (torch.from_numpy(d[k]) for k in ("qweight", "qzeros", "scales"))
    for world in (2, 4, 8):
        for rank in range(world):
            a = tp.shard_awq_column(qw, qz, sc, rank, world)
            assert a[0].shape == (1024, 64 // world) and a[2].shape == (8, 512 // world)
            b = tp.shard_awq_row(qw, qz, sc, rank, world, 128)
            assert b[0].shape == (1024 // world, 64) and b[1].shape == (8 // world, 64)
    # reassembly is exact
    parts = [tp.shard_awq_row(qw, qz, sc, r, 4, 128)[0] for r in range(4)]
    assert torch.equal(torch.cat(parts, 0), qw)
    with pytest.raises(ValueError):
        tp.shard_awq_row(qw, qz, sc, 0, 16, 128)  # 1024/16 = 64 rows: not whole groups


def test_silent_rank_is_detected():
    res = _run(_silent_rank_body, timeout=90)
    assert res[1] == ("ok", "skipped")
    status, out = res[0]
    assert status == "err", "rank 0's collective should fail when rank 1 never joins"
