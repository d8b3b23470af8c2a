"""The one-shot peer all-reduce (include/lmrs_comm.h) on 2 GPUs: bit-identical
on both ranks, equal to the fp32 sum in rank order rounded once, across sizes,
repeated calls (alternating buffer phases) and CUDA-graph replays.  Skipped
with fewer than two GPUs."""
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, out_path):
    import datetime
    import torch.distributed as dist
    from lmrs_b200.comm import PeerAllReduce
    import lmrs_b200 as L
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    results = {}
    try:
        ar = PeerAllReduce(1 << 20)
        for dtype in (torch.bfloat16, torch.float16):
            for n in (2, 8192, 16384 * 4, 262144, 1 << 20):
                for rep in range(3):
                    g = torch.Generator(device=dev).manual_seed(1000 * rep + n + rank)
                    x = (torch.randn(n, generator=g, device=dev) * (rank + 1)).to(dtype)
                    parts = [torch.empty_like(x) for _ in range(world)]
                    dist.all_gather(parts, x)
                    ref = parts[0].float()
                    for p in parts[1:]:
                        ref = ref + p.float()
                    ar(x)
                    ok = torch.equal(x, ref.to(dtype))
                    allx = [torch.empty_like(x) for _ in range(world)]
                    dist.all_gather(allx, x)
                    same = all(torch.equal(allx[0], a) for a in allx)
                    results[(str(dtype), n, rep)] = (ok, same)
        # graph capture: 5 all-reduces per replay, inputs refilled between replays
        buf = torch.empty(8192, dtype=torch.bfloat16, device=dev)
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            ar(buf.fill_(1))
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            for _ in range(5):
                ar(buf)
        for it in range(4):
            buf.fill_(float(it + rank))
            gr.replay()
            torch.cuda.synchronize()
            # each all-reduce sums world copies: value v -> v * world ... over 5 calls
            v = float(it) * world + sum(range(world)) if world else 0.0
            expect = torch.tensor(v, dtype=torch.float32)
            for _ in range(4):
                expect = expect * world
            results[("graph", it)] = (bool(torch.all(buf.float() == expect.item())), True)
        del gr
        results["device_error"] = L.read_device_error()
        ar.close()
        if rank == 0:
            torch.save(results, out_path)
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_peer_allreduce_2gpu(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    out = str(tmp_path / "ar.pt")
    mp.start_processes(_worker, args=(2, _free_port(), out), nprocs=2, join=True,
                       start_method="spawn")
    res = torch.load(out, weights_only=False)
    assert res.pop("device_error") == 0
    bad = {k: v for k, v in res.items() if not (v[0] and v[1])}
    assert not bad, bad
