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
        # the two-stage form (reduce-scatter + all-gather; by default from 4
        # ranks), forced here at 2: the same exact sums, slices uneven or empty
        try:
            L.set_tuning("ar_two_stage_min_world", 2)
            L.set_tuning("ar_two_stage_min_elems", 2)
            for dtype in (torch.bfloat16, torch.float16):
                for n in (2, 8194, 262144):
                    for rep in range(2):
                        g = torch.Generator(device=dev).manual_seed(77 * rep + n + rank)
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
                        results[("two-stage", str(dtype), n, rep)] = (ok, same)
        finally:
            L.set_tuning("ar_two_stage_min_world", 4)
            L.set_tuning("ar_two_stage_min_elems", 131072)
        # the fused all-reduce + residual add + RMSNorm against the all-reduce
        # followed by the norm kernel; identical on both ranks
        from lmrs_b200 import decode_ops as DO
        for dtype in (torch.bfloat16, torch.float16):
            for rows, H in ((1, 8192), (32, 8192), (7, 4096), (200, 4096)):
                g = torch.Generator(device=dev).manual_seed(rows + H)  # same on every rank
                h0 = torch.randn(rows, H, generator=g, device=dev).to(dtype)
                w = (1.0 + 0.1 * torch.randn(H, generator=g, device=dev)).to(dtype)
                gp = torch.Generator(device=dev).manual_seed(rows + H + 100 * (rank + 1))
                part = torch.randn(rows, H, generator=gp, device=dev).to(dtype)
                red = part.clone()
                ar(red)
                h_ref = h0.clone()
                ref = DO.rmsnorm(h_ref, w, 1e-5, red)
                h = h0.clone()
                out = ar.rmsnorm(part, h, w, 1e-5)
                hq = h0.clone()
                q, sc = ar.rmsnorm_fp8(part, hq, w, 1e-5)
                ok = (torch.equal(h, h_ref) and torch.equal(hq, h_ref)
                      and _ulp_close(out, ref, dtype))
                same = True
                for t in (out, q, sc):
                    allt = [torch.empty_like(t) for _ in range(world)]
                    dist.all_gather(allt, t)
                    same = same and all(torch.equal(allt[0], a) for a in allt)
                results[("fused", str(dtype), rows, H)] = (ok, same)
        results["device_error"] = L.read_device_error()
        ar.close()
        if rank == 0:
            torch.save(results, out_path)
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_wait_gives_up_without_peer():
    """The all-reduce's bounded wait, made to run out on one GPU: a 2-rank call
    whose second rank is only a local buffer nobody writes into.  With the wait
    limit lowered to ~1 ms the call must return, flag kErrWaitPeer in the device
    error word and leave NaN where the missing rank's packets belong; after the
    limit and the buffers are reset, the next call is clean.  No kernel waits on
    another launch: rank 1's packets simply never come."""
    import ctypes
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import lmrs_b200 as L
    from lmrs_b200 import _lib
    lib = _lib.load()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    n, world = 4096, 2
    nbytes = lib.lmrs_allreduce_buffer_bytes(world, n)
    bufs = (ctypes.c_void_p * world)()

    def alloc():  # zero-filled receive buffers (epoch 0)
        for r in range(world):
            p = ctypes.c_void_p()
            _lib.check("lmrs_comm_alloc", lib.lmrs_comm_alloc(ctypes.byref(p), nbytes))
            bufs[r] = p

    def free():
        torch.cuda.synchronize()
        for r in range(world):
            lib.lmrs_comm_free(bufs[r])
            bufs[r] = None

    alloc()
    stream = torch.cuda.current_stream().cuda_stream
    x = torch.ones(n, dtype=torch.bfloat16, device=dev)
    y = torch.zeros_like(x)
    try:
        assert L.read_device_error() == 0
        L.set_tuning("wait_limit_kcycles", 2000)  # ~1 ms at 1.9 GHz
        _lib.check("lmrs_allreduce_sum", lib.lmrs_allreduce_sum(
            y.data_ptr(), x.data_ptr(), n, _lib.DTYPE_BF16, 0, world, bufs, n, stream))
        torch.cuda.synchronize()
        assert L.read_device_error() & (1 << 5), "kErrWaitPeer not flagged"
        assert bool(torch.isnan(y.float()).all()), "a missing peer must not yield a sum"
        # reset: default limit, fresh buffers; a single-rank call is then exact and clean
        L.set_tuning("wait_limit_kcycles", 0)
        free()
        alloc()
        y2 = torch.empty_like(x)
        _lib.check("lmrs_allreduce_sum", lib.lmrs_allreduce_sum(
            y2.data_ptr(), x.data_ptr(), n, _lib.DTYPE_BF16, 0, 1, bufs, n, stream))
        torch.cuda.synchronize()
        assert torch.equal(y2, x)
        assert L.read_device_error() == 0
    finally:
        L.set_tuning("wait_limit_kcycles", 0)
        free()


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


def _ulp_close(a, b, dtype):
    """Equal up to one unit in the last place of dtype (the norm's sum of squares
    is reduced in a different order by the fused kernel, so 1/rms may differ in
    its last bit)."""
    ulp = 2.0 ** (-7 if dtype == torch.bfloat16 else -10)
    d = (a.float() - b.float()).abs()
    return bool((d <= ulp * b.float().abs().clamp_min(1e-30)).all())


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("rows,H", [(1, 8192), (5, 4096), (64, 1280), (300, 8192), (3, 14336)])
def test_allreduce_rmsnorm_single_rank(dtype, rows, H):
    """The fused all-reduce + residual add + RMSNorm (lmrs_allreduce_rmsnorm and
    its FP8 form) with one rank, against lmrs_rmsnorm[_fp8] with the partial as
    the delta: the updated residual bit for bit, the output within one ulp (FP8:
    the same e4m3 bytes wherever the scale agrees), over repeated calls (the
    buffers' phases alternate) and CUDA-graph replays.  Rows beyond the grid's
    clusters (300) exercise the clusters' row loop; H = 1280 leaves columns of
    the last CTA unused."""
    import ctypes
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import lmrs_b200 as L
    from lmrs_b200 import _lib
    from lmrs_b200 import decode_ops as DO
    lib = _lib.load()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    n = rows * H
    nbytes = lib.lmrs_allreduce_buffer_bytes(1, n)
    own = ctypes.c_void_p()
    _lib.check("lmrs_comm_alloc", lib.lmrs_comm_alloc(ctypes.byref(own), nbytes))
    bufs = (ctypes.c_void_p * 1)(own.value)
    code = _lib.DTYPE_BF16 if dtype == torch.bfloat16 else _lib.DTYPE_F16
    stream = torch.cuda.current_stream().cuda_stream
    g = torch.Generator(device=dev).manual_seed(rows * 7 + H)
    h0 = torch.randn(rows, H, generator=g, device=dev).to(dtype)
    w = (1.0 + 0.1 * torch.randn(H, generator=g, device=dev)).to(dtype)
    eps = 1e-5
    try:
        for rep in range(3):
            part = (torch.randn(rows, H, generator=g, device=dev) * (rep + 1)).to(dtype)
            # plain form
            h_ref, h = h0.clone(), h0.clone()
            ref = DO.rmsnorm(h_ref, w, eps, part)
            out = torch.empty_like(h)
            _lib.check("lmrs_allreduce_rmsnorm", lib.lmrs_allreduce_rmsnorm(
                out.data_ptr(), h.data_ptr(), part.data_ptr(), w.data_ptr(), rows, H, eps, code,
                0, 1, bufs, n, stream))
            torch.cuda.synchronize()
            assert torch.equal(h, h_ref), rep
            assert _ulp_close(out, ref, dtype), rep
            # FP8 form
            h_ref, h = h0.clone(), h0.clone()
            qr, sr = DO.rmsnorm_fp8(h_ref, w, eps, part)
            q = torch.empty(rows, H, dtype=torch.uint8, device=dev)
            sc = torch.empty(rows, dtype=torch.float32, device=dev)
            _lib.check("lmrs_allreduce_rmsnorm_fp8", lib.lmrs_allreduce_rmsnorm_fp8(
                q.data_ptr(), sc.data_ptr(), h.data_ptr(), part.data_ptr(), w.data_ptr(), rows, H,
                eps, code, 0, 1, bufs, n, stream))
            torch.cuda.synchronize()
            assert torch.equal(h, h_ref), rep
            assert bool((((sc - sr).abs() / sr.abs().clamp_min(1e-30)) <= 2.0 ** -6).all()), rep
            # decoded values within one e4m3 step; nearly all bytes identical
            dq = q.view(torch.float8_e4m3fn).float() * sc[:, None]
            dr = qr.view(torch.float8_e4m3fn).float() * sr[:, None]
            assert bool(((dq - dr).abs() <= 2.0 ** -3 * dr.abs() + 2.0 ** -9 * sr[:, None]).all()), rep
            assert (q != qr).float().mean().item() < 1e-3, rep
        # graph capture: two fused calls per replay (phases alternate inside the graph)
        part = torch.randn(rows, H, generator=g, device=dev).to(dtype)
        h = h0.clone()
        out = torch.empty_like(h)
        call = lambda: lib.lmrs_allreduce_rmsnorm(
            out.data_ptr(), h.data_ptr(), part.data_ptr(), w.data_ptr(), rows, H, eps, code, 0, 1,
            bufs, n, torch.cuda.current_stream().cuda_stream)
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            call()
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            call()
            call()
        for _ in range(3):
            h.copy_(h0)
            h_ref = h0.clone()
            DO.rmsnorm(h_ref, w, eps, part)
            ref = DO.rmsnorm(h_ref, w, eps, part)
            gr.replay()
            torch.cuda.synchronize()
            assert torch.equal(h, h_ref)
            assert _ulp_close(out, ref, dtype)
        del gr
        assert L.read_device_error() == 0
    finally:
        torch.cuda.synchronize()
        lib.lmrs_comm_free(own)
