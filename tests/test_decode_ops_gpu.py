"""Decode-step kernels around the quantized linears (include/lmrs_decode.h) on the
B200, against plain torch fp32 references of the reference's semantics:
rmsnorm (kernels/ffi/norm_ffi.cu), silu_mul (kernels/ops/activation_kernels.cuh),
rope (kernels/ffi/pos_embed_ffi.cu) and paged decode attention
(kernels/attention/paged_attention.cuh).  The FP8 fused forms must equal the
unfused kernel followed by fp8_quant_rows byte for byte."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu

DTS = [torch.bfloat16, torch.float16]


def _ulp_close(got, ref, dtype):
    """got within one unit in the last place of ref (the same fp32 value computed
    in a different order, rounded once to the I/O type)."""
    mant = 7 if dtype == torch.bfloat16 else 10
    r = ref.float()
    _, e = torch.frexp(r)
    ulp = torch.ldexp(torch.ones_like(r), e - 1 - mant)
    diff = (got.float() - r).abs()
    return bool((diff <= ulp).all()), float((diff / ulp).max())


@pytest.mark.parametrize("dtype", DTS)
@pytest.mark.parametrize("rows,H", [(1, 4096), (7, 8192), (64, 4096), (3, 1032), (2, 32768),
                                    (5, 16392)])
@pytest.mark.parametrize("with_delta", [False, True])
def test_rmsnorm(cuda, dtype, rows, H, with_delta):
    from lmrs_b200 import decode_ops as DO
    torch.manual_seed(rows + H)
    x = (torch.randn(rows, H, device=cuda) * 3).to(dtype)
    w = (1 + 0.1 * torch.randn(H, device=cuda)).to(dtype)
    d = (torch.randn(rows, H, device=cuda)).to(dtype) if with_delta else None
    resid = x.clone()
    y = DO.rmsnorm(resid, w, 1e-5, delta=d)
    xs = (x.float() + d.float()).to(dtype) if with_delta else x
    assert torch.equal(resid, xs)  # the residual add rounds once
    xf = xs.float()
    ref = (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-5) * w.float()).to(dtype)
    ok, worst = _ulp_close(y, ref, dtype)
    assert ok, worst


@pytest.mark.parametrize("dtype", DTS)
@pytest.mark.parametrize("rows,H", [(1, 8192), (32, 4096), (5, 1040), (2, 32768)])
def test_rmsnorm_fp8_equals_unfused(cuda, dtype, rows, H):
    import lmrs_b200 as L
    from lmrs_b200 import decode_ops as DO
    torch.manual_seed(H)
    x = (torch.randn(rows, H, device=cuda) * 2).to(dtype)
    x[0] = 0  # all-zero row -> scale 0, bytes 0
    w = (1 + 0.1 * torch.randn(H, device=cuda)).to(dtype)
    d = torch.randn(rows, H, device=cuda).to(dtype)
    r1, r2 = x.clone(), x.clone()
    q, s = DO.rmsnorm_fp8(r1, w, 1e-5, delta=d)
    y = DO.rmsnorm(r2, w, 1e-5, delta=d)
    q_ref, s_ref = L.fp8_quant_rows(y)
    assert torch.equal(r1, r2)
    assert torch.equal(s, s_ref) and torch.equal(q, q_ref)


@pytest.mark.parametrize("dtype", DTS)
@pytest.mark.parametrize("rows,inter", [(1, 14336), (16, 7168), (40, 1024), (3, 1032), (2, 28672),
                                        (1, 40000), (3, 8200), (1, 65536)])
def test_silu_mul(cuda, dtype, rows, inter):
    import lmrs_b200 as L
    from lmrs_b200 import decode_ops as DO
    torch.manual_seed(inter)
    gu = (torch.randn(rows, 2 * inter, device=cuda) * 3).to(dtype)
    y = DO.silu_mul(gu)
    g, u = gu[:, :inter].float(), gu[:, inter:].float()
    ref = ((g / (1 + torch.exp(-g))) * u).to(dtype)
    ok, worst = _ulp_close(y, ref, dtype)
    assert ok, worst
    if inter % 16 or inter > 65536:
        return  # the standalone quantiser takes K % 16 == 0
    q, s = DO.silu_mul_fp8(gu)
    q_ref, s_ref = L.fp8_quant_rows(y)
    assert torch.equal(s, s_ref) and torch.equal(q, q_ref)


def _paged_cache(seqs, hkv, d, block_size, max_blocks, dtype, dev, seed):
    g = torch.Generator(device=dev).manual_seed(seed)
    nblocks = seqs * max_blocks + 3
    kc = torch.randn(nblocks, hkv, block_size, d, generator=g, device=dev).to(dtype)
    vc = torch.randn(nblocks, hkv, block_size, d, generator=g, device=dev).to(dtype)
    perm = torch.randperm(nblocks, generator=g, device=dev)[: seqs * max_blocks]
    tables = perm.view(seqs, max_blocks).to(torch.int32).contiguous()
    return kc, vc, tables


def _gather(cache, tables, s, n, h):
    """positions [0, n) of sequence s, KV head h -> [n, d]"""
    bs = cache.shape[2]
    idx = torch.arange(n, device=cache.device)
    blk = tables[s, idx // bs].long()
    return cache[blk, h, idx % bs]


@pytest.mark.parametrize("dtype", DTS)
@pytest.mark.parametrize("seqs,hq,hkv,block_size,lens,kv_map", [
    (1, 32, 8, 16, [2048], 1),
    (3, 8, 8, 16, [1, 65, 700], 1),
    (4, 64, 8, 32, [4096, 100, 0, 33], 1),
    (2, 16, 1, 16, [513, 64], 1),
    (2, 8, 2, 16, [77, 300], 0),
    (64, 32, 8, 2048, [2048] * 64, 1),
])
def test_paged_attention_decode(cuda, dtype, seqs, hq, hkv, block_size, lens, kv_map):
    from lmrs_b200 import decode_ops as DO
    d = 128
    max_ctx = max(lens)
    max_blocks = max(1, (max_ctx + block_size - 1) // block_size)
    kc, vc, tables = _paged_cache(seqs, hkv, d, block_size, max_blocks, dtype, cuda, seqs + hq)
    torch.manual_seed(7)
    q = torch.randn(seqs, hq, d, device=cuda).to(dtype)
    ctx = torch.tensor(lens, dtype=torch.int32, device=cuda)
    scale = 1 / math.sqrt(d)
    out = DO.paged_attention_decode(q, kc, vc, tables, ctx, max_ctx, scale, kv_head_map=kv_map)
    G = hq // hkv
    for s in range(seqs):
        n = lens[s]
        for h in range(hq):
            kvh = h // G if kv_map else h % hkv
            if n == 0:
                assert torch.all(out[s, h] == 0)
                continue
            K = _gather(kc, tables, s, n, kvh).float()
            V = _gather(vc, tables, s, n, kvh).float()
            p = torch.softmax(q[s, h].float() @ K.t() * scale, -1)
            ref = p @ V
            err = ((out[s, h].float() - ref).abs().max() / ref.abs().max()).item()
            # P enters the PV MMA in the I/O type (bf16: 8 significant bits)
            assert err < (2e-2 if dtype == torch.bfloat16 else 4e-3), (s, h, err)


@pytest.mark.parametrize("dtype", DTS)
@pytest.mark.parametrize("d", [128, 64, 72])  # 16-byte vector path (d % 16 == 0) and the general one
def test_rope_kv_write(cuda, dtype, d):
    from lmrs_b200 import decode_ops as DO
    seqs, hq, hkv, bs, mb = 5, 8, 2, 16, 6
    kc, vc, tables = _paged_cache(seqs, hkv, d, bs, mb, dtype, cuda, 3)
    k0, v0 = kc.clone(), vc.clone()
    torch.manual_seed(3)
    qkv = torch.randn(seqs, (hq + 2 * hkv) * d, device=cuda).to(dtype)
    pos = torch.tensor([0, 5, 17, 63, 95], dtype=torch.int32, device=cuda)
    inv = 1.0 / (500000.0 ** (torch.arange(0, d, 2, device=cuda).float() / d))
    ang = 37.0 * inv
    cos, sin = ang.cos().to(dtype), ang.sin().to(dtype)
    q = DO.rope_kv_write(qkv, cos, sin, kc, vc, tables, pos, hq, hkv, d)

    def rope(x):  # [..., d] rotate-half with the same tables, fp32 math, one rounding
        x = x.float()
        half = d // 2
        c, s_ = cos.float(), sin.float()
        return torch.cat([x[..., :half] * c - x[..., half:] * s_,
                          x[..., half:] * c + x[..., :half] * s_], -1).to(dtype)

    qr = rope(qkv[:, : hq * d].view(seqs, hq, d))
    ok, worst = _ulp_close(q, qr, dtype)
    assert ok, worst
    kr = rope(qkv[:, hq * d: (hq + hkv) * d].view(seqs, hkv, d))
    vr = qkv[:, (hq + hkv) * d:].view(seqs, hkv, d)
    touched = torch.zeros_like(kc, dtype=torch.bool)
    for s in range(seqs):
        p = int(pos[s])
        blk = int(tables[s, p // bs])
        ok, worst = _ulp_close(kc[blk, :, p % bs], kr[s], dtype)
        assert ok, worst
        assert torch.equal(vc[blk, :, p % bs], vr[s])
        touched[blk, :, p % bs] = True
    assert torch.equal(kc[~touched], k0[~touched]) and torch.equal(vc[~touched], v0[~touched])


def test_decode_ops_status(cuda):
    from lmrs_b200 import _lib
    lib = _lib.load()
    x = torch.zeros(2, 64, dtype=torch.float32, device=cuda)
    s = torch.cuda.current_stream().cuda_stream
    assert lib.lmrs_rmsnorm(x.data_ptr(), x.data_ptr(), None, x.data_ptr(), 2, 64, 1e-5, 2,
                            s) == _lib.LMRS_ERR_DTYPE
    assert lib.lmrs_rmsnorm(x.data_ptr(), x.data_ptr(), None, x.data_ptr(), 2, 60, 1e-5, 0,
                            s) == _lib.LMRS_ERR_SHAPE
    assert lib.lmrs_rmsnorm(x.data_ptr(), x.data_ptr(), None, x.data_ptr(), 2, 32776, 1e-5, 0,
                            s) == _lib.LMRS_ERR_SHAPE
    assert lib.lmrs_paged_attention_decode(x.data_ptr(), x.data_ptr(), x.data_ptr(), x.data_ptr(),
                                           x.data_ptr(), x.data_ptr(), 1, 8, 8, 64, 16, 1, 16,
                                           0.1, 1, 0, None, 0, s) == _lib.LMRS_ERR_SHAPE
    import lmrs_b200 as L
    assert L.read_device_error() == 0


@pytest.mark.parametrize("cps", [1, 2, 4, 16])
def test_paged_attention_cluster_splits(cuda, cps):
    """Context splits from 1 to 8 (one thread-block cluster per sequence and KV
    head, merged in distributed shared memory), with a short and an empty
    sequence among full ones; deterministic across calls."""
    import lmrs_b200 as L
    from lmrs_b200 import decode_ops as DO
    d, hq, hkv, bs = 128, 32, 8, 16
    lens = [2048, 37, 0, 1500]
    seqs, max_ctx = len(lens), max(lens)
    max_blocks = (max_ctx + bs - 1) // bs
    kc, vc, tables = _paged_cache(seqs, hkv, d, bs, max_blocks, torch.float16, cuda, 99)
    torch.manual_seed(3)
    q = torch.randn(seqs, hq, d, device=cuda).half()
    ctx = torch.tensor(lens, dtype=torch.int32, device=cuda)
    scale = 1 / math.sqrt(d)
    try:
        L.set_tuning("attn_ctas_per_sm", cps)
        out = DO.paged_attention_decode(q, kc, vc, tables, ctx, max_ctx, scale)
        again = DO.paged_attention_decode(q, kc, vc, tables, ctx, max_ctx, scale)
    finally:
        L.set_tuning("attn_ctas_per_sm", 2)
    assert torch.equal(out, again)
    G = hq // hkv
    for s in range(seqs):
        n = lens[s]
        for h in range(hq):
            if n == 0:
                assert torch.all(out[s, h] == 0)
                continue
            K = _gather(kc, tables, s, n, h // G).float()
            V = _gather(vc, tables, s, n, h // G).float()
            ref = torch.softmax(q[s, h].float() @ K.t() * scale, -1) @ V
            assert (out[s, h].float() - ref).abs().max().item() < 2e-3
    assert L.read_device_error() == 0


@pytest.mark.parametrize("seqs,hq,hkv,lens", [(1, 8, 1, [4096]), (1, 64, 8, [4096]),
                                              (2, 32, 8, [2100, 700]), (3, 16, 2, [4096, 0, 129])])
def test_paged_attention_workspace_merge(cuda, seqs, hq, hkv, lens):
    """Small batches with long contexts split the context over several 8-CTA
    clusters (one 64-position tile per CTA at batch 1 with one KV head; 2100
    positions leave trailing splits empty), each cluster's merged partial going
    through the workspace to the last cluster of the (sequence, KV head) to
    arrive: against an fp32 softmax, equal across calls and CUDA-graph replays
    (the arrival counters return to zero), and close to the one-cluster path."""
    import lmrs_b200 as L
    from lmrs_b200 import _lib
    from lmrs_b200 import decode_ops as DO
    d, bs = 128, 16
    max_ctx = max(lens)
    max_blocks = (max_ctx + bs - 1) // bs
    assert _lib.load().lmrs_paged_attention_workspace_bytes(seqs, hq, hkv, max_ctx) > 0
    kc, vc, tables = _paged_cache(seqs, hkv, d, bs, max_blocks, torch.bfloat16, cuda, 41 + hq)
    torch.manual_seed(5)
    q = torch.randn(seqs, hq, d, device=cuda).bfloat16()
    ctx = torch.tensor(lens, dtype=torch.int32, device=cuda)
    scale = 1 / math.sqrt(d)
    ws = DO.AttentionWorkspace()
    out = DO.paged_attention_decode(q, kc, vc, tables, ctx, max_ctx, scale, workspace=ws)
    for _ in range(2):
        assert torch.equal(DO.paged_attention_decode(q, kc, vc, tables, ctx, max_ctx, scale,
                                                     workspace=ws), out)
    g = torch.cuda.CUDAGraph()
    buf = torch.empty_like(out)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        buf.copy_(DO.paged_attention_decode(q, kc, vc, tables, ctx, max_ctx, scale, workspace=ws))
    torch.cuda.current_stream().wait_stream(s)
    with torch.cuda.graph(g):
        buf.copy_(DO.paged_attention_decode(q, kc, vc, tables, ctx, max_ctx, scale, workspace=ws))
    for _ in range(3):
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(buf, out)
    del g
    try:
        L.set_tuning("attn_global_merge", 0)
        clus = DO.paged_attention_decode(q, kc, vc, tables, ctx, max_ctx, scale, workspace=ws)
    finally:
        L.set_tuning("attn_global_merge", 1)
    G = hq // hkv
    for si in range(seqs):
        n = lens[si]
        for h in range(hq):
            if n == 0:
                assert torch.all(out[si, h] == 0)
                continue
            K = _gather(kc, tables, si, n, h // G).float()
            V = _gather(vc, tables, si, n, h // G).float()
            ref = torch.softmax(q[si, h].float() @ K.t() * scale, -1) @ V
            err = ((out[si, h].float() - ref).abs().max() / ref.abs().max()).item()
            assert err < 2e-2, (si, h, err)
    assert ((out.float() - clus.float()).abs().max() / clus.float().abs().max()).item() < 2e-2
    assert L.read_device_error() == 0


@pytest.mark.parametrize("dtype", DTS)
@pytest.mark.parametrize("seqs,hq,hkv,ctx", [
    (1, 8, 1, 4096),     # one KV head, clusters merged through the workspace
    (1, 8, 1, 1000),     # one KV head, one cluster of splits
    (64, 8, 1, 512),     # one KV head, one cluster per sequence
    (300, 16, 1, 200),   # one KV head, one CTA per sequence
    (2, 32, 8, 700),     # eight KV heads: attention, then the row quant
])
def test_paged_attention_fp8_output(cuda, dtype, seqs, hq, hkv, ctx):
    """lmrs_paged_attention_decode_fp8: the e4m3 bytes and scales of the output
    rows, equal byte for byte to lmrs_fp8_quant_rows of the plain call's output,
    which it also writes unchanged; with one KV head the attention's own merge
    quantises (every merge path), otherwise a second launch does."""
    import lmrs_b200 as L
    from lmrs_b200 import decode_ops as DO
    d, bs = 128, 16
    max_blocks = (ctx + bs - 1) // bs
    kc, vc, tables = _paged_cache(seqs, hkv, d, bs, max_blocks, dtype, cuda, 90 + seqs)
    g = torch.Generator(device=cuda).manual_seed(seqs + hq)
    q = torch.randn(seqs, hq, d, generator=g, device=cuda).to(dtype)
    lens = torch.randint(max(1, ctx // 2), ctx + 1, (seqs,), generator=g, device=cuda).to(torch.int32)
    lens[0] = ctx
    scale = 1 / math.sqrt(d)
    ws = DO.AttentionWorkspace()
    ref = DO.paged_attention_decode(q, kc, vc, tables, lens, ctx, scale, workspace=ws)
    qr, sr = L.fp8_quant_rows(ref.reshape(seqs, hq * d).contiguous())
    for _ in range(2):   # repeated calls: the workspace counters return to zero
        qq, sq, out = DO.paged_attention_decode_fp8(q, kc, vc, tables, lens, ctx, scale,
                                                    workspace=ws)
        torch.cuda.synchronize()
        assert torch.equal(out, ref)
        assert torch.equal(sq, sr)
        assert torch.equal(qq, qr)
    assert L.read_device_error() == 0


@pytest.mark.parametrize("dtype", DTS)
@pytest.mark.parametrize("seqs,hq,hkv,ctx,fp8", [
    (1, 8, 1, 4096, True),    # one KV head, clusters merged through the workspace
    (1, 32, 8, 2048, False),  # one cluster of splits per (sequence, KV head)
    (64, 8, 1, 512, True),    # one cluster per sequence
    (300, 16, 2, 200, True),  # one CTA per (sequence, KV head); FP8 output by a second launch
    (5, 64, 8, 700, False),
])
def test_rope_paged_attention_fused(cuda, dtype, seqs, hq, hkv, ctx, fp8):
    """lmrs_rope_paged_attention_decode against lmrs_rope_kv_write (positions =
    context_lens - 1) followed by the attention: the same output, the same cache
    contents (the new token's rotated k and v in place, nothing else touched) and,
    with the FP8 output, the same e4m3 bytes and scales."""
    import lmrs_b200 as L
    from lmrs_b200 import decode_ops as DO
    d, bs = 128, 16
    max_blocks = (ctx + bs - 1) // bs
    kc, vc, tables = _paged_cache(seqs, hkv, d, bs, max_blocks, dtype, cuda, 123 + seqs)
    g = torch.Generator(device=cuda).manual_seed(5 * seqs + hq)
    qkv = torch.randn(seqs, (hq + 2 * hkv) * d, generator=g, device=cuda).to(dtype)
    lens = torch.randint(1, ctx + 1, (seqs,), generator=g, device=cuda).to(torch.int32)
    lens[0] = ctx
    inv = 1.0 / (500000.0 ** (torch.arange(0, d, 2, device=cuda).float() / d))
    ang = float(ctx - 1) * inv
    cos, sin = ang.cos().to(dtype).contiguous(), ang.sin().to(dtype).contiguous()
    scale = 1 / math.sqrt(d)
    k1, v1 = kc.clone(), vc.clone()
    q = DO.rope_kv_write(qkv, cos, sin, k1, v1, tables, lens - 1, hq, hkv, d)
    ws = DO.AttentionWorkspace()
    if fp8:
        qr, sr, ref = DO.paged_attention_decode_fp8(q, k1, v1, tables, lens, ctx, scale, workspace=ws)
    else:
        ref = DO.paged_attention_decode(q, k1, v1, tables, lens, ctx, scale, workspace=ws)
    k2, v2 = kc.clone(), vc.clone()
    for _ in range(2):  # the second call rewrites the same k / v, reads the same cache
        got = DO.rope_paged_attention_decode(qkv, cos, sin, k2, v2, tables, lens, ctx, hq, hkv,
                                             scale, workspace=ws, fp8=fp8)
        torch.cuda.synchronize()
        if fp8:
            qq, sq, out = got
            assert torch.equal(sq, sr) and torch.equal(qq, qr)
        else:
            out = got
        assert torch.equal(out, ref)
        assert torch.equal(k2, k1) and torch.equal(v2, v1)
    assert L.read_device_error() == 0
