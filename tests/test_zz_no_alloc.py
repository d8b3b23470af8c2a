"""lmrs_fp8_linear_noalloc: the FP8 W8A8 linear for callers that cannot allocate.

Some hosts cannot hand this library a device workspace: their device memory
belongs to a pool they do not control, or their decode loop may not allocate
after warm-up.  For them the quantised activations live in a scratch array
compiled into the library instead of a caller-provided workspace.  This test
calls the entry point through the C-ABI twice in a row (a larger problem, then
a smaller one, so stale bytes from the first call sit in the shared array) and
requires each result to equal the regular entry point's output bit for bit:
both run the same kernels on the same inputs, so any difference is a scratch
bug.  It lives in its own file, collected last, and is written
to pass alone in a fresh process as well as after the rest of the suite.
"""
import pytest

from lmrs_b200 import _lib

pytestmark = pytest.mark.gpu


def _regular(lib, torch, x, wq, sw, bias, M, K, N):
    y = torch.empty(M, N, dtype=torch.bfloat16, device=x.device)
    need = lib.lmrs_fp8_linear_workspace_bytes(M, K, N)
    ws = torch.empty(need, dtype=torch.uint8, device=x.device)
    rc = lib.lmrs_fp8_linear(y.data_ptr(), x.data_ptr(), wq.data_ptr(), sw.data_ptr(),
                             None if bias is None else bias.data_ptr(), M, K, N, ws.data_ptr(),
                             need, torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.LMRS_OK, _lib.status_string(rc)
    return y


def _noalloc(lib, torch, x, wq, sw, bias, M, K, N):
    y = torch.empty(M, N, dtype=torch.bfloat16, device=x.device)
    rc = lib.lmrs_fp8_linear_noalloc(y.data_ptr(), x.data_ptr(), wq.data_ptr(), sw.data_ptr(),
                                     None if bias is None else bias.data_ptr(), M, K, N,
                                     torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.LMRS_OK, _lib.status_string(rc)
    return y


def test_noalloc_matches_regular_two_calls(cuda):
    import torch
    lib = _lib.load()
    torch.manual_seed(123)
    # call 1: GEMM path (M > 32), 512*4096 bytes of scratch; call 2: GEMV path, smaller
    cases = [(512, 4096, 1024, True), (5, 2048, 768, False)]
    for M, K, N, with_bias in cases:
        x = torch.randn(M, K, device=cuda).bfloat16()
        w = (torch.randn(N, K, device=cuda) * 0.02).bfloat16()
        wq = torch.empty(N, K, dtype=torch.uint8, device=cuda)
        sw = torch.empty(N, dtype=torch.float32, device=cuda)
        assert lib.lmrs_fp8_quant_rows(wq.data_ptr(), sw.data_ptr(), w.data_ptr(), N, K, 0,
                                       torch.cuda.current_stream().cuda_stream) == 0
        bias = torch.randn(N, device=cuda).bfloat16() if with_bias else None
        y_ref = _regular(lib, torch, x, wq, sw, bias, M, K, N)
        y = _noalloc(lib, torch, x, wq, sw, bias, M, K, N)
        torch.cuda.synchronize()
        assert torch.equal(y, y_ref), (M, K, N, "no-alloc result differs from the regular path")


def test_noalloc_rejects_oversize(cuda):
    import torch
    lib = _lib.load()
    M, K, N = 1024, 8192, 64  # 8 MiB of e4m3 activations > 4 MiB scratch
    assert lib.lmrs_fp8_linear_workspace_bytes(M, K, N) > _lib.FP8_NOALLOC_SCRATCH_BYTES
    x = torch.zeros(M, K, dtype=torch.bfloat16, device=cuda)
    wq = torch.zeros(N, K, dtype=torch.uint8, device=cuda)
    sw = torch.ones(N, device=cuda)
    y = torch.full((M, N), 7.0, dtype=torch.bfloat16, device=cuda)
    rc = lib.lmrs_fp8_linear_noalloc(y.data_ptr(), x.data_ptr(), wq.data_ptr(), sw.data_ptr(),
                                     None, M, K, N, torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.LMRS_ERR_TOO_LARGE
    torch.cuda.synchronize()
    assert bool((y == 7.0).all()), "a rejected call must not launch anything"
