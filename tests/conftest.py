import ctypes
import pathlib
import sys

import numpy as np
import pytest

ROOT = pathlib.Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

REF_LIB = ROOT / "oracle" / "_ref" / "libref_ffi.so"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU")
    config.addinivalue_line("markers", "slow: full-size parity case")


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")


@pytest.fixture(scope="session")
def ref_ffi():
    """The reference's own kernels/ffi/tensor_ffi.cu, built unchanged for sm_100a."""
    if not REF_LIB.exists():
        pytest.skip("oracle/_ref/libref_ffi.so not built (needs the reference sources)")
    lib = ctypes.CDLL(str(REF_LIB))
    P, I = ctypes.c_void_p, ctypes.c_int
    lib.linear_fwd.argtypes = [P, P, P, P, I, I, I, I, P]
    lib.linear_fwd.restype = None
    return lib


def to_dev(a, device, dtype=None):
    import torch
    t = torch.from_numpy(np.ascontiguousarray(a))
    if dtype is not None:
        t = t.view(dtype)
    return t.to(device)


def bf16_dev(bits, device):
    import torch
    return to_dev(np.asarray(bits, dtype=np.uint16), device, torch.bfloat16)


def bits16(t):
    """torch fp16/bf16 tensor -> numpy uint16 bit patterns."""
    import torch
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def ref_linear(ref_ffi, x, w_nk, bias, dtype_code):
    """Run the reference's linear_fwd (kernels/ffi/tensor_ffi.cu:820-841) on device tensors."""
    import torch
    M, K = x.shape
    N = w_nk.shape[0]
    y = torch.empty((M, N), dtype=x.dtype, device=x.device)
    ref_ffi.linear_fwd(ctypes.c_void_p(y.data_ptr()), ctypes.c_void_p(x.data_ptr()),
                       ctypes.c_void_p(w_nk.data_ptr()),
                       None if bias is None else ctypes.c_void_p(bias.data_ptr()),
                       M, K, N, dtype_code,
                       ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    return y
