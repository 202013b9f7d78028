"""The no-allocation HiF8 entry point, called through its exported C symbol.

Some callers cannot allocate GPU memory at the point of the call (a fixed memory
budget, a pre-reserved pool, or host code that must not call cudaMalloc or a
caching allocator); ``osp_hif8_qdq_noalloc`` serves them with a fixed scratch
array compiled into the library.  This file is collected last so a failure here
cannot hide the results of the other GPU tests; it passes alone and after them.
"""
import ctypes

import pytest
import torch

from osp_next_b200 import ops
from osp_next_b200.ops._ext import so_path

pytestmark = pytest.mark.gpu

CUDA_ERROR_INVALID_VALUE = 1
MAX_ELEMS = 16384 * 4096


def _entry():
    ops.ext()                                    # the extension (and libtorch) are loaded
    lib = ctypes.CDLL(so_path(), mode=ctypes.RTLD_GLOBAL)
    fn = lib.osp_hif8_qdq_noalloc
    fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float,
                   ctypes.c_void_p]
    fn.restype = ctypes.c_int
    return fn


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_noalloc_matches_allocating_entry_point(dtype):
    fn = _entry()
    stream = torch.cuda.current_stream().cuda_stream
    code = 0 if dtype == torch.float32 else 1
    for call in range(2):                        # two calls in a row share the scratch array
        torch.manual_seed(call)
        x = (torch.randn(3_000_003 + 7 * call, device="cuda") * (1.0 + 3 * call)).to(dtype)
        out = torch.empty_like(x)
        assert fn(x.data_ptr(), out.data_ptr(), x.numel(), code, 15.0, stream) == 0
        want = ops.hif8_quant_dequant(x, 15.0)   # existing (allocating) entry point
        torch.cuda.synchronize()
        # same tolerance as the other HiF8 GPU test: exact agreement
        assert torch.equal(out, want), (out.float() - want.float()).abs().max()


def test_noalloc_rejects_oversized_input():
    fn = _entry()
    x = torch.zeros(16, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    assert fn(x.data_ptr(), x.data_ptr(), MAX_ELEMS + 1, 0, 15.0, stream) == CUDA_ERROR_INVALID_VALUE
    assert fn(x.data_ptr(), x.data_ptr(), 16, 7, 15.0, stream) == CUDA_ERROR_INVALID_VALUE
