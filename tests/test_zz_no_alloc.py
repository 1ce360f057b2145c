"""The allocation-free GEMM entry point, called through its exported C symbol.

Callers such as inference-runtime plugins, allocator hooks or fixed-budget
real-time loops cannot allocate GPU memory while they run; this entry point
serves them with a fixed scratch array compiled into the library.  The test
compares it with the regular GEMM op, on two calls in a row, and checks that
neither call allocated device memory.  It is collected last on purpose.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _rel(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / (b.norm() + 1e-6)).item()


@pytest.fixture(scope="module")
def lib():
    from kunserve_b200.ops import native
    C = native()
    so = ctypes.CDLL(C.__file__)
    fn = so.kus_gemm_bf16_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int,
                   ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    flag = so.kus_noalloc_error_flag
    flag.restype = ctypes.c_longlong
    flag.argtypes = [ctypes.c_int]
    fn.error_flag = flag
    return C, fn


def _call(fn, A, B, out):
    M, K = A.shape
    N = B.shape[0]
    stream = torch.cuda.current_stream().cuda_stream
    return fn(A.data_ptr(), K, B.data_ptr(), K, out.data_ptr(), N, M, N, K, stream)


@pytest.mark.parametrize("shapes", [((16, 4096, 4096), (300, 1024, 2048))])
def test_noalloc_gemm_matches_regular_entry_point(lib, shapes):
    C, fn = lib
    torch.manual_seed(11)
    cases = []
    for M, N, K in shapes:
        A = torch.randn(M, K, device="cuda").bfloat16()
        B = (torch.randn(N, K, device="cuda") * 0.05).bfloat16()
        ref = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        C.gemm(A, B, ref, C.EPI_BF16, None, 0, 16)
        out = torch.full((M, N), float("nan"), device="cuda", dtype=torch.bfloat16)
        cases.append((A, B, ref, out))
    torch.cuda.synchronize()
    alloc0 = torch.cuda.memory_allocated()
    # first call: sets up the scratch address for this device
    assert _call(fn, *cases[0][:2], cases[0][3]) == 0
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    # second call, different problem, right after the first
    assert _call(fn, *cases[1][:2], cases[1][3]) == 0
    torch.cuda.synchronize()
    free2, _ = torch.cuda.mem_get_info()
    assert torch.cuda.memory_allocated() == alloc0
    assert free2 == free1, "the second call changed free device memory"
    # the library's device error flag, read through the C API: zero means
    # both calls' outputs are complete
    assert fn.error_flag(0) == 0
    for A, B, ref, out in cases:
        assert _rel(out, ref) < 1e-2
        assert _rel(out, A.float() @ B.float().t()) < 1e-2
    from kunserve_b200.ops import check_error
    check_error()


def test_noalloc_rejects_bad_arguments(lib):
    C, fn = lib
    A = torch.zeros(4, 12, device="cuda", dtype=torch.bfloat16)
    B = torch.zeros(8, 12, device="cuda", dtype=torch.bfloat16)
    out = torch.zeros(4, 8, device="cuda", dtype=torch.bfloat16)
    assert _call(fn, A, B, out) == -1          # K = 12 is not a multiple of 8
