"""Fixed-scratch split-K GEMM entry point (C ABI, no allocation at call time).

The entry point serves callers that must not allocate while they run (code
inside a device allocator or its out-of-memory path, servers that fix their
device footprint at start-up); it is declared in ``ops/csrc/uno_noalloc.h``.

Collected last on purpose: it must agree with the regular entry point both
when it runs alone and after every other test has used the device.
"""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

OK, BAD_ARGS, TOO_LARGE = 0, 1, 2


def _lib():
    from uno_b200.ops import cuda as C

    lib = ctypes.CDLL(C.ext().__file__)
    fn = lib.uno_gemm_splitk_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_longlong, ctypes.c_void_p, ctypes.c_longlong, ctypes.c_void_p,
                   ctypes.c_longlong, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    lib.uno_gemm_noalloc_setup.restype = ctypes.c_int
    lib.uno_noalloc_last_error.restype = ctypes.c_char_p
    lib.uno_noalloc_error_flag.restype = ctypes.c_int
    lib.uno_noalloc_error_flag.argtypes = [ctypes.c_int]
    return C, lib, fn


def _call(fn, a, b, out, splits):
    M, K = a.shape
    N = b.shape[0]
    stream = torch.cuda.current_stream().cuda_stream
    return fn(a.data_ptr(), a.stride(0), b.data_ptr(), b.stride(0), out.data_ptr(), out.stride(0), M, N, K, splits,
              stream)


# 32-column tiles with explicit and automatic splits; CTA-pair 256x256 tiles with two automatic K splits
# (M = 384 is an odd multiple of 128: the pair kernel indexes four 128-row tiles); an automatic split
# of 128x128 tiles that needs more partials than the fixed scratch holds, which runs unsplit.
@pytest.mark.parametrize("M,N,K,splits", [(512, 64, 4096, 4), (384, 192, 4096, 0), (200, 256, 2048, 2),
                                          (512, 512, 6144, 0), (384, 768, 8192, 0), (384, 1024, 4096, 0)])
def test_no_alloc_gemm_matches_regular_entry_point(M, N, K, splits):
    C, lib, fn = _lib()
    torch.manual_seed(M + N)
    a = torch.randn(M, K, device="cuda").bfloat16()
    b = torch.randn(N, K, device="cuda").bfloat16()
    expected = C.gemm(a, b, splits=splits)  # regular entry point, allocator-backed scratch
    assert lib.uno_gemm_noalloc_setup() == OK, lib.uno_noalloc_last_error()
    ref32 = a.float() @ b.float().t()
    for _ in range(2):  # counters must be back at zero for the second call
        out = torch.full((M, N), float("nan"), device="cuda", dtype=torch.bfloat16)
        rc = _call(fn, a, b, out, splits)
        torch.cuda.synchronize()
        assert rc == OK, lib.uno_noalloc_last_error()
        assert lib.uno_noalloc_error_flag(0) == 0  # no bounded wait of this entry point gave up
        torch.testing.assert_close(out.float(), expected.float(), rtol=1e-2, atol=1e-2)
        assert ((out.float() - ref32).norm() / ref32.norm()).item() < 1e-2
    assert C.error_flag() == 0


def test_no_alloc_gemm_rejects_oversized_requests():
    C, lib, fn = _lib()
    a = torch.zeros(4096, 8192, device="cuda", dtype=torch.bfloat16)
    b = torch.zeros(256, 8192, device="cuda", dtype=torch.bfloat16)
    out = torch.zeros(4096, 256, device="cuda", dtype=torch.bfloat16)
    rc = _call(fn, a, b, out, 8)  # an explicit split count that does not fit is an error, not a fallback
    assert rc == TOO_LARGE
    assert b"scratch too small" in lib.uno_noalloc_last_error()
    bad = torch.zeros(64, 100, device="cuda", dtype=torch.bfloat16)  # leading dimension not a multiple of 8
    assert _call(fn, bad, bad, torch.zeros(64, 64, device="cuda", dtype=torch.bfloat16), 1) == BAD_ARGS
    assert lib.uno_noalloc_error_flag(1) == 0
