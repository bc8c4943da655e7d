"""qmc_matmul_nt_q_noalloc: the prefill entry point for callers that cannot call cudaMalloc (code running
during CUDA graph capture, or hosts whose own allocator owns all device memory).  It must give the same
result as the allocating qmc_matmul_nt_q -- bit for bit, the tolerance the prefill tests use -- on
consecutive calls that reuse its fixed scratch, and reject shapes whose scratch exceeds the fixed size.
Collected last (file name) so a stop-at-first-failure run has already run every other test."""
import ctypes as C

import numpy as np
import pytest
import torch

import quillm_b200 as qb
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _dev(a):
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    torch.cuda.synchronize()
    return t


@pytest.mark.parametrize("dt", [O.Q8_0, O.Q4_0])
def test_noalloc_prefill_matches_allocating_entry_point(cuda_dev, dt):
    lib = qb.cuda()
    lib.qmc_matmul_nt_q_noalloc.restype = C.c_int
    lib.qmc_matmul_nt_q_noalloc.argtypes = [C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64, C.c_int64,
                                            C.c_int64, C.c_void_p]
    rng = np.random.default_rng(31 + dt)
    N, K = 1100, 4096
    W = _dev(O.quantize(dt, (rng.standard_normal((N, K)) * 0.02).astype(np.float32)))
    # two calls in a row through the fixed scratch: a large T, then a smaller one with new inputs, so a
    # stale scratch row from the first call would show up in the second
    for T in (96, 33):
        A = _dev(rng.standard_normal((T, K)).astype(np.float32))
        want = torch.empty((T, N), device="cuda")
        got = torch.full((T, N), float("nan"), device="cuda")
        torch.cuda.synchronize()
        qb.check(lib.qmc_matmul_nt_q(dt, W.data_ptr(), A.data_ptr(), want.data_ptr(), T, N, K, None), "matmul_nt_q")
        qb.check(lib.qmc_sync())
        qb.check(lib.qmc_matmul_nt_q_noalloc(dt, W.data_ptr(), A.data_ptr(), got.data_ptr(), T, N, K, None),
                 "matmul_nt_q_noalloc")
        torch.cuda.synchronize()
        assert torch.equal(got.view(torch.int32), want.view(torch.int32)), T


def test_noalloc_rejects_oversized_scratch(cuda_dev):
    lib = qb.cuda()
    lib.qmc_matmul_nt_q_noalloc.restype = C.c_int
    lib.qmc_matmul_nt_q_noalloc.argtypes = [C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64, C.c_int64,
                                            C.c_int64, C.c_void_p]
    buf = torch.zeros(1 << 20, dtype=torch.uint8, device="cuda")
    # T * ceil(K/32) * 36 = 4096 * 128 * 36 bytes = 18 MiB > 8 MiB: refused before touching any pointer
    rc = lib.qmc_matmul_nt_q_noalloc(O.Q8_0, buf.data_ptr(), buf.data_ptr(), buf.data_ptr(), 4096, 8, 4096, None)
    assert rc == -1 and b"fixed" in qb.cuda().qmc_last_error()
    # sizes whose byte count would wrap a 64-bit product (T * 36 > 2^64) are refused the same way
    for T, K in ((2**62 + 1, 32), (2**40, 2**40)):
        rc = lib.qmc_matmul_nt_q_noalloc(O.Q8_0, buf.data_ptr(), buf.data_ptr(), buf.data_ptr(), T, 8, K, None)
        assert rc == -1 and b"fixed" in qb.cuda().qmc_last_error(), (T, K)
