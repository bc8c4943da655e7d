"""GPU kernels through the C ABI vs the CPU oracle, on the reference's own edge cases:
bit-exact quantization, matvec within the reference's accumulation bound (tests/test_kernels.c:13),
prefill equal to the scalar matvec bit for bit, elementwise ops."""
import ctypes as C
import os

import numpy as np
import pytest
import torch

import quillm_b200 as qb
from oracle import oracle as O

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")


_keep = []


def dev(a, d):
    """device copy of a numpy array, kept alive for the test (the library only sees the raw address) and
    complete before the library's own stream uses it"""
    t = torch.from_numpy(np.ascontiguousarray(a)).to(d)
    torch.cuda.synchronize()
    _keep.append(t)
    return t


@pytest.fixture(autouse=True)
def _release():
    yield
    _keep.clear()


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def sync():
    qb.check(qb.cuda().qmc_sync(), "sync")


# ------------------------------------------------------------------ quantization
def test_quantize_golden_bytes(cuda_dev):
    x = np.fromfile(os.path.join(GOLD, "qin.f32"), np.float32).reshape(5, 100)
    for dt, name in ((O.Q8_0, "qin.q8"), (O.Q4_0, "qin.q4")):
        want = np.fromfile(os.path.join(GOLD, name), np.uint8).reshape(5, -1)
        out = torch.zeros(want.shape, dtype=torch.uint8, device=cuda_dev)
        qb.check(qb.cuda().qmc_quantize_rows(dt, qb.ptr(dev(x, cuda_dev)), qb.ptr(out), 5, 100, None))
        sync()
        assert np.array_equal(host(out), want), name


def test_quantize_random_rows_bit_exact(cuda_dev):
    """>= 1e5 rows: scales 2^-12..2^12, K not a multiple of 32, zero blocks, outliers, tiny/huge values"""
    rng = np.random.default_rng(1)
    total = 0
    for K in (1, 7, 31, 32, 33, 100, 288, 1000):
        rows = 400000 // max(K, 8) + 64
        x = rng.standard_normal((rows, K)).astype(np.float32)
        x *= np.ldexp(1.0, rng.integers(-12, 13, (rows, 1))).astype(np.float32)
        x[::9, : min(K, 40)] = 0.0
        x[::11, 0] *= 50.0
        x[5::13] *= np.float32(1e-30)  # subnormal fp16 scales and below
        x[7::17] *= np.float32(1e4)    # fp16 scale overflow -> inf
        for dt in (O.Q8_0, O.Q4_0):
            want = O.quantize(dt, x)
            out = torch.zeros(want.shape, dtype=torch.uint8, device=cuda_dev)
            qb.check(qb.cuda().qmc_quantize_rows(dt, qb.ptr(dev(x, cuda_dev)), qb.ptr(out), rows, K, None))
            sync()
            got = host(out)
            bad = np.where(~np.all(got == want, axis=1))[0]
            assert bad.size == 0, (dt, K, bad[:5])
        total += rows
    assert total >= 100000


def test_dequantize_matches_oracle(cuda_dev):
    rng = np.random.default_rng(2)
    x = rng.standard_normal((37, 77)).astype(np.float32)
    for dt in (O.Q8_0, O.Q4_0):
        q = O.quantize(dt, x)
        want = np.zeros((37, 77), np.float32)
        for r in range(37):
            O.orc().orc_dequantize_row(dt, q[r].ctypes.data, want[r].ctypes.data, 77)
        out = torch.zeros((37, 77), dtype=torch.float32, device=cuda_dev)
        qb.check(qb.cuda().qmc_dequantize_rows(dt, qb.ptr(dev(q, cuda_dev)), qb.ptr(out), 37, 77, None))
        sync()
        assert np.array_equal(host(out).view(np.uint32), want.view(np.uint32))


# ------------------------------------------------------------------ matvec
def run_matvec(d, dt, W, rows, cols, x):
    y = torch.zeros(rows, dtype=torch.float32, device=d)
    xq = torch.zeros(O.row_bytes(O.Q8_0, cols), dtype=torch.uint8, device=d)
    qb.check(qb.cuda().qmc_matvec(dt, qb.ptr(dev(W, d)), rows, cols, qb.ptr(dev(x, d)), qb.ptr(y), qb.ptr(xq), None),
             "matvec")
    sync()
    return host(y), host(xq)


def check_matvec(d, dt, Wf, x):
    rows, cols = Wf.shape
    W = Wf if dt == O.F32 else O.quantize(dt, Wf)
    y, xq = run_matvec(d, dt, W, rows, cols, x)
    _, xq_ref = O.matvec(dt, W, rows, cols, x)
    if dt != O.F32:
        assert np.array_equal(xq, xq_ref), "activation blocks differ"
    ref, tol = O.matvec_bound(dt, W, rows, cols, x, xq_ref)
    err = np.abs(y.astype(np.float64) - ref)
    assert np.all(err <= tol), (dt, rows, cols, float((err / tol).max()))


@pytest.mark.parametrize("dt", [O.F32, O.Q8_0, O.Q4_0])
def test_matvec_ragged_shapes(cuda_dev, dt):
    rng = np.random.default_rng(3 + dt)
    shapes = [(1, 1), (1, 31), (3, 33), (31, 288), (288, 288), (300, 1000), (17, 4096), (768, 288), (288, 768)]
    shapes += [(int(rng.integers(1, 400)), int(rng.integers(1, 1500))) for _ in range(25)]
    for rows, cols in shapes:
        Wf = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32)
        x = rng.standard_normal(cols).astype(np.float32)
        check_matvec(cuda_dev, dt, Wf, x)


@pytest.mark.parametrize("dt", [O.Q8_0, O.Q4_0])
@pytest.mark.parametrize("shape", [(4096, 4096), (11008, 4096), (4096, 11008), (32000, 4096), (28672, 8192)])
def test_matvec_sweep_shapes(cuda_dev, dt, shape):
    """the BASELINE matvec sweep shapes, seeded N(0, 0.02) weights and N(0, 1) activations"""
    rows, cols = shape
    Wf = O.synth_rows(17, 1, 0, rows, cols, 0.02)
    x = np.random.default_rng(4).standard_normal(cols).astype(np.float32)
    check_matvec(cuda_dev, dt, Wf, x)


def test_matvec_deterministic(cuda_dev):
    rng = np.random.default_rng(5)
    W = O.quantize(O.Q4_0, rng.standard_normal((4096, 4096)).astype(np.float32))
    x = rng.standard_normal(4096).astype(np.float32)
    a, _ = run_matvec(cuda_dev, O.Q4_0, W, 4096, 4096, x)
    b, _ = run_matvec(cuda_dev, O.Q4_0, W, 4096, 4096, x)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_matvec_rejects_unaligned_weights(cuda_dev):
    buf = torch.zeros(34 * 64 + 64, dtype=torch.uint8, device=cuda_dev)
    x = torch.zeros(64, device=cuda_dev)
    y = torch.zeros(2, device=cuda_dev)
    rc = qb.cuda().qmc_matvec(O.Q8_0, qb.ptr(buf) + 2, 2, 64, qb.ptr(x), qb.ptr(y), None, None)
    assert rc == -1 and b"aligned" in qb.cuda().qmc_last_error()


# ------------------------------------------------------------------ prefill
@pytest.mark.parametrize("dt", [O.Q8_0, O.Q4_0])
def test_matmul_q_bitwise_equals_scalar_matvec(cuda_dev, dt):
    rng = np.random.default_rng(6)
    for T, N, K in [(1, 64, 64), (8, 300, 288), (33, 130, 1000), (70, 257, 4096), (128, 1024, 512)]:
        Wf = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
        W = O.quantize(dt, Wf)
        A = rng.standard_normal((T, K)).astype(np.float32)
        want = np.zeros((T, N), np.float32)
        O.orc().orc_matmul_q(dt, W.ctypes.data, N, K, A.ctypes.data, T, want.ctypes.data)
        Cd = torch.zeros((T, N), dtype=torch.float32, device=cuda_dev)
        qb.check(qb.cuda().qmc_matmul_nt_q(dt, qb.ptr(dev(W, cuda_dev)), qb.ptr(dev(A, cuda_dev)), qb.ptr(Cd), T, N, K,
                                           None), "matmul_q")
        sync()
        assert np.array_equal(host(Cd).view(np.uint32), want.view(np.uint32)), (T, N, K)


@pytest.mark.parametrize("dt", [O.Q8_0, O.Q4_0])
def test_matmul_tensor_core_bitwise_equals_scalar_matvec(cuda_dev, dt):
    """the tcgen05 kind::i8 contraction on split-row weights: bit-identical to the reference's scalar matvec
    of every row, on ragged T / N / K (partial 128-row and 32-token tiles, a last stage of 1-3 blocks),
    and with extreme block scales and saturated int8 values"""
    rng = np.random.default_rng(16)
    shapes = [(1, 64, 64), (8, 300, 288), (33, 130, 1000), (70, 257, 4096), (128, 1024, 512), (31, 128, 96),
              (200, 384, 4096), (5, 129, 32), (512, 4096, 256), (520, 4200, 100)]
    for T, N, K in shapes:
        Wf = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
        A = rng.standard_normal((T, K)).astype(np.float32)
        if T == 200:  # outliers: some blocks dominated by one huge value, a zero block, tiny scales
            Wf[3, :32] = 0.0
            Wf[5, 7] = 40.0
            A[1, 100] = 1e4
            A[2, :32] *= 1e-6
        W = O.quantize(dt, Wf)
        want = np.zeros((T, N), np.float32)
        O.orc().orc_matmul_q(dt, W.ctypes.data, N, K, A.ctypes.data, T, want.ctypes.data)
        rb = qb.cuda().qmc_split_row_bytes(dt, K)
        assert rb > 0 and rb % 16 == 0
        Ws = torch.zeros(N * rb + 256, dtype=torch.uint8, device=cuda_dev)
        qb.check(qb.cuda().qmc_repack_split(dt, qb.ptr(dev(W, cuda_dev)), N, K, qb.ptr(Ws), None), "repack_split")
        Cd = torch.full((T, N), float("nan"), dtype=torch.float32, device=cuda_dev)
        qb.check(qb.cuda().qmc_matmul_split_q(dt, qb.ptr(Ws), qb.ptr(dev(A, cuda_dev)), qb.ptr(Cd), T, N, K, None),
                 "matmul_split_q")
        sync()
        assert qb.cuda().qmc_check_device_error() == 0
        got = host(Cd)
        bad = np.argwhere(got.view(np.uint32) != want.view(np.uint32))
        assert len(bad) == 0, (T, N, K, len(bad), bad[:4].tolist())


def test_matmul_f32_within_bound(cuda_dev):
    rng = np.random.default_rng(7)
    for M, N, K in [(4, 4, 8), (1, 150, 600), (40, 150, 600), (37, 65, 1), (128, 96, 333)]:
        A = rng.standard_normal((M, K)).astype(np.float32)
        B = rng.standard_normal((N, K)).astype(np.float32)
        ref = np.zeros((M, N)), np.zeros((M, N))
        O.orc().orc_gemm_exact(A.ctypes.data, B.ctypes.data, ref[0].ctypes.data, ref[1].ctypes.data, M, N, K)
        Cd = torch.zeros((M, N), dtype=torch.float32, device=cuda_dev)
        qb.check(qb.cuda().qmc_matmul_nt(qb.ptr(dev(A, cuda_dev)), qb.ptr(dev(B, cuda_dev)), qb.ptr(Cd), M, N, K, None))
        sync()
        tol = 4.0 * (K + 16) * 6e-8 * ref[1] + 1e-30
        assert np.all(np.abs(host(Cd) - ref[0]) <= tol)


# ------------------------------------------------------------------ elementwise
def test_rmsnorm_rope_swiglu_softmax(cuda_dev):
    o = O.orc()
    rng = np.random.default_rng(8)
    x = rng.standard_normal(4096).astype(np.float32)
    w = rng.standard_normal(4096).astype(np.float32)
    want = np.zeros_like(x)
    o.orc_rmsnorm(want.ctypes.data, x.ctypes.data, w.ctypes.data, 4096, 1e-5)
    out = torch.zeros(4096, device=cuda_dev)
    qb.check(qb.cuda().qmc_rmsnorm(qb.ptr(out), qb.ptr(dev(x, cuda_dev)), qb.ptr(dev(w, cuda_dev)), 4096, 1e-5, None))
    sync()
    ulp = np.abs(host(out).view(np.int32).astype(np.int64) - want.view(np.int32))
    assert ulp.max() <= 2  # the double sum's order can move inv by one rounding
    for nh, hd, pos in [(32, 128, 0), (32, 128, 383), (6, 48, 255), (8, 12, 19)]:
        v = rng.standard_normal(nh * hd).astype(np.float32)
        want = v.copy()
        o.orc_rope(want.ctypes.data, nh, hd, pos, 10000.0)
        t = dev(v, cuda_dev)
        qb.check(qb.cuda().qmc_rope(qb.ptr(t), nh, hd, pos, 10000.0, None))
        sync()
        assert np.array_equal(host(t).view(np.uint32), want.view(np.uint32)), (nh, hd, pos)
    g = (rng.standard_normal(11008) * 3).astype(np.float32)
    u = rng.standard_normal(11008).astype(np.float32)
    want = g.copy()
    o.orc_swiglu(want.ctypes.data, u.ctypes.data, 11008)
    t = dev(g, cuda_dev)
    qb.check(qb.cuda().qmc_swiglu(qb.ptr(t), qb.ptr(dev(u, cuda_dev)), 11008, None))
    sync()
    np.testing.assert_allclose(host(t), want, rtol=4e-7, atol=1e-30)
    s = (rng.standard_normal(1000) * 10).astype(np.float32)
    s[[3, 700]] = 1000.0
    want = s.copy()
    o.orc_softmax(want.ctypes.data, 1000)
    t = dev(s, cuda_dev)
    qb.check(qb.cuda().qmc_softmax(qb.ptr(t), 1000, None))
    sync()
    np.testing.assert_allclose(host(t), want, rtol=1e-6, atol=1e-30)


def test_argmax_first_maximum(cuda_dev):
    rng = np.random.default_rng(9)
    out = torch.zeros(1, dtype=torch.int32, device=cuda_dev)
    for n in (1, 2, 31, 32000, 100000):
        x = rng.standard_normal(n).astype(np.float32)
        if n > 10:
            x[[n // 3, n // 2, n - 1]] = x.max() + 1.0  # ties: the first index wins
        qb.check(qb.cuda().qmc_argmax(qb.ptr(dev(x, cuda_dev)), n, qb.ptr(out), None))
        sync()
        assert int(host(out)[0]) == O.orc().orc_argmax(x.ctypes.data, n) == int(np.argmax(x))


@pytest.mark.parametrize("dt", [O.F32, O.Q8_0, O.Q4_0])
def test_dot_within_bound(cuda_dev, dt):
    rng = np.random.default_rng(10)
    n = 999
    w = rng.standard_normal(n).astype(np.float32)
    x = rng.standard_normal(n).astype(np.float32)
    out = torch.zeros(1, device=cuda_dev)
    if dt == O.F32:
        qb.check(qb.cuda().qmc_dot(dt, qb.ptr(dev(w, cuda_dev)), qb.ptr(dev(x, cuda_dev)), n, qb.ptr(out), None))
        ref, tol = O.matvec_bound(dt, w, 1, n, x, np.zeros(64, np.uint8))
    else:
        W = O.quantize(dt, w[None])
        xq = O.quantize(O.Q8_0, x[None])[0]
        qb.check(qb.cuda().qmc_dot(dt, qb.ptr(dev(W, cuda_dev)), qb.ptr(dev(xq, cuda_dev)), n, qb.ptr(out), None))
        ref, tol = O.matvec_bound(dt, W, 1, n, x, xq)
    sync()
    assert abs(float(host(out)[0]) - ref[0]) <= tol[0]
