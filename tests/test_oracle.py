"""Pins the CPU oracle before anything is checked against it:
  * against the reference's own golden vectors (tests/golden, made by the reference's tools/qlm.py), and
  * bit for bit against the reference itself compiled from its sources (oracle/_ref)."""
import ctypes as C
import os

import numpy as np
import pytest

from oracle import oracle as O

GOLD = os.path.join(os.path.dirname(__file__), "golden")
needs_ref = pytest.mark.skipif(not O.ref_available(), reason="oracle/_ref not built (reference sources absent)")


def test_fp16_known_values():
    """tests/test_fp16.c:29-38 of the reference"""
    o = O.orc()
    assert o.orc_fp32_to_fp16(1.0) == 0x3C00
    assert o.orc_fp32_to_fp16(-2.0) == 0xC000
    assert o.orc_fp32_to_fp16(65504.0) == 0x7BFF
    assert o.orc_fp32_to_fp16(65519.0) == 0x7BFF
    assert o.orc_fp32_to_fp16(65520.0) == 0x7C00
    assert o.orc_fp32_to_fp16(5.9604644775390625e-08) == 0x0001
    assert o.orc_fp32_to_fp16(2.98023223876953125e-08) == 0x0000
    assert o.orc_fp32_to_fp16(-0.0) == 0x8000
    assert o.orc_fp16_to_fp32(0x3555) == np.float32(0.333251953125)
    h = o.orc_fp32_to_fp16(float("nan"))
    assert (h & 0x7C00) == 0x7C00 and (h & 0x3FF)


def test_fp16_matches_numpy_everywhere():
    """all 65536 halves decode like numpy; 2M random floats (+ boundaries) round like numpy's RNE"""
    o = O.orc()
    h = np.arange(65536, dtype=np.uint16)
    dec = np.array([o.orc_fp16_to_fp32(int(v)) for v in h[::7]], np.float32)
    ref = h[::7].view(np.float16).astype(np.float32)
    finite = ~np.isnan(ref)
    assert np.array_equal(dec[finite].view(np.uint32), ref[finite].view(np.uint32))
    assert np.all(np.isnan(dec[~finite]))
    rng = np.random.default_rng(3)
    f = rng.integers(0, 2**32, 20000, dtype=np.uint64).astype(np.uint32).view(np.float32)
    f = np.concatenate([f, np.float32([65504, 65519, 65520, 6e-8, 2.98e-8, 3e-8, 1e-10, -0.0, 0.0, np.inf])])
    f = f[~np.isnan(f)]
    mine = np.array([o.orc_fp32_to_fp16(float(v)) for v in f], np.uint16)
    with np.errstate(over="ignore"):
        want = f.astype(np.float16).view(np.uint16)
    assert np.array_equal(mine, want)


def test_quantizer_matches_numpy_golden():
    """byte-exact with the reference's numpy quantizer (gen_fixtures.py:72-77, test_quant.c:77-98)"""
    x = np.fromfile(os.path.join(GOLD, "qin.f32"), np.float32).reshape(5, 100)
    for dt, name in ((O.Q8_0, "qin.q8"), (O.Q4_0, "qin.q4")):
        want = np.fromfile(os.path.join(GOLD, name), np.uint8).reshape(5, -1)
        assert np.array_equal(O.quantize(dt, x), want), name


def test_q8_scale_known_answer():
    """tests/test_python.py:32-36: amax 254 -> d = fp16(2.0), q = -127"""
    x = np.zeros((1, 32), np.float32)
    x[0, 3] = -254.0
    b = O.quantize(O.Q8_0, x)[0]
    assert int(b[0]) | (int(b[1]) << 8) == 0x4000 and np.int8(b[2 + 3]) == -127


@needs_ref
def test_quantizer_and_fp16_bitwise_vs_reference():
    r = O.ref()
    rng = np.random.default_rng(11)
    for it in range(300):
        n = int(rng.integers(1, 700))
        x = (rng.standard_normal(n) * np.ldexp(1.0, int(rng.integers(-12, 13)))).astype(np.float32)
        if it % 5 == 0:
            x[: min(n, 40)] = 0.0
        for dt in (O.Q8_0, O.Q4_0):
            mine = O.quantize(dt, x[None, :])[0]
            theirs = np.zeros_like(mine)
            r.ref_quantize_row(dt, x.ctypes.data, theirs.ctypes.data, n)
            assert np.array_equal(mine, theirs), (dt, n)
    f = rng.standard_normal(5000).astype(np.float32) * np.float32(1e3)
    for v in f:
        assert O.orc().orc_fp32_to_fp16(float(v)) == r.ref_fp32_to_fp16(float(v))


@needs_ref
def test_scalar_dots_and_matvec_bitwise_vs_reference():
    r = O.ref()
    rng = np.random.default_rng(12)
    for _ in range(60):
        rows, cols = int(rng.integers(1, 90)), int(rng.integers(1, 700))
        Wf = rng.standard_normal((rows, cols)).astype(np.float32)
        x = rng.standard_normal(cols).astype(np.float32)
        for dt in (O.F32, O.Q8_0, O.Q4_0):
            W = Wf.copy() if dt == O.F32 else O.quantize(dt, Wf)
            y, xq = O.matvec(dt, W, rows, cols, x)
            yr = np.zeros(rows, np.float32)
            xqr = np.zeros(xq.size + 64, np.uint8)
            assert r.ref_isa_select(O.ISA_SCALAR) == 0
            r.ref_matvec(dt, W.ctypes.data, rows, cols, x.ctypes.data, yr.ctypes.data, xqr.ctypes.data, 1)
            assert np.array_equal(y.view(np.uint32), yr.view(np.uint32)), dt
            if dt != O.F32:
                assert np.array_equal(xq, xqr[: xq.size])
            ref, tol = O.matvec_bound(dt, W, rows, cols, x, xq)
            assert np.all(np.abs(y - ref) <= tol)


@needs_ref
def test_elementwise_bitwise_vs_reference():
    r, o = O.ref(), O.orc()
    rng = np.random.default_rng(13)
    x = rng.standard_normal(777).astype(np.float32)
    w = rng.standard_normal(777).astype(np.float32)
    a, b = np.zeros_like(x), np.zeros_like(x)
    o.orc_rmsnorm(a.ctypes.data, x.ctypes.data, w.ctypes.data, 777, 1e-5)
    r.qm_rmsnorm(b.ctypes.data, x.ctypes.data, w.ctypes.data, 777, 1e-5)
    assert np.array_equal(a, b)
    for fn_o, fn_r, args in ((o.orc_softmax, r.qm_softmax, (777,)), (o.orc_rope, r.qm_rope, (7, 111 - 111 % 2, 37, 10000.0))):
        a, b = x.copy(), x.copy()
        if len(args) == 1:
            fn_o(a.ctypes.data, *args)
            fn_r(b.ctypes.data, *args)
        else:
            v = np.ascontiguousarray(x[: 7 * 110])
            a, b = v.copy(), v.copy()
            fn_o(a.ctypes.data, 7, 110, 37, 10000.0)
            fn_r(b.ctypes.data, 7, 110, 37, 10000.0)
        assert np.array_equal(a, b)
    a, b = x.copy(), x.copy()
    o.orc_swiglu(a.ctypes.data, w.ctypes.data, 777)
    r.qm_swiglu(b.ctypes.data, w.ctypes.data, 777)
    assert np.array_equal(a, b)


CASES = [("small_f32", 1e-5, 1e-5), ("odd_f32", 1e-5, 1e-5), ("l2c_f32", 1e-5, 1e-5), ("small_q8_0", 2e-2, 3e-2),
         ("odd_q8_0", 2e-2, 3e-2), ("small_q4_0", 2e-2, 0.5), ("odd_q4_0", 2e-2, 0.5)]


@pytest.mark.parametrize("name,tol_deq,tol_fp", CASES)
def test_oracle_forward_vs_golden_logits(name, tol_deq, tol_fp):
    """the oracle forward against the reference's float64 numpy logits (tests/test_model.c:50-53)"""
    toks, V = O.read_tokens(os.path.join(GOLD, f"{name}.tokens"))
    ref = np.fromfile(os.path.join(GOLD, f"{name}.ref.f32"), np.float32).reshape(len(toks), V)
    fp_path = os.path.join(GOLD, f"{name}.reffp.f32")
    reffp = np.fromfile(fp_path, np.float32).reshape(len(toks), V) if os.path.exists(fp_path) else ref
    m = O.OracleModel(os.path.join(GOLD, f"{name}.qlm"))
    got = np.stack([m.forward(t, p) for p, t in enumerate(toks)])
    assert np.abs(got - ref).max() / np.abs(ref).max() < tol_deq
    assert np.abs(got - reffp).max() / np.abs(reffp).max() < tol_fp
    if tol_deq <= 1e-5:
        assert np.array_equal(got.argmax(1), ref.argmax(1))


@pytest.mark.parametrize("name", [c[0] for c in CASES])
def test_oracle_fp16_cache_option(name):
    """the oracle's fp16 KV cache (the checker of the device's optional fp16 cache): off, it is the
    reference's forward bit for bit; on, it moves f32-weight logits by fp16-rounding amounts (more than
    the fp32 tolerance, under 1e-3 of the float64 truth) with the greedy tokens unchanged, and quantized
    models stay within 3e-2 of the truth"""
    toks, V = O.read_tokens(os.path.join(GOLD, f"{name}.tokens"))
    ref = np.fromfile(os.path.join(GOLD, f"{name}.ref.f32"), np.float32).reshape(len(toks), V)
    path = os.path.join(GOLD, f"{name}.qlm")
    a, b = O.OracleModel(path), O.OracleModel(path, kv_f16=True)
    ga = np.stack([a.forward(t, p) for p, t in enumerate(toks)])
    gb = np.stack([b.forward(t, p) for p, t in enumerate(toks)])
    e = np.abs(gb - ref).max() / np.abs(ref).max()
    if name.endswith("f32"):
        assert 1e-5 < np.abs(gb - ga).max() / np.abs(ga).max() and e < 1e-3, e
        assert np.array_equal(gb.argmax(1), ref.argmax(1))
    else:
        assert e < 3e-2, e


@needs_ref
@pytest.mark.parametrize("name", [c[0] for c in CASES])
def test_oracle_forward_bitwise_vs_reference_scalar(name):
    toks, _ = O.read_tokens(os.path.join(GOLD, f"{name}.tokens"))
    path = os.path.join(GOLD, f"{name}.qlm")
    m = O.OracleModel(path)
    rm = O.RefModel(path, threads=1, isa=O.ISA_SCALAR)
    for p, t in enumerate(toks):
        assert np.array_equal(m.forward(t, p), rm.forward(t, p)), p


def test_synth_deterministic_and_distributed(tmp_path):
    cfg = dict(dim=64, hidden_dim=96, n_layers=1, n_heads=4, n_kv_heads=2, vocab_size=300, max_seq=16)
    a, b, c = (str(tmp_path / n) for n in ("a.qlm", "b.qlm", "c.qlm"))
    O.synth_write(a, cfg, O.Q8_0, 5, 0.02, threads=3)
    O.synth_write(b, cfg, O.Q8_0, 5, 0.02, threads=1)
    O.synth_write(c, cfg, O.Q8_0, 6, 0.02)
    assert open(a, "rb").read() == open(b, "rb").read()
    assert open(a, "rb").read() != open(c, "rb").read()
    z = O.synth_rows(7, 3, 0, 200, 1000, 1.0).ravel()
    assert abs(z.mean()) < 0.01 and abs(z.std() - 1.0) < 0.01
    assert abs(np.mean(np.abs(z) > 1.96) - 0.05) < 0.003  # tails of the normal are right
    m = O.OracleModel(a)
    assert m.cfg["dim"] == 64 and np.all(np.isfinite(m.forward(3, 0)))


@pytest.mark.parametrize("name", ["small_q8_0", "odd_q4_0", "l2c_f32"])
def test_float64_forward_restatement_matches_golden(name):
    """oracle/forward_ref.py reproduces the reference's numpy forward_ref logits (the .ref.f32 fixtures)"""
    from oracle import forward_ref as F

    toks, V = O.read_tokens(os.path.join(GOLD, f"{name}.tokens"))
    ref = np.fromfile(os.path.join(GOLD, f"{name}.ref.f32"), np.float32).reshape(len(toks), V)
    cfg, W = F.load(os.path.join(GOLD, f"{name}.qlm"))
    got = F.forward(cfg, W, toks).astype(np.float32)
    assert np.abs(got - ref).max() <= 1e-6 * np.abs(ref).max()
