"""The decode kernel quantizes activations without a division per element (quant_block and
quant_near_half in quillm_b200/csrc/cuda/decode.cu): q = rint(v * RN(1/sc)), and for the rare element
whose product lies within 1e-4 of a half-integer an exact decision against h * sc.  This restates those
float32 steps in numpy and checks them against the reference's rint(v / sc) (src/quant.c:47-50), with
the inputs concentrated where the two could differ: quotients near and exactly at half-integers, and
ulp-neighbours of them.  The kernel itself is checked bit-exact against the golden fixtures on the GPU.
"""
import numpy as np

F32 = np.float32
KROUND = F32(12582912.0)  # 1.5 * 2^23


def device_quant(v, sc):
    """the kernel's steps, one float32 rounding per operation as the CUDA intrinsics do"""
    with np.errstate(all="ignore"):
        rs = (F32(1) / sc).astype(F32)
        r = (v * rs).astype(F32)
    c = np.clip(r, F32(-127), F32(127)).astype(F32)
    cr = (c + KROUND).astype(F32)
    q = np.where((sc != 0) & (r == r), cr.view(np.int32) - 0x4B400000, 0).astype(np.int64)
    near = np.abs((r - (cr - KROUND).astype(F32)).astype(F32)) > F32(0.4999)
    # quant_near_half
    fl = np.floor(r).astype(F32)
    h = (fl + F32(0.5)).astype(F32)
    hs = h.astype(np.float64) * sc.astype(np.float64)
    assert np.all(hs[near] == hs[near].astype(F32)), "h * sc must be exact in float32"
    d64 = v.astype(np.float64) - hs
    d = d64.astype(F32)  # fmaf(-h, sc, v): one rounding of the exact difference
    assert np.all(d64[near] == d[near]), "v - h * sc must be exact in float32"
    u = ((h.view(np.int32) & 0x7F800000) - (24 << 23)).astype(np.int32).view(F32)
    toward0 = (d < 0) == (h > 0)
    lim = (np.where((np.abs(h) == 0.5) & toward0, F32(0.5) * u, u) * sc).astype(F32)
    f = (fl + KROUND).astype(F32).view(np.int32).astype(np.int64) - 0x4B400000
    qn = np.clip(np.where(np.abs(d) <= lim, f + (f & 1), np.where(d > 0, f + 1, f)), -127, 127)
    return np.where(near, qn, q), int(near.sum())


def reference_quant(v, sc):
    with np.errstate(all="ignore"):
        x = (v / sc).astype(F32)
    r = np.clip(np.rint(x), -127, 127)
    return np.where(np.isnan(r), 0, r).astype(np.int64)


def _scales(rng, n):
    sc = rng.uniform(1e-6, 10, n).astype(np.float16).astype(F32)  # fp16 scales, subnormals included
    return np.where(sc == 0, F32(2.0**-24), sc)


def test_division_free_rounding_matches_ieee_quotient():
    rng = np.random.default_rng(7)
    n, near_total = 1 << 19, 0
    for it in range(12):
        sc = _scales(rng, n)
        k = rng.integers(-127, 127, n).astype(np.float64)
        mode = it % 3
        if mode == 0:  # quotients near half-integers
            delta = rng.choice([0.0, 1e-7, -1e-7, 3e-6, -3e-6, 5e-5, -5e-5, 1e-3], n) * rng.uniform(0, 1, n)
            v = ((k + 0.5 + delta) * sc).astype(F32)
        elif mode == 1:  # exactly at half-integers and a few ulps either side
            v = ((k + 0.5) * sc).astype(F32)
            v = (v.view(np.int32) + rng.integers(-3, 4, n).astype(np.int32)).view(F32)
        else:  # anywhere in the block's range
            v = (rng.uniform(-127.5, 127.5, n) * sc).astype(F32)
        got, nn = device_quant(v, sc)
        near_total += nn
        want = reference_quant(v, sc)
        bad = np.flatnonzero(got != want)
        assert bad.size == 0, (v[bad[0]], sc[bad[0]], got[bad[0]], want[bad[0]])
    assert near_total > 100000  # the exact path was exercised


def test_division_free_rounding_at_plus_minus_half():
    """|h| = 0.5 is the one half-integer that is a power of two: its rounding interval is narrower
    towards zero"""
    rng = np.random.default_rng(8)
    for sgn in (1.0, -1.0):
        sc = rng.uniform(1e-4, 10, 1 << 18).astype(np.float16).astype(F32)
        v = (F32(0.5 * sgn) * sc).astype(F32)
        v = (v.view(np.int32) + rng.integers(-4, 5, v.size).astype(np.int32)).view(F32)
        got, nn = device_quant(v, sc)
        assert nn > 0
        np.testing.assert_array_equal(got, reference_quant(v, sc))
