""".qlm loader (host C11): parses every golden model like the reference parser does, rejects every
truncation, and accepts / rejects randomly mutated headers exactly when the reference loader does
(the reference's tests/test_format.c:42-84 strategy, with the reference itself as the judge)."""
import ctypes as C
import os

import numpy as np
import pytest

import quillm_b200 as qb
from oracle import oracle as O

GOLD = os.path.join(os.path.dirname(__file__), "golden")
needs_ref = pytest.mark.skipif(not O.ref_available(), reason="oracle/_ref not built")


def parse(lib, buf: bytes):
    f = qb.QlmFile()
    arr = (C.c_uint8 * max(len(buf), 1)).from_buffer_copy(buf or b"\0")
    err = C.create_string_buffer(256)
    lib.qlm_parse.restype = C.c_int
    lib.qlm_parse.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t, C.c_char_p, C.c_size_t]
    lib.qlm_close.argtypes = [C.c_void_p]
    rc = lib.qlm_parse(C.byref(f), arr, len(buf), err, 256)
    info = None
    if rc == 0:
        info = [(f.tensors[i].name, f.tensors[i].type, tuple(f.tensors[i].ne[:f.tensors[i].ndim]),
                 f.tensors[i].data - C.addressof(arr)) for i in range(f.n_tensors)]
        info.append(("n_kv", f.n_kv))
        lib.qlm_close(C.byref(f))
    return rc, info, err.value


def header_len(buf: bytes) -> int:
    return int.from_bytes(buf[16:24], "little")


@pytest.mark.parametrize("name", ["small_q8_0", "odd_q4_0", "l2c_f32"])
def test_golden_models_parse(name):
    buf = open(os.path.join(GOLD, f"{name}.qlm"), "rb").read()
    rc, info, _ = parse(qb.host(), buf)
    assert rc == 0 and any(t[0] == b"tok_embd" for t in info[:-1])


def test_truncations_rejected():
    buf = open(os.path.join(GOLD, "small_q4_0.qlm"), "rb").read()
    for n in list(range(0, header_len(buf) + 1, 3)) + [len(buf) - 64]:  # the last 64 bytes hold data
        rc, _, err = parse(qb.host(), buf[:n])
        assert rc == -1 and err, n


def test_bad_magic_and_version():
    buf = bytearray(open(os.path.join(GOLD, "small_q8_0.qlm"), "rb").read())
    b2 = bytearray(buf)
    b2[0] = ord("X")
    assert parse(qb.host(), bytes(b2))[2] == b"bad magic"
    b3 = bytearray(buf)
    b3[4] = 2
    assert parse(qb.host(), bytes(b3))[2] == b"unsupported version 2"


@needs_ref
def test_random_mutations_agree_with_reference():
    mine, ref = qb.host(), C.CDLL(O.REF_LIB)
    rng = np.random.default_rng(9)
    for name in ("small_q8_0", "odd_f32"):
        buf = open(os.path.join(GOLD, f"{name}.qlm"), "rb").read()
        hl = header_len(buf)
        for it in range(3000):
            b = bytearray(buf[: hl + 4096] if it % 3 else buf)
            for _ in range(int(rng.integers(1, 4))):
                i = int(rng.integers(0, hl))
                b[i] = int(rng.integers(0, 256)) if rng.random() < 0.7 else b[i] ^ (1 << int(rng.integers(0, 8)))
            a = parse(mine, bytes(b))
            r = parse(ref, bytes(b))
            assert a[0] == r[0], (name, it)
            assert a[1] == r[1], (name, it)


def test_model_metadata_errors(tmp_path):
    """a non-model file is rejected by qm_model_load with a message (tests/test_model.c:143-145)"""
    h = qb.host()
    m = qb.QmModel()
    err = C.create_string_buffer(256)
    p = tmp_path / "x.bin"
    p.write_bytes(b"\0" * 100)
    assert h.qm_model_load(C.byref(m), str(p).encode(), 1, 0, err, 256) == -1
    assert err.value == b"bad magic"
