"""The C-ABI libraries load without a GPU, export every function include/*.h declares, and fail loudly
(error status / NaN + message, never a CPU fallback) when no CUDA device is present."""
import ctypes as C
import glob
import os
import re
import subprocess

import numpy as np
import pytest

import quillm_b200 as qb

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = {}
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        src = re.sub(r"//[^\n]*", "", src)
        src = re.sub(r"\{[^{}]*\}", ";", src)  # drop inline bodies / struct bodies
        for m in re.finditer(r"([A-Za-z_][A-Za-z0-9_]*)\s*\([^;()]*(?:\([^()]*\)[^;()]*)*\)\s*;", src):
            name = m.group(1)
            if name in ("sizeof", "_Static_assert") or name.startswith("__"):
                continue
            names.setdefault(name, os.path.basename(h))
    return names


def exported(lib_path):
    out = subprocess.run(["nm", "-D", "--defined-only", lib_path], capture_output=True, text=True, check=True).stdout
    return {line.split()[-1] for line in out.splitlines() if line.split()[1] in ("T", "D", "R", "B")}


def test_every_declared_symbol_is_exported():
    decl = declared_functions()
    assert len(decl) > 60
    have = exported(qb.CUDA_LIB) | exported(qb.HOST_LIB)
    inline = {"qm_nblocks"}  # static inline in qm_base.h
    missing = sorted(n for n in decl if n not in have and n not in inline)
    assert not missing, missing
    assert "qm_kernels_cuda" in have


def test_libraries_load_and_bind():
    cu, h = qb.cuda(), qb.host()
    assert cu.qmc_last_error is not None and h.qm_row_bytes(2, 4096) == 128 * 34
    assert h.qm_row_bytes(3, 4096) == 128 * 18 and h.qm_row_bytes(0, 7) == 28
    assert h.qm_dtype_name(3) == b"q4_0" and h.qm_dtype_valid(1) == 0
    assert h.qm_isa_name(4) == b"cuda" and h.qm_isa_from_name(b"cuda") == 4 and h.qm_cpu_best() == 4


def test_host_fp16_matches_oracle():
    from oracle import oracle as O

    h, o = qb.host(), O.orc()
    for v in range(0, 65536, 3):
        a, b = h.qm_fp16_to_fp32(v), o.orc_fp16_to_fp32(v)
        assert (a == b) or (a != a and b != b)
    rng = np.random.default_rng(0)
    for f in rng.integers(0, 2**32, 20000, dtype=np.uint64).astype(np.uint32).view(np.float32):
        assert h.qm_fp32_to_fp16(float(f)) == o.orc_fp32_to_fp16(float(f))


@pytest.mark.skipif(os.environ.get("CUDA_VISIBLE_DEVICES") is None and os.path.exists("/dev/nvidia0"),
                    reason="a GPU is present")
def test_no_gpu_fails_loudly():
    """without a device every op reports an error: no silent CPU path"""
    cu, h = qb.cuda(), qb.host()
    n = C.c_int(-1)
    rc = cu.qmc_device_count(C.byref(n))
    assert rc != 0 or n.value == 0
    x = np.ones(64, np.float32)
    W = np.zeros(2 * 34 * 4, np.uint8)
    t = qb.QmTensor(b"w", 2, 2, (C.c_int64 * 4)(4, 64, 0, 0), W.ctypes.data)
    y = np.zeros(4, np.float32)
    h.qm_matvec(None, C.byref(t), x.ctypes.data, y.ctypes.data, None)
    assert np.all(np.isnan(y)) and b"CUDA" in h.qm_last_error()
    m = qb.QmModel()
    err = C.create_string_buffer(256)
    path = os.path.join(ROOT, "tests", "golden", "small_q8_0.qlm")
    assert h.qm_model_load(C.byref(m), path.encode(), 1, 0, err, 256) == -1 and err.value
    assert h.qm_kernels_for(4) is None and h.qm_kernels_select(0) == -1
