"""ctypes bindings of the CPU oracle -- TEST / BASELINE INFRASTRUCTURE ONLY.

  liboracle.so            own C restatement of the reference's scalar algorithms (qm_oracle.c)
  _ref/libquillm_ref.so   the reference compiled from its own sources + argument-marshalling harness

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference legs import this module.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_LIB = os.path.join(HERE, "liboracle.so")
REF_LIB = os.path.join(HERE, "_ref", "libquillm_ref.so")
F32, Q8_0, Q4_0 = 0, 2, 3
ISA_SCALAR, ISA_AVX2, ISA_AVX512 = 0, 1, 2

_orc = None
_ref = None
V, I, I32, I64, F, D, S = C.c_void_p, C.c_int, C.c_int32, C.c_int64, C.c_float, C.c_double, C.c_size_t


def build() -> None:
    """(Re)build the oracle libraries (the reference part only where its sources are present)."""
    subprocess.run(["make", "-s", "-C", HERE, "all"], check=True)


def orc():
    global _orc
    if _orc is None:
        if not os.path.exists(ORACLE_LIB):
            build()
        lib = C.CDLL(ORACLE_LIB)
        sig = {
            "orc_fp16_to_fp32": (F, [C.c_uint16]), "orc_fp32_to_fp16": (C.c_uint16, [F]),
            "orc_row_bytes": (S, [I, I64]), "orc_quantize_row": (None, [I, V, V, I64]),
            "orc_quantize_rows": (None, [I, V, V, I64, I64]), "orc_dequantize_row": (None, [I, V, V, I64]),
            "orc_dot_f32": (F, [V, V, I64]), "orc_dot_q8": (F, [V, V, I64]), "orc_dot_q4": (F, [V, V, I64]),
            "orc_matvec": (None, [I, V, I64, I64, V, V, V]),
            "orc_matvec_exact": (None, [I, V, I64, I64, V, V, V, V]),
            "orc_accum_tol": (D, [I64, D]), "orc_gemm_exact": (None, [V, V, V, V, I64, I64, I64]),
            "orc_matmul_q": (None, [I, V, I64, I64, V, I64, V]),
            "orc_rmsnorm": (None, [V, V, V, I64, F]), "orc_softmax": (None, [V, I64]),
            "orc_rope": (None, [V, I64, I64, I64, F]), "orc_swiglu": (None, [V, V, I64]),
            "orc_argmax": (I32, [V, I32]),
            "orc_model_open": (V, [C.c_char_p, I, C.c_char_p, S]), "orc_model_close": (None, [V]),
            "orc_model_config": (None, [V, V, V]), "orc_model_forward": (C.POINTER(F), [V, I32, I32]),
            "orc_model_set_kv_f16": (None, [V, I]),
            "orc_synth_normal": (D, [C.c_uint64, C.c_uint64, C.c_uint64]),
            "orc_synth_rows": (None, [C.c_uint64, C.c_uint64, I64, I64, I64, D, V]),
            "orc_synth_write": (I, [C.c_char_p, V, F, F, I, C.c_uint64, D, I]),
        }
        for n, (r, a) in sig.items():
            fn = getattr(lib, n)
            fn.restype, fn.argtypes = r, a
        _orc = lib
    return _orc


def ref_available() -> bool:
    return os.path.exists(REF_LIB)


def ref():
    """The reference itself (compiled from its sources by oracle/Makefile)."""
    global _ref
    if _ref is None:
        if not ref_available():
            build()
        if not ref_available():
            raise RuntimeError(f"{REF_LIB} missing (reference sources unavailable and no prebuilt copy)")
        lib = C.CDLL(REF_LIB)
        sig = {
            "ref_isa_supported": (I, [I]), "ref_isa_select": (I, [I]), "ref_isa_active": (I, []),
            "ref_isa_best": (I, []),
            "ref_fp16_to_fp32": (F, [C.c_uint16]), "ref_fp32_to_fp16": (C.c_uint16, [F]),
            "ref_quantize_row": (None, [I, V, V, I64]), "ref_dot": (F, [I, I, V, V, V, I64]),
            "ref_matvec": (None, [I, V, I64, I64, V, V, V, I]),
            "ref_matvec_time": (D, [I, V, I64, I64, V, V, V, I, D]),
            "ref_matmul_nt": (None, [V, V, V, I64, I64, I64, I]),
            "ref_model_load": (V, [C.c_char_p, I, I, C.c_char_p, S]), "ref_model_free": (None, [V]),
            "ref_model_config": (None, [V, V]), "ref_model_forward": (C.POINTER(F), [V, I32, I32]),
            "ref_greedy_run": (I, [V, V, I, I, V, V, V]),
            "ref_decode_time": (D, [V, I32, I32, I, V]),
            "qm_rmsnorm": (None, [V, V, V, I64, F]), "qm_softmax": (None, [V, I64]),
            "qm_rope": (None, [V, I64, I64, I64, F]), "qm_swiglu": (None, [V, V, I64]),
            "qm_sample": (I32, [V, V]), "qm_rng_uniform": (F, [V]),
        }
        for n, (r, a) in sig.items():
            fn = getattr(lib, n)
            fn.restype, fn.argtypes = r, a
        _ref = lib
    return _ref


class _QmSampler(C.Structure):
    """the reference's qm_sampler (src/sampler.h:8-16)"""
    _fields_ = [("temperature", C.c_float), ("top_k", C.c_int), ("top_p", C.c_float), ("rng", C.c_uint64),
                ("n_vocab", C.c_int32), ("probs", C.POINTER(C.c_float)), ("idx", C.POINTER(C.c_int32))]


class RefSampler:
    """The reference's own qm_sample (src/sampler.c) on host logits, its settings normalised as
    qm_sampler_init does (src/sampler.c:6-16) with the scratch owned here instead of an arena."""

    def __init__(self, n_vocab: int, temperature: float, top_k: int = 0, top_p: float = 1.0, seed: int = 0):
        import numpy as np
        self.lib = ref()
        self._probs = np.zeros(n_vocab, np.float32)
        self._idx = np.zeros(n_vocab, np.int32)
        self.s = _QmSampler(max(temperature, 0.0), max(top_k, 0), 1.0 if (top_p <= 0 or top_p > 1) else top_p,
                            seed or 0x9E3779B97F4A7C15, n_vocab,
                            self._probs.ctypes.data_as(C.POINTER(C.c_float)), self._idx.ctypes.data_as(C.POINTER(C.c_int32)))

    def sample(self, logits) -> int:
        import numpy as np
        lg = np.ascontiguousarray(logits, np.float32)
        return int(self.lib.qm_sample(C.byref(self.s), lg.ctypes.data))

    @property
    def rng(self) -> int:
        return int(self.s.rng)


# ------------------------------------------------------------------ numpy conveniences
def row_bytes(dtype: int, n: int) -> int:
    nb = (n + 31) // 32
    return n * 4 if dtype == F32 else nb * (34 if dtype == Q8_0 else 18)


def quantize(dtype: int, x: np.ndarray) -> np.ndarray:
    """rows of a 2-D float32 array -> uint8 [rows, row_bytes] (oracle quantizer)"""
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, x.shape[-1])
    out = np.zeros((x.shape[0], row_bytes(dtype, x.shape[1])), dtype=np.uint8)
    orc().orc_quantize_rows(dtype, x.ctypes.data, out.ctypes.data, x.shape[0], x.shape[1])
    return out


def matvec(dtype: int, W: np.ndarray, rows: int, cols: int, x: np.ndarray):
    """scalar-reference matvec: (y float32[rows], xq uint8 Q8_0 blocks)"""
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.zeros(rows, np.float32)
    xq = np.zeros(row_bytes(Q8_0, cols) + 64, np.uint8)
    orc().orc_matvec(dtype, W.ctypes.data, rows, cols, x.ctypes.data, y.ctypes.data, xq.ctypes.data)
    return y, xq[: row_bytes(Q8_0, cols)]


def matvec_bound(dtype: int, W: np.ndarray, rows: int, cols: int, x: np.ndarray, xq: np.ndarray):
    """float64 truth and the reference's accumulation tolerance per row"""
    ref = np.zeros(rows, np.float64)
    ab = np.zeros(rows, np.float64)
    x = np.ascontiguousarray(x, dtype=np.float32)
    orc().orc_matvec_exact(dtype, W.ctypes.data, rows, cols, x.ctypes.data, xq.ctypes.data, ref.ctypes.data,
                           ab.ctypes.data)
    n = cols if dtype == F32 else ((cols + 31) // 32) * 8
    tol = 4.0 * (n + 16) * 6e-8 * ab + 1e-30
    return ref, tol


def synth_rows(seed: int, tid: int, r0: int, nrows: int, cols: int, std: float) -> np.ndarray:
    out = np.zeros((nrows, cols), np.float32)
    orc().orc_synth_rows(seed, tid, r0, nrows, cols, std, out.ctypes.data)
    return out


def synth_write(path: str, cfg: dict, dtype: int, seed: int, std: float, threads: int | None = None) -> None:
    c = (C.c_int32 * 7)(cfg["dim"], cfg["hidden_dim"], cfg["n_layers"], cfg["n_heads"], cfg["n_kv_heads"],
                        cfg["vocab_size"], cfg["max_seq"])
    rc = orc().orc_synth_write(path.encode(), c, cfg.get("rope_theta", 10000.0), cfg.get("norm_eps", 1e-5), dtype,
                               seed, std, threads or os.cpu_count() or 1)
    if rc != 0:
        raise RuntimeError(f"orc_synth_write({path}) failed")


class OracleModel:
    """the restated forward (qm_oracle.c) on a .qlm file"""

    def __init__(self, path: str, max_seq: int = 0, kv_f16: bool = False):
        err = C.create_string_buffer(256)
        self.h = orc().orc_model_open(path.encode(), max_seq, err, 256)
        if not self.h:
            raise RuntimeError(err.value.decode())
        if kv_f16:
            orc().orc_model_set_kv_f16(self.h, 1)
        cfg = (C.c_int32 * 7)()
        fc = (C.c_float * 2)()
        orc().orc_model_config(self.h, cfg, fc)
        self.cfg = dict(zip(["dim", "hidden_dim", "n_layers", "n_heads", "n_kv_heads", "vocab_size", "max_seq"], cfg))
        self.cfg["rope_theta"], self.cfg["norm_eps"] = fc[0], fc[1]

    def forward(self, token: int, pos: int) -> np.ndarray:
        p = orc().orc_model_forward(self.h, token, pos)
        if not p:
            raise ValueError("bad token/pos")
        return np.ctypeslib.as_array(p, (self.cfg["vocab_size"],)).copy()

    def close(self):
        if self.h:
            orc().orc_model_close(self.h)
            self.h = None

    def __del__(self):
        self.close()


class RefModel:
    """the reference's own qm_model_load / qm_model_forward (compiled reference)"""

    def __init__(self, path: str, threads: int = 1, max_seq: int = 0, isa: int | None = None):
        r = ref()
        if isa is not None and r.ref_isa_select(isa) != 0:
            raise RuntimeError(f"ISA {isa} unavailable")
        err = C.create_string_buffer(256)
        self.h = r.ref_model_load(path.encode(), threads, max_seq, err, 256)
        if not self.h:
            raise RuntimeError(err.value.decode())
        cfg = (C.c_int32 * 7)()
        r.ref_model_config(self.h, cfg)
        self.cfg = dict(zip(["dim", "hidden_dim", "n_layers", "n_heads", "n_kv_heads", "vocab_size", "max_seq"], cfg))

    def forward(self, token: int, pos: int) -> np.ndarray:
        p = ref().ref_model_forward(self.h, token, pos)
        if not p:
            raise ValueError("bad token/pos")
        return np.ctypeslib.as_array(p, (self.cfg["vocab_size"],)).copy()

    def greedy(self, prompt, n_gen: int):
        p = np.ascontiguousarray(prompt, np.int32)
        out = np.zeros(max(n_gen, 1), np.int32)
        ps, gs = C.c_double(0), C.c_double(0)
        if ref().ref_greedy_run(self.h, p.ctypes.data, len(p), n_gen, out.ctypes.data, C.byref(ps), C.byref(gs)):
            raise RuntimeError("greedy run failed")
        return out[:n_gen], ps.value, gs.value

    def close(self):
        if self.h:
            ref().ref_model_free(self.h)
            self.h = None

    def __del__(self):
        self.close()


def read_tokens(path: str):
    with open(path) as f:
        T, Vv = map(int, f.readline().split())
        toks = list(map(int, f.readline().split()))
    return toks[:T], Vv
