"""quillm-b200: ctypes bindings to the in-tree native libraries.

  lib/libquillm_cuda.so   the hand-written sm_100a kernels behind the qmc_* C ABI (include/quillm_cuda.h)
  lib/libquillm.so        the C11 drop-in for quillm's qm_* / qlm_* API (include/*.h)

There is no Python or CPU fallback: importing `cuda()` / `host()` raises if a library is missing, and
every compute call fails (non-zero status) without a CUDA device.  Build with `make -C quillm_b200/csrc`
(or `__graft_entry__.build()`).
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIBDIR = os.path.join(HERE, "lib")
CUDA_LIB = os.path.join(LIBDIR, "libquillm_cuda.so")
HOST_LIB = os.path.join(LIBDIR, "libquillm.so")

QMC_F32, QMC_F16, QMC_Q8_0, QMC_Q4_0 = 0, 1, 2, 3  # QMC_F16: KV cache only
(QMC_T_TOK_EMBD, QMC_T_NORM, QMC_T_OUTPUT, QMC_T_ATTN_NORM, QMC_T_WQ, QMC_T_WK, QMC_T_WV, QMC_T_WO,
 QMC_T_FFN_NORM, QMC_T_W1, QMC_T_W2, QMC_T_W3) = range(12)
STATUS = {0: "ok", -1: "invalid argument", -2: "cuda error", -3: "out of memory", -4: "nccl error",
          -5: "device wait timed out", -6: "bad state"}


class QmcError(RuntimeError):
    pass


class QmcConfig(C.Structure):
    _fields_ = [("dim", C.c_int32), ("hidden_dim", C.c_int32), ("n_layers", C.c_int32), ("n_heads", C.c_int32),
                ("n_kv_heads", C.c_int32), ("vocab_size", C.c_int32), ("max_seq", C.c_int32),
                ("rope_theta", C.c_float), ("norm_eps", C.c_float)]


class QmTensor(C.Structure):  # include/ops.h qm_tensor
    _fields_ = [("name", C.c_char * 64), ("type", C.c_int), ("ndim", C.c_int), ("ne", C.c_int64 * 4),
                ("data", C.c_void_p)]


class QmArena(C.Structure):
    _fields_ = [("base", C.c_void_p), ("cap", C.c_size_t), ("used", C.c_size_t), ("peak", C.c_size_t)]


class QlmFile(C.Structure):
    _fields_ = [("map", C.c_void_p), ("map_size", C.c_size_t), ("n_kv", C.c_uint32), ("n_tensors", C.c_uint32),
                ("kv", C.c_void_p), ("tensors", C.POINTER(QmTensor))]


class QmConfig(C.Structure):
    _fields_ = QmcConfig._fields_


class QmModel(C.Structure):  # include/model.h qm_model
    _fields_ = [("cfg", QmConfig), ("file", QlmFile), ("tok_embd", C.c_void_p), ("norm", C.c_void_p),
                ("output", C.c_void_p), ("layers", C.c_void_p), ("arena", QmArena),
                ("logits", C.POINTER(C.c_float)), ("pool", C.c_void_p), ("n_threads", C.c_int),
                ("gpu", C.c_void_p)]


_cuda = None
_host = None
V, P, I, I32, I64, F, D, S = C.c_void_p, C.c_void_p, C.c_int, C.c_int32, C.c_int64, C.c_float, C.c_double, C.c_size_t

_CUDA_SIGS = {
    "qmc_last_error": (C.c_char_p, []),
    "qmc_device_count": (I, [C.POINTER(I)]),
    "qmc_set_device": (I, [I]),
    "qmc_get_device": (I, [C.POINTER(I)]),
    "qmc_stream": (I, [C.POINTER(V)]),
    "qmc_sync": (I, []),
    "qmc_check_device_error": (I, []),
    "qmc_split_row_bytes": (I64, [I, I64]),
    "qmc_repack_split": (I, [I, P, I64, I64, P, V]),
    "qmc_matmul_split_q": (I, [I, P, P, P, I64, I64, I64, V]),
    "qmc_wait_selftest": (I, [I, C.POINTER(F)]),
    "qmc_malloc": (I, [C.POINTER(V), S]),
    "qmc_free": (I, [V]),
    "qmc_memcpy_h2d": (I, [V, V, S, V]),
    "qmc_memcpy_d2h": (I, [V, V, S, V]),
    "qmc_host_alloc": (I, [C.POINTER(V), S]),
    "qmc_host_free": (I, [V]),
    "qmc_quantize_rows": (I, [I, P, P, I64, I64, V]),
    "qmc_dequantize_rows": (I, [I, P, P, I64, I64, V]),
    "qmc_matvec": (I, [I, P, I64, I64, P, P, P, V]),
    "qmc_matmul_nt": (I, [P, P, P, I64, I64, I64, V]),
    "qmc_matmul_nt_q": (I, [I, P, P, P, I64, I64, I64, V]),
    "qmc_rmsnorm": (I, [P, P, P, I64, F, V]),
    "qmc_softmax": (I, [P, I64, V]),
    "qmc_rope": (I, [P, I64, I64, I64, F, V]),
    "qmc_swiglu": (I, [P, P, I64, V]),
    "qmc_argmax": (I, [P, I32, P, V]),
    "qmc_dot": (I, [I, P, P, I64, P, V]),
    "qmc_nccl_unique_id": (I, [V]),
    "qmc_model_create": (I, [C.POINTER(QmcConfig), I, I, V, C.POINTER(V)]),
    "qmc_model_upload": (I, [V, I, I, I, I64, I64, V]),
    "qmc_host_register": (I, [V, S]),
    "qmc_host_unregister": (I, [V]),
    "qmc_model_synthesize": (I, [V, I, C.c_uint64, D]),
    "qmc_model_forward": (I, [V, I32, I32, P, P]),
    "qmc_model_generate": (I, [V, P, I32, I32, P]),
    "qmc_model_prefill": (I, [V, P, I32, I32, P, P]),
    "qmc_model_enqueue_decode": (I, [V, I32, I32, I32]),
    "qmc_model_state": (I, [V, C.POINTER(I32), C.POINTER(I32)]),
    "qmc_model_logits": (I, [V, C.POINTER(V)]),
    "qmc_model_config": (I, [V, C.POINTER(QmcConfig)]),
    "qmc_model_step_bytes": (I, [V, I32, C.POINTER(D)]),
    "qmc_model_decode_info": (I, [V, C.POINTER(I32), C.POINTER(I32)]),
    "qmc_model_set_kv_dtype": (I, [V, I]),
    "qmc_model_kv_dtype": (I, [V, C.POINTER(I)]),
    "qmc_model_free": (I, [V]),
    "qmc_sampler_create": (I, [I32, F, I32, F, C.c_uint64, P]),
    "qmc_sampler_enqueue": (I, [V, P, P, V]),
    "qmc_sampler_sample": (I, [V, P, P]),
    "qmc_sampler_rng": (I, [V, P]),
    "qmc_sampler_free": (I, [V]),
    "qmc_model_forward_sample": (I, [V, I32, I32, V, P]),
}

_HOST_SIGS = {
    "qm_fp16_to_fp32": (F, [C.c_uint16]),
    "qm_fp32_to_fp16": (C.c_uint16, [F]),
    "qm_row_bytes": (S, [I, I64]),
    "qm_dtype_name": (C.c_char_p, [I]),
    "qm_dtype_valid": (I, [C.c_uint32]),
    "qm_quantize_row_q8": (None, [P, P, I64]),
    "qm_quantize_row_q4": (None, [P, P, I64]),
    "qm_dequantize_row_q8": (None, [P, P, I64]),
    "qm_dequantize_row_q4": (None, [P, P, I64]),
    "qm_row_to_f32": (None, [I, P, P, I64]),
    "qm_cpu_supports": (I, [I]),
    "qm_cpu_best": (I, []),
    "qm_isa_name": (C.c_char_p, [I]),
    "qm_isa_from_name": (I, [C.c_char_p]),
    "qm_last_error": (C.c_char_p, []),
    "qm_kernels_for": (V, [I]),
    "qm_kernels_active": (V, []),
    "qm_kernels_select": (I, [I]),
    "qm_matvec": (None, [V, C.POINTER(QmTensor), P, P, P]),
    "qm_matmul_nt": (None, [V, P, P, P, I64, I64, I64]),
    "qm_matmul_nt_q": (None, [V, C.POINTER(QmTensor), P, P, I64]),
    "qm_rmsnorm": (None, [P, P, P, I64, F]),
    "qm_softmax": (None, [P, I64]),
    "qm_rope": (None, [P, I64, I64, I64, F]),
    "qm_swiglu": (None, [P, P, I64]),
    "qm_tensor_upload": (I, [C.POINTER(QmTensor)]),
    "qm_tensor_release": (None, [C.POINTER(QmTensor)]),
    "qm_pool_create": (V, [I]),
    "qm_pool_destroy": (None, [V]),
    "qm_pool_size": (I, [V]),
    "qlm_parse": (I, [V, P, S, C.c_char_p, S]),
    "qlm_open": (I, [V, C.c_char_p, C.c_char_p, S]),
    "qlm_close": (None, [V]),
    "qm_model_load": (I, [C.POINTER(QmModel), C.c_char_p, I, I, C.c_char_p, S]),
    "qm_model_load_tp": (I, [C.POINTER(QmModel), C.c_char_p, I, I, I, V, C.c_char_p, S]),
    "qm_model_free": (None, [C.POINTER(QmModel)]),
    "qm_model_forward": (C.POINTER(C.c_float), [C.POINTER(QmModel), I32, I32]),
    "qm_model_generate": (I, [C.POINTER(QmModel), P, I32, I32, P]),
    "qm_model_prefill": (C.POINTER(C.c_float), [C.POINTER(QmModel), P, I32, I32]),
    "qm_model_set_kv_dtype": (I, [C.POINTER(QmModel), I]),
}


def _bind(lib, sigs):
    for name, (res, args) in sigs.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args


def cuda():
    """libquillm_cuda.so (raises if it was not built)."""
    global _cuda
    if _cuda is None:
        if not os.path.exists(CUDA_LIB):
            raise QmcError(f"{CUDA_LIB} is missing: build it with `make -C quillm_b200/csrc` (no CPU fallback)")
        lib = C.CDLL(CUDA_LIB)
        _bind(lib, _CUDA_SIGS)
        _cuda = lib
    return _cuda


def host():
    """libquillm.so, the C11 drop-in API (raises if it was not built)."""
    global _host
    if _host is None:
        cuda()
        if not os.path.exists(HOST_LIB):
            raise QmcError(f"{HOST_LIB} is missing: build it with `make -C quillm_b200/csrc` (no CPU fallback)")
        lib = C.CDLL(HOST_LIB)
        _bind(lib, _HOST_SIGS)
        _host = lib
    return _host


def last_error() -> str:
    return (cuda().qmc_last_error() or b"").decode(errors="replace")


def check(rc: int, what: str = "qmc call") -> None:
    if rc != 0:
        raise QmcError(f"{what}: {STATUS.get(rc, rc)}: {last_error()}")


def ptr(t) -> int:
    """device (or host) address of a torch tensor / numpy array"""
    if hasattr(t, "data_ptr"):
        return t.data_ptr()
    return t.ctypes.data


class Sampler:
    """device-side sampler (temperature / top-k / top-p, the reference's xorshift64* stream)"""

    def __init__(self, n_vocab: int, temperature: float, top_k: int = 0, top_p: float = 1.0, seed: int = 0):
        self.lib = cuda()
        self.h = C.c_void_p()
        check(self.lib.qmc_sampler_create(n_vocab, temperature, top_k, top_p, seed, C.byref(self.h)), "sampler_create")

    def sample(self, dev_logits: int) -> int:
        """one draw from float32 logits at device address dev_logits"""
        t = C.c_int32(0)
        check(self.lib.qmc_sampler_sample(self.h, C.c_void_p(dev_logits), C.byref(t)), "sampler_sample")
        return t.value

    def rng(self) -> int:
        st = C.c_uint64(0)
        check(self.lib.qmc_sampler_rng(self.h, C.byref(st)), "sampler_rng")
        return st.value

    def close(self) -> None:
        if self.h:
            self.lib.qmc_sampler_free(self.h)
            self.h = C.c_void_p()


class Model:
    """A libquillm_cuda model (qmc_model*) on the current device."""

    def __init__(self, cfg: dict, tp_rank: int = 0, tp_size: int = 1, nccl_id: bytes | None = None,
                 kv_dtype: int = QMC_F32):
        self.lib = cuda()
        self.cfg = QmcConfig(cfg["dim"], cfg["hidden_dim"], cfg["n_layers"], cfg["n_heads"], cfg["n_kv_heads"],
                             cfg["vocab_size"], cfg["max_seq"], cfg.get("rope_theta", 10000.0),
                             cfg.get("norm_eps", 1e-5))
        self.h = C.c_void_p()
        idbuf = C.create_string_buffer(nccl_id, 128) if nccl_id else None
        check(self.lib.qmc_model_create(C.byref(self.cfg), tp_rank, tp_size, idbuf, C.byref(self.h)), "model_create")
        if kv_dtype != QMC_F32:
            self.set_kv_dtype(kv_dtype)

    def set_kv_dtype(self, dtype: int) -> None:
        """KV cache element type, QMC_F32 (default) or QMC_F16; before the first step only"""
        check(self.lib.qmc_model_set_kv_dtype(self.h, dtype), "set_kv_dtype")

    def kv_dtype(self) -> int:
        d = C.c_int(0)
        check(self.lib.qmc_model_kv_dtype(self.h, C.byref(d)), "kv_dtype")
        return d.value

    def synthesize(self, dtype: int, seed: int, std: float) -> None:
        check(self.lib.qmc_model_synthesize(self.h, dtype, seed, std), "model_synthesize")

    def upload(self, kind: int, layer: int, dtype: int, rows: int, cols: int, host_array) -> None:
        check(self.lib.qmc_model_upload(self.h, kind, layer, dtype, rows, cols, host_array.ctypes.data), "upload")

    def forward(self, token: int, pos: int, logits=None) -> int:
        nxt = C.c_int32(0)
        check(self.lib.qmc_model_forward(self.h, token, pos, None if logits is None else logits.ctypes.data,
                                         C.byref(nxt)), "model_forward")
        return nxt.value

    def forward_sample(self, token: int, pos: int, sampler: "Sampler") -> int:
        """one decode step whose next token the sampler draws on the device"""
        nxt = C.c_int32(0)
        check(self.lib.qmc_model_forward_sample(self.h, token, pos, sampler.h, C.byref(nxt)), "model_forward_sample")
        return nxt.value

    def prefill(self, tokens, pos0: int = 0, logits=None) -> int:
        """the prompt's tokens through every layer at once (KV slots pos0 .. pos0+len-1); returns the
        last token's greedy argmax and fills `logits` (float32[vocab]) when given"""
        import numpy as np

        t = np.ascontiguousarray(tokens, dtype=np.int32)
        nxt = C.c_int32(0)
        check(self.lib.qmc_model_prefill(self.h, t.ctypes.data, len(t), pos0,
                                         None if logits is None else logits.ctypes.data, C.byref(nxt)), "model_prefill")
        return nxt.value

    def generate(self, prompt, n_gen: int):
        import numpy as np
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.zeros(max(n_gen, 1), dtype=np.int32)
        check(self.lib.qmc_model_generate(self.h, p.ctypes.data, len(p), n_gen, out.ctypes.data), "generate")
        return out[:n_gen]

    def enqueue_decode(self, token: int, pos: int, steps: int) -> None:
        check(self.lib.qmc_model_enqueue_decode(self.h, token, pos, steps), "enqueue_decode")

    def state(self):
        t, p = C.c_int32(0), C.c_int32(0)
        check(self.lib.qmc_model_state(self.h, C.byref(t), C.byref(p)), "model_state")
        return t.value, p.value

    def step_bytes(self, pos: int) -> float:
        b = C.c_double(0)
        check(self.lib.qmc_model_step_bytes(self.h, pos, C.byref(b)), "step_bytes")
        return b.value

    def decode_info(self) -> tuple[int, bool]:
        """(kernel launches per decode step, whether the single-launch persistent path runs)"""
        n, pers = C.c_int32(0), C.c_int32(0)
        check(self.lib.qmc_model_decode_info(self.h, C.byref(n), C.byref(pers)), "decode_info")
        return n.value, bool(pers.value)

    def close(self) -> None:
        if self.h:
            self.lib.qmc_model_free(self.h)
            self.h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def load_qlm_into(model: Model, path: str) -> None:
    """Upload every tensor of a .qlm file (parsed by libquillm's qlm_open) into a Model."""
    h = host()
    f = QlmFile()
    err = C.create_string_buffer(256)
    if h.qlm_open(C.byref(f), path.encode(), err, 256) != 0:
        raise QmcError(f"qlm_open: {err.value.decode()}")
    try:
        L = model.cfg.n_layers
        kinds = {"tok_embd": (QMC_T_TOK_EMBD, -1), "norm": (QMC_T_NORM, -1), "output": (QMC_T_OUTPUT, -1)}
        per = {"attn_norm": QMC_T_ATTN_NORM, "wq": QMC_T_WQ, "wk": QMC_T_WK, "wv": QMC_T_WV, "wo": QMC_T_WO,
               "ffn_norm": QMC_T_FFN_NORM, "w1": QMC_T_W1, "w2": QMC_T_W2, "w3": QMC_T_W3}
        for l in range(L):
            for k, v in per.items():
                kinds[f"layers.{l}.{k}"] = (v, l)
        # page-lock the mapping for the uploads: DMA straight from the file's pages
        pinned = model.lib.qmc_host_register(f.map, f.map_size) == 0
        try:
            for i in range(f.n_tensors):
                t = f.tensors[i]
                name = t.name.decode()
                if name not in kinds:
                    continue
                kind, layer = kinds[name]
                cols = t.ne[1] if t.ndim == 2 else 0
                check(model.lib.qmc_model_upload(model.h, kind, layer, t.type, t.ne[0], cols, t.data), f"upload {name}")
        finally:
            if pinned:
                model.lib.qmc_host_unregister(f.map)
    finally:
        h.qlm_close(C.byref(f))
