"""fp16 KV cache (qm_model_set_kv_dtype / qmc_model_set_kv_dtype, dtype 1).

Storing K (after RoPE) and V as fp16 changes the numerics beyond the reference's contract, so the cache
type has its own parity bar, in two parts:
  - the same algorithm: logits within the fp32-cache path's own tolerances of the oracle's forward with
    the same fp16 cache (oracle/qm_oracle.c orc_model_set_kv_f16: every stored K/V element rounded
    to nearest-even fp16), except that f32-weight models get 1e-4 instead of 1e-5, because a K value
    within a float ulp of an fp16 rounding boundary may round the other way;
  - the cost of the cache type: logits within the third column of CASES of the reference's float64
    golden logits (1e-3 relative for f32 weights, where fp16's 2^-11 rounding is all that differs; 3e-2 for
    quantized weights, where activation quantization noise dominates), greedy tokens unchanged on the
    f32-weight models."""
import ctypes as C
import os

import numpy as np
import pytest

import quillm_b200 as qb
from oracle import oracle as O

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")
QMC_ESTATE, QMC_EINVAL = -6, -1
# name, tolerance vs the fp16-cache oracle, tolerance vs the float64 golden logits
CASES = [("small_f32", 1e-4, 1e-3), ("odd_f32", 1e-4, 1e-3), ("l2c_f32", 1e-4, 1e-3), ("small_q8_0", 2e-2, 3e-2),
         ("odd_q8_0", 2e-2, 3e-2), ("small_q4_0", 2e-2, 3e-2), ("odd_q4_0", 2e-2, 3e-2)]


def rel(a, b):
    return float(np.abs(a - b).max() / np.abs(b).max())


class DropIn:
    def __init__(self, path, kv_dtype=1):
        self.h = qb.host()
        self.m = qb.QmModel()
        err = C.create_string_buffer(256)
        assert self.h.qm_model_load(C.byref(self.m), path.encode(), 1, 0, err, 256) == 0, err.value
        assert self.h.qm_model_set_kv_dtype(C.byref(self.m), kv_dtype) == 0
        self.V = self.m.cfg.vocab_size

    def forward(self, tok, pos):
        p = self.h.qm_model_forward(C.byref(self.m), tok, pos)
        return None if not p else np.ctypeslib.as_array(p, (self.V,)).copy()

    def prefill(self, toks, pos0):
        t = np.asarray(toks, np.int32)
        p = self.h.qm_model_prefill(C.byref(self.m), t.ctypes.data, len(t), pos0)
        return None if not p else np.ctypeslib.as_array(p, (self.V,)).copy()

    def close(self):
        self.h.qm_model_free(C.byref(self.m))


@pytest.mark.parametrize("name,tol_orc,tol_gold", CASES)
def test_kv16_golden_models(cuda_dev, name, tol_orc, tol_gold):
    toks, V = O.read_tokens(os.path.join(GOLD, f"{name}.tokens"))
    ref = np.fromfile(os.path.join(GOLD, f"{name}.ref.f32"), np.float32).reshape(len(toks), V)
    path = os.path.join(GOLD, f"{name}.qlm")
    m = DropIn(path)
    got = np.stack([m.forward(t, p) for p, t in enumerate(toks)])
    orc = O.OracleModel(path, kv_f16=True)
    want = np.stack([orc.forward(t, p) for p, t in enumerate(toks)])
    e_orc, e_gold = rel(got, want), rel(got, ref)
    print(f"{name}: vs fp16-cache oracle {e_orc:.3g}, vs golden {e_gold:.3g}")
    assert e_orc < tol_orc and e_gold < tol_gold, (e_orc, e_gold)
    if tol_orc <= 1e-4:
        assert np.array_equal(got.argmax(1), ref.argmax(1))
    # the prompt's first half through the batched forward, then decode on the slots it wrote
    m2 = DropIn(path)
    n = max(1, len(toks) // 2)
    assert rel(m2.prefill(toks[:n], 0), want[n - 1]) < tol_orc
    for p in range(n, len(toks)):
        assert rel(m2.forward(toks[p], p), want[p]) < tol_orc, p
    m2.close()
    m.close()


def test_kv16_persistent_path_and_state_rules(cuda_dev):
    path = os.path.join(GOLD, "small_q8_0.qlm")
    cfg = O.OracleModel(path).cfg
    a = qb.Model(cfg)
    lib = qb.cuda()
    assert lib.qmc_model_set_kv_dtype(a.h, qb.QMC_Q8_0) == QMC_EINVAL  # cache types: F32 or F16 only
    a.set_kv_dtype(qb.QMC_F16)
    assert a.kv_dtype() == qb.QMC_F16
    a.set_kv_dtype(qb.QMC_F32)  # switching back before the first step is allowed
    a.set_kv_dtype(qb.QMC_F16)
    qb.load_qlm_into(a, path)
    lg = np.zeros(cfg["vocab_size"], np.float32)
    a.forward(3, 0, lg)
    launches, persistent = a.decode_info()
    assert persistent and launches == 1  # quantized single-GPU model: the one-launch decode kernel
    assert lib.qmc_model_set_kv_dtype(a.h, qb.QMC_F32) == QMC_ESTATE  # the cache already holds a position
    assert a.kv_dtype() == qb.QMC_F16
    a.close()


@pytest.mark.parametrize("dt", [qb.QMC_Q8_0, qb.QMC_Q4_0])
def test_kv16_long_prompt_gqa(cuda_dev, dt):
    """a 61-token prompt on a synthesized GQA model (8 query / 2 KV heads) with the fp16 cache: the
    batched forward and the one-launch decode agree with feeding the prompt token by token, and the
    fp16 cache stays close to the fp32 one"""
    cfg = dict(dim=256, hidden_dim=688, n_layers=3, n_heads=8, n_kv_heads=2, vocab_size=2000, max_seq=128)
    prompt = np.random.default_rng(3).integers(0, cfg["vocab_size"], 61).astype(np.int32)
    V = cfg["vocab_size"]
    a = qb.Model(dict(cfg), kv_dtype=qb.QMC_F16)
    a.synthesize(dt, 21, 0.05)
    b = qb.Model(dict(cfg), kv_dtype=qb.QMC_F16)
    b.synthesize(dt, 21, 0.05)
    f = qb.Model(dict(cfg))  # fp32 cache
    f.synthesize(dt, 21, 0.05)
    la, lb, lf = np.zeros(V, np.float32), np.zeros(V, np.float32), np.zeros(V, np.float32)
    a.prefill(prompt, 0, la)
    for p, t in enumerate(prompt):
        b.forward(int(t), p, lb)
        f.forward(int(t), p, lf)
    assert rel(la, lb) < 2e-2, rel(la, lb)
    assert rel(lb, lf) < 5e-2, rel(lb, lf)
    for p in range(61, 70):  # decode after the prefill vs after the token-by-token feed
        t = int(np.argmax(lb))
        a.forward(t, p, la)
        b.forward(t, p, lb)
        assert rel(la, lb) < 2e-2, (p, rel(la, lb))
    for m in (a, b, f):
        m.close()
