"""Whole-model decode on the GPU vs the reference (tests/test_model.c strategy):
golden numpy logits within the reference's tolerances, teacher-forced logits vs the reference's own C
forward, greedy tokens identical (tie-aware), run-to-run determinism, error returns, device synthesis
== file synthesis."""
import ctypes as C
import os

import numpy as np
import pytest

import quillm_b200 as qb
from oracle import oracle as O

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")
CASES = [("small_f32", 1e-5, 1e-5), ("odd_f32", 1e-5, 1e-5), ("l2c_f32", 1e-5, 1e-5), ("small_q8_0", 2e-2, 3e-2),
         ("odd_q8_0", 2e-2, 3e-2), ("small_q4_0", 2e-2, 0.5), ("odd_q4_0", 2e-2, 0.5)]


class DropIn:
    """the reference-facing API: qm_model_load / qm_model_forward from libquillm.so"""

    def __init__(self, path, max_seq=0):
        self.h = qb.host()
        self.m = qb.QmModel()
        err = C.create_string_buffer(256)
        assert self.h.qm_model_load(C.byref(self.m), path.encode(), 1, max_seq, err, 256) == 0, err.value
        self.V = self.m.cfg.vocab_size

    def forward(self, tok, pos):
        p = self.h.qm_model_forward(C.byref(self.m), tok, pos)
        return None if not p else np.ctypeslib.as_array(p, (self.V,)).copy()

    def generate(self, prompt, n):
        pr = np.asarray(prompt, np.int32)
        out = np.zeros(n, np.int32)
        assert self.h.qm_model_generate(C.byref(self.m), pr.ctypes.data, len(pr), n, out.ctypes.data) == 0
        return out

    def close(self):
        self.h.qm_model_free(C.byref(self.m))


@pytest.mark.parametrize("name,tol_deq,tol_fp", CASES)
def test_golden_models(cuda_dev, name, tol_deq, tol_fp):
    toks, V = O.read_tokens(os.path.join(GOLD, f"{name}.tokens"))
    ref = np.fromfile(os.path.join(GOLD, f"{name}.ref.f32"), np.float32).reshape(len(toks), V)
    fp_path = os.path.join(GOLD, f"{name}.reffp.f32")
    reffp = np.fromfile(fp_path, np.float32).reshape(len(toks), V) if os.path.exists(fp_path) else ref
    path = os.path.join(GOLD, f"{name}.qlm")
    m = DropIn(path)
    got = np.stack([m.forward(t, p) for p, t in enumerate(toks)])
    e = np.abs(got - ref).max() / np.abs(ref).max()
    efp = np.abs(got - reffp).max() / np.abs(reffp).max()
    assert e < tol_deq and efp < tol_fp, (e, efp)
    if tol_deq <= 1e-5:
        assert np.array_equal(got.argmax(1), ref.argmax(1))
    # same weights, same activation quantization: the reference's own C forward
    orc = O.OracleModel(path)
    want = np.stack([orc.forward(t, p) for p, t in enumerate(toks)])
    e_c = np.abs(got - want).max() / np.abs(want).max()
    print(f"{name}: rel err vs numpy float64 {e:.3e} (fp32 weights {efp:.3e}), vs the C forward {e_c:.3e}")
    # both sides quantize the activations bit-exactly, so only the accumulation order differs: far inside
    # the reference's own tolerance (observed at most ~1e-7 on these models)
    assert e_c < 1e-5, e_c
    # run-to-run determinism (bitwise) and error returns
    again = np.stack([m.forward(t, p) for p, t in enumerate(toks)])
    assert np.array_equal(got.view(np.uint32), again.view(np.uint32))
    assert m.forward(0, m.m.cfg.max_seq) is None and m.forward(V, 0) is None and m.forward(-1, 0) is None
    m.close()


def test_device_greedy_equals_forward_argmax(cuda_dev):
    path = os.path.join(GOLD, "small_q8_0.qlm")
    m = DropIn(path)
    prompt = [0, 5, 9]
    gen = m.generate(prompt, 30)
    seq = list(prompt)
    for p in range(len(prompt) + 29):
        lg = m.forward(seq[p], p)
        if p >= len(prompt) - 1:
            seq.append(int(np.argmax(lg)))
    assert list(gen) == seq[len(prompt):]
    m.close()


def test_device_synthesis_equals_file_synthesis(cuda_dev, tmp_path):
    cfg = dict(dim=128, hidden_dim=352, n_layers=2, n_heads=4, n_kv_heads=2, vocab_size=1000, max_seq=64)
    for dt in (O.Q8_0, O.Q4_0):
        path = str(tmp_path / f"s{dt}.qlm")
        O.synth_write(path, cfg, dt, 42, 0.02)
        a = qb.Model(cfg)
        qb.load_qlm_into(a, path)
        b = qb.Model(cfg)
        b.synthesize(dt, 42, 0.02)
        la, lb = np.zeros(1000, np.float32), np.zeros(1000, np.float32)
        for p, t in enumerate([1, 7, 300, 999, 5]):
            a.forward(t, p, la)
            b.forward(t, p, lb)
            assert np.array_equal(la.view(np.uint32), lb.view(np.uint32)), (dt, p)
        a.close()
        b.close()


def greedy_parity(model_fwd, model_gen, rm: O.RefModel, prompt, n_gen):
    """tie-aware greedy protocol: the reference (scalar ISA) generates; the GPU is teacher-forced on the
    reference's sequence; a differing argmax is accepted only where the reference's top-2 gap is within
    twice the observed logit difference (a tie).  Returns (per-position rel errs, tie steps)."""
    R, _, _ = rm.greedy(prompt, n_gen)
    seq = list(prompt) + list(R)
    rels, ties = [], []
    for p in range(len(prompt) + n_gen - 1):
        want = rm.forward(seq[p], p)
        got = model_fwd(seq[p], p)
        diff = float(np.abs(got - want).max())
        rels.append(diff / float(np.abs(want).max()))
        if p >= len(prompt) - 1:
            g, r = int(np.argmax(got)), int(np.argmax(want))
            assert r == seq[p + 1]
            if g != r:
                top2 = np.sort(want)[-2:]
                gap = float(top2[1] - top2[0])
                assert gap <= 2 * diff, f"step {p}: argmax {g} vs {r}, gap {gap} > 2*diff {2 * diff}"
                ties.append(p)
    gen = model_gen(prompt, n_gen)
    k = (ties[0] - (len(prompt) - 1)) if ties else n_gen  # free-running tokens agree up to the first tie
    assert list(gen[:k]) == list(R[:k])
    return np.asarray(rels), ties


def test_stories15m_q8_greedy_parity(cuda_dev, tmp_path):
    """stories15M-shaped, Q8_0, N(0,0.02) seed 1, 4 random prompt ids, 64 greedy tokens"""
    cfg = dict(dim=288, hidden_dim=768, n_layers=6, n_heads=6, n_kv_heads=6, vocab_size=32000, max_seq=256)
    path = str(tmp_path / "stories15m_q8.qlm")
    O.synth_write(path, cfg, O.Q8_0, 1, 0.02)
    prompt = [int(v) for v in np.random.default_rng(2024).integers(3, 32000, 4)]
    rm = O.RefModel(path, threads=1, isa=O.ISA_SCALAR)
    m = DropIn(path)
    rels, ties = greedy_parity(m.forward, m.generate, rm, prompt, 64)
    # the reference's own SIMD path against its scalar path on the same tokens: its spread at this shape
    # (the reference's ISA choice is process-wide: all scalar logits first, then the SIMD ones)
    R, _, _ = rm.greedy(prompt, 64)
    seq = list(prompt) + list(R)
    scal = [rm.forward(seq[p], p) for p in range(len(seq) - 1)]
    best = O.ref().ref_isa_best()
    rs = O.RefModel(path, threads=1, isa=best)
    isa = np.asarray([np.abs(rs.forward(seq[p], p) - scal[p]).max() / np.abs(scal[p]).max() for p in range(len(seq) - 1)])
    rs.close()
    O.ref().ref_isa_select(O.ISA_SCALAR)
    print(f"stories15M q8: rel logit err vs reference scalar over {len(rels)} positions: max {rels.max():.3e}, "
          f"median {np.median(rels):.3e}; the reference's ISA {best} vs its scalar: max {isa.max():.3e}, "
          f"median {np.median(isa):.3e}; tie steps {ties}")
    # the reference's same-weights tolerance (tests/test_model.c:50-53) bounds every position, and the GPU
    # must stay as close to the scalar path as the reference's own SIMD path is (1.5x): an int8 rounding
    # step of one activation (the sums are ordered differently) propagates through the KV cache
    assert rels.max() < 2e-2 and rels.max() <= max(1e-5, 1.5 * isa.max())
    assert np.median(rels) <= max(1e-5, 1.5 * np.median(isa))
    m.close()


@pytest.mark.parametrize("dt", [O.Q8_0, O.Q4_0])
def test_gqa_long_context_vs_float64(cuda_dev, tmp_path, dt):
    """GQA (8 q heads / 2 kv heads), hidden not a multiple of 256, 600 positions (split attention with
    many chunks): logits within the reference's same-weights tolerance (tests/test_model.c:50-53) of
    the float64 forward, like the reference's own C forward on the same file."""
    from oracle import forward_ref as F

    cfg = dict(dim=256, hidden_dim=704, n_layers=3, n_heads=8, n_kv_heads=2, vocab_size=3000, max_seq=700)
    path = str(tmp_path / f"gqa{dt}.qlm")
    O.synth_write(path, cfg, dt, 3, 0.05)
    toks = [int(t) for t in np.random.default_rng(1).integers(0, 3000, 600)]
    fcfg, W = F.load(path)
    truth = F.forward(fcfg, W, toks)
    m = DropIn(path)
    rm = O.RefModel(path, threads=4, isa=O.ref().ref_isa_best())
    got = np.stack([m.forward(t, p) for p, t in enumerate(toks)])
    cref = np.stack([rm.forward(t, p) for p, t in enumerate(toks)])
    e_gpu = np.abs(got - truth).max() / np.abs(truth).max()
    e_ref = np.abs(cref - truth).max() / np.abs(truth).max()
    print(f"gqa dt={dt}: rel err vs float64: gpu {e_gpu:.3e}, reference C {e_ref:.3e}")
    # over 600 positions activation-quantization flips push the reference itself past 2e-2 here, so the
    # bound is the reference's own error on the same file (with 25% slack)
    assert e_gpu <= max(2e-2, 1.25 * e_ref)
    m.close()
