"""Batched prompt forward (qm_model_prefill / qmc_model_prefill): the prompt's tokens go through every layer
together, filling their KV-cache slots.  Teacher-forced parity: the last prompt token's logits equal the
golden logits at that position (the token-at-a-time reference, tests/test_model.c tolerances), and decode
steps after the prefill continue on those golden logits, which checks the cache slots the prefill wrote."""
import ctypes as C
import os

import numpy as np
import pytest

import quillm_b200 as qb
from oracle import oracle as O

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")
CASES = [("small_f32", 1e-5), ("odd_f32", 1e-5), ("l2c_f32", 1e-5), ("small_q8_0", 2e-2), ("odd_q8_0", 2e-2),
         ("small_q4_0", 2e-2), ("odd_q4_0", 2e-2)]


class DropIn:
    def __init__(self, path):
        self.h = qb.host()
        self.m = qb.QmModel()
        err = C.create_string_buffer(256)
        assert self.h.qm_model_load(C.byref(self.m), path.encode(), 1, 0, err, 256) == 0, err.value
        self.V = self.m.cfg.vocab_size

    def prefill(self, toks, pos0):
        t = np.asarray(toks, np.int32)
        p = self.h.qm_model_prefill(C.byref(self.m), t.ctypes.data, len(t), pos0)
        return None if not p else np.ctypeslib.as_array(p, (self.V,)).copy()

    def forward(self, tok, pos):
        p = self.h.qm_model_forward(C.byref(self.m), tok, pos)
        return None if not p else np.ctypeslib.as_array(p, (self.V,)).copy()

    def close(self):
        self.h.qm_model_free(C.byref(self.m))


def rel(a, b):
    return float(np.abs(a - b).max() / np.abs(b).max())


@pytest.mark.parametrize("name,tol", CASES)
def test_prefill_matches_token_at_a_time_reference(cuda_dev, name, tol):
    toks, V = O.read_tokens(os.path.join(GOLD, f"{name}.tokens"))
    ref = np.fromfile(os.path.join(GOLD, f"{name}.ref.f32"), np.float32).reshape(len(toks), V)
    m = DropIn(os.path.join(GOLD, f"{name}.qlm"))
    n = max(1, len(toks) // 2)
    lg = m.prefill(toks[:n], 0)
    assert rel(lg, ref[n - 1]) < tol, rel(lg, ref[n - 1])
    for p in range(n, len(toks)):  # decode on the cache slots the prefill wrote
        got = m.forward(toks[p], p)
        assert rel(got, ref[p]) < tol, (p, rel(got, ref[p]))
    # the same prompt in two chunks (the second at pos0 > 0), then one decode step
    k = max(1, n // 3)
    m.prefill(toks[:k], 0)
    lg2 = m.prefill(toks[k:n], k) if k < n else m.prefill(toks[:n], 0)
    assert rel(lg2, ref[n - 1]) < tol
    assert rel(m.forward(toks[n], n), ref[n]) < tol
    # errors: empty prompt, past max_seq, token out of range
    S = m.m.cfg.max_seq
    assert m.prefill([], 0) is None
    assert m.prefill([0] * 2, S - 1) is None
    assert m.prefill([V], 0) is None and m.prefill([-1], 0) is None
    m.close()


@pytest.mark.parametrize("heads,kv_heads,n_prompt", [(8, 2, 61), (32, 8, 200), (32, 8, 300)])
def test_prefill_long_prompt_gqa(cuda_dev, heads, kv_heads, n_prompt):
    """a long prompt on a synthesized GQA model: the prefill's logits and the decode steps after it agree
    with feeding the prompt token by token.  On a 148-SM B200 the three cases take the attention kernel's
    8-, 16- and 32-token query tiles (the largest tile that still gives every SM two blocks)"""
    cfg = dict(dim=256 if heads == 8 else 512, hidden_dim=688, n_layers=3 if heads == 8 else 2, n_heads=heads,
               n_kv_heads=kv_heads, vocab_size=2000, max_seq=128 if n_prompt < 100 else 320)
    rng = np.random.default_rng(3)
    prompt = rng.integers(0, cfg["vocab_size"], n_prompt).astype(np.int32)
    for dt in (qb.QMC_Q8_0, qb.QMC_Q4_0):
        a = qb.Model(dict(cfg))
        a.synthesize(dt, 21, 0.05)
        la = np.zeros(cfg["vocab_size"], np.float32)
        nxt_a = a.prefill(prompt, 0, la)
        b = qb.Model(dict(cfg))
        b.synthesize(dt, 21, 0.05)
        lb = np.zeros(cfg["vocab_size"], np.float32)
        for p, t in enumerate(prompt):
            nxt_b = b.forward(int(t), p, lb)
        assert rel(la, lb) < 2e-2, rel(la, lb)
        assert nxt_a == int(np.argmax(la))
        # both continue on the same tokens (b's greedy choices): the logits agree step by step, which
        # checks the cache slots the prefill wrote without depending on near-tie argmax choices
        t = nxt_b
        for p in range(len(prompt), len(prompt) + 8):
            a.forward(t, p, la)
            t = b.forward(t, p, lb)
            assert rel(la, lb) < 2e-2, (p, rel(la, lb))
        a.close(), b.close()
