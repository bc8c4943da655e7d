"""Device-side sampler (qmc_sampler_*) against the reference's own qm_sample (src/sampler.c, compiled from
its sources into oracle/_ref): same-seed draw sequences and RNG state on the same logits, the
distribution and edge-case checks of tests/test_sampler.c run on the device, and sampled decoding through
qmc_model_forward_sample."""
import ctypes as C
import os

import numpy as np
import pytest

import quillm_b200 as qb
from oracle import oracle as O

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")
SIX = np.array([1.0, 3.0, 0.5, 2.5, -1.0, 3.0], np.float32)  # tests/test_sampler.c:8


def dev(x):
    import torch
    return torch.tensor(np.asarray(x, np.float32), device="cuda")


def draws(logits, n, temperature, top_k, top_p, seed):
    """n device draws and n reference draws with the same settings and seed, plus the final rng states"""
    import torch
    d = dev(logits)
    s = qb.Sampler(len(logits), temperature, top_k, top_p, seed)
    got = [s.sample(d.data_ptr()) for _ in range(n)]
    st = s.rng()
    s.close()
    r = O.RefSampler(len(logits), temperature, top_k, top_p, seed)
    want = [r.sample(logits) for _ in range(n)]
    torch.cuda.synchronize()
    return np.array(got), np.array(want), st, r.rng


@pytest.mark.parametrize("T,k,p", [(0.7, 0, 1.0), (1.0, 3, 1.0), (1.0, 0, 0.6), (1.5, 0, 1.0), (1.0, 2, 0.5)])
def test_same_seed_sequences_match_reference_six(cuda_dev, T, k, p):
    got, want, st, rst = draws(SIX, 400, T, k, p, 123)
    assert st == rst  # the xorshift64* stream advanced identically
    assert (got == want).mean() >= 0.995, np.flatnonzero(got != want)[:10]


@pytest.mark.parametrize("V,T,k,p", [(300, 1.0, 0, 0.8), (5000, 0.9, 40, 0.9), (32000, 0.8, 0, 0.95),
                                     (32000, 1.2, 50, 1.0), (32000, 0.6, 0, 0.5)])
def test_same_seed_sequences_match_reference_large(cuda_dev, V, T, k, p):
    rng = np.random.default_rng(V)
    lg = (rng.standard_normal(V) * 3).astype(np.float32)
    got, want, st, rst = draws(lg, 300, T, k, p, 11)
    assert st == rst
    assert (got == want).mean() >= 0.99, np.flatnonzero(got != want)[:10]


def test_reference_properties_on_device(cuda_dev):
    """tests/test_sampler.c's checks, run through the device sampler"""
    d = dev(SIX)
    def sampler(*a):
        return qb.Sampler(6, *a)
    s = sampler(0.0, 0, 1.0, 1)
    assert s.sample(d.data_ptr()) == 1  # greedy: first maximum
    s.close()
    s = sampler(1.0, 1, 1.0, 1)
    assert s.sample(d.data_ptr()) == 1  # top_k = 1 is greedy
    s.close()
    s = sampler(1.0, 0, 1e-6, 1)
    assert all(s.sample(d.data_ptr()) == 1 for _ in range(50))  # tiny top_p: the first-ranked token
    s.close()
    N, T = 20000, 0.7
    pr = np.exp(SIX / T) / np.exp(SIX / T).sum()
    s = sampler(T, 0, 1.0, 123)
    cnt = np.bincount([s.sample(d.data_ptr()) for _ in range(N)], minlength=6)
    s.close()
    assert np.all(np.abs(cnt / N - pr) < 4 * np.sqrt(pr * (1 - pr) / N) + 1e-3)
    s = sampler(1.0, 3, 1.0, 7)  # top-k = 3: only {1, 5, 3}, renormalised
    cnt = np.bincount([s.sample(d.data_ptr()) for _ in range(N)], minlength=6)
    s.close()
    assert cnt[0] == 0 and cnt[2] == 0 and cnt[4] == 0
    assert abs(cnt[3] / N - np.exp(2.5) / (2 * np.exp(3.0) + np.exp(2.5))) < 0.015
    s = sampler(1.0, 0, 0.6, 9)  # top-p = 0.6: nucleus {1, 5}
    cnt = np.bincount([s.sample(d.data_ptr()) for _ in range(N)], minlength=6)
    s.close()
    assert cnt[1] + cnt[5] == N and abs(cnt[1] / N - 0.5) < 0.015
    seqs = []
    for seed in (99, 99, 100):  # determinism
        s = sampler(1.5, 0, 1.0, seed)
        seqs.append([s.sample(d.data_ptr()) for _ in range(200)])
        s.close()
    assert seqs[0] == seqs[1] and seqs[0] != seqs[2]
    flat = dev(np.zeros(1000, np.float32))  # near-uniform + tiny top_p: prefilter empties -> first-ranked
    s = qb.Sampler(1000, 1.0, 0, 1e-6, 4)
    assert all(s.sample(flat.data_ptr()) == 0 for _ in range(50))
    s.close()
    rng = np.random.default_rng(5)  # the prefiltered top-p path equals the top_k = V path, draw by draw
    lg = dev((rng.standard_normal(300) * 2).astype(np.float32))
    a, b = qb.Sampler(300, 1.0, 0, 0.8, 11), qb.Sampler(300, 1.0, 300, 0.8, 11)
    assert [a.sample(lg.data_ptr()) for _ in range(3000)] == [b.sample(lg.data_ptr()) for _ in range(3000)]
    a.close(), b.close()


def test_model_forward_sample(cuda_dev):
    """sampled decoding with only the token copied back: greedy settings give forward's argmax; with a
    temperature the draws follow the reference sampler applied to forward's logits, step by step"""
    path = os.path.join(GOLD, "small_q8_0.qlm")
    cfg_m = qb.QmModel()
    h = qb.host()
    err = C.create_string_buffer(256)
    assert h.qm_model_load(C.byref(cfg_m), path.encode(), 1, 0, err, 256) == 0, err.value
    gpu = C.c_void_p(cfg_m.gpu)
    V = cfg_m.cfg.vocab_size
    lib = qb.cuda()
    s = qb.Sampler(V, 0.0)
    lg = np.zeros(V, np.float32)
    nxt, nxt_s = C.c_int32(0), C.c_int32(0)
    for p, t in enumerate([3, 7, 11, 2]):
        qb.check(lib.qmc_model_forward(gpu, t, p, lg.ctypes.data, C.byref(nxt)), "forward")
        qb.check(lib.qmc_model_forward_sample(gpu, t, p, s.h, C.byref(nxt_s)), "forward_sample")
        assert nxt_s.value == nxt.value == int(np.argmax(lg))
    s.close()
    s = qb.Sampler(V, 0.9, 0, 0.9, 77)
    r = O.RefSampler(V, 0.9, 0, 0.9, 77)
    same, tok = 0, 5
    for p in range(40):
        qb.check(lib.qmc_model_forward(gpu, tok, p, lg.ctypes.data, C.byref(nxt)), "forward")
        want = r.sample(lg)
        qb.check(lib.qmc_model_forward_sample(gpu, tok, p, s.h, C.byref(nxt_s)), "forward_sample")
        same += nxt_s.value == want
        tok = want
    assert same >= 39
    assert s.rng() == r.rng
    s.close()
    h.qm_model_free(C.byref(cfg_m))
