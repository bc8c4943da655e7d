"""Model-level parity at the shapes the benchmark runs (tests/test_model.c strategy, applied to the
benchmark's own models), through the drop-in qm_model_load / qm_model_forward / qm_model_prefill:

  - the full Llama-7B-shaped Q4_0 model (seed 7, the benchmark's 128-token prompt, head_dim 128,
    32 layers, vocab 32000): the decode kernel whose speed the benchmark reports, at its own shape;
  - a Llama-70B-shaped GQA Q8_0 model cut to 2 layers (dim 8192, hidden 28672, 64 query heads over 8 KV
    heads: group 8, head_dim 128): the attention units that span more than one group of query heads;
  - Llama-7B dims in Q8_0, 2 layers.

The oracle is the reference itself (src/model.c:158-191 compiled from its sources, best ISA): it runs
greedily from the prompt and its logits at every position are the teacher-forced targets.  Protocol
(tie-aware greedy, as for the stories15M case):
  * per position, the GPU's logits on the reference's token sequence are as close to the reference's as
    the reference's own second-best ISA is (its other SIMD path, same file, same tokens, teacher
    forced): max and median over positions within 1.5x of that spread, and never looser than the
    reference's same-weights tolerance (2e-2 relative, tests/test_model.c:50-53) or 2e-3 median.
    Both sides quantize activations bit-exactly, but the dot products sum in different orders; where
    that moves an activation across an int8 rounding boundary the two quantize it one step apart, the
    step propagates through the KV cache and later layers, and on these random N(0, 0.02) models the
    logits drift by percents over 32 layers -- between the reference's own scalar, AVX2 and AVX-512
    paths alike (measured: 5e-2 median at Llama-7B shape).  Both spreads are printed;
  * a differing argmax is accepted only where the reference's top-2 gap is within twice the observed
    logit difference (a tie); the tie steps are printed;
  * free-running greedy tokens from the GPU equal the reference's up to the first tie;
  * the batched prompt forward's last-token logits agree with the reference's at that position.
"""
import ctypes as C
import os
import sys

import numpy as np
import pytest

import quillm_b200 as qb
from oracle import oracle as O

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
import bench  # noqa: E402  (workload definitions and the shared model-file cache)

pytestmark = pytest.mark.gpu

TOL = 2e-2  # tests/test_model.c:50-53, same weights
MEDIAN = 2e-3  # floor of the bound on the median over positions
SLACK = 1.5  # bound = SLACK x the reference's own ISA spread


def _host_model(path: str, max_seq: int):
    h = qb.host()
    m = qb.QmModel()
    err = C.create_string_buffer(256)
    assert h.qm_model_load(C.byref(m), path.encode(), 1, max_seq, err, 256) == 0, err.value
    return h, m


def _forward(h, m, V, tok, pos):
    p = h.qm_model_forward(C.byref(m), tok, pos)
    assert p, h.qm_last_error()
    return np.ctypeslib.as_array(p, (V,)).copy()


def _ref_greedy_logits(rm: O.RefModel, prompt, n_gen: int):
    """the reference fed the prompt, then its own greedy tokens: (sequence, logits at every position)"""
    seq, want = list(prompt), []
    for p in range(len(prompt) + n_gen - 1):
        lg = rm.forward(seq[p], p)
        want.append(lg)
        if p >= len(prompt) - 1:
            seq.append(int(np.argmax(lg)))
    return seq, want


def _rel(a, b):
    return float(np.abs(a - b).max() / np.abs(b).max())


def _check(name, path, prompt, n_gen, max_seq, threads=None):
    threads = threads or os.cpu_count() or 1
    best = O.ref().ref_isa_best()
    rm = O.RefModel(path, threads=threads, max_seq=max_seq, isa=best)
    V = rm.cfg["vocab_size"]
    seq, want = _ref_greedy_logits(rm, prompt, n_gen)
    rm.close()
    # the reference's second-best ISA on the same sequence: its own spread at this shape
    other = next((i for i in (O.ISA_AVX2, O.ISA_SCALAR) if i != best and O.ref().ref_isa_supported(i)), None)
    isa_rels = None
    if other is not None:
        ro = O.RefModel(path, threads=threads, max_seq=max_seq, isa=other)
        isa_rels = np.asarray([_rel(ro.forward(seq[p], p), want[p]) for p in range(len(seq) - 1)])
        ro.close()
    h, m = _host_model(path, max_seq)
    try:
        rels, ties = [], []
        for p in range(len(seq) - 1):
            got = _forward(h, m, V, seq[p], p)
            diff = float(np.abs(got - want[p]).max())
            rels.append(diff / float(np.abs(want[p]).max()))
            if p >= len(prompt) - 1:
                g, r = int(np.argmax(got)), int(np.argmax(want[p]))
                if g != r:
                    top2 = np.sort(want[p])[-2:]
                    gap = float(top2[1] - top2[0])
                    assert gap <= 2 * diff, f"{name} step {p}: argmax {g} vs {r}, gap {gap} > 2*diff {2 * diff}"
                    ties.append(p)
        # free-running greedy on the device (the token-at-a-time prompt, then n_gen steps)
        pr = np.asarray(prompt, np.int32)
        out = np.zeros(n_gen, np.int32)
        assert h.qm_model_generate(C.byref(m), pr.ctypes.data, len(pr), n_gen, out.ctypes.data) == 0
        k = (ties[0] - (len(prompt) - 1)) if ties else n_gen
        assert list(out[:k]) == seq[len(prompt):len(prompt) + k], name
        # the batched prompt forward (tensor-core contraction): last prompt token's logits
        lp = h.qm_model_prefill(C.byref(m), pr.ctypes.data, len(pr), 0)
        assert lp, h.qm_last_error()
        pf = np.ctypeslib.as_array(lp, (V,)).copy()
        w = want[len(prompt) - 1]
        pf_rel = float(np.abs(pf - w).max() / np.abs(w).max())
        n_launch, pers = C.c_int32(0), C.c_int32(0)
        qb.check(qb.cuda().qmc_model_decode_info(m.gpu, C.byref(n_launch), C.byref(pers)), "decode_info")
        path_name = "persistent decode kernel" if pers.value else f"per-operation graph ({n_launch.value} launches)"
    finally:
        h.qm_model_free(C.byref(m))
    rels = np.asarray(rels)
    bmax, bmed = TOL, MEDIAN
    spread = ""
    if isa_rels is not None:
        bmax = max(TOL, SLACK * float(isa_rels.max()))
        bmed = max(MEDIAN, SLACK * float(np.median(isa_rels)))
        spread = f"; the reference's ISA {other} vs {best}: max {isa_rels.max():.3e}, median {np.median(isa_rels):.3e}"
    print(f"{name} [{path_name}]: rel logit err vs the reference (ISA {best}) over {len(rels)} positions: "
          f"max {rels.max():.3e}, median {np.median(rels):.3e}{spread}; tie steps {ties}; "
          f"prefill last-token rel err {pf_rel:.3e}")
    assert rels.max() <= bmax and np.median(rels) <= bmed, (name, rels.max(), np.median(rels), bmax, bmed)
    assert pf_rel <= bmax, (name, pf_rel)


def test_llama7b_q4_0_full_model(cuda_dev):
    """BASELINE config 4 at full size: seed 7, the benchmark's 128 random prompt ids, 32 greedy tokens"""
    wl = bench.WORKLOADS["llama7b_q4_0"]
    path = bench.model_file(wl, "llama7b_q4_0")
    _check("llama7b_q4_0", path, [int(t) for t in bench.prompt_ids(wl)], 32, 256)


def _cut_model(tmp_dir, name, cfg, dt, seed):
    d = os.environ.get("QUILLM_BENCH_DIR", "/tmp/quillm_bench")
    os.makedirs(d, exist_ok=True)
    path = os.path.join(d, f"{name}_seed{seed}.qlm")
    if not os.path.exists(path + ".ok"):
        O.synth_write(path, cfg, dt, seed, 0.02, os.cpu_count())
        open(path + ".ok", "w").close()
    return path


def test_llama70b_gqa8_q8_0_two_layers(cuda_dev, tmp_path):
    """BASELINE config 5's layer shapes (GQA group 8, head_dim 128) in 2 layers; 160 prompt ids spread
    the attention over several position segments per KV head"""
    cfg = dict(dim=8192, hidden_dim=28672, n_layers=2, n_heads=64, n_kv_heads=8, vocab_size=32000, max_seq=512)
    path = _cut_model(tmp_path, "llama70b2_q8_0", cfg, O.Q8_0, 70)
    prompt = [int(t) for t in np.random.default_rng(1070).integers(3, 32000, 160)]
    _check("llama70b2_q8_0", path, prompt, 24, 512)


def test_llama7b_dims_q8_0_two_layers(cuda_dev, tmp_path):
    cfg = dict(dim=4096, hidden_dim=11008, n_layers=2, n_heads=32, n_kv_heads=32, vocab_size=32000, max_seq=256)
    path = _cut_model(tmp_path, "llama7b2_q8_0", cfg, O.Q8_0, 8)
    prompt = [int(t) for t in np.random.default_rng(1008).integers(3, 32000, 64)]
    _check("llama7b2_q8_0", path, prompt, 32, 256)


def test_llama7b_dims_gqa8_q4_0_two_layers(cuda_dev, tmp_path):
    """the persistent decode kernel at GQA group 8 and head_dim 128 (32 query heads over 4 KV heads):
    each KV head's query group spans two attention units"""
    cfg = dict(dim=4096, hidden_dim=11008, n_layers=2, n_heads=32, n_kv_heads=4, vocab_size=32000, max_seq=256)
    path = _cut_model(tmp_path, "llama7b2gqa8_q4_0", cfg, O.Q4_0, 9)
    prompt = [int(t) for t in np.random.default_rng(1009).integers(3, 32000, 100)]
    _check("llama7b2gqa8_q4_0", path, prompt, 32, 256)
