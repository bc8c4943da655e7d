"""Weight upload from a .qlm file through the pinned staging path (chunks of 32 MiB, two in flight): a
model loaded from a file written by the oracle's synthesiser gives bit-identical logits to the same
model synthesised on the device, with matrices large enough to take the staged path (the output
projection spans two chunks)."""
import os
import time

import numpy as np
import pytest

import quillm_b200 as qb
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def test_staged_upload_equals_device_synthesis(cuda_dev, tmp_path):
    cfg = dict(dim=1024, hidden_dim=2816, n_layers=2, n_heads=8, n_kv_heads=8, vocab_size=32000, max_seq=64)
    path = str(tmp_path / "big.qlm")
    O.synth_write(path, cfg, O.Q8_0, 5, 0.02)
    a = qb.Model(dict(cfg))
    t0 = time.perf_counter()
    qb.load_qlm_into(a, path)
    dt = time.perf_counter() - t0
    print(f"loaded {os.path.getsize(path) / 1e6:.0f} MB .qlm in {dt * 1e3:.0f} ms")
    b = qb.Model(dict(cfg))
    b.synthesize(O.Q8_0, 5, 0.02)
    la, lb = np.zeros(cfg["vocab_size"], np.float32), np.zeros(cfg["vocab_size"], np.float32)
    for p, t in enumerate([1, 70, 31999, 5]):
        a.forward(t, p, la)
        b.forward(t, p, lb)
        assert np.array_equal(la.view(np.uint32), lb.view(np.uint32)), p
    a.close()
    b.close()


def test_reupload_after_steps_refreshes_only_that_tensor(cuda_dev):
    """The persistent path keeps only its split-row weight copies (the file-layout buffers are released
    once repacked).  Uploading one tensor after the model has run allocates its buffer again and
    repacks only its rows: the result must equal a model that had the new tensors from the start."""
    cfg = dict(dim=256, hidden_dim=704, n_layers=2, n_heads=8, n_kv_heads=4, vocab_size=3000, max_seq=32)
    rng = np.random.default_rng(9)
    kv = cfg["dim"] // cfg["n_heads"] * cfg["n_kv_heads"]
    new = {(qb.QMC_T_WK, 1): O.quantize(O.Q8_0, (rng.standard_normal((kv, 256)) * 0.05).astype(np.float32)),
           (qb.QMC_T_W3, 0): O.quantize(O.Q8_0, (rng.standard_normal((704, 256)) * 0.05).astype(np.float32)),
           (qb.QMC_T_OUTPUT, -1): O.quantize(O.Q8_0, (rng.standard_normal((3000, 256)) * 0.05).astype(np.float32))}

    def upload_new(m):
        for (kind, layer), w in new.items():
            m.upload(kind, layer, O.Q8_0, w.shape[0], 256, w)

    a = qb.Model(dict(cfg))
    a.synthesize(O.Q8_0, 5, 0.02)
    la = np.zeros(3000, np.float32)
    for p, t in enumerate([3, 8, 13]):
        a.forward(t, p, la)
    assert a.decode_info()[1], "expected the persistent decode path"
    upload_new(a)
    b = qb.Model(dict(cfg))
    b.synthesize(O.Q8_0, 5, 0.02)
    upload_new(b)
    lb = np.zeros(3000, np.float32)
    for p, t in enumerate([1, 70, 2999, 5]):
        a.forward(t, p, la)
        b.forward(t, p, lb)
        assert np.array_equal(la.view(np.uint32), lb.view(np.uint32)), p
    a.close()
    b.close()
