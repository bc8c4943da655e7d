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
