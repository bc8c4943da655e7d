"""Multi-rank host logic of bench.py (one process per GPU, launched by torchrun): exchange of the NCCL
unique id, barriers, the max-over-ranks timing reduction, and the reference arm running on rank 0 only.
Two gloo ranks on the CPU (no GPU needed); the tensor-parallel decode itself is checked on GPUs by
test_tp_matches_single_gpu below when two are present."""
import os
import socket
import subprocess
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, out_dir: str) -> None:
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port))
    sys.path.insert(0, ROOT)
    import bench

    d = bench.Dist("gloo")
    ident = bytes(range(128)) if rank == 0 else None
    got = d.broadcast_bytes(ident)
    d.barrier()
    mx = d.max(1.5 + rank)
    args = type("A", (), {"workload": "stories15m_q8_0", "warmup": 3, "steps": 1})()
    ref = bench.reference_arm(args, dict(bench.WORKLOADS["stories15m_q8_0"])) if rank != 0 else "skipped"
    d.close()
    with open(os.path.join(out_dir, f"rank{rank}.txt"), "w") as f:
        f.write(f"{got == bytes(range(128))} {mx} {ref}\n")


def test_two_gloo_ranks_share_id_and_reduce_max(tmp_path):
    import torch.multiprocessing as mp

    port = _free_port()
    mp.start_processes(_rank_main, args=(2, port, str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    lines = [open(tmp_path / f"rank{r}.txt").read().split() for r in range(2)]
    for r, (ok, mx, ref) in enumerate(lines):
        assert ok == "True", r  # rank 1 received rank 0's 128-byte id
        assert float(mx) == 2.5, r  # max over ranks, seen by every rank
    assert lines[1][2] == "None"  # the reference arm does no work off rank 0


@pytest.mark.gpu
@pytest.mark.parametrize("world", [2, 4, 8])
def test_tp_matches_single_gpu(tmp_path, world):
    """tensor-parallel decode over 2, 4 or 8 GPUs (NCCL, one process per GPU; GQA group 2, so at 8 ranks
    each holds one KV head and its two query heads) gives the single-GPU tokens and logits within the
    reference's tolerance (tests/test_model.c:50-53, 2e-2 relative); so does the tensor-parallel batched
    prompt forward (qm_model_prefill), and the greedy decode that continues from it"""
    import torch

    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    script = tmp_path / "tp.py"
    script.write_text(f"""
import os, sys, numpy as np
sys.path.insert(0, {ROOT!r})
import ctypes as C, torch, torch.distributed as dist
import quillm_b200 as qb
rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
torch.cuda.set_device(rank)
qb.check(qb.cuda().qmc_set_device(rank))
dist.init_process_group("gloo")
cfg = dict(dim=512, hidden_dim=1024, n_layers=3, n_heads=16, n_kv_heads=8, vocab_size=3000, max_seq=64)
buf = C.create_string_buffer(128)
if rank == 0:
    qb.check(qb.cuda().qmc_nccl_unique_id(buf))
obj = [buf.raw if rank == 0 else None]
dist.broadcast_object_list(obj, src=0)
outs = []
for tp in ((1, 0), (world, rank)):
    if tp[0] == 1 and rank != 0:
        outs.append(None)
        continue
    m = qb.Model(cfg, tp[1], tp[0], obj[0] if tp[0] > 1 else None)
    m.synthesize(3, 11, 0.05)
    lg = np.zeros(cfg["vocab_size"], np.float32)
    toks, t = [], 5
    for p in range(12):
        t = m.forward(t, p, lg)
        toks.append(t)
    # the batched prompt forward over the same cache slots, then greedy decode from its token
    lp = np.zeros(cfg["vocab_size"], np.float32)
    t = m.prefill([(7 * i + 3) % cfg["vocab_size"] for i in range(20)], 0, lp)
    ptoks = [t]
    for p in range(20, 24):
        t = m.forward(t, p)
        ptoks.append(t)
    outs.append((toks, lg.copy(), ptoks, lp))
    m.close()
dist.barrier()
if rank == 0:
    (t1, l1, p1, lp1), (t2, l2, p2, lp2) = outs
    rel = float(np.max(np.abs(l1 - l2)) / np.max(np.abs(l1)))
    prel = float(np.max(np.abs(lp1 - lp2)) / np.max(np.abs(lp1)))
    open({str(tmp_path / "res.txt")!r}, "w").write(f"{{t1 == t2}} {{rel}} {{p1 == p2}} {{prel}}")
dist.destroy_process_group()
""")
    port = _free_port()
    cmd = ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node", str(world), "--master-addr", "127.0.0.1", "--master-port", str(port), str(script)]
    r = subprocess.run(cmd, capture_output=True, text=True, env=dict(os.environ, NCCL_NVLS_ENABLE="0"))
    assert r.returncode == 0, r.stderr[-3000:]
    same, rel, psame, prel = open(tmp_path / "res.txt").read().split()
    print(f"tp{world} vs tp1: identical greedy tokens {same}, max rel logit diff {float(rel):.2e}; "
          f"batched prompt forward: identical tokens after it {psame}, last-token rel logit diff {float(prel):.2e}")
    assert same == "True" and psame == "True"
    assert float(rel) < 2e-2 and float(prel) < 2e-2
