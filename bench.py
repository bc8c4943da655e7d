#!/usr/bin/env python3
"""quillm-b200 benchmark: batch-1 greedy decode tok/s (+ matvec HBM GB/s, prefill) on N GPUs of one node.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--workload llama7b_q4_0|llama70b_q8_0|stories15m_q8_0]
  python bench.py --impl reference ...      the reference's own CPU path (oracle/_ref) on this host's cores

A step is one decode token.  The model (seeded N(0, 0.02) weights, synthesized in HBM) first consumes
the workload's random prompt one token per step, then W untimed and K timed greedy decode steps run as
a device-resident chain of CUDA-graph replays (value); `e2e` repeats K steps through the public
per-token call with host buffers (token in, logits + next token out, copies inside the timed region).
N > 1 (launched by torchrun): tensor parallelism over NCCL, timing = max over ranks, rank 0 prints.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "batch-1 decode tok/s + matvec achieved HBM GB/s vs 8 TB/s peak"
Q8_0, Q4_0 = 2, 3
WORKLOADS = {
    "llama7b_q4_0": dict(cfg=dict(dim=4096, hidden_dim=11008, n_layers=32, n_heads=32, n_kv_heads=32,
                                  vocab_size=32000, max_seq=2048), dtype=Q4_0, seed=7, prompt=128,
                         model="Llama-7B-shaped, Q4_0, N(0,0.02) seed 7"),
    "llama70b_q8_0": dict(cfg=dict(dim=8192, hidden_dim=28672, n_layers=80, n_heads=64, n_kv_heads=8,
                                   vocab_size=32000, max_seq=4096), dtype=Q8_0, seed=70, prompt=512,
                          model="Llama-70B-shaped GQA, Q8_0, N(0,0.02) seed 70"),
    "stories15m_q8_0": dict(cfg=dict(dim=288, hidden_dim=768, n_layers=6, n_heads=6, n_kv_heads=6,
                                     vocab_size=32000, max_seq=256), dtype=Q8_0, seed=1, prompt=4,
                            model="stories15M-shaped, Q8_0, N(0,0.02) seed 1"),
}
STD = 0.02
DTYPE_NAME = {Q8_0: "q8_0", Q4_0: "q4_0"}


def row_bytes(dt: int, n: int) -> int:
    return ((n + 31) // 32) * (34 if dt == Q8_0 else 18)


def prompt_ids(wl: dict) -> np.ndarray:
    rng = np.random.default_rng(wl["seed"] + 1000)
    return rng.integers(3, wl["cfg"]["vocab_size"], wl["prompt"]).astype(np.int32)


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


# ------------------------------------------------------------------ distributed plumbing
class Dist:
    """rank / world from torchrun's environment; torch.distributed only for id exchange, barriers and the
    max-over-ranks timing reduction"""

    def __init__(self, backend: str):
        self.rank = int(os.environ.get("RANK", 0))
        self.world = int(os.environ.get("WORLD_SIZE", 1))
        self.local = int(os.environ.get("LOCAL_RANK", 0))
        self.pg = None
        if self.world > 1:
            import datetime

            import torch.distributed as dist

            kw = {}
            if backend == "nccl":
                import torch

                kw["device_id"] = torch.device(f"cuda:{self.local}")
            dist.init_process_group(backend, timeout=datetime.timedelta(seconds=180), **kw)
            self.pg = dist

    def broadcast_bytes(self, b: bytes | None) -> bytes:
        if self.world == 1:
            return b
        obj = [b]
        self.pg.broadcast_object_list(obj, src=0)
        return obj[0]

    def broadcast_object(self, obj):
        if self.world == 1:
            return obj
        box = [obj]
        self.pg.broadcast_object_list(box, src=0)
        return box[0]

    def barrier(self):
        if self.world > 1:
            self.pg.barrier()

    def max(self, v: float) -> float:
        if self.world == 1:
            return v
        import torch

        dev = "cuda" if self.pg.get_backend() == "nccl" else "cpu"
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        if self.pg is not None:
            self.pg.destroy_process_group()


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 100 ms while running"""

    Q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                       "-lms", "100", "-i", str(index)], stdout=subprocess.PIPE,
                                      stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.p = None

    def stop(self) -> dict:
        if not self.p:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.15)
        self.p.terminate()
        out, _ = self.p.communicate(timeout=10)
        rows = [[c.strip() for c in line.split(",")] for line in out.splitlines() if line.count(",") >= 7]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[0]) for r in rows if r[0].replace(".", "").isdigit()]
        mx = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        busy = [s for s in sm if mx and s > 0.5 * max(mx)] or sm
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[4 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(busy) if busy else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


# ------------------------------------------------------------------ GPU arm
def cuda_events(stream_ptr: int):
    import torch

    st = torch.cuda.ExternalStream(stream_ptr)
    return st, torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)


def _graph_time(torch, launch, n: int) -> float:
    """seconds per launch of `launch(stream_ptr)` replayed n times from one captured CUDA graph (no host
    launch overhead in the timing), CUDA events on the capture stream"""
    st = torch.cuda.Stream()
    torch.cuda.synchronize()
    with torch.cuda.stream(st):
        for _ in range(3):
            launch(st.cuda_stream)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=st):
        for i in range(n):
            launch(st.cuda_stream, i)
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(st):
        e0.record(st)
        g.replay()
        e1.record(st)
    torch.cuda.synchronize()
    del g
    return e0.elapsed_time(e1) / 1e3 / n


def matvec_operands(torch, dt: int, rows: int, cols: int):
    """rotating weight copies (> 2x L2 in total, so every launch streams from HBM) with valid fp16 scales"""
    rb = row_bytes(dt, cols)
    wbytes = rows * rb
    copies = max(2, -(-256 * 2**20 // wbytes))
    g = torch.Generator(device="cuda").manual_seed(rows * 7 + cols)
    Ws = [torch.randint(0, 256, (wbytes + 256,), dtype=torch.uint8, device="cuda", generator=g) for _ in range(copies)]
    for w in Ws:  # fp16 0.01 as every block's scale keeps the arithmetic finite
        v = w[:wbytes].view(rows, -1, 34 if dt == Q8_0 else 18)
        v[:, :, 0] = 0x1F
        v[:, :, 1] = 0x21
    x = torch.randn(cols, device="cuda")
    y = torch.empty(rows, device="cuda")
    xq = torch.empty(34 * ((cols + 31) // 32), dtype=torch.uint8, device="cuda")
    torch.cuda.synchronize()
    algo = wbytes + 4 * cols + 34 * ((cols + 31) // 32) + 4 * rows
    return Ws, x, y, xq, float(algo)


def time_matvec(qb, torch, dt: int, rows: int, cols: int, iters: int = 64) -> tuple[float, float]:
    """(seconds per launch, algorithmic bytes) of qmc_matvec"""
    Ws, x, y, xq, algo = matvec_operands(torch, dt, rows, cols)
    lib = qb.cuda()

    def launch(stream, i=0):
        qb.check(lib.qmc_matvec(dt, Ws[i % len(Ws)].data_ptr(), rows, cols, x.data_ptr(), y.data_ptr(),
                                xq.data_ptr(), stream))

    sec = _graph_time(torch, launch, iters)
    del Ws
    return sec, algo


def time_prefill(qb, torch, T: int, N: int, K: int, iters: int = 10) -> tuple[float, float]:
    """seconds per launch of the Q8_0 prefill contraction: (tensor cores on the split-row copy, the model's
    path; CUDA cores on the file layout, qmc_matmul_nt_q)"""
    W = torch.randint(0, 256, (N * row_bytes(Q8_0, K) + 256,), dtype=torch.uint8, device="cuda")
    v = W[: N * row_bytes(Q8_0, K)].view(N, -1, 34)
    v[:, :, 0] = 0x1F
    v[:, :, 1] = 0x21
    lib = qb.cuda()
    Ws = torch.empty(N * lib.qmc_split_row_bytes(Q8_0, K) + 256, dtype=torch.uint8, device="cuda")
    qb.check(lib.qmc_repack_split(Q8_0, W.data_ptr(), N, K, Ws.data_ptr(), None))
    A = torch.randn(T, K, device="cuda")
    Cm = torch.empty(T, N, device="cuda")

    def tc(stream, i=0):
        qb.check(lib.qmc_matmul_split_q(Q8_0, Ws.data_ptr(), A.data_ptr(), Cm.data_ptr(), T, N, K, stream))

    def cc(stream, i=0):
        qb.check(lib.qmc_matmul_nt_q(Q8_0, W.data_ptr(), A.data_ptr(), Cm.data_ptr(), T, N, K, stream))

    return _graph_time(torch, tc, iters), _graph_time(torch, cc, iters)


def profile_decode(layers: int, workload: str = "llama7b_q4_0") -> None:
    """--profile-decode LAYERS: the workload's model cut to LAYERS layers decodes positions 0..133 (a few
    GB on the device), for ncu captures of decode_step_kernel at a position like the bench's"""
    import quillm_b200 as qb

    wl = WORKLOADS[workload]
    cfg = dict(wl["cfg"], n_layers=layers)
    qb.check(qb.cuda().qmc_set_device(0))
    m = qb.Model(cfg)
    m.synthesize(wl["dtype"], wl["seed"], STD)
    m.enqueue_decode(1, 0, 130)
    qb.check(qb.cuda().qmc_sync())
    m.enqueue_decode(-1, 0, 4)
    qb.check(qb.cuda().qmc_sync())
    print("decode_info", m.decode_info())
    m.close()


def profile_matvec(spec: str) -> None:
    """--profile-matvec ROWSxCOLS:DTYPE[:N]: N plain qmc_matvec launches (for ncu captures)"""
    import torch

    import quillm_b200 as qb

    shape, dts, *rest = spec.split(":")
    rows, cols = map(int, shape.split("x"))
    dt = {"q8_0": Q8_0, "q4_0": Q4_0}[dts]
    n = int(rest[0]) if rest else 4
    qb.check(qb.cuda().qmc_set_device(0))
    Ws, x, y, xq, _ = matvec_operands(torch, dt, rows, cols)
    for i in range(n):
        qb.check(qb.cuda().qmc_matvec(dt, Ws[i % len(Ws)].data_ptr(), rows, cols, x.data_ptr(), y.data_ptr(),
                                      xq.data_ptr(), None))
    qb.check(qb.cuda().qmc_sync())
    print(f"profile-matvec {spec}: {n} launches ok")


def profile_prefill(spec: str) -> None:
    """--profile-prefill TxNxK:DTYPE[:N]: N launches of the tensor-core prefill contraction (ncu captures)"""
    import torch

    import quillm_b200 as qb

    shape, dts, *rest = spec.split(":")
    T, N, K = map(int, shape.split("x"))
    dt = {"q8_0": Q8_0, "q4_0": Q4_0}[dts]
    n = int(rest[0]) if rest else 3
    lib = qb.cuda()
    qb.check(lib.qmc_set_device(0))
    rb = row_bytes(dt, K)
    W = torch.randint(0, 256, (N * rb + 256,), dtype=torch.uint8, device="cuda")
    v = W[: N * rb].view(N, -1, 34 if dt == Q8_0 else 18)
    v[:, :, 0] = 0x1F  # fp16 0.01 scales
    v[:, :, 1] = 0x21
    Ws = torch.empty(N * lib.qmc_split_row_bytes(dt, K) + 256, dtype=torch.uint8, device="cuda")
    qb.check(lib.qmc_repack_split(dt, W.data_ptr(), N, K, Ws.data_ptr(), None))
    A = torch.randn(T, K, device="cuda")
    Cm = torch.empty(T, N, device="cuda")
    for _ in range(n):
        qb.check(lib.qmc_matmul_split_q(dt, Ws.data_ptr(), A.data_ptr(), Cm.data_ptr(), T, N, K, None))
    qb.check(lib.qmc_sync())
    print(f"profile-prefill {spec}: {n} launches ok")


def profile_prompt(T: int) -> None:
    """--profile-prompt T: the 7B Q4_0 model's batched forward of a T-token prompt, twice (ncu launch lists)"""
    import quillm_b200 as qb

    wl = WORKLOADS["llama7b_q4_0"]
    qb.check(qb.cuda().qmc_set_device(0))
    m = qb.Model(dict(wl["cfg"]))
    m.synthesize(wl["dtype"], wl["seed"], STD)
    prompt = np.random.default_rng(wl["seed"] + 2000).integers(3, wl["cfg"]["vocab_size"], T).astype(np.int32)
    for _ in range(2):
        m.prefill(prompt, 0)
    m.close()
    print(f"profile-prompt {T}: 2 prefills ok")


def traffic_from_profiles(tag: str):
    """DRAM bytes per launch recorded from an ncu capture (profiles/*.md line `traffic[<tag>] = <bytes>`)"""
    pdir = os.path.join(ROOT, "profiles")
    if not os.path.isdir(pdir):
        return None
    for fn in sorted(os.listdir(pdir)):
        if fn.endswith((".md", ".txt")):
            for line in open(os.path.join(pdir, fn)):
                if line.strip().startswith(f"traffic[{tag}]"):
                    try:
                        return float(line.split("=")[1].split()[0])
                    except (IndexError, ValueError):
                        pass
    return None


def gpu_arm(args, wl: dict) -> dict | None:
    import torch

    import quillm_b200 as qb

    d = Dist("nccl")
    torch.cuda.set_device(d.local)
    qb.check(qb.cuda().qmc_set_device(d.local), "set_device")
    cfg = dict(wl["cfg"])
    nid = None
    if d.world > 1:
        buf = C.create_string_buffer(128)
        if d.rank == 0:
            qb.check(qb.cuda().qmc_nccl_unique_id(buf))
        nid = d.broadcast_bytes(buf.raw if d.rank == 0 else None)
    model = qb.Model(cfg, d.rank, d.world, nid)
    model.synthesize(wl["dtype"], wl["seed"], STD)
    prompt = prompt_ids(wl)
    W, K = args.warmup, args.steps
    npos = len(prompt)
    if npos + W + 2 * K > cfg["max_seq"]:
        raise SystemExit(f"{npos}+{W}+2*{K} positions exceed max_seq {cfg['max_seq']}")
    s = C.c_void_p()
    qb.check(qb.cuda().qmc_stream(C.byref(s)))
    st, e0, e1 = cuda_events(s.value)

    # prompt, one token per step like the reference (device-resident chain); one untimed step first builds
    # the decode graph and the split-row weight copies, one-time costs kept out of the timing
    model.generate(prompt[:1], 1)
    d.barrier()
    qb.check(qb.cuda().qmc_sync())
    e0.record(st)
    first = int(model.generate(prompt, 1)[0])
    e1.record(st)
    qb.check(qb.cuda().qmc_sync())
    prompt_s = d.max(e0.elapsed_time(e1) / 1e3)

    clocks = ClockSampler(d.local)
    model.enqueue_decode(first, npos, W)
    qb.check(qb.cuda().qmc_sync())
    pos0 = npos + W
    d.barrier()
    qb.check(qb.cuda().qmc_sync())
    e0.record(st)
    model.enqueue_decode(-1, 0, K)
    e1.record(st)
    qb.check(qb.cuda().qmc_sync())
    d.barrier()
    clk = clocks.stop()
    sec = d.max(e0.elapsed_time(e1) / 1e3)
    tok, pos = model.state()
    assert pos == pos0 + K, (pos, pos0, K)

    # e2e: the public per-token call, host buffers, copies inside the timed region, over the same
    # positions as the device-timed steps (their cache slots are rewritten), so that both figures carry
    # the same attention length
    logits = np.zeros(cfg["vocab_size"], np.float32)
    model.forward(tok, pos0 - 1, logits)  # warm
    d.barrier()
    t0 = time.perf_counter()
    t = tok
    for i in range(K):
        t = model.forward(t, pos0 + i, logits)
    e2e_s = d.max(time.perf_counter() - t0)

    # sampled decoding through the public call: temperature 0.8 / top-p 0.9 drawn on the device, only the
    # 4-byte token copied back per step (the reference's loop copies the logits and samples on the host)
    sampler = qb.Sampler(cfg["vocab_size"], 0.8, 0, 0.9, 1234)
    t = model.forward_sample(tok, pos0 - 1, sampler)  # warm
    d.barrier()
    t0 = time.perf_counter()
    for i in range(K):
        t = model.forward_sample(t, pos0 + i, sampler)
    e2e_sampled_s = d.max(time.perf_counter() - t0)
    sampler.close()

    # batched prompt forward: the same prompt through every layer at once, timed through the public call
    # (host token copy in, logits copy out, one synchronisation); under tensor parallelism every rank
    # runs it (its wo / w2 all-reduces are collectives) and the time is the max over ranks
    # (a failure here is reported in the line instead of losing the decode figures: the same calls fail on
    # every rank, so the ranks still take the same collective steps afterwards)
    try:
        model.prefill(prompt, 0, logits)  # allocates the row buffers
        reps = 5
        d.barrier()
        e0.record(st)
        for _ in range(reps):
            model.prefill(prompt, 0, logits)
        e1.record(st)
        qb.check(qb.cuda().qmc_sync())
        pf_s = d.max(e0.elapsed_time(e1) / 1e3 / reps)
        prefill = {"tokens": npos, "tok_s": npos / pf_s, "ms": pf_s * 1e3,
                   "token_at_a_time_tok_s": npos / prompt_s, "speedup": prompt_s / pf_s}
    except Exception as e:  # noqa: BLE001
        prefill = {"tokens": npos, "error": str(e)[:300]}

    per_gpu_bytes = np.mean([model.step_bytes(p) for p in range(pos0, pos0 + K)])
    launches, persistent = model.decode_info()
    tp_par = tp_parity(qb, wl, model, prompt, d) if d.world > 1 else None
    hbm, tflops, src = peaks()
    step_time = sec / K
    achieved = per_gpu_bytes / step_time / 1e9
    kname = "decode_step_kernel (one launch per token)" if persistent else "decode step (per-operation kernels)"
    out = {
        "metric": METRIC, "value": K / sec, "unit": "tok/s", "n_gpus": d.world, "steps": K, "warmup": W,
        "ms_per_step": step_time * 1e3, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "i8xi8->i32 dp4a, f32 scale/accumulate",
        "data": f"synthetic: {wl['model']}; random prompt ids (numpy default_rng({wl['seed'] + 1000}))",
        "config": {"workload": f"{args.workload}_decode", "model": wl["model"], "global_batch": 1,
                   "seq_len": cfg["max_seq"], "prompt_tokens": npos, "decode_positions": [pos0, pos0 + K - 1],
                   "parallelism": f"tp{d.world}",
                   "l2": f"inputs larger than L2: {per_gpu_bytes / 1e9:.2f} GB streamed per step per GPU"},
        # the dominant kernel: a whole decode step is one launch, so its duration is the step time
        "roofline": {"bound": "hbm", "kernel": kname, "achieved": achieved, "peak": hbm, "unit": "GB/s",
                     "frac": achieved / hbm, "traffic": traffic_from_profiles(f"decode_step {args.workload}")
                     if persistent and d.world == 1 else None,
                     "bytes_per_step_per_gpu": per_gpu_bytes,
                     "peak_source": f"{src} (MEASURED_PEAKS.json hbm_gbs)" if src == "measured" else src},
        "prompt_tok_s": npos / prompt_s,
        "prefill": prefill,
        "e2e": {"value": K / e2e_s, "unit": "tok/s", "h2d_bytes_per_step": 16,
                "d2h_bytes_per_step": cfg["vocab_size"] * 4 + 4},
        "e2e_sampled": {"value": K / e2e_sampled_s, "unit": "tok/s", "sampling": "temperature 0.8, top-p 0.9, on the device",
                        "h2d_bytes_per_step": 16, "d2h_bytes_per_step": 4},
        "gpu_launches": K * launches,
        "clocks": clk,
    }
    if tp_par is not None:
        out["tp_parity"] = tp_par
    model.close()
    if d.rank == 0 and d.world == 1 and not args.quick:
        out.update(kernel_sweeps(qb, torch, wl, hbm, tflops, src))
        out["long_context"] = long_context(qb, wl, st, e0, e1, hbm)
    if d.rank == 0 and d.world == 1 and not args.no_cpu_baseline:
        out["cpu_baseline"] = cpu_baseline(args, wl)
    if "matvec" in out:  # last, where a tail of the line keeps it: shape, dtype, fraction of the HBM peak
        out["matvec_sweep_frac"] = {f"{r['dtype']} {r['shape']}": round(r["frac"], 3) for r in out["matvec"]}
    d.close()
    return out if d.rank == 0 else None


TP_PARITY_TOKENS = 16


def tp_parity(qb, wl: dict, model, prompt, d) -> dict | None:
    """The tensor-parallel model against the same model on one GPU, teacher forced.  Rank 0 first runs
    the whole model (TP=1) greedily from the prompt and keeps its logits at each generated position; every
    rank then feeds that token sequence to the tensor-parallel model.  Per position: the relative logit
    difference, and whether the greedy token agrees -- a different argmax counts as a tie when TP=1's
    top-2 gap is within twice the observed difference (the summation order differs across the ranks'
    shards, as it does between the reference's own SIMD paths).  Rank 0 returns the summary."""
    P, T = len(prompt), TP_PARITY_TOKENS
    seq, ref, why = None, None, None
    if d.rank == 0:  # every rank reaches the broadcast below, with None when the TP=1 run failed
        m1 = None
        try:
            m1 = qb.Model(dict(wl["cfg"]))
            m1.synthesize(wl["dtype"], wl["seed"], STD)
            gen = [int(t) for t in m1.generate(prompt, T)]
            ref = []
            for p in range(P - 1, P + T - 1):  # the cache holds the sequence: the same K/V are rewritten
                lg = np.zeros(wl["cfg"]["vocab_size"], np.float32)
                m1.forward(([int(t) for t in prompt] + gen)[p], p, lg)
                ref.append(lg)
            seq = [int(t) for t in prompt] + gen
        except Exception as e:  # e.g. the whole model does not fit beside this rank's shard
            why = str(e)
        finally:
            if m1 is not None:
                m1.close()
    seq = d.broadcast_object(seq)
    if seq is None:
        return {"reference": "the same model on 1 GPU (TP=1)", "unavailable": why} if d.rank == 0 else None
    model.generate(seq[:P], 1)  # the prompt's cache slots, device-resident
    rels, ties, disagree = [], 0, 0
    for j, p in enumerate(range(P - 1, P + T - 1)):
        lg = np.zeros(wl["cfg"]["vocab_size"], np.float32)
        model.forward(seq[p], p, lg)
        if d.rank == 0:
            diff = float(np.abs(lg - ref[j]).max())
            rels.append(diff / float(np.abs(ref[j]).max()))
            if int(np.argmax(lg)) != int(np.argmax(ref[j])):
                top2 = np.sort(ref[j])[-2:]
                if float(top2[1] - top2[0]) <= 2 * diff:
                    ties += 1
                else:
                    disagree += 1
    if d.rank != 0:
        return None
    return {"reference": "the same model on 1 GPU (TP=1), teacher forced on its greedy tokens",
            "positions": [P - 1, P + T - 2], "max_rel_logit_diff": max(rels),
            "median_rel_logit_diff": float(np.median(rels)), "argmax_ties": ties, "argmax_disagreements": disagree,
            "tokens_identical_up_to_ties": disagree == 0}


def long_context(qb, wl: dict, st, e0, e1, hbm: float, steps: int = 64) -> list:
    """decode at the end of the context window, where the KV cache is a large share of the bytes a step
    reads: the prompt (max_seq - steps - 8 random ids) goes in through the batched forward (timed), then
    `steps` greedy steps are timed, once with the fp32 cache (the reference's) and once with the fp16 cache"""
    cfg = dict(wl["cfg"])
    n = cfg["max_seq"] - steps - 8
    prompt = np.random.default_rng(wl["seed"] + 2000).integers(3, cfg["vocab_size"], n).astype(np.int32)
    res = []
    for kv, name in ((0, "f32"), (1, "f16")):
        m = qb.Model(cfg, kv_dtype=kv)
        m.synthesize(wl["dtype"], wl["seed"], STD)
        m.prefill(prompt, 0)  # first call: row buffers, split-row copies
        e0.record(st)
        first = m.prefill(prompt, 0)  # the whole prompt through the batched forward, timed
        e1.record(st)
        qb.check(qb.cuda().qmc_sync())
        pf_s = e0.elapsed_time(e1) / 1e3
        m.enqueue_decode(first, n, 4)
        qb.check(qb.cuda().qmc_sync())
        e0.record(st)
        m.enqueue_decode(-1, 0, steps)
        e1.record(st)
        qb.check(qb.cuda().qmc_sync())
        sec = e0.elapsed_time(e1) / 1e3
        b = float(np.mean([m.step_bytes(p) for p in range(n + 4, n + 4 + steps)]))
        res.append({"kv_cache": name, "prompt_tokens": n, "prefill_ms": pf_s * 1e3, "prefill_tok/s": n / pf_s,
                    "decode_positions": [n + 4, n + 3 + steps], "tok/s": steps / sec,
                    "bytes_per_step": b, "GB/s": b * steps / sec / 1e9, "frac": b * steps / sec / 1e9 / hbm})
        m.close()
    return res


def kernel_sweeps(qb, torch, wl: dict, hbm: float, tflops: float, src: str) -> dict:
    """matvec sweep, the decode GEMV mix (roofline of the dominant kernel), prefill"""
    res = {"matvec": []}
    for dt in (Q4_0, Q8_0):
        for rows, cols in ((4096, 4096), (11008, 4096), (4096, 11008), (32000, 4096), (28672, 8192)):
            sec, algo = time_matvec(qb, torch, dt, rows, cols)
            res["matvec"].append({"shape": f"{rows}x{cols}", "dtype": DTYPE_NAME[dt], "us": sec * 1e6,
                                  "GB/s": algo / sec / 1e9, "frac": algo / sec / 1e9 / hbm})
    c = wl["cfg"]
    D, H, V, L = c["dim"], c["hidden_dim"], c["vocab_size"], c["n_layers"]
    kvd = D // c["n_heads"] * c["n_kv_heads"]
    mix = [(D + 2 * kvd, D, L), (D, D, L), (2 * H, D, L), (D, H, L), (V, D, 1)]
    tot_b = tot_t = 0.0
    for rows, cols, n in mix:
        sec, algo = time_matvec(qb, torch, wl["dtype"], rows, cols)
        tot_b += n * algo
        tot_t += n * sec
    tag = f"{DTYPE_NAME[wl['dtype']]} decode mix"
    traffic = traffic_from_profiles(f"gemv {DTYPE_NAME[wl['dtype']]} 11008x4096")
    res["matvec_roofline"] = {"bound": "hbm", "kernel": f"gemv_q_kernel<{DTYPE_NAME[wl['dtype']].upper()}> ({tag})",
                       "achieved": tot_b / tot_t / 1e9, "peak": hbm, "unit": "GB/s",
                       "frac": tot_b / tot_t / 1e9 / hbm, "traffic": traffic,
                       "traffic_note": "DRAM bytes per 11008x4096 launch from ncu (algorithmic 25.43 MB)",
                       "peak_source": f"{src} (MEASURED_PEAKS.json hbm_gbs)" if src == "measured" else src}
    # Q8_0 prefill contraction: tensor cores (tcgen05 kind::i8, the model's batched forward) against the
    # CUDA-core dp4a kernel; "TOP/s" counts 2 int8 operations per multiply-add
    res["prefill_contraction"] = []
    for N, Kd in ((4096, 4096), (11008, 4096)):
        for T in (1, 8, 32, 128, 512):
            sec, sec_cc = time_prefill(qb, torch, T, N, Kd)
            res["prefill_contraction"].append({"T": T, "N": N, "K": Kd, "kernel": "matmul_q_tc_kernel (tcgen05 kind::i8)",
                                   "tok/s": T / sec, "TOP/s": 2 * T * N * Kd / sec / 1e12, "us": sec * 1e6,
                                   "cuda_core_us": sec_cc * 1e6})
    return res


# ------------------------------------------------------------------ CPU baseline / reference arm
def model_file(wl: dict, name: str) -> str:
    from oracle import oracle as O

    d = os.environ.get("QUILLM_BENCH_DIR", "/tmp/quillm_bench")
    os.makedirs(d, exist_ok=True)
    path = os.path.join(d, f"{name}_seed{wl['seed']}.qlm")
    if not os.path.exists(path + ".ok"):
        O.synth_write(path, wl["cfg"], wl["dtype"], wl["seed"], STD, os.cpu_count())
        open(path + ".ok", "w").close()
    return path


def ref_model(wl: dict, name: str, threads: int):
    """the reference's best ISA on this host (AVX2 vs AVX-512, as its README recommends measuring) at
    the given thread count"""
    from oracle import oracle as O

    path = model_file(wl, name)
    best = None
    for isa in (O.ISA_AVX512, O.ISA_AVX2):
        if not O.ref().ref_isa_supported(isa):
            continue
        m = O.RefModel(path, threads=threads, isa=isa, max_seq=wl["cfg"]["max_seq"])
        m.forward(int(prompt_ids(wl)[0]), 0)
        t0 = time.perf_counter()
        m.forward(int(prompt_ids(wl)[1 % wl["prompt"]]), 1)
        m.forward(int(prompt_ids(wl)[2 % wl["prompt"]]), 2)
        dt = time.perf_counter() - t0
        if best is None or dt < best[0]:
            if best:
                best[2].close()
            best = (dt, isa, m)
        else:
            m.close()
    if best is None:
        m = O.RefModel(path, threads=threads, isa=O.ISA_SCALAR, max_seq=wl["cfg"]["max_seq"])
        return m, O.ISA_SCALAR
    return best[2], best[1]


def cpu_model() -> str:
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown CPU"


def host_ram_bytes() -> int:
    try:
        return os.sysconf("SC_PAGE_SIZE") * os.sysconf("SC_PHYS_PAGES")
    except (ValueError, OSError):
        return 0


def model_file_bytes(wl: dict) -> int:
    c = wl["cfg"]
    D, H, L, V = c["dim"], c["hidden_dim"], c["n_layers"], c["vocab_size"]
    kv = D // c["n_heads"] * c["n_kv_heads"]
    rb = lambda n: row_bytes(wl["dtype"], n)  # noqa: E731
    return L * ((D + 2 * kv) * rb(D) + D * rb(D) + 2 * H * rb(D) + D * rb(H)) + 2 * V * rb(D)


def ref_threads(wl: dict) -> list:
    """thread counts to time: all host cores, and for models of a few tens of MB also one thread, which
    the reference's README finds faster there (its pool's wake-ups dominate, README.md:157-159,194-195)"""
    n = os.cpu_count() or 1
    return [n, 1] if n > 1 and model_file_bytes(wl) < 64 * 2**20 else [n]


def ref_decode(wl: dict, name: str, warmup: int, steps: int, time_cap: float | None = None, threads: int | None = None):
    """the reference's CPU decode as its own loop runs it (src/main.c:127-146): the whole prompt one
    token at a time (untimed), `warmup` greedy steps, then up to `steps` timed greedy steps (fewer when
    time_cap seconds run out).  Returns (steps timed, seconds, ISA name, threads, first timed position)."""
    from oracle import oracle as O

    threads = threads or os.cpu_count() or 1
    m, isa = ref_model(wl, name, threads)
    prompt = prompt_ids(wl)
    if model_file_bytes(wl) > CPU_SHORT_PROMPT_BYTES:  # the CPU feeds ~1 token/s here: a short prompt
        prompt = prompt[:CPU_SHORT_PROMPT]
    lg = None
    for p, t in enumerate(prompt):
        lg = m.forward(int(t), p)
    tok = int(np.argmax(lg))
    pos = len(prompt)
    for _ in range(warmup):
        tok = int(np.argmax(m.forward(tok, pos)))
        pos += 1
    first, n, t0 = pos, 0, time.perf_counter()
    while n < steps and (time_cap is None or n < 3 or time.perf_counter() - t0 < time_cap):
        tok = int(np.argmax(m.forward(tok, pos)))
        pos += 1
        n += 1
    sec = time.perf_counter() - t0
    m.close()
    names = {O.ISA_SCALAR: "scalar", O.ISA_AVX2: "avx2", O.ISA_AVX512: "avx512"}
    return n, sec, names[isa], threads, first


# models above this size (the 70B-shaped one, ~75 GB) take about a second per token on the host cores:
# their CPU legs feed only the first CPU_SHORT_PROMPT prompt tokens before the timed steps (the weights
# dominate each token's time; the shorter context barely changes it)
CPU_SHORT_PROMPT_BYTES, CPU_SHORT_PROMPT = 16 << 30, 8


def ram_refusal(wl: dict) -> str | None:
    need, have = model_file_bytes(wl), host_ram_bytes()
    if have and need > 0.8 * have:
        return f"not run (host RAM): the {need / 1e9:.0f} GB model file does not fit in {have / 1e9:.0f} GB of host memory"
    return None


def cpu_baseline(args, wl: dict) -> dict:
    why = ram_refusal(wl)
    if why:
        return {"value": None, "unit": "tok/s", "cores": os.cpu_count() or 1, "kind": "reference", "sample": why}
    runs = [ref_decode(wl, args.workload, args.warmup, args.steps, time_cap=10.0, threads=t) for t in ref_threads(wl)]
    n, sec, isa, threads, first = max(runs, key=lambda r: r[0] / r[1])
    return {"value": n / sec, "unit": "tok/s", "cores": threads, "kind": "reference", "cpu": cpu_model(),
            "sample": f"reference qm_model_forward ({isa}, {threads} threads on {cpu_model()}), {args.workload}: "
                      f"{first - args.warmup} prompt tokens and {args.warmup} warm-up steps untimed, then {n} greedy "
                      f"decode steps timed at positions {first}-{first + n - 1}"
                      + (" (the reference arm's)" if first - args.warmup == wl["prompt"] else
                         f" (a short prompt: the model takes about a second per token on the host)")}


def reference_arm(args, wl: dict) -> dict | None:
    rank = int(os.environ.get("RANK", 0))
    if rank != 0:
        return None
    why = ram_refusal(wl)
    if why:
        return {"impl": "reference", "unavailable": why}
    runs = [ref_decode(wl, args.workload, args.warmup, args.steps, threads=t) for t in ref_threads(wl)]
    n, sec, isa, threads, first = max(runs, key=lambda r: r[0] / r[1])
    prompt = prompt_ids(wl)
    pos = first + n
    v = args.steps / sec
    c = wl["cfg"]
    return {"metric": METRIC, "impl": "reference", "value": v, "unit": "tok/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": sec / args.steps * 1e3,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "i8xi8->i32, f32",
            "data": f"synthetic: {wl['model']}; random prompt ids (numpy default_rng({wl['seed'] + 1000}))",
            "config": {"workload": f"{args.workload}_decode", "model": wl["model"], "global_batch": 1,
                       "seq_len": c["max_seq"], "prompt_tokens": len(prompt),
                       "decode_positions": [len(prompt) + args.warmup, pos - 1], "parallelism": "cpu"},
            "cpu_baseline": {"value": v, "unit": "tok/s", "cores": threads, "kind": "reference", "cpu": cpu_model(),
                             "sample": f"reference qm_model_forward ({isa}, {threads} threads on {cpu_model()}): "
                                       f"{len(prompt)} prompt tokens untimed, {args.warmup} warm-up and "
                                       f"{args.steps} timed greedy decode steps"},
            "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", choices=["quillm_b200", "reference"], default="quillm_b200")
    ap.add_argument("--workload", choices=list(WORKLOADS), default="llama7b_q4_0")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--quick", action="store_true", help="skip the matvec / prefill sweeps")
    ap.add_argument("--prompt", type=int, default=None, help="override the workload's prompt length")
    ap.add_argument("--profile-matvec", default=None, metavar="ROWSxCOLS:DTYPE[:N]",
                    help="only launch N plain matvecs (a small case for ncu captures)")
    ap.add_argument("--profile-decode", type=int, default=None, metavar="LAYERS",
                    help="only decode 134 positions of the workload's model cut to LAYERS layers (ncu)")
    ap.add_argument("--profile-prefill", default=None, metavar="TxNxK:DTYPE[:N]",
                    help="only launch N tensor-core prefill contractions (a small case for ncu captures)")
    ap.add_argument("--profile-prompt", type=int, default=None, metavar="T",
                    help="only run the 7B Q4_0 model's batched forward of a T-token prompt twice (ncu)")
    args = ap.parse_args()
    if args.profile_prompt:
        profile_prompt(args.profile_prompt)
        return
    if args.profile_prefill:
        profile_prefill(args.profile_prefill)
        return
    if args.profile_matvec:
        profile_matvec(args.profile_matvec)
        return
    if args.profile_decode:
        profile_decode(args.profile_decode, args.workload)
        return
    if args.warmup < 3:
        args.warmup = 3
    wl = dict(WORKLOADS[args.workload])
    if args.prompt is not None:
        wl["prompt"] = max(1, args.prompt)
    out = reference_arm(args, wl) if args.impl == "reference" else gpu_arm(args, wl)
    if out is not None:
        print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
