"""float64 numpy forward pass on dequantized weights -- TEST INFRASTRUCTURE ONLY.

Restates the reference's numpy oracle (tools/qlm.py: dequantize :70-80, read_qlm :135-182,
_rmsnorm/_rope :264-276, forward_ref :279-310) so GPU model tests can use the reference's own float64
truth and tolerances (tests/test_model.c:50-53) on models the reference's fixture set does not contain.
Loads a .qlm written by any writer (the golden fixtures, the oracle's synthesiser).
"""
from __future__ import annotations

import struct

import numpy as np

Q8_DT = np.dtype([("d", "<u2"), ("qs", "i1", 32)])
Q4_DT = np.dtype([("d", "<u2"), ("qs", "u1", 16)])


def dequantize(blocks: np.ndarray, n: int) -> np.ndarray:
    d = blocks["d"].view(np.float16).astype(np.float32)
    if blocks.dtype == Q8_DT:
        q = blocks["qs"].astype(np.float32)
    else:
        qs = blocks["qs"]
        q = np.empty(qs.shape[:-1] + (32,), np.float32)
        q[..., 0::2] = (qs & 0xF).astype(np.float32) - 8
        q[..., 1::2] = (qs >> 4).astype(np.float32) - 8
    return (d[..., None] * q).reshape(blocks.shape[0], -1)[:, :n]


def load(path: str):
    """(config dict, {name: float32 array}) from a .qlm file"""
    buf = open(path, "rb").read()
    assert buf[:4] == b"QLMF"
    _, n_kv, n_t, data_off = struct.unpack_from("<IIIQ", buf, 4)
    p = 24

    def take_str():
        nonlocal p
        (n,) = struct.unpack_from("<I", buf, p)
        p += 4 + n
        return buf[p - n:p]

    kv = {}
    for _ in range(n_kv):
        k = take_str().decode()
        (ty,) = struct.unpack_from("<I", buf, p)
        p += 4
        if ty in (0, 1):
            (kv[k],) = struct.unpack_from("<I" if ty == 0 else "<f", buf, p)
            p += 4
        elif ty == 2:
            kv[k] = take_str()
        else:
            (n,) = struct.unpack_from("<I", buf, p)
            p += 4 + 4 * n
    W = {}
    for _ in range(n_t):
        name = take_str().decode()
        dt, nd = struct.unpack_from("<II", buf, p)
        p += 8
        shape = struct.unpack_from(f"<{nd}Q", buf, p)
        p += 8 * nd
        (off,) = struct.unpack_from("<Q", buf, p)
        p += 8
        rows = int(np.prod(shape[:-1])) if nd > 1 else 1
        nb = (shape[-1] + 31) // 32
        o = data_off + off
        if dt == 0:
            W[name] = np.frombuffer(buf, np.float32, rows * shape[-1], o).reshape(shape).copy()
        else:
            bdt = Q8_DT if dt == 2 else Q4_DT
            W[name] = dequantize(np.frombuffer(buf, bdt, rows * nb, o).reshape(rows, nb), shape[-1])
    cfg = {k.split(".")[1]: v for k, v in kv.items() if k.startswith("llama.")}
    cfg.setdefault("rope_theta", 10000.0)
    cfg.setdefault("norm_eps", 1e-5)
    return cfg, W


def _rmsnorm(x, w, eps):
    return x / np.sqrt(np.mean(x * x) + eps) * w


def _rope(v, n_heads, hd, pos, theta):
    v = v.reshape(n_heads, hd).copy()
    i = np.arange(hd // 2)
    ang = pos * theta ** (-2.0 * i / hd)
    c, s = np.cos(ang), np.sin(ang)
    a, b = v[:, 0::2].copy(), v[:, 1::2].copy()
    v[:, 0::2] = a * c - b * s
    v[:, 1::2] = a * s + b * c
    return v.reshape(-1)


def forward(cfg: dict, W: dict, tokens) -> np.ndarray:
    """logits [len(tokens), vocab] in float64, whole sequence from position 0"""
    W = {k: np.asarray(v, np.float64) for k, v in W.items()}
    D, L = cfg["dim"], cfg["n_layers"]
    hd = D // cfg["n_heads"]
    grp = cfg["n_heads"] // cfg["n_kv_heads"]
    theta, eps = float(cfg["rope_theta"]), float(cfg["norm_eps"])
    kc, vc, out = [[] for _ in range(L)], [[] for _ in range(L)], []
    for pos, tok in enumerate(tokens):
        x = W["tok_embd"][tok].copy()
        for l in range(L):
            p = f"layers.{l}."
            xb = _rmsnorm(x, W[p + "attn_norm"], eps)
            q = _rope(W[p + "wq"] @ xb, cfg["n_heads"], hd, pos, theta)
            kc[l].append(_rope(W[p + "wk"] @ xb, cfg["n_kv_heads"], hd, pos, theta))
            vc[l].append(W[p + "wv"] @ xb)
            K, V = np.stack(kc[l]), np.stack(vc[l])
            att = np.zeros(D)
            for h in range(cfg["n_heads"]):
                g = h // grp
                sc = K[:, g * hd:(g + 1) * hd] @ q[h * hd:(h + 1) * hd] / np.sqrt(hd)
                sc = np.exp(sc - sc.max())
                sc /= sc.sum()
                att[h * hd:(h + 1) * hd] = sc @ V[:, g * hd:(g + 1) * hd]
            x = x + W[p + "wo"] @ att
            xb = _rmsnorm(x, W[p + "ffn_norm"], eps)
            g1 = W[p + "w1"] @ xb
            x = x + W[p + "w2"] @ (g1 / (1 + np.exp(-g1)) * (W[p + "w3"] @ xb))
        out.append(W["output"] @ _rmsnorm(x, W["norm"], eps))
    return np.stack(out)
