"""Seeded synthetic inputs with the shapes and distributions of the benchmark configs.

The reference has no checked-in weights (its .gitignore drops weights/), and no
GGUF file is available here, so every run uses synthetic data:

* weights: fp32 ~ N(0, 0.02), quantised to GGUF Q4_0 along K in blocks of 32 with
  the GGUF rule d = (signed value of max|x|) / -8 stored fp16,
  q = min(15, (int)(x * (1/d) + 8.5)), two nibbles per byte (low = element j,
  high = element j+16);
* q/k/v biases ~ N(0, 0.02); RMSNorm gammas 1 + N(0, 0.02);
* activations x ~ N(0, 1).
"""
from __future__ import annotations

import numpy as np

QK, Q4_BYTES, Q8_BYTES = 32, 18, 34

# Model shapes of the benchmark configurations (Qwen2.5 0.5B / 1.5B / 7B / 72B).
CONFIGS = {
    0: dict(hidden=896, n_q_heads=14, n_kv_heads=2, head_dim=64, intermediate=4864),
    1: dict(hidden=1536, n_q_heads=12, n_kv_heads=2, head_dim=128, intermediate=8960),
    2: dict(hidden=3584, n_q_heads=28, n_kv_heads=4, head_dim=128, intermediate=18944),
    3: dict(hidden=3584, n_q_heads=28, n_kv_heads=4, head_dim=128, intermediate=18944),
    4: dict(hidden=8192, n_q_heads=64, n_kv_heads=8, head_dim=128, intermediate=29568),
}
for _c in CONFIGS.values():
    _c.setdefault("rope_theta", 1e6)
    _c.setdefault("rms_eps", 1e-6)


def q4_0_quantize(w: np.ndarray) -> np.ndarray:
    """fp32 [rows, K] -> GGUF Q4_0 bytes [rows, K/32*18] (float32 arithmetic)."""
    w = np.ascontiguousarray(w, np.float32)
    rows, k = w.shape
    nb = k // QK
    x = w.reshape(rows, nb, QK)
    idx = np.argmax(np.abs(x), axis=2)
    smax = np.take_along_axis(x, idx[..., None], axis=2)[..., 0]
    d = (smax / np.float32(-8.0)).astype(np.float32)
    with np.errstate(divide="ignore"):
        inv = np.where(d != 0, np.float32(1.0) / np.where(d != 0, d, np.float32(1.0)),
                       np.float32(0.0)).astype(np.float32)
    q = (x * inv[..., None]).astype(np.float32) + np.float32(8.5)
    qi = np.minimum(q.astype(np.int32), 15).astype(np.uint8)
    out = np.empty((rows, nb, Q4_BYTES), np.uint8)
    out[..., :2] = d.astype(np.float16).view(np.uint8).reshape(rows, nb, 2)
    out[..., 2:] = qi[..., :16] | (qi[..., 16:] << 4)
    return out.reshape(rows, nb * Q4_BYTES)


def q4_0_dequantize(q: np.ndarray, k: int) -> np.ndarray:
    rows = q.shape[0]
    b = q.reshape(rows, k // QK, Q4_BYTES)
    d = b[..., :2].copy().view(np.float16).astype(np.float32)[..., 0]
    lo = (b[..., 2:] & 15).astype(np.float32) - 8
    hi = (b[..., 2:] >> 4).astype(np.float32) - 8
    return (np.concatenate([lo, hi], axis=2) * d[..., None]).reshape(rows, k)


def random_q4(rng: np.random.Generator, rows: int, k: int, std: float = 0.02) -> np.ndarray:
    return q4_0_quantize(rng.normal(0.0, std, size=(rows, k)).astype(np.float32))


def random_layer(dims: dict, seed: int, mlp: bool = True, norms: bool = True,
                 biases: bool = True) -> dict:
    """Host layer dict with GGUF Q4_0 matrices and fp32 vectors."""
    rng = np.random.default_rng(seed)
    H, D = dims["hidden"], dims["head_dim"]
    QD, KVD = dims["n_q_heads"] * D, dims["n_kv_heads"] * D
    L = {
        "wq": random_q4(rng, QD, H), "wk": random_q4(rng, KVD, H),
        "wv": random_q4(rng, KVD, H), "wo": random_q4(rng, H, QD),
        "norm": None, "bq": None, "bk": None, "bv": None,
        "w_gate": None, "w_up": None, "w_down": None, "norm2": None,
    }
    if norms:
        L["norm"] = (1.0 + rng.normal(0.0, 0.02, H)).astype(np.float32)
    if biases:
        L["bq"] = rng.normal(0.0, 0.02, QD).astype(np.float32)
        L["bk"] = rng.normal(0.0, 0.02, KVD).astype(np.float32)
        L["bv"] = rng.normal(0.0, 0.02, KVD).astype(np.float32)
    if mlp and dims.get("intermediate", 0):
        I = dims["intermediate"]
        L["w_gate"] = random_q4(rng, I, H)
        L["w_up"] = random_q4(rng, I, H)
        L["w_down"] = random_q4(rng, H, I)
        L["norm2"] = (1.0 + rng.normal(0.0, 0.02, H)).astype(np.float32) if norms else None
    return L


def q8_split(blocks: np.ndarray, k: int):
    """Reference block_q8_0 bytes [M, K/32*34] -> (qs int8 [M, K], d fp16-bits [M, K/32])."""
    b = np.ascontiguousarray(blocks).reshape(-1, k // QK, Q8_BYTES)
    d = b[..., :2].copy().view(np.uint16)[..., 0]
    qs = b[..., 2:].copy().view(np.int8).reshape(b.shape[0], k)
    return qs, d
