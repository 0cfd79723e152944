"""Shared test helpers: import paths and deterministic inputs.

Inputs for parity cases come from the reference's own xorshift32 generator
(qwen_one_layer.c:88-96, restated as oc_random_fill in the oracle), so every
case is reproducible from a seed on any machine without storing weights.
"""
from __future__ import annotations

import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "simple-inference_b200")
for p in (ROOT, PKG, os.path.join(ROOT, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)

from oracle import Oracle, Reference, QK, Q8_BYTES  # noqa: E402,F401
from sib200 import synth  # noqa: E402

GOLDEN = os.path.join(ROOT, "tests", "golden")

DIMS_15B = dict(hidden=1536, n_q_heads=12, n_kv_heads=2, head_dim=128, intermediate=8960,
                rope_theta=1e6, rms_eps=1e-6)


def stream(oc: Oracle, seed: int, n: int, scale: float = 1.0, offset: float = 0.0):
    oc.seed(seed)
    return oc.random_floats(n, scale, offset)


def xs_layer(oc: Oracle, dims: dict, seed: int, mlp: bool = False, norms: bool = True,
             biases: bool = True, wscale: float = 0.05) -> dict:
    """A layer whose fp32 weights are one xorshift stream, quantised to Q4_0."""
    H, D = dims["hidden"], dims["head_dim"]
    QD, KVD = dims["n_q_heads"] * D, dims["n_kv_heads"] * D
    oc.seed(seed)

    def mat(rows, cols):
        return synth.q4_0_quantize(oc.random_floats(rows * cols, wscale).reshape(rows, cols))

    L = {"wq": mat(QD, H), "wk": mat(KVD, H), "wv": mat(KVD, H), "wo": mat(H, QD),
         "norm": None, "bq": None, "bk": None, "bv": None,
         "w_gate": None, "w_up": None, "w_down": None, "norm2": None}
    if norms:
        L["norm"] = oc.random_floats(H, 0.02, 1.0)
    if biases:
        L["bq"] = oc.random_floats(QD, 0.02)
        L["bk"] = oc.random_floats(KVD, 0.02)
        L["bv"] = oc.random_floats(KVD, 0.02)
    if mlp:
        I = dims["intermediate"]
        L["w_gate"] = mat(I, H)
        L["w_up"] = mat(I, H)
        L["w_down"] = mat(H, I)
        L["norm2"] = oc.random_floats(H, 0.02, 1.0) if norms else None
    return L


def xs_kv_history(oc: Oracle, seed: int, context: int, kvdim: int, kscale=0.25, vscale=0.25,
                  f32: bool = False, total: int | None = None):
    """History rows [0, context-1) like fill_kv_history (qwen_one_layer.c:228-235);
    rows up to `total` stay zero."""
    total = total or context
    k = stream(oc, seed, (context - 1) * kvdim, kscale)
    v = stream(oc, seed ^ 0x5bd1e995, (context - 1) * kvdim, vscale)
    dt = np.float32 if f32 else np.uint16
    kc = np.zeros(total * kvdim, dt)
    vc = np.zeros(total * kvdim, dt)
    if f32:
        kc[:k.size], vc[:v.size] = k, v
    else:
        kc[:k.size] = k.astype(np.float16).view(np.uint16)
        vc[:v.size] = v.astype(np.float16).view(np.uint16)
    return kc, vc


def assert_layer_close(ref, got, rel=1e-3, what=""):
    """Layer-output bar (1e-3 relative): ||got-ref|| <= rel*||ref|| and every
    element within rel * max|ref|.  Near-zero elements are judged against the
    vector's scale, since a flipped Q8 rounding of one activation moves every
    output by roughly dx*dw regardless of that output's own size."""
    ref = np.asarray(ref, np.float64)
    got = np.asarray(got, np.float64)
    assert np.all(np.isfinite(got)), f"{what}: non-finite output"
    d = got - ref
    n = np.linalg.norm(d) / max(np.linalg.norm(ref), 1e-30)
    m = np.max(np.abs(d)) / max(np.max(np.abs(ref)), 1e-30)
    assert n <= rel and m <= rel, f"{what}: rel-L2 {n:.3g}, max/scale {m:.3g} (bar {rel})"


def assert_close(ref, got, atol, rtol, what=""):
    ref = np.asarray(ref, np.float64)
    got = np.asarray(got, np.float64)
    assert np.all(np.isfinite(got)), f"{what}: non-finite output"
    bad = np.abs(ref - got) > atol + rtol * np.maximum(np.abs(ref), np.abs(got))
    if bad.any():
        i = int(np.argmax(bad))
        raise AssertionError(f"{what}: {int(bad.sum())}/{bad.size} outside tolerance; first "
                             f"at {i}: ref={ref.flat[i]!r} got={got.flat[i]!r}")
