#!/usr/bin/env python3
"""Generate tests/golden/reference_golden.npz from the reference implementation itself.

Runs the reference's own portable C kernels (qwen_one_layer.c and the headers it
includes, compiled in place from the reference checkout by oracle/Makefile into
oracle/_ref/libsiref.so) and the reference's repack_weights.py on deterministic
inputs, and stores their outputs.  Inputs come from the reference's xorshift32
stream (qwen_one_layer.c:88-96) so only small inputs are stored; large ones are
regenerated from seeds by tests/common.py.

Usage:  python tests/golden/make_golden.py [--ref-dir /path/to/reference]
Needs the reference checkout; the committed .npz is what the tests read.
"""
from __future__ import annotations

import argparse
import hashlib
import os
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
from common import (DIMS_15B, Oracle, Reference, stream, xs_kv_history, xs_layer)  # noqa: E402
from oracle import reference_dir  # noqa: E402

OUT = os.path.join(HERE, "reference_golden.npz")
LAYER_SEED = 0x1234
RUN_CASES = [  # (context, kv history scale, x pattern) -- audit_fusion_timing.c:143-162
    (1, 0.25, "random"), (2, 0.0125, "alternating"), (17, 1.0, "random"),
    (64, 0.0, "spikes"), (200, 0.5, "random"),
]


def q8_inputs(oc: Oracle) -> np.ndarray:
    rows = [stream(oc, 11, 1536),                                  # uniform [-1, 1)
            stream(oc, 12, 1536) * 3.0,
            np.zeros(1536, np.float32),                            # d = 0 -> inv = 0
            stream(oc, 13, 1536, 1e-6),                            # fp16-subnormal d
            stream(oc, 14, 1536, 3e4),                             # large d
            ]
    ties = stream(oc, 15, 1536)
    # x = (k + 0.5) * d exactly for an exactly representable d: exercises lrintf's
    # round-half-even on the Q8 grid.
    blk = ties.reshape(48, 32)
    blk[:, 0] = 127.0 / 64.0
    blk[:, 1:] = (np.round(blk[:, 1:] * 100) + 0.5) / 64.0
    rows.append(blk.reshape(-1))
    spikes = stream(oc, 16, 1536, 0.1)
    spikes[::13] = 0.8
    rows.append(spikes)
    return np.stack(rows).astype(np.float32)


def x_pattern(oc: Oracle, kind: str, seed: int) -> np.ndarray:
    r = stream(oc, seed, 1536)
    if kind == "alternating":
        i = np.arange(1536)
        return np.where(i & 1, -0.125 - np.abs(r), 0.125 + np.abs(r)).astype(np.float32)
    if kind == "spikes":
        i = np.arange(1536)
        return np.where(i % 13 == 0, 0.8, r * 0.1).astype(np.float32)
    return r


def run_repack(ref_dir: str, layer: dict) -> dict:
    """Run the reference's repack_weights.py on the layer; return the tile files."""
    with tempfile.TemporaryDirectory() as d:
        for k, name in (("wq", "q"), ("wk", "k"), ("wv", "v"), ("wo", "o")):
            layer[k].tofile(os.path.join(d, f"{name}.q4_0"))
        subprocess.run([sys.executable, os.path.join(ref_dir, "repack_weights.py"), "--weights", d],
                       check=True, capture_output=True)
        return {n: np.fromfile(os.path.join(d, f"{n}.colsoa"), np.uint8) for n in ("q", "kv", "o")}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref-dir", default=reference_dir(),
                    help="the reference checkout (default: $SI_REFERENCE_DIR, else a "
                         "checkout named reference beside this repository)")
    args = ap.parse_args()
    if not args.ref_dir:
        sys.exit("no reference checkout: pass --ref-dir or set SI_REFERENCE_DIR")
    ref, oc = Reference(), Oracle()
    g: dict[str, np.ndarray] = {}

    # f16 conversions: all 65536 halves and a spread of float bit patterns.
    halves = np.arange(65536, dtype=np.uint32)
    f32 = np.array([ref.lib.ref_f16_to_f32(int(h)) for h in halves], np.float32)
    g["f16_to_f32_sha256"] = np.frombuffer(hashlib.sha256(f32.view(np.uint32).tobytes())
                                           .digest(), np.uint8)
    bits = np.concatenate([np.arange(0, 1 << 32, 524309, dtype=np.uint64).astype(np.uint32),
                           np.array([0x7f800000, 0xff800000, 0x7fc00000, 0x38000000, 0x33000000,
                                     0x477fe000, 0x477ff000, 0x387fc000], np.uint32)])
    g["f32_bits"] = bits
    g["f32_to_f16"] = np.array([ref.lib.ref_f32_to_f16(float(v)) for v in bits.view(np.float32)],
                               np.uint16)

    # Q8_0 quantiser.
    qx = q8_inputs(oc)
    g["q8_x"] = qx
    g["q8_out"] = np.stack([ref.quantize_q8(r) for r in qx])

    # Q4_0 x Q8_0 GEMV, 256 rows of a 1536-input matrix, with and without bias.
    layer = xs_layer(oc, DIMS_15B, LAYER_SEED)
    xin = stream(oc, 21, 1536)
    q8 = ref.quantize_q8(xin)
    w = layer["wq"][:256]
    g["mv_out_bias"] = ref.matvec(w, q8, 1536, 256, layer["bq"][:256])
    g["mv_out"] = ref.matvec(w, q8, 1536, 256, None)
    g["mv_isum"] = np.array([[ref.lib.ref_dot_32_q4q8(np.ascontiguousarray(w[r, b * 18:(b + 1) * 18]),
                                                      q8[b * 34 + 2:(b + 1) * 34].view(np.int8).copy())
                              for b in range(48)] for r in range(256)], np.int32)

    # RMSNorm with and without the gamma vector.
    rx = stream(oc, 31, 1536, 2.0)
    g["rms_out"] = ref.rmsnorm(rx, layer["norm"])
    g["rms_out_noweight"] = ref.rmsnorm(rx, None)

    # RoPE at several positions.
    g["rope_pos"] = np.array([0, 1, 2, 63, 1000, 4095, 32767], np.int32)
    heads = stream(oc, 41, 12 * 128)
    g["rope_out"] = np.stack([ref.rope(heads, 12, int(p)) for p in g["rope_pos"]])

    # Attention (verify_fused_projections.c:121-139 style, seed 0x91be2145).
    qa = stream(oc, 0x91BE2145, 1536, 1.5)
    kc = (stream(oc, 0x91BE2146, 64 * 256, 1.5)).astype(np.float16).view(np.uint16)
    vc = (stream(oc, 0x91BE2147, 64 * 256, 1.5)).astype(np.float16).view(np.uint16)
    g["attn_ctx"] = np.array([1, 2, 17, 64], np.int32)
    g["attn_flash"] = np.stack([ref.attention(qa, kc, vc, int(c), 1) for c in g["attn_ctx"]])
    g["attn_standard"] = np.stack([ref.attention(qa, kc, vc, int(c), 0) for c in g["attn_ctx"]])

    # Staged decode run_layer over the audit's adversarial cases.
    for i, (ctx, kscale, kind) in enumerate(RUN_CASES):
        x = x_pattern(oc, kind, 100 + i)
        k0, v0 = xs_kv_history(oc, 200 + i, ctx, 256, kscale=kscale)
        for method in (1, 0):
            kcm, vcm = k0.copy(), v0.copy()
            y, att, q8o = ref.run_layer(layer, x, kcm, vcm, ctx, method)
            tag = f"run{i}_{'flash' if method else 'standard'}"
            g[tag + "_y"], g[tag + "_attn"], g[tag + "_q8"] = y, att, q8o
            g[tag + "_knew"] = kcm[(ctx - 1) * 256:ctx * 256].copy()
            g[tag + "_vnew"] = vcm[(ctx - 1) * 256:ctx * 256].copy()

    # Column-SoA repack (repack_weights.py) and the fused paths that read it.
    tiles = run_repack(args.ref_dir, layer)
    for n, t in tiles.items():
        g[f"colsoa_{n}_sha256"] = np.frombuffer(hashlib.sha256(t.tobytes()).digest(), np.uint8)
    g["fcm_q_tile0"] = ref.fused_column_matvec(tiles["q"][:245760], q8, 48, layer["bq"][:128],
                                               layer["bq"][128:256])
    for i, (ctx, kscale, kind) in enumerate(RUN_CASES[:4]):
        x = x_pattern(oc, kind, 100 + i)
        kcm, vcm = xs_kv_history(oc, 200 + i, ctx, 256, kscale=kscale)
        y, att, q8o = ref.run_layer_fused(layer, tiles, x, kcm, vcm, ctx)
        g[f"fused{i}_y"], g[f"fused{i}_attn"], g[f"fused{i}_q8"] = y, att, q8o

    np.savez_compressed(OUT, **g)
    print(f"wrote {OUT} ({os.path.getsize(OUT)} bytes, {len(g)} arrays)")


if __name__ == "__main__":
    main()
