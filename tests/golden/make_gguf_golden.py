#!/usr/bin/env python3
"""Generate tests/golden/gguf_extract_golden.json from the reference's own
GGUF extractor (extract_weights.py in the reference checkout).

Builds a seeded synthetic Qwen2 GGUF at the reference extractor's dimensions
(hidden 1536, 12 Q / 2 KV heads, head_dim 128 -- extract_weights.py checks
them; a small feed-forward width keeps the file small), runs the reference's
extract_weights.py on layers 0 and 1, and records the sha256 of the GGUF and
of every file the extractor writes (the manifest excepted: it names paths).
Layer 1 stores its norms and biases as F16 and lacks attn_k.bias, so the
golden covers the extractor's F16 -> F32 widening and its optional-tensor
path.  tests/test_gguf.py rebuilds the same file and compares the library's
extractor with these hashes.

Usage:  python tests/golden/make_gguf_golden.py [--ref-dir /path/to/reference]
Needs the reference checkout; the committed JSON is what the tests read.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import subprocess
import sys
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
import common  # noqa: E402,F401  (import paths)
from gguf_writer import make_qwen2_gguf  # noqa: E402
from oracle import reference_dir  # noqa: E402

OUT = os.path.join(HERE, "gguf_extract_golden.json")
DIMS = dict(hidden=1536, n_q_heads=12, n_kv_heads=2, head_dim=128, intermediate=256,
            rope_theta=1e6, rms_eps=1e-6)
SEED = 77
LAYERS = (0, 1)


def sha(path: str) -> str:
    with open(path, "rb") as f:
        return hashlib.sha256(f.read()).hexdigest()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref-dir", default=reference_dir(),
                    help="the reference checkout (default: $SI_REFERENCE_DIR, else a "
                         "checkout named reference beside this repository)")
    args = ap.parse_args()
    if not args.ref_dir:
        sys.exit("no reference checkout: pass --ref-dir or set SI_REFERENCE_DIR")
    script = os.path.join(args.ref_dir, "extract_weights.py")
    with tempfile.TemporaryDirectory() as tmp:
        gguf = os.path.join(tmp, "synthetic.gguf")
        make_qwen2_gguf(gguf, DIMS, SEED)
        golden = {"dims": DIMS, "seed": SEED, "gguf_sha256": sha(gguf), "layers": {}}
        for layer in LAYERS:
            out = os.path.join(tmp, f"layer{layer}")
            subprocess.run([sys.executable, script, gguf, "--layer", str(layer), "--out", out],
                           check=True, capture_output=True)
            golden["layers"][str(layer)] = {
                name: sha(os.path.join(out, name))
                for name in sorted(os.listdir(out)) if name != "manifest.json"}
    with open(OUT, "w", encoding="utf-8") as f:
        json.dump(golden, f, indent=2, sort_keys=True)
        f.write("\n")
    print(f"wrote {OUT}")


if __name__ == "__main__":
    main()
