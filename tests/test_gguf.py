"""GGUF loading (the role of the reference's extract_weights.py).

CPU: the library's extractor writes the same files, byte for byte, as the
reference's own extract_weights.py on a seeded synthetic Qwen2 GGUF (hashes
recorded by tests/golden/make_gguf_golden.py from the reference run); the
index, the dimensions and the layer tensors round-trip; malformed files and
non-Q4_0 matrices are rejected.  GPU: a layer built from a GGUF file decodes
bit-identically to the same weights uploaded directly.
"""
from __future__ import annotations

import hashlib
import json
import os

import numpy as np
import pytest

from common import GOLDEN
from gguf_writer import T_Q8_0, make_qwen2_gguf
from sib200 import gguf

with open(os.path.join(GOLDEN, "gguf_extract_golden.json"), encoding="utf-8") as _f:
    GOLD = json.load(_f)
DIMS = GOLD["dims"]
# The file stores rope theta and eps as float32: the values the kernels use.
DIMS_F32 = dict(DIMS, rope_theta=float(np.float32(DIMS["rope_theta"])),
                rms_eps=float(np.float32(DIMS["rms_eps"])))


def _sha(path):
    with open(path, "rb") as f:
        return hashlib.sha256(f.read()).hexdigest()


@pytest.fixture(scope="module")
def synthetic(tmp_path_factory):
    path = str(tmp_path_factory.mktemp("gguf") / "synthetic.gguf")
    layers = make_qwen2_gguf(path, DIMS, GOLD["seed"])
    return path, layers


def test_synthetic_file_matches_the_golden_one(synthetic):
    path, _ = synthetic
    assert _sha(path) == GOLD["gguf_sha256"]


@pytest.mark.parametrize("layer", [0, 1])
def test_extract_matches_reference_extractor(synthetic, tmp_path, layer):
    path, _ = synthetic
    out = str(tmp_path / f"layer{layer}")
    manifest = gguf.extract(path, out, layer)
    got = {n: _sha(os.path.join(out, n)) for n in sorted(os.listdir(out)) if n != "manifest.json"}
    assert got == GOLD["layers"][str(layer)]
    assert set(manifest["tensors"]) == {n.split(".")[0] for n in got}


def test_command_line(synthetic, tmp_path):
    import subprocess
    import sys
    from common import PKG
    path, _ = synthetic
    out = str(tmp_path / "cli")
    env = dict(os.environ, PYTHONPATH=PKG)
    r = subprocess.run([sys.executable, "-m", "sib200.gguf", path, "--layer", "0", "--out", out],
                       capture_output=True, text=True, env=env)
    assert r.returncode == 0, r.stdout + r.stderr
    got = {n: _sha(os.path.join(out, n)) for n in sorted(os.listdir(out)) if n != "manifest.json"}
    assert got == GOLD["layers"]["0"]
    r = subprocess.run([sys.executable, "-m", "sib200.gguf", path, "--list"],
                       capture_output=True, text=True, env=env)
    assert r.returncode == 0 and "blk.0.attn_q.weight" in r.stdout and "Q4_0" in r.stdout
    r = subprocess.run([sys.executable, "-m", "sib200.gguf", path + ".missing"],
                       capture_output=True, text=True, env=env)
    assert r.returncode == 1


def test_extract_removes_a_stale_optional_file(synthetic, tmp_path):
    path, _ = synthetic
    out = str(tmp_path / "x")
    os.makedirs(out)
    with open(os.path.join(out, "k_bias.f32"), "wb") as f:
        f.write(b"stale")
    gguf.extract(path, out, 1)  # layer 1 has no attn_k.bias
    assert not os.path.exists(os.path.join(out, "k_bias.f32"))


def test_index_and_dims(synthetic):
    path, _ = synthetic
    idx = gguf.read_index(path)
    assert idx.version == 3 and idx.alignment == 32 and idx.data_start % 32 == 0
    assert idx.meta["tokenizer.ggml.tokens"] == 64  # arrays are skipped, counted
    d = gguf.qwen2_dims(idx)
    assert d.pop("n_layers") == 2
    assert d == DIMS_F32
    t = idx.tensors["blk.0.attn_k.weight"]
    assert t.dims == [1536, 256] and t.type == gguf.Q4_0 and t.nbytes == 256 * 48 * 18


def test_layer_host_round_trip(synthetic):
    path, layers = synthetic
    for li, want in enumerate(layers):
        d, host = gguf.layer_host(path, li)
        assert d == DIMS_F32
        for key, v in want.items():
            if v is None:
                assert host[key] is None, key
            else:
                np.testing.assert_array_equal(host[key], v, err_msg=key)
    d, host = gguf.layer_host(path, 0, mlp=False)
    assert d["intermediate"] == 0 and host["w_gate"] is None and host["norm2"] is None


def test_rejects_bad_files(synthetic, tmp_path):
    path, _ = synthetic
    raw = open(path, "rb").read()
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"GGUX" + raw[4:])
    with pytest.raises(gguf.GGUFError, match="magic"):
        gguf.read_index(str(bad))
    bad.write_bytes(raw[: len(raw) // 2])
    with pytest.raises(gguf.GGUFError, match="beyond the end|truncated"):
        gguf.read_index(str(bad))
    bad.write_bytes(raw[:100])
    with pytest.raises(gguf.GGUFError, match="truncated"):
        gguf.read_index(str(bad))
    with pytest.raises(gguf.GGUFError, match="dims"):
        gguf.layer_host(path, 0, dims=dict(DIMS, hidden=1024))
    with pytest.raises(gguf.GGUFError, match="not found"):
        gguf.layer_host(path, 5)


def test_rejects_a_non_q4_0_matrix(tmp_path):
    path = str(tmp_path / "q8.gguf")
    dims = dict(DIMS, intermediate=0)
    name = "blk.0.attn_q.weight"
    q8 = bytes(1536 * 48 * 34)  # a Q8_0 tensor of the same shape
    make_qwen2_gguf(path, dims, 5, n_layers=1, overrides={name: (T_Q8_0, q8)})
    with pytest.raises(gguf.GGUFError, match="not Q4_0"):
        gguf.layer_host(path, 0)
    with pytest.raises(gguf.GGUFError, match="not Q4_0"):
        gguf.extract(path, str(tmp_path / "out"), 0)


@pytest.mark.gpu
def test_gguf_layer_decodes_like_the_direct_upload(tmp_path):
    """Config-0 dims: a layer read from a GGUF file and the same host tensors
    uploaded directly give bit-identical decode outputs over four steps."""
    import torch
    import sib200
    dims = dict(hidden=896, n_q_heads=14, n_kv_heads=2, head_dim=64, intermediate=4864,
                rope_theta=1e6, rms_eps=1e-6)
    path = str(tmp_path / "c0.gguf")
    layers = make_qwen2_gguf(path, dims, 3, n_layers=1, f16_vectors_layer=None, drop=())
    ctx = sib200.Context(0, 256, 1e6, 64)
    try:
        la, lb = ctx.layer_gguf(path, 0), ctx.layer(dims, layers[0])
        kva, kvb = ctx.kv(dims, 1, 64, True), ctx.kv(dims, 1, 64, True)
        g = torch.Generator("cuda").manual_seed(4)
        X = torch.randn(4, dims["hidden"], device="cuda", generator=g)
        ya, yb = torch.zeros_like(X), torch.zeros_like(X)
        torch.cuda.synchronize()
        for t in range(4):
            la.decode_dev(kva, X[t], [t + 1], ya[t], sib200.SI_LAYER_FULL)
            lb.decode_dev(kvb, X[t], [t + 1], yb[t], sib200.SI_LAYER_FULL)
        ctx.status()
        assert torch.isfinite(ya).all()
        assert torch.equal(ya, yb)
        for o in (kva, kvb, la, lb):
            o.free()
    finally:
        ctx.close()
