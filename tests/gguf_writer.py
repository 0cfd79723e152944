"""Test infrastructure: write small GGUF v3 files (public GGUF format) with
Qwen2 decoder-layer tensors, deterministically from a seed.

Used by tests/test_gguf.py and tests/golden/make_gguf_golden.py; nothing in
the library imports it.  Layout written: magic "GGUF", u32 version 3, u64
tensor count, u64 metadata count, metadata (key, u32 type, value), tensor
infos (name, u32 rank, u64 dims fastest first, u32 type, u64 offset), zero
padding to `general.alignment`, then each tensor's bytes at its (aligned)
offset.
"""
from __future__ import annotations

import struct

import numpy as np

from sib200 import synth

U32, F32T, STRING, ARRAY = 4, 6, 8, 9
T_F32, T_F16, T_Q4_0, T_Q8_0 = 0, 1, 2, 8


def _string(s: str) -> bytes:
    b = s.encode("utf-8")
    return struct.pack("<Q", len(b)) + b


def _value(typ: int, v) -> bytes:
    if typ == U32:
        return struct.pack("<I", v)
    if typ == F32T:
        return struct.pack("<f", v)
    if typ == STRING:
        return _string(v)
    if typ == ARRAY:
        inner, items = v
        out = struct.pack("<IQ", inner, len(items))
        return out + b"".join(_value(inner, x) for x in items)
    raise ValueError(typ)


def write_gguf(path: str, meta: list, tensors: list, alignment: int = 32) -> None:
    """meta: [(key, type, value)]; tensors: [(name, dims fastest-first, type, bytes)]."""
    head = bytearray(b"GGUF" + struct.pack("<IQQ", 3, len(tensors), len(meta)))
    for key, typ, v in meta:
        head += _string(key) + struct.pack("<I", typ) + _value(typ, v)
    offsets, off = [], 0
    for _, _, _, data in tensors:
        offsets.append(off)
        off = (off + len(data) + alignment - 1) // alignment * alignment
    for (name, dims, typ, _), o in zip(tensors, offsets):
        head += _string(name) + struct.pack("<I", len(dims))
        head += b"".join(struct.pack("<Q", d) for d in dims)
        head += struct.pack("<IQ", typ, o)
    pad = (-len(head)) % alignment
    with open(path, "wb") as f:
        f.write(bytes(head) + b"\0" * pad)
        for (_, _, _, data), o in zip(tensors, offsets):
            f.write(data)
            f.write(b"\0" * ((-len(data)) % alignment))


def qwen2_meta(dims: dict, n_layers: int, alignment: int = 32) -> list:
    H, hq = dims["hidden"], dims["n_q_heads"]
    meta = [
        ("general.architecture", STRING, "qwen2"),
        ("general.name", STRING, "synthetic-qwen2"),
        ("general.alignment", U32, alignment),
        ("qwen2.block_count", U32, n_layers),
        ("qwen2.embedding_length", U32, H),
        ("qwen2.feed_forward_length", U32, dims["intermediate"]),
        ("qwen2.attention.head_count", U32, hq),
        ("qwen2.attention.head_count_kv", U32, dims["n_kv_heads"]),
        ("qwen2.attention.key_length", U32, dims["head_dim"]),
        ("qwen2.attention.value_length", U32, dims["head_dim"]),
        ("qwen2.rope.freq_base", F32T, float(dims["rope_theta"])),
        ("qwen2.attention.layer_norm_rms_epsilon", F32T, float(dims["rms_eps"])),
        # A tokenizer-sized array the reader must skip.
        ("tokenizer.ggml.tokens", ARRAY, (STRING, [f"tok{i}" for i in range(64)])),
        ("tokenizer.ggml.scores", ARRAY, (F32T, [float(i) for i in range(64)])),
    ]
    return meta


def make_qwen2_gguf(path: str, dims: dict, seed: int, n_layers: int = 2,
                    f16_vectors_layer: int | None = 1, drop: tuple = ("blk.1.attn_k.bias",),
                    overrides: dict | None = None, alignment: int = 32) -> list:
    """Write a Qwen2-shaped GGUF; return the per-layer host dicts it encodes.

    Layer `f16_vectors_layer` stores its norms and biases as F16 (the host
    dict then holds their exact float32 widening); tensors named in `drop`
    are left out; `overrides` maps a tensor name to (type, bytes) to plant
    a wrong type.
    """
    layers, tensors = [], []
    for li in range(n_layers):
        L = synth.random_layer(dims, seed + li)
        H, D, I = dims["hidden"], dims["head_dim"], dims["intermediate"]
        QD, KVD = dims["n_q_heads"] * D, dims["n_kv_heads"] * D
        spec = [("wq", "attn_q.weight", [H, QD]), ("wk", "attn_k.weight", [H, KVD]),
                ("wv", "attn_v.weight", [H, KVD]), ("wo", "attn_output.weight", [QD, H]),
                ("bq", "attn_q.bias", [QD]), ("bk", "attn_k.bias", [KVD]),
                ("bv", "attn_v.bias", [KVD]), ("norm", "attn_norm.weight", [H]),
                ("w_gate", "ffn_gate.weight", [H, I]), ("w_up", "ffn_up.weight", [H, I]),
                ("w_down", "ffn_down.weight", [I, H]), ("norm2", "ffn_norm.weight", [H])]
        for key, suffix, gdims in spec:
            name = f"blk.{li}.{suffix}"
            v = L[key]
            if v is None:  # a layer without an MLP
                continue
            if name in drop:
                L[key] = None
                continue
            if key.startswith("w"):
                typ, data = T_Q4_0, np.ascontiguousarray(v, np.uint8).tobytes()
            elif li == f16_vectors_layer:
                h = v.astype(np.float16)
                L[key] = h.astype(np.float32)
                typ, data = T_F16, h.astype("<f2").tobytes()
            else:
                typ, data = T_F32, np.ascontiguousarray(v, "<f4").tobytes()
            if overrides and name in overrides:
                typ, data = overrides[name]
            tensors.append((name, gdims, typ, data))
        layers.append(L)
    write_gguf(path, qwen2_meta(dims, n_layers, alignment), tensors, alignment)
    return layers
