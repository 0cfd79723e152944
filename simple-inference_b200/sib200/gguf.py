"""GGUF (v2/v3) reader for Qwen2 decoder layers.

The reference gets real weights into its layer through extract_weights.py
(extract_weights.py:77-203): it indexes a single-file GGUF, checks the Qwen2
attention tensors' shapes and types (Q4_0 matrices, F32/F16 vectors) and
copies their bytes unchanged into the files `load_layer` reads
(qwen_one_layer.c:210-221).  This module does the same job for this library:

* `read_index`   -- header, metadata and tensor table of a GGUF file;
* `qwen2_dims`   -- the layer dimensions from the metadata;
* `layer_host`   -- one layer's tensors as the host dict `Context.layer`
                    uploads (GGUF Q4_0 rows as-is; the GPU repacks them);
* `extract`      -- the reference extractor's output files (q/k/v/o `.q4_0`,
                    norm and bias `.f32`), byte for byte.

Q4_0 bytes are never dequantised or re-quantised: a tensor of another type
where a Q4_0 matrix is required is an error, as in the reference.  The file
format follows the public GGUF specification (little-endian): magic "GGUF",
u32 version, u64 tensor count, u64 metadata count, the metadata key/value
pairs, the tensor infos (name, rank, dims with the fastest first, type,
offset), then the tensor data from the next multiple of `general.alignment`.
"""
from __future__ import annotations

import json
import math
import os
import struct
from dataclasses import dataclass, field

import numpy as np

# Metadata value types of the GGUF specification.
_SCALAR = {0: "B", 1: "b", 2: "H", 3: "h", 4: "I", 5: "i", 6: "f", 7: "?",
           10: "Q", 11: "q", 12: "d"}
_STRING, _ARRAY = 8, 9
# Tensor types this loader reads.
F32, F16, Q4_0, Q8_0 = 0, 1, 2, 8
TYPE_NAMES = {0: "F32", 1: "F16", 2: "Q4_0", 3: "Q4_1", 6: "Q5_0", 7: "Q5_1", 8: "Q8_0",
              10: "Q2_K", 11: "Q3_K", 12: "Q4_K", 13: "Q5_K", 14: "Q6_K"}
_MAX_STRING = 1 << 30
_MAX_ARRAY = 1 << 31


class GGUFError(ValueError):
    """A malformed, truncated or unsupported GGUF file."""


@dataclass
class TensorInfo:
    name: str
    dims: list          # fastest-varying first (GGUF order): [K, N] for an N x K matrix
    type: int
    offset: int         # from the start of the data section

    @property
    def nbytes(self) -> int:
        return tensor_nbytes(self.dims, self.type)


@dataclass
class GGUFIndex:
    path: str
    version: int
    meta: dict = field(default_factory=dict)      # scalars and strings; arrays as their length
    tensors: dict = field(default_factory=dict)   # name -> TensorInfo
    alignment: int = 32
    data_start: int = 0


def tensor_nbytes(dims, typ) -> int:
    n = math.prod(dims)
    if typ == Q4_0:
        if n % 32:
            raise GGUFError(f"Q4_0 element count {n} is not a multiple of 32")
        return n // 32 * 18
    if typ == Q8_0:
        if n % 32:
            raise GGUFError(f"Q8_0 element count {n} is not a multiple of 32")
        return n // 32 * 34
    if typ == F32:
        return 4 * n
    if typ == F16:
        return 2 * n
    raise GGUFError(f"unsupported tensor type {TYPE_NAMES.get(typ, typ)}")


class _Reader:
    def __init__(self, f):
        self.f = f

    def take(self, n: int) -> bytes:
        b = self.f.read(n)
        if len(b) != n:
            raise GGUFError("truncated GGUF file")
        return b

    def num(self, fmt: str):
        return struct.unpack("<" + fmt, self.take(struct.calcsize(fmt)))[0]

    def string(self) -> str:
        n = self.num("Q")
        if n > _MAX_STRING:
            raise GGUFError("GGUF string longer than 1 GiB")
        return self.take(n).decode("utf-8")

    def value(self, typ: int, depth: int = 0):
        if typ in _SCALAR:
            return self.num(_SCALAR[typ])
        if typ == _STRING:
            return self.string()
        if typ == _ARRAY:
            if depth > 4:
                raise GGUFError("GGUF metadata arrays nested too deep")
            inner, count = self.num("I"), self.num("Q")
            if count > _MAX_ARRAY:
                raise GGUFError("GGUF metadata array too long")
            if inner in _SCALAR:  # e.g. token scores: skip without decoding
                self.f.seek(count * struct.calcsize(_SCALAR[inner]), os.SEEK_CUR)
            else:
                for _ in range(count):
                    self.value(inner, depth + 1)
            return count
        raise GGUFError(f"unsupported GGUF metadata type {typ}")


def read_index(path: str) -> GGUFIndex:
    """Header, metadata and tensor table of a GGUF v2/v3 file."""
    with open(path, "rb") as f:
        r = _Reader(f)
        if r.take(4) != b"GGUF":
            raise GGUFError("not a little-endian GGUF file (magic)")
        version = r.num("I")
        if version not in (2, 3):
            raise GGUFError(f"GGUF version {version} (2 and 3 are supported)")
        ntensors, nmeta = r.num("Q"), r.num("Q")
        idx = GGUFIndex(path=path, version=version)
        for _ in range(nmeta):
            key = r.string()
            idx.meta[key] = r.value(r.num("I"))
        for _ in range(ntensors):
            name = r.string()
            rank = r.num("I")
            if not 1 <= rank <= 4:
                raise GGUFError(f"tensor {name}: rank {rank}")
            dims = [r.num("Q") for _ in range(rank)]
            t = TensorInfo(name, dims, r.num("I"), r.num("Q"))
            if name in idx.tensors:
                raise GGUFError(f"duplicate tensor {name}")
            idx.tensors[name] = t
        align = int(idx.meta.get("general.alignment", 32))
        if align < 8 or align % 8:
            raise GGUFError(f"general.alignment {align}")
        idx.alignment = align
        idx.data_start = (f.tell() + align - 1) // align * align
        size = os.fstat(f.fileno()).st_size
    for t in idx.tensors.values():
        if t.type in (F32, F16, Q4_0, Q8_0) and idx.data_start + t.offset + t.nbytes > size:
            raise GGUFError(f"tensor {t.name}: data beyond the end of the file")
    return idx


def tensor_bytes(idx: GGUFIndex, name: str) -> bytes:
    t = idx.tensors[name]
    with open(idx.path, "rb") as f:
        f.seek(idx.data_start + t.offset)
        return _Reader(f).take(t.nbytes)


def qwen2_dims(idx: GGUFIndex) -> dict:
    """Layer dimensions (the keys `Context.layer` takes) from Qwen2 metadata."""
    m = idx.meta
    arch = m.get("general.architecture", "qwen2")
    if arch != "qwen2":
        raise GGUFError(f"architecture {arch!r}, expected 'qwen2'")

    def need(key):
        if key not in m:
            raise GGUFError(f"metadata {key} missing")
        return m[key]
    hidden, hq = int(need("qwen2.embedding_length")), int(need("qwen2.attention.head_count"))
    hkv = int(m.get("qwen2.attention.head_count_kv", hq))
    head_dim = int(m.get("qwen2.attention.key_length", hidden // hq))
    return dict(hidden=hidden, n_q_heads=hq, n_kv_heads=hkv, head_dim=head_dim,
                intermediate=int(m.get("qwen2.feed_forward_length", 0)),
                rope_theta=float(m.get("qwen2.rope.freq_base", 1e6)),
                rms_eps=float(m.get("qwen2.attention.layer_norm_rms_epsilon", 1e-6)),
                n_layers=int(m.get("qwen2.block_count", 0)))


# Layer tensors: host-dict key -> (GGUF name suffix, is a matrix, dims(d) in GGUF order).
def _layer_tensors(d: dict) -> dict:
    H, D, I = d["hidden"], d["head_dim"], d["intermediate"]
    QD, KVD = d["n_q_heads"] * D, d["n_kv_heads"] * D
    return {
        "wq": ("attn_q.weight", True, [H, QD]), "wk": ("attn_k.weight", True, [H, KVD]),
        "wv": ("attn_v.weight", True, [H, KVD]), "wo": ("attn_output.weight", True, [QD, H]),
        "bq": ("attn_q.bias", False, [QD]), "bk": ("attn_k.bias", False, [KVD]),
        "bv": ("attn_v.bias", False, [KVD]), "norm": ("attn_norm.weight", False, [H]),
        "w_gate": ("ffn_gate.weight", True, [H, I]), "w_up": ("ffn_up.weight", True, [H, I]),
        "w_down": ("ffn_down.weight", True, [I, H]), "norm2": ("ffn_norm.weight", False, [H]),
    }


def _check(idx: GGUFIndex, name: str, matrix: bool, dims: list) -> TensorInfo:
    t = idx.tensors[name]
    if t.dims != dims:
        raise GGUFError(f"{name}: dims {t.dims}, expected {dims} (GGUF order)")
    if matrix and t.type != Q4_0:
        raise GGUFError(f"{name} is {TYPE_NAMES.get(t.type, t.type)}, not Q4_0 "
                        "(weights are never dequantised or re-quantised)")
    if not matrix and t.type not in (F32, F16):
        raise GGUFError(f"{name} must be F32 or F16, is {TYPE_NAMES.get(t.type, t.type)}")
    return t


def _vector(idx: GGUFIndex, t: TensorInfo) -> np.ndarray:
    raw = tensor_bytes(idx, t.name)
    if t.type == F32:
        return np.frombuffer(raw, "<f4").astype(np.float32)
    return np.frombuffer(raw, "<f2").astype(np.float32)  # exact widening


def layer_host(path: str, layer: int, dims: dict | None = None, mlp: bool = True) -> tuple:
    """(dims, host dict) of decoder layer `layer`, ready for `Context.layer`.

    Matrices stay GGUF Q4_0 rows (N rows of K/32 18-byte blocks, uint8);
    norms and biases become float32.  Missing norms/biases are None (identity
    norm, zero bias), as in the reference's loader; missing matrices are
    errors.  With mlp=False (or no feed_forward_length) the MLP is omitted.
    """
    idx = read_index(path)
    d = dict(dims) if dims is not None else qwen2_dims(idx)
    if not mlp:
        d["intermediate"] = 0
    host = {}
    for key, (suffix, matrix, gdims) in _layer_tensors(d).items():
        if key in ("w_gate", "w_up", "w_down", "norm2") and not d["intermediate"]:
            host[key] = None
            continue
        name = f"blk.{layer}.{suffix}"
        if name not in idx.tensors:
            if matrix:
                raise GGUFError(f"required tensor {name} not found")
            host[key] = None
            continue
        t = _check(idx, name, matrix, gdims)
        if matrix:  # N rows of K/32 blocks of 18 bytes
            host[key] = np.frombuffer(tensor_bytes(idx, name), np.uint8).reshape(
                gdims[1], gdims[0] // 32 * 18).copy()
        else:
            host[key] = _vector(idx, t)
    d.pop("n_layers", None)
    return d, host


# The reference extractor's output files for one attention sublayer:
# short name -> (GGUF suffix, Q4_0 matrix?).
_EXTRACT = {"q": ("attn_q.weight", True), "k": ("attn_k.weight", True),
            "v": ("attn_v.weight", True), "o": ("attn_output.weight", True),
            "norm": ("attn_norm.weight", False), "q_bias": ("attn_q.bias", False),
            "k_bias": ("attn_k.bias", False), "v_bias": ("attn_v.bias", False)}


def extract(path: str, out_dir: str, layer: int = 0, dims: dict | None = None) -> dict:
    """Write `<short>.q4_0` / `<short>.f32` files for layer `layer`'s attention.

    The files are those of extract_weights.py (extract_weights.py:139-203):
    Q4_0 matrices copied byte for byte, F32 vectors copied, F16 vectors widened
    to F32; a missing optional vector leaves no file (a stale one is removed).
    Every tensor is validated before any file is written.  Returns a manifest
    (also written as manifest.json).
    """
    idx = read_index(path)
    d = dict(dims) if dims is not None else qwen2_dims(idx)
    shapes = {k: v[2] for k, v in _layer_tensors(d).items()}
    want = {"q": shapes["wq"], "k": shapes["wk"], "v": shapes["wv"], "o": shapes["wo"],
            "norm": shapes["norm"], "q_bias": shapes["bq"], "k_bias": shapes["bk"],
            "v_bias": shapes["bv"]}
    found = {}
    for short, (suffix, matrix) in _EXTRACT.items():
        name = f"blk.{layer}.{suffix}"
        if name not in idx.tensors:
            if matrix:
                raise GGUFError(f"required tensor {name} not found")
            continue
        found[short] = _check(idx, name, matrix, want[short])
    os.makedirs(out_dir, exist_ok=True)
    manifest = {"source": str(path), "layer": layer, "tensors": {}}
    for short, (suffix, matrix) in _EXTRACT.items():
        dest = os.path.join(out_dir, short + (".q4_0" if matrix else ".f32"))
        t = found.get(short)
        if t is None:
            if os.path.exists(dest):
                os.unlink(dest)  # never leave a previous extraction's file behind
            continue
        data = tensor_bytes(idx, t.name)
        if not matrix and t.type == F16:
            data = np.frombuffer(data, "<f2").astype("<f4").tobytes()
        with open(dest, "wb") as f:
            f.write(data)
        manifest["tensors"][short] = {"name": t.name, "gguf_shape": t.dims,
                                      "gguf_type": TYPE_NAMES.get(t.type, str(t.type)),
                                      "file": os.path.basename(dest), "bytes": len(data)}
    with open(os.path.join(out_dir, "manifest.json"), "w", encoding="utf-8") as f:
        json.dump(manifest, f, indent=2)
        f.write("\n")
    return manifest


def main(argv=None) -> int:
    """Command line of the reference extractor (extract_weights.py:206-224):
    `python -m sib200.gguf model.gguf [--layer N] [--out DIR] [--list]`."""
    import argparse
    ap = argparse.ArgumentParser(prog="python -m sib200.gguf",
                                 description="Extract one Qwen2 attention sublayer from a GGUF file.")
    ap.add_argument("gguf", help="local single-file Q4_0 GGUF")
    ap.add_argument("--layer", type=int, default=0, help="layer number, default 0")
    ap.add_argument("--out", default="weights", help="output directory")
    ap.add_argument("--list", action="store_true", help="list the layer's tensors; do not extract")
    args = ap.parse_args(argv)
    try:
        if args.list:
            idx = read_index(args.gguf)
            for name, t in idx.tensors.items():
                if name.startswith(f"blk.{args.layer}."):
                    print(f"{name:<36} {TYPE_NAMES.get(t.type, t.type):<8} {t.dims}")
            print("model metadata:", {k: v for k, v in idx.meta.items() if k.startswith("qwen2.")})
        else:
            m = extract(args.gguf, args.out, args.layer)
            for short, t in m["tensors"].items():
                print(f"  {t['name']:<34} {t['gguf_type']:<6} {str(t['gguf_shape']):<15} -> "
                      f"{os.path.join(args.out, t['file'])}")
    except (OSError, GGUFError, struct.error) as exc:
        print(f"sib200.gguf: {exc}")
        return 1
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
