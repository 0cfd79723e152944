"""TEST INFRASTRUCTURE ONLY: ctypes bindings to the CPU oracle and the reference.

``Oracle`` wraps oracle/liboracle.so, the dims-parametrised C restatement of the
reference hot path (oracle/si_oracle.c).  ``Reference`` wraps oracle/_ref/libsiref.so,
the reference's own qwen_one_layer.c translation unit built in place from the
reference checkout (oracle/ref_shim.c); it exists only where that checkout exists.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs may import
this module: it is the checker, never the product path.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_ORACLE = os.path.join(HERE, "liboracle.so")
LIB_REF = os.path.join(HERE, "_ref", "libsiref.so")

QK, Q4_BYTES, Q8_BYTES = 32, 18, 34

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
_i8p = np.ctypeslib.ndpointer(np.int8, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")


def reference_dir():
    """The reference checkout: $SI_REFERENCE_DIR, else a checkout named
    `reference` beside this repository; None when neither exists."""
    cand = os.environ.get("SI_REFERENCE_DIR") or os.path.join(HERE, "..", "..", "reference")
    cand = os.path.abspath(cand)
    return cand if os.path.exists(os.path.join(cand, "qwen_one_layer.c")) else None


def build(quiet: bool = True) -> None:
    """Compile oracle/liboracle.so (and oracle/_ref when the reference exists)."""
    out = subprocess.run(["make", "-C", HERE, "all"], capture_output=True, text=True)
    if out.returncode != 0:
        raise RuntimeError("oracle build failed:\n" + out.stdout + out.stderr)
    if not quiet:
        print(out.stdout)


class Dims(C.Structure):
    _fields_ = [("hidden", C.c_int), ("n_q_heads", C.c_int), ("n_kv_heads", C.c_int),
                ("head_dim", C.c_int), ("intermediate", C.c_int),
                ("rope_theta", C.c_float), ("rms_eps", C.c_float)]


class LayerPtrs(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in
                ("wq", "wk", "wv", "wo", "norm", "bq", "bk", "bv",
                 "w_gate", "w_up", "w_down", "norm2")]


def _ptr(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def make_dims(d) -> Dims:
    return Dims(d["hidden"], d["n_q_heads"], d["n_kv_heads"], d["head_dim"],
                d.get("intermediate", 0), d.get("rope_theta", 1e6), d.get("rms_eps", 1e-6))


class Oracle:
    def __init__(self, path: str = LIB_ORACLE):
        if not os.path.exists(path):
            build()
        L = self.lib = C.CDLL(path)
        L.oc_f16_to_f32.restype = C.c_float
        L.oc_f16_to_f32.argtypes = [C.c_uint16]
        L.oc_f32_to_f16.restype = C.c_uint16
        L.oc_f32_to_f16.argtypes = [C.c_float]
        L.oc_quantize_q8.restype = C.c_int
        L.oc_quantize_q8.argtypes = [_f32p, _u8p, C.c_int]
        L.oc_matvec_q4q8.argtypes = [_u8p, _u8p, C.c_int, C.c_int, C.c_void_p, _f32p]
        L.oc_block_isums.argtypes = [_u8p, _u8p, C.c_int, C.c_int, _i32p]
        L.oc_rmsnorm.argtypes = [_f32p, C.c_void_p, _f32p, C.c_int, C.c_float]
        L.oc_rope.argtypes = [_f32p, C.c_int, C.c_int, C.c_int, C.c_float]
        L.oc_rope_table.argtypes = [C.c_int, C.c_int, C.c_int, C.c_float, _f32p, _f32p]
        for fn in (L.oc_attention_flash,):
            fn.argtypes = [C.POINTER(Dims), _f32p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, _f32p]
        L.oc_attention_flash_heads.argtypes = [C.POINTER(Dims), _f32p, C.c_void_p, C.c_void_p,
                                               C.c_int, C.c_int, _f32p, C.c_int, C.c_int]
        L.oc_attention_standard.argtypes = [C.POINTER(Dims), _f32p, C.c_void_p, C.c_void_p,
                                            C.c_int, C.c_int, _f32p, _f32p]
        L.oc_run_layer.argtypes = [C.POINTER(Dims), C.POINTER(LayerPtrs), _f32p, C.c_void_p,
                                   C.c_void_p, C.c_int, C.c_int, _f32p, C.c_int, C.c_void_p,
                                   C.c_void_p, C.c_void_p]
        L.oc_mlp.argtypes = [C.POINTER(Dims), C.POINTER(LayerPtrs), _f32p, _f32p,
                             C.c_void_p, C.c_void_p]
        L.oc_decoder_layer.argtypes = [C.POINTER(Dims), C.POINTER(LayerPtrs), _f32p, C.c_void_p,
                                       C.c_void_p, C.c_int, C.c_int, _f32p]
        L.oc_prefill_sequential.argtypes = [C.POINTER(Dims), C.POINTER(LayerPtrs), _f32p, C.c_int,
                                            C.c_int, C.c_void_p, C.c_void_p, C.c_int, _f32p, C.c_int]
        L.oc_fused_column_matvec.argtypes = [_u8p, _u8p, C.c_int, C.c_void_p, C.c_void_p,
                                             _f32p, C.c_int]
        L.oc_pack_colsoa_tile.argtypes = [_u8p, _u8p, _u8p, C.c_int, C.c_int, C.c_int,
                                          C.c_int, C.c_int]
        L.oc_quantize_q4_0.argtypes = [_f32p, _u8p, C.c_int, C.c_int]
        L.oc_rng_seed.argtypes = [C.c_uint32]
        L.oc_random_float.restype = C.c_float
        L.oc_random_fill.argtypes = [_f32p, C.c_size_t, C.c_float, C.c_float]

    # -- primitives -------------------------------------------------------
    def quantize_q8(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32).reshape(-1)
        out = np.zeros(x.size // QK * Q8_BYTES, np.uint8)
        if self.lib.oc_quantize_q8(x, out, x.size) != 0:
            raise ValueError("Q8 quantization length must be multiple of 32")
        return out

    def matvec(self, w: np.ndarray, q8: np.ndarray, inputs: int, outputs: int,
               bias: np.ndarray | None = None) -> np.ndarray:
        out = np.zeros(outputs, np.float32)
        b = None if bias is None else np.ascontiguousarray(bias, np.float32)
        self.lib.oc_matvec_q4q8(np.ascontiguousarray(w).reshape(-1),
                                np.ascontiguousarray(q8).reshape(-1), inputs, outputs, _ptr(b), out)
        return out

    def block_isums(self, w, q8, inputs, outputs) -> np.ndarray:
        out = np.zeros((outputs, inputs // QK), np.int32)
        self.lib.oc_block_isums(np.ascontiguousarray(w).reshape(-1),
                                np.ascontiguousarray(q8).reshape(-1), inputs, outputs, out)
        return out

    def rmsnorm(self, x, w=None, eps=1e-6) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        out = np.zeros_like(x)
        wc = None if w is None else np.ascontiguousarray(w, np.float32)
        self.lib.oc_rmsnorm(x, _ptr(wc), out, x.size, eps)
        return out

    def rope(self, heads, nheads, pos, head_dim, theta=1e6) -> np.ndarray:
        h = np.array(heads, np.float32, copy=True)
        self.lib.oc_rope(h, nheads, pos, head_dim, theta)
        return h

    def rope_table(self, pos0, npos, head_dim, theta=1e6):
        c = np.zeros((npos, head_dim // 2), np.float32)
        s = np.zeros_like(c)
        self.lib.oc_rope_table(pos0, npos, head_dim, theta, c, s)
        return c, s

    def attention(self, dims, q, kc, vc, context, method=1) -> np.ndarray:
        d = make_dims(dims)
        kv_f32 = int(kc.dtype == np.float32)
        out = np.zeros(dims["n_q_heads"] * dims["head_dim"], np.float32)
        q = np.ascontiguousarray(q, np.float32)
        kc = np.ascontiguousarray(kc)
        vc = np.ascontiguousarray(vc)
        if method:
            self.lib.oc_attention_flash(C.byref(d), q, _ptr(kc), _ptr(vc), kv_f32, context, out)
        else:
            scores = np.zeros(dims["n_q_heads"] * max(context, 1), np.float32)
            self.lib.oc_attention_standard(C.byref(d), q, _ptr(kc), _ptr(vc), kv_f32, context,
                                           out, scores)
        return out

    # -- layer-level ------------------------------------------------------
    @staticmethod
    def _layer(layer) -> LayerPtrs:
        names = [f[0] for f in LayerPtrs._fields_]
        keep = {k: (None if layer.get(k) is None else np.ascontiguousarray(layer[k]))
                for k in names}
        lp = LayerPtrs(*[_ptr(keep[f[0]]) for f in LayerPtrs._fields_])
        lp._keep = keep
        return lp

    def run_layer(self, dims, layer, x, kc, vc, context, method=1, captures=False):
        d = make_dims(dims)
        lp = self._layer(layer)
        H = dims["hidden"]
        QD = dims["n_q_heads"] * dims["head_dim"]
        out = np.zeros(H, np.float32)
        attn = np.zeros(QD, np.float32) if captures else None
        q8 = np.zeros(QD // QK * Q8_BYTES, np.uint8) if captures else None
        self.lib.oc_run_layer(C.byref(d), C.byref(lp), np.ascontiguousarray(x, np.float32),
                              _ptr(kc), _ptr(vc), int(kc.dtype == np.float32), context, out,
                              method, None, _ptr(attn), _ptr(q8))
        return (out, attn, q8) if captures else out

    def mlp(self, dims, layer, h, captures=False):
        d = make_dims(dims)
        lp = self._layer(layer)
        out = np.zeros(dims["hidden"], np.float32)
        I = dims["intermediate"]
        act = np.zeros(I, np.float32) if captures else None
        q8 = np.zeros(I // QK * Q8_BYTES, np.uint8) if captures else None
        self.lib.oc_mlp(C.byref(d), C.byref(lp), np.ascontiguousarray(h, np.float32), out,
                        _ptr(act), _ptr(q8))
        return (out, act, q8) if captures else out

    def decoder_layer(self, dims, layer, x, kc, vc, context):
        d = make_dims(dims)
        lp = self._layer(layer)
        y = np.zeros(dims["hidden"], np.float32)
        self.lib.oc_decoder_layer(C.byref(d), C.byref(lp), np.ascontiguousarray(x, np.float32),
                                  _ptr(kc), _ptr(vc), int(kc.dtype == np.float32), context, y)
        return y

    def prefill_sequential(self, dims, layer, x, prefix, kc, vc, full_layer=False):
        d = make_dims(dims)
        lp = self._layer(layer)
        x = np.ascontiguousarray(x, np.float32)
        ntok = x.shape[0]
        y = np.zeros_like(x)
        self.lib.oc_prefill_sequential(C.byref(d), C.byref(lp), x, ntok, prefix, _ptr(kc),
                                       _ptr(vc), int(kc.dtype == np.float32), y, int(full_layer))
        return y

    def fused_column_matvec(self, tile, q8, nblocks, bias_lo=None, bias_hi=None, out=None, add=0):
        if out is None:
            out = np.zeros(256, np.float32)
        self.lib.oc_fused_column_matvec(np.ascontiguousarray(tile).reshape(-1),
                                        np.ascontiguousarray(q8).reshape(-1), nblocks,
                                        _ptr(bias_lo), _ptr(bias_hi), out, add)
        return out

    def pack_colsoa_tile(self, low_src, high_src, src_cols, low_base, high_base, input_base,
                         nblocks) -> np.ndarray:
        out = np.zeros(nblocks * 5120, np.uint8)
        self.lib.oc_pack_colsoa_tile(out, np.ascontiguousarray(low_src).reshape(-1),
                                     np.ascontiguousarray(high_src).reshape(-1), src_cols,
                                     low_base, high_base, input_base, nblocks)
        return out

    def quantize_q4_0(self, w: np.ndarray) -> np.ndarray:
        w = np.ascontiguousarray(w, np.float32)
        rows, k = w.shape
        out = np.zeros((rows, k // QK * Q4_BYTES), np.uint8)
        self.lib.oc_quantize_q4_0(w, out, rows, k)
        return out

    def seed(self, s: int) -> None:
        self.lib.oc_rng_seed(s)

    def random_floats(self, n: int, scale: float = 1.0, offset: float = 0.0) -> np.ndarray:
        out = np.zeros(n, np.float32)
        self.lib.oc_random_fill(out, n, scale, offset)
        return out


class Reference:
    """The reference's own kernels (compile-time 1.5B dims)."""

    def __init__(self, path: str = LIB_REF):
        if not os.path.exists(path):
            raise FileNotFoundError(path)
        L = self.lib = C.CDLL(path)
        dims = (C.c_int * 5)()
        L.ref_dims(dims)
        self.hidden, self.qheads, self.kvheads, self.hdim, _ = list(dims)
        self.kvdim = self.kvheads * self.hdim
        L.ref_f16_to_f32.restype = C.c_float
        L.ref_f16_to_f32.argtypes = [C.c_uint16]
        L.ref_f32_to_f16.restype = C.c_uint16
        L.ref_f32_to_f16.argtypes = [C.c_float]
        L.ref_quantize_q8.argtypes = [_f32p, _u8p, C.c_int]
        L.ref_dot_32_q4q8.restype = C.c_int32
        L.ref_dot_32_q4q8.argtypes = [_u8p, _i8p]
        L.ref_matvec_q4q8.argtypes = [_u8p, _u8p, C.c_int, C.c_int, C.c_void_p, _f32p]
        L.ref_rmsnorm.argtypes = [_f32p, C.c_void_p, _f32p]
        L.ref_rope.argtypes = [_f32p, C.c_int, C.c_int]
        L.ref_attention_flash.argtypes = [_f32p, _u16p, _u16p, C.c_int, _f32p]
        L.ref_attention_standard.argtypes = [_f32p, _u16p, _u16p, C.c_int, _f32p, _f32p]
        L.ref_run_layer.argtypes = [C.c_void_p] * 8 + [_f32p, _u16p, _u16p, C.c_int, _f32p,
                                                       C.c_int, C.c_void_p, C.c_void_p, C.c_void_p]
        L.ref_fused_column_matvec.argtypes = [_u8p, _u8p, C.c_int, C.c_void_p, C.c_void_p,
                                              _f32p, C.c_int]
        L.ref_fused_attention_pair.argtypes = [_f32p, _u16p, _u16p, C.c_int, C.c_int, _f32p]
        L.ref_run_layer_fused.argtypes = [C.c_void_p] * 11 + [_f32p, _u16p, _u16p, C.c_int,
                                                              _f32p, C.c_void_p, C.c_void_p]
        L.ref_seed.argtypes = [C.c_uint32]
        L.ref_random_float.restype = C.c_float
        L.ref_fill_kv_history.argtypes = [_u16p, _u16p, C.c_int]

    def quantize_q8(self, x):
        x = np.ascontiguousarray(x, np.float32)
        out = np.zeros(x.size // QK * Q8_BYTES, np.uint8)
        self.lib.ref_quantize_q8(x, out, x.size)
        return out

    def matvec(self, w, q8, inputs, outputs, bias=None):
        out = np.zeros(outputs, np.float32)
        self.lib.ref_matvec_q4q8(np.ascontiguousarray(w).reshape(-1),
                                 np.ascontiguousarray(q8).reshape(-1), inputs, outputs,
                                 _ptr(bias), out)
        return out

    def rmsnorm(self, x, w=None):
        out = np.zeros(self.hidden, np.float32)
        self.lib.ref_rmsnorm(np.ascontiguousarray(x, np.float32), _ptr(w), out)
        return out

    def rope(self, heads, nheads, pos):
        h = np.array(heads, np.float32, copy=True)
        self.lib.ref_rope(h, nheads, pos)
        return h

    def attention(self, q, kc, vc, context, method=1):
        out = np.zeros(self.qheads * self.hdim, np.float32)
        if method:
            self.lib.ref_attention_flash(q, kc, vc, context, out)
        else:
            scores = np.zeros(self.qheads * context, np.float32)
            self.lib.ref_attention_standard(q, kc, vc, context, out, scores)
        return out

    def run_layer(self, layer, x, kc, vc, context, method=1):
        out = np.zeros(self.hidden, np.float32)
        attn = np.zeros(self.hidden, np.float32)
        q8 = np.zeros(self.hidden // QK * Q8_BYTES, np.uint8)
        scores = np.zeros(self.qheads * context, np.float32)
        ptrs = [_ptr(layer.get(k)) for k in ("wq", "wk", "wv", "wo", "norm", "bq", "bk", "bv")]
        self.lib.ref_run_layer(*ptrs, np.ascontiguousarray(x, np.float32), kc, vc, context, out,
                               method, _ptr(scores), _ptr(attn), _ptr(q8))
        return out, attn, q8

    def run_layer_fused(self, layer, colsoa, x, kc, vc, context):
        out = np.zeros(self.hidden, np.float32)
        attn = np.zeros(self.hidden, np.float32)
        q8 = np.zeros(self.hidden // QK * Q8_BYTES, np.uint8)
        ptrs = [_ptr(layer.get(k)) for k in ("wq", "wk", "wv", "wo", "norm", "bq", "bk", "bv")]
        ptrs += [_ptr(colsoa[k]) for k in ("q", "kv", "o")]
        self.lib.ref_run_layer_fused(*ptrs, np.ascontiguousarray(x, np.float32), kc, vc, context,
                                     out, _ptr(attn), _ptr(q8))
        return out, attn, q8

    def fused_column_matvec(self, tile, q8, nblocks, bias_lo=None, bias_hi=None, out=None, add=0):
        if out is None:
            out = np.zeros(256, np.float32)
        self.lib.ref_fused_column_matvec(np.ascontiguousarray(tile).reshape(-1),
                                         np.ascontiguousarray(q8).reshape(-1), nblocks,
                                         _ptr(bias_lo), _ptr(bias_hi), out, add)
        return out

    def seed(self, s):
        self.lib.ref_seed(s)

    def random_floats(self, n):
        return np.array([self.lib.ref_random_float() for _ in range(n)], np.float32)

    def fill_kv_history(self, context):
        kc = np.zeros(context * self.kvdim, np.uint16)
        vc = np.zeros_like(kc)
        self.lib.ref_fill_kv_history(kc, vc, context)
        return kc, vc
