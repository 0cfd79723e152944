"""ctypes bindings to libsi_b200.so (the C ABI in include/si_b200.h).

The library is the product; this module only loads it and converts arguments.
Device buffers are passed as raw pointers (ints): callers use torch tensors
purely as device memory.  If the shared library is missing or cannot load, every
entry point raises -- there is no fallback implementation.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

from . import synth  # noqa: F401

PKG_DIR = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.path.join(PKG_DIR, "lib", "libsi_b200.so")

SI_OK = 0
SI_ERR_INVALID, SI_ERR_CUDA, SI_ERR_OOM, SI_ERR_NO_DEVICE = 1, 2, 3, 4
SI_ERR_DEVICE, SI_ERR_TIMEOUT, SI_ERR_IO, SI_ERR_UNSUPPORTED = 5, 6, 7, 8
SI_LAYER_ATTN, SI_LAYER_FULL = 0, 1


class SiError(RuntimeError):
    def __init__(self, status: int, where: str, detail: str):
        super().__init__(f"{where}: status {status} ({detail})")
        self.status = status


def kernel_launches() -> int:
    """Kernels libsi_b200 has queued so far in this process."""
    return int(lib().si_kernel_launches())


def build(jobs: int = 8) -> str:
    """Compile libsi_b200.so (sm_100a) in-tree with nvcc."""
    out = subprocess.run(["make", "-C", PKG_DIR, f"-j{jobs}"], capture_output=True, text=True)
    if out.returncode != 0:
        raise RuntimeError("libsi_b200 build failed:\n" + out.stdout[-4000:] + out.stderr[-8000:])
    return LIB_PATH


class Dims(C.Structure):
    _fields_ = [("hidden", C.c_int), ("n_q_heads", C.c_int), ("n_kv_heads", C.c_int),
                ("head_dim", C.c_int), ("intermediate", C.c_int),
                ("rope_theta", C.c_float), ("rms_eps", C.c_float)]

    @classmethod
    def of(cls, d: dict) -> "Dims":
        return cls(d["hidden"], d["n_q_heads"], d["n_kv_heads"], d["head_dim"],
                   d.get("intermediate", 0), d.get("rope_theta", 1e6), d.get("rms_eps", 1e-6))


class LayerHost(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in ("wq", "wk", "wv", "wo", "w_gate", "w_up", "w_down",
                                          "norm", "bq", "bk", "bv", "norm2")]


class Captures(C.Structure):
    _fields_ = [("attn", C.c_void_p), ("attn_q8", C.c_void_p), ("qkv", C.c_void_p)]


_lib = None


def lib() -> C.CDLL:
    """Load libsi_b200.so once; raise if it is absent (no silent fallback)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is missing: build it with sib200.build()")
    L = C.CDLL(LIB_PATH)
    vp, i32, f32, u64 = C.c_void_p, C.c_int, C.c_float, C.c_uint64
    pp = C.POINTER(C.c_void_p)
    sigs = {
        "si_status_str": (C.c_char_p, [i32]),
        "si_last_error": (C.c_char_p, []),
        "si_ctx_create": (i32, [i32, i32, f32, i32, pp]),
        "si_ctx_destroy": (None, [vp]),
        "si_ctx_synchronize": (i32, [vp]),
        "si_ctx_status": (i32, [vp]),
        "si_ctx_stream": (vp, [vp]),
        "si_ctx_scratch_bytes": (C.c_size_t, [vp]),
        "si_kernel_launches": (C.c_ulonglong, []),
        "si_tc_i8_peak_dev": (i32, [vp, i32, i32, C.POINTER(C.c_double)]),
        "si_matrix_upload": (i32, [vp, vp, i32, i32, pp]),
        "si_matrix_upload_dev": (i32, [vp, vp, i32, i32, pp]),
        "si_matrix_synth": (i32, [vp, i32, i32, u64, f32, pp]),
        "si_matrix_free": (None, [vp]),
        "si_matrix_rows": (i32, [vp]),
        "si_matrix_cols": (i32, [vp]),
        "si_matrix_layout": (i32, [vp, pp, pp]),
        "si_matrix_download": (i32, [vp, vp, vp]),
        "si_q8_quantize_dev": (i32, [vp, vp, i32, i32, vp, vp]),
        "si_q8_to_blocks_dev": (i32, [vp, vp, vp, i32, i32, vp]),
        "si_q8_from_blocks_dev": (i32, [vp, vp, i32, i32, vp, vp]),
        "si_matmul_dev": (i32, [vp, vp, vp, vp, i32, vp, vp]),
        "si_matmul_dev_kernel": (i32, [vp, vp, vp, vp, i32, vp, vp, i32]),
        "si_matmul_tc_static_dev": (i32, [vp, vp, vp, vp, i32, vp, vp]),
        "si_block_isums_dev": (i32, [vp, vp, vp, i32, vp]),
        "si_gateup_q8_dev": (i32, [vp, vp, vp, vp, vp, i32, vp, vp, vp]),
        "si_gateup_q8_dev_kernel": (i32, [vp, vp, vp, vp, vp, i32, vp, vp, vp, i32]),
        "si_rmsnorm_q8_dev": (i32, [vp, vp, vp, i32, i32, f32, vp, vp, vp]),
        "si_layer_upload": (i32, [vp, C.POINTER(Dims), C.POINTER(LayerHost), pp]),
        "si_layer_synth": (i32, [vp, C.POINTER(Dims), u64, pp]),
        "si_layer_free": (None, [vp]),
        "si_layer_matrix": (i32, [vp, i32, pp]),
        "si_layer_vectors_download": (i32, [vp, vp, vp, vp, vp]),
        "si_kv_create": (i32, [vp, C.POINTER(Dims), i32, i32, i32, pp]),
        "si_kv_free": (None, [vp]),
        "si_kv_write": (i32, [vp, vp, i32, i32, i32, vp, vp]),
        "si_kv_read": (i32, [vp, vp, i32, i32, i32, vp, vp]),
        "si_kv_fill_synth": (i32, [vp, vp, u64, f32, i32]),
        "si_kv_device_ptr": (vp, [vp, i32]),
        "si_decode_step": (i32, [vp, vp, vp, vp, i32, vp, vp, i32, C.POINTER(Captures)]),
        "si_decode_step_dev": (i32, [vp, vp, vp, vp, i32, vp, vp, i32, C.POINTER(Captures)]),
        "si_prefill": (i32, [vp, vp, vp, i32, vp, i32, i32, vp, i32]),
        "si_prefill_dev": (i32, [vp, vp, vp, i32, vp, i32, i32, vp, i32]),
        "si_graph_kernel_nodes": (i32, [vp]),
        "si_tp_split": (None, [i32, i32, i32, C.POINTER(C.c_int), C.POINTER(C.c_int)]),
        "si_tp_unique_id": (i32, [vp]),
        "si_tp_create": (i32, [vp, vp, i32, i32, pp]),
        "si_tp_free": (None, [vp]),
        "si_tp_set_options": (i32, [vp, i32, i32]),
        "si_tp_probe_wait": (i32, [vp, i32]),
        "si_tp_local_dims": (i32, [C.POINTER(Dims), i32, i32, C.POINTER(Dims),
                                   C.POINTER(C.c_int)]),
        "si_layer_tp_synth": (i32, [vp, C.POINTER(Dims), u64, i32, i32, pp]),
        "si_decode_step_tp_dev": (i32, [vp, vp, vp, vp, vp, i32, vp, vp, i32]),
        "si_prefill_tp_dev": (i32, [vp, vp, vp, vp, i32, vp, i32, i32, vp, i32]),
        "si_attention_decode_dev": (i32, [vp, vp, C.POINTER(Dims), vp, i32, vp, vp]),
        "si_attention_prefill_dev": (i32, [vp, vp, C.POINTER(Dims), vp, i32, i32, i32, vp]),
        "si_ctx_set_exact_attention": (i32, [vp, i32]),
        "si_matvec_gguf_dev": (i32, [vp, vp, i32, i32, vp, vp, i32, vp, vp]),
        "si_decode_state_create": (i32, [vp, i32, vp, i32, pp]),
        "si_decode_state_free": (None, [vp]),
        "si_decode_state_advance": (i32, [vp, vp]),
        "si_decode_state_set": (i32, [vp, vp, vp]),
        "si_decode_state_read": (i32, [vp, vp, vp]),
        "si_decode_step_state_dev": (i32, [vp, vp, vp, vp, vp, vp, i32]),
        "si_decode_step_state_tp_dev": (i32, [vp, vp, vp, vp, vp, vp, vp, i32]),
        "si_graph_begin": (i32, [vp]),
        "si_graph_end": (i32, [vp, pp]),
        "si_graph_launch": (i32, [vp, vp]),
        "si_graph_free": (None, [vp]),
        "quantize_q8": (None, [vp, vp, i32]),
        "matvec_q4q8": (None, [vp, vp, i32, i32, vp, vp]),
        "si_forget_host_weights": (None, [vp]),
        "si_ref_rmsnorm": (None, [vp, vp, vp, i32, f32]),
        "si_ref_rope": (None, [vp, i32, i32, i32, f32]),
        "si_ref_attention": (None, [i32, vp, vp, vp, i32, vp, vp, i32, i32, i32]),
    }
    for name, (res, args) in sigs.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def check(status: int, where: str) -> None:
    if status != SI_OK:
        L = lib()
        raise SiError(status, where, L.si_last_error().decode(errors="replace"))


def _p(x):
    """Pointer of a numpy array / torch tensor / int / None."""
    if x is None:
        return None
    if isinstance(x, int):
        return x
    if hasattr(x, "data_ptr"):
        return x.data_ptr()
    return x.ctypes.data


class Context:
    def __init__(self, device: int = 0, max_positions: int = 32768, rope_theta: float = 1e6,
                 head_dim: int = 128):
        self.L = lib()
        h = C.c_void_p()
        check(self.L.si_ctx_create(device, max_positions, rope_theta, head_dim, C.byref(h)),
              "si_ctx_create")
        self.h = h
        self.device = device

    def close(self):
        if self.h:
            self.L.si_ctx_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def stream(self) -> int:
        return self.L.si_ctx_stream(self.h)

    def sync(self):
        check(self.L.si_ctx_synchronize(self.h), "si_ctx_synchronize")

    def tc_i8_peak(self, n: int, iters: int) -> float:
        """Queue the int8 tensor-core probe; returns its int8 ops per launch."""
        ops = C.c_double()
        check(self.L.si_tc_i8_peak_dev(self.h, n, iters, C.byref(ops)), "si_tc_i8_peak_dev")
        return ops.value

    def scratch_bytes(self) -> int:
        """Device bytes held by the context's on-demand buffers."""
        return int(self.L.si_ctx_scratch_bytes(self.h))

    def status(self):
        check(self.L.si_ctx_status(self.h), "si_ctx_status")

    def capture(self, fn) -> "Graph":
        """Capture the library calls made by fn() into a replayable CUDA graph."""
        check(self.L.si_graph_begin(self.h), "si_graph_begin")
        try:
            fn()
        finally:
            g = C.c_void_p()
            st = self.L.si_graph_end(self.h, C.byref(g))
        check(st, "si_graph_end")
        return Graph(self, g)

    # -- matrices -----------------------------------------------------------
    def matrix(self, gguf, rows: int, cols: int) -> "Matrix":
        h = C.c_void_p()
        check(self.L.si_matrix_upload(self.h, _p(gguf), rows, cols, C.byref(h)),
              "si_matrix_upload")
        return Matrix(self, h)

    def matrix_synth(self, rows: int, cols: int, seed: int, std: float = 0.02) -> "Matrix":
        h = C.c_void_p()
        check(self.L.si_matrix_synth(self.h, rows, cols, seed, std, C.byref(h)),
              "si_matrix_synth")
        return Matrix(self, h)

    def q8_quantize(self, x, M, K, qs, d):
        check(self.L.si_q8_quantize_dev(self.h, _p(x), M, K, _p(qs), _p(d)), "si_q8_quantize_dev")

    def q8_to_blocks(self, qs, d, M, K, blocks):
        check(self.L.si_q8_to_blocks_dev(self.h, _p(qs), _p(d), M, K, _p(blocks)),
              "si_q8_to_blocks_dev")

    def q8_from_blocks(self, blocks, M, K, qs, d):
        check(self.L.si_q8_from_blocks_dev(self.h, _p(blocks), M, K, _p(qs), _p(d)),
              "si_q8_from_blocks_dev")

    def matmul(self, w: "Matrix", qs, d, M, bias, out, kernel: int | None = None):
        if kernel is None:
            check(self.L.si_matmul_dev(self.h, w.h, _p(qs), _p(d), M, _p(bias), _p(out)),
                  "si_matmul_dev")
        else:
            check(self.L.si_matmul_dev_kernel(self.h, w.h, _p(qs), _p(d), M, _p(bias), _p(out),
                                              kernel), "si_matmul_dev_kernel")

    def matvec_gguf(self, w_gguf, rows, cols, qs, d, M, bias, out):
        """GEMV straight from row-major GGUF Q4_0 bytes on the device (no repack)."""
        check(self.L.si_matvec_gguf_dev(self.h, _p(w_gguf), rows, cols, _p(qs), _p(d), M,
                                        _p(bias), _p(out)), "si_matvec_gguf_dev")

    def block_isums(self, w: "Matrix", qs, M, out):
        check(self.L.si_block_isums_dev(self.h, w.h, _p(qs), M, _p(out)), "si_block_isums_dev")

    def gateup_q8(self, gate, up, qs, d, M, act_qs, act_d, act_f32=None,
                  kernel: int | None = None):
        if kernel is None:
            check(self.L.si_gateup_q8_dev(self.h, gate.h, up.h, _p(qs), _p(d), M, _p(act_qs),
                                          _p(act_d), _p(act_f32)), "si_gateup_q8_dev")
        else:
            check(self.L.si_gateup_q8_dev_kernel(self.h, gate.h, up.h, _p(qs), _p(d), M,
                                                 _p(act_qs), _p(act_d), _p(act_f32), kernel),
                  "si_gateup_q8_dev_kernel")

    def rmsnorm_q8(self, x, w, M, n, eps, out=None, qs=None, d=None):
        check(self.L.si_rmsnorm_q8_dev(self.h, _p(x), _p(w), M, n, eps, _p(out), _p(qs), _p(d)),
              "si_rmsnorm_q8_dev")

    # -- layers / KV --------------------------------------------------------
    def layer(self, dims: dict, host: dict) -> "Layer":
        lh = LayerHost(*[_p(host.get(f[0])) for f in LayerHost._fields_])
        dm = Dims.of(dims)
        h = C.c_void_p()
        check(self.L.si_layer_upload(self.h, C.byref(dm), C.byref(lh), C.byref(h)),
              "si_layer_upload")
        return Layer(self, h, dims)

    def layer_gguf(self, path: str, layer: int, mlp: bool = True) -> "Layer":
        """Decoder layer `layer` of a Qwen2 GGUF file (Q4_0 matrices, F32/F16
        vectors), dimensions from the file's metadata; see sib200.gguf."""
        from . import gguf
        dims, host = gguf.layer_host(path, layer, mlp=mlp)
        return self.layer(dims, host)

    def layer_synth(self, dims: dict, seed: int) -> "Layer":
        dm = Dims.of(dims)
        h = C.c_void_p()
        check(self.L.si_layer_synth(self.h, C.byref(dm), seed, C.byref(h)), "si_layer_synth")
        return Layer(self, h, dims)

    def tp(self, uid: bytes, rank: int, world: int) -> "TP":
        """Join the tensor-parallel group identified by uid (from tp_unique_id)."""
        h = C.c_void_p()
        buf = C.create_string_buffer(bytes(uid), 128)
        check(self.L.si_tp_create(self.h, buf, rank, world, C.byref(h)), "si_tp_create")
        return TP(self, h, rank, world)

    def tp_probe_wait(self, timeout_us: int) -> int:
        """Status of the fused TP reduction's bounded wait on a flag nothing sets."""
        return self.L.si_tp_probe_wait(self.h, timeout_us)

    def layer_tp_synth(self, full: dict, seed: int, rank: int, world: int) -> "Layer":
        dm = Dims.of(full)
        h = C.c_void_p()
        check(self.L.si_layer_tp_synth(self.h, C.byref(dm), seed, rank, world, C.byref(h)),
              "si_layer_tp_synth")
        return Layer(self, h, tp_local_dims(full, rank, world)[0])

    def kv(self, dims: dict, batch: int, max_ctx: int, kv_f32: bool) -> "KV":
        dm = Dims.of(dims)
        h = C.c_void_p()
        check(self.L.si_kv_create(self.h, C.byref(dm), batch, max_ctx, int(kv_f32), C.byref(h)),
              "si_kv_create")
        return KV(self, h, dims, batch, max_ctx, kv_f32)

    def attention_prefill(self, kv: "KV", dims: dict, q, ntok, seq, prefix, out):
        dm = Dims.of(dims)
        check(self.L.si_attention_prefill_dev(self.h, kv.h, C.byref(dm), _p(q), ntok, seq, prefix,
                                              _p(out)), "si_attention_prefill_dev")

    def decode_state(self, ctx_lens, max_ctx: int) -> "DecodeState":
        """Device-resident decode positions for a batch (see si_decode_state_create)."""
        lens = (C.c_int * len(ctx_lens))(*ctx_lens)
        h = C.c_void_p()
        check(self.L.si_decode_state_create(self.h, len(ctx_lens), lens, max_ctx, C.byref(h)),
              "si_decode_state_create")
        return DecodeState(self, h, len(ctx_lens))

    def set_exact_attention(self, exact: bool):
        """True: prefill attention by the fp32 kernel (bit-identical to decode
        steps); False (default): the tcgen05 tensor-core kernel."""
        check(self.L.si_ctx_set_exact_attention(self.h, int(exact)), "si_ctx_set_exact_attention")

    def attention_decode(self, kv: "KV", dims: dict, q, batch, ctx_lens, out):
        dm = Dims.of(dims)
        lens = (C.c_int * batch)(*ctx_lens)
        check(self.L.si_attention_decode_dev(self.h, kv.h, C.byref(dm), _p(q), batch, lens,
                                             _p(out)), "si_attention_decode_dev")


class DecodeState:
    def __init__(self, ctx: "Context", h, batch: int):
        self.ctx, self.h, self.batch = ctx, h, batch

    def advance(self):
        check(self.ctx.L.si_decode_state_advance(self.ctx.h, self.h), "si_decode_state_advance")

    def set(self, ctx_lens):
        lens = (C.c_int * len(ctx_lens))(*ctx_lens)
        check(self.ctx.L.si_decode_state_set(self.ctx.h, self.h, lens), "si_decode_state_set")

    def lens(self) -> list:
        out = (C.c_int * self.batch)()
        check(self.ctx.L.si_decode_state_read(self.ctx.h, self.h, out), "si_decode_state_read")
        return list(out)

    def free(self):
        if self.h:
            self.ctx.L.si_decode_state_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class Graph:
    def __init__(self, ctx: Context, h):
        self.ctx, self.h = ctx, h

    def launch(self):
        check(self.ctx.L.si_graph_launch(self.ctx.h, self.h), "si_graph_launch")

    def kernels(self) -> int:
        """Kernel launches per replay."""
        return self.ctx.L.si_graph_kernel_nodes(self.h)

    def free(self):
        if self.h:
            self.ctx.L.si_graph_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class Matrix:
    def __init__(self, ctx: Context, h, owned: bool = True):
        self.ctx, self.h, self.owned = ctx, h, owned
        self.rows = ctx.L.si_matrix_rows(h)
        self.cols = ctx.L.si_matrix_cols(h)

    def download(self, out):
        check(self.ctx.L.si_matrix_download(self.ctx.h, self.h, _p(out)), "si_matrix_download")

    def download_gguf(self):
        """GGUF row-major Q4_0 bytes as a new numpy array."""
        out = np.zeros(self.rows * (self.cols // 32) * 18, np.uint8)
        self.download(out)
        return out

    def layout(self):
        nib, scl = C.c_void_p(), C.c_void_p()
        check(self.ctx.L.si_matrix_layout(self.h, C.byref(nib), C.byref(scl)), "si_matrix_layout")
        return nib.value, scl.value

    def free(self):
        if self.h and self.owned:
            self.ctx.L.si_matrix_free(self.h)
        self.h = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class Layer:
    def __init__(self, ctx: Context, h, dims):
        self.ctx, self.h, self.dims = ctx, h, dims

    def host(self) -> dict:
        """The layer as a host dict in the reference's formats (GGUF Q4_0 rows,
        fp32 vectors), e.g. for checking a synthetic layer against the oracle."""
        d = self.dims
        H, D = d["hidden"], d["head_dim"]
        QD, KVD = d["n_q_heads"] * D, d["n_kv_heads"] * D
        norm, norm2 = np.zeros(H, np.float32), np.zeros(H, np.float32)
        bias = np.zeros(QD + 2 * KVD, np.float32)
        check(self.ctx.L.si_layer_vectors_download(self.ctx.h, self.h, _p(norm), _p(norm2),
                                                   _p(bias)), "si_layer_vectors_download")
        qkv = self.matrix(0).download_gguf()
        rb = H // 32 * 18
        out = {"wq": qkv[:QD * rb], "wk": qkv[QD * rb:(QD + KVD) * rb],
               "wv": qkv[(QD + KVD) * rb:], "wo": self.matrix(1).download_gguf(),
               "norm": norm, "bq": bias[:QD], "bk": bias[QD:QD + KVD], "bv": bias[QD + KVD:],
               "w_gate": None, "w_up": None, "w_down": None, "norm2": None}
        if d.get("intermediate", 0) > 0:
            out.update(w_gate=self.matrix(2).download_gguf(), w_up=self.matrix(3).download_gguf(),
                       w_down=self.matrix(4).download_gguf(), norm2=norm2)
        return out

    def matrix(self, which: int) -> Matrix:
        m = C.c_void_p()
        check(self.ctx.L.si_layer_matrix(self.h, which, C.byref(m)), "si_layer_matrix")
        return Matrix(self.ctx, m, owned=False)  # borrowed: the layer owns it

    def free(self):
        if self.h:
            self.ctx.L.si_layer_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass

    def decode(self, kv: "KV", x_host, ctx_lens, y_host, mode=SI_LAYER_ATTN, captures=None):
        lens = (C.c_int * len(ctx_lens))(*ctx_lens)
        cap = None
        if captures is not None:
            cap = Captures(_p(captures.get("attn")), _p(captures.get("attn_q8")),
                           _p(captures.get("qkv")))
        check(self.ctx.L.si_decode_step(self.ctx.h, self.h, kv.h, _p(x_host), len(ctx_lens),
                                        lens, _p(y_host), mode,
                                        C.byref(cap) if cap is not None else None),
              "si_decode_step")

    def decode_dev(self, kv: "KV", x, ctx_lens, y, mode=SI_LAYER_ATTN):
        lens = (C.c_int * len(ctx_lens))(*ctx_lens)
        check(self.ctx.L.si_decode_step_dev(self.ctx.h, self.h, kv.h, _p(x), len(ctx_lens),
                                            lens, _p(y), mode, None), "si_decode_step_dev")

    def decode_state_dev(self, kv: "KV", x, state: "DecodeState", y, mode=SI_LAYER_ATTN):
        check(self.ctx.L.si_decode_step_state_dev(self.ctx.h, self.h, kv.h, _p(x), state.h,
                                                  _p(y), mode), "si_decode_step_state_dev")

    def prefill(self, kv: "KV", seq, x_host, ntok, prefix, y_host, mode=SI_LAYER_ATTN):
        check(self.ctx.L.si_prefill(self.ctx.h, self.h, kv.h, seq, _p(x_host), ntok, prefix,
                                    _p(y_host), mode), "si_prefill")

    def prefill_dev(self, kv: "KV", seq, x, ntok, prefix, y, mode=SI_LAYER_ATTN):
        check(self.ctx.L.si_prefill_dev(self.ctx.h, self.h, kv.h, seq, _p(x), ntok, prefix,
                                        _p(y), mode), "si_prefill_dev")


def tp_split(units: int, rank: int, world: int) -> tuple[int, int]:
    """(first, count) of the units rank owns (host-only; no GPU needed)."""
    f, c = C.c_int(), C.c_int()
    lib().si_tp_split(units, rank, world, C.byref(f), C.byref(c))
    return f.value, c.value


def tp_local_dims(full: dict, rank: int, world: int) -> tuple[dict, int]:
    """Shard dims and first owned MLP row (host-only)."""
    dm, out, first = Dims.of(full), Dims(), C.c_int()
    check(lib().si_tp_local_dims(C.byref(dm), rank, world, C.byref(out), C.byref(first)),
          "si_tp_local_dims")
    d = dict(full)
    d.update(n_q_heads=out.n_q_heads, n_kv_heads=out.n_kv_heads, intermediate=out.intermediate)
    return d, first.value


def tp_unique_id() -> bytes:
    buf = C.create_string_buffer(128)
    check(lib().si_tp_unique_id(buf), "si_tp_unique_id")
    return buf.raw


class TP:
    def __init__(self, ctx: Context, h, rank, world):
        self.ctx, self.h, self.rank, self.world = ctx, h, rank, world

    def decode_dev(self, layer: "Layer", kv: "KV", x, ctx_lens, y, mode=SI_LAYER_FULL):
        lens = (C.c_int * len(ctx_lens))(*ctx_lens)
        check(self.ctx.L.si_decode_step_tp_dev(self.ctx.h, self.h, layer.h, kv.h, _p(x),
                                               len(ctx_lens), lens, _p(y), mode),
              "si_decode_step_tp_dev")

    def decode_state_dev(self, layer: "Layer", kv: "KV", x, state, y, mode=SI_LAYER_FULL):
        check(self.ctx.L.si_decode_step_state_tp_dev(self.ctx.h, self.h, layer.h, kv.h, _p(x),
                                                     state.h, _p(y), mode),
              "si_decode_step_state_tp_dev")

    def prefill_dev(self, layer: "Layer", kv: "KV", seq, x, ntok, prefix, y, mode=SI_LAYER_FULL):
        check(self.ctx.L.si_prefill_tp_dev(self.ctx.h, self.h, layer.h, kv.h, seq, _p(x), ntok,
                                           prefix, _p(y), mode), "si_prefill_tp_dev")

    def set_options(self, fused: bool = True, timeout_ms: int = 5000):
        check(self.ctx.L.si_tp_set_options(self.h, int(fused), timeout_ms), "si_tp_set_options")

    def free(self):
        if self.h:
            self.ctx.L.si_tp_free(self.h)
            self.h = None


class KV:
    def __init__(self, ctx: Context, h, dims, batch, max_ctx, kv_f32):
        self.ctx, self.h, self.dims = ctx, h, dims
        self.batch, self.max_ctx, self.kv_f32 = batch, max_ctx, kv_f32

    def write(self, seq, pos0, k, v):
        npos = k.shape[0]
        check(self.ctx.L.si_kv_write(self.ctx.h, self.h, seq, pos0, npos, _p(k), _p(v)),
              "si_kv_write")

    def read(self, seq, pos0, npos, k, v):
        check(self.ctx.L.si_kv_read(self.ctx.h, self.h, seq, pos0, npos, _p(k), _p(v)),
              "si_kv_read")

    def fill_synth(self, seed, std, npos):
        check(self.ctx.L.si_kv_fill_synth(self.ctx.h, self.h, seed, std, npos),
              "si_kv_fill_synth")

    def free(self):
        if self.h:
            self.ctx.L.si_kv_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass
