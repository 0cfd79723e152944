"""GPU parity of the column-SoA (fused) entry points and the batched prefill,
called with the reference's signatures through the C ABI.

* fused_column_matvec (fused_layer.h:169) on tiles packed by the oracle's
  restatement of repack_weights.py (itself pinned to the reference's tiles by
  sha256 in test_oracle.py): bit-exact against the reference's own output.
* run_layer_fused (register_fusion.h:344) against the reference's fused
  outputs: same bars as run_layer.
* pf_run_batch (prefill_weight_stationary.h:183) against the reference's
  prefill oracle, sequential decode with context prefix+t+1
  (bench_ai_dma_prefill.c:104-108).
"""
import ctypes as C

import numpy as np
import pytest

from common import DIMS_15B, assert_close, assert_layer_close, stream, xs_kv_history, xs_layer
from golden.make_golden import LAYER_SEED, RUN_CASES, x_pattern

pytestmark = pytest.mark.gpu

ATT_ATOL, ATT_RTOL = 1e-5, 1e-4
LAYER_RTOL = 1e-3


class LayerT(C.Structure):  # defines.h:30-33
    _fields_ = [(n, C.c_void_p) for n in ("wq", "wk", "wv", "wo", "norm", "bq", "bk", "bv")]


class FusedWeightsT(C.Structure):  # fused_layer.h:59-66
    _fields_ = [("q", C.c_void_p), ("kv", C.c_void_p), ("o", C.c_void_p), ("tcm_fd", C.c_int),
                ("tcm_map", C.c_void_p), ("tcm_tile", C.c_void_p), ("tcm_map_bytes", C.c_size_t),
                ("tcm_block", C.c_int)]


class PhaseT(C.Structure):  # defines.h:35-37
    _fields_ = [(n, C.c_float) for n in ("rms", "q8_input", "q_proj", "k_proj", "v_proj",
                                         "rope_cache", "attention", "q8_output", "out_proj")]


class FusedStatsT(C.Structure):  # fused_layer.h:68-71
    _fields_ = [("phase", PhaseT), ("tcm_stage", C.c_double)]


class PfWorkspaceT(C.Structure):  # prefill_weight_stationary.h:149-155
    _fields_ = [("xin", C.c_void_p), ("oq", C.c_void_p), ("acc", C.c_void_p), ("cv", C.c_void_p),
                ("sv", C.c_void_p), ("capacity", C.c_int)]


def colsoa_tiles(oc, layer):
    """q / kv / o column-SoA blobs, as repack_weights.py writes them."""
    q = np.concatenate([oc.pack_colsoa_tile(layer["wq"], layer["wq"], 1536, p * 256,
                                            p * 256 + 128, 0, 48) for p in range(6)])
    kv = np.concatenate([oc.pack_colsoa_tile(layer["wk"], layer["wv"], 1536, g * 128, g * 128,
                                             0, 48) for g in range(2)])
    o = np.concatenate([oc.pack_colsoa_tile(layer["wo"], layer["wo"], 1536, t * 256,
                                            t * 256 + 128, p * 256, 8)
                        for p in range(6) for t in range(6)])
    return {"q": q, "kv": kv, "o": o}


def layer_t(layer):
    return LayerT(*[layer[k].ctypes.data if layer[k] is not None else None
                    for k in ("wq", "wk", "wv", "wo", "norm", "bq", "bk", "bv")])


def fused_t(tiles):
    return FusedWeightsT(tiles["q"].ctypes.data, tiles["kv"].ctypes.data, tiles["o"].ctypes.data,
                         -1, None, None, 0, 0)


def bind(L):
    L.fused_column_matvec.restype = None
    L.fused_column_matvec.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p,
                                      C.c_void_p, C.c_int]
    L.si_ref_run_layer_fused.restype = FusedStatsT
    L.si_ref_run_layer_fused.argtypes = ([C.c_void_p] * 5 + [C.c_int] + [C.c_void_p] * 3 +
                                         [C.c_int] * 4 + [C.c_float] * 2)
    L.si_ref_pf_workspace_open.restype = None
    L.si_ref_pf_workspace_open.argtypes = [C.c_void_p, C.c_int, C.c_int]
    L.pf_workspace_close.restype = None
    L.pf_workspace_close.argtypes = [C.c_void_p]
    L.si_ref_pf_run_batch.restype = None
    L.si_ref_pf_run_batch.argtypes = ([C.c_void_p] * 5 + [C.c_int] * 2 + [C.c_void_p] * 3 +
                                      [C.c_int] * 4 + [C.c_float] * 2)
    L.fused_weights_free.restype = None
    L.fused_weights_free.argtypes = [C.c_void_p]
    return L


def forget(L, layer, tiles):
    for k in ("wq", "wk", "wv", "wo"):
        L.si_forget_host_weights(layer[k].ctypes.data)
    for t in tiles.values():
        L.si_forget_host_weights(t.ctypes.data)


def test_fused_column_matvec_golden(si_ctx, golden, oc):
    L = bind(si_ctx.L)
    layer = xs_layer(oc, DIMS_15B, LAYER_SEED)
    tiles = colsoa_tiles(oc, layer)
    q8 = oc.quantize_q8(stream(oc, 21, 1536))
    bq = np.ascontiguousarray(layer["bq"][:256])
    out = np.zeros(256, np.float32)
    tile0 = np.ascontiguousarray(tiles["q"][:245760])
    L.fused_column_matvec(tile0.ctypes.data, q8.ctypes.data, 48, bq.ctypes.data,
                          bq[128:].ctypes.data, out.ctypes.data, 0)
    np.testing.assert_array_equal(out, golden["fcm_q_tile0"])
    # add mode over an O subtile (8 groups), twice in a row: output accumulates
    # in block order exactly as the oracle's restatement does.
    sub = np.ascontiguousarray(tiles["o"][:8 * 5120])
    acc = stream(oc, 22, 256, 0.5)
    want = oc.fused_column_matvec(sub, q8, 8, None, None, acc.copy(), add=1)
    want = oc.fused_column_matvec(sub, q8, 8, None, None, want, add=1)
    got = acc.copy()
    for _ in range(2):
        L.fused_column_matvec(sub.ctypes.data, q8.ctypes.data, 8, None, None, got.ctypes.data, 1)
    np.testing.assert_array_equal(got, want)
    L.si_forget_host_weights(tile0.ctypes.data)
    L.si_forget_host_weights(sub.ctypes.data)


@pytest.mark.parametrize("case", range(4))
def test_run_layer_fused_golden(si_ctx, golden, oc, case):
    L = bind(si_ctx.L)
    ctx, kscale, kind = RUN_CASES[case]
    layer = xs_layer(oc, DIMS_15B, LAYER_SEED)
    tiles = colsoa_tiles(oc, layer)
    x = x_pattern(oc, kind, 100 + case)
    kc, vc = xs_kv_history(oc, 200 + case, ctx, 256, kscale=kscale)
    lt, fw = layer_t(layer), fused_t(tiles)
    y = np.zeros(1536, np.float32)
    att = np.zeros(1536, np.float32)
    q8 = np.zeros(48 * 34, np.uint8)
    st = L.si_ref_run_layer_fused(C.addressof(lt), C.addressof(fw), x.ctypes.data, kc.ctypes.data,
                                  vc.ctypes.data, ctx, y.ctypes.data, att.ctypes.data,
                                  q8.ctypes.data, 1536, 12, 2, 128, 1e6, 1e-6)
    assert st.tcm_stage == 0.0 and st.phase.attention > 0
    tag = f"fused{case}"
    assert_close(golden[tag + "_attn"], att, ATT_ATOL, ATT_RTOL, "attention output")
    ref_blocks = golden[tag + "_q8"].reshape(48, 34)
    diff = int((q8.reshape(48, 34) != ref_blocks).any(axis=1).sum())
    assert diff <= 2, f"{diff}/48 Q8 blocks differ"
    if diff == 0:
        np.testing.assert_array_equal(y, golden[tag + "_y"])
    assert_layer_close(golden[tag + "_y"], y, LAYER_RTOL, "layer output")
    # The fused schedule computes run_layer: the new KV slot matches the
    # reference's run_layer on the same input.
    k2, v2 = kc.copy(), vc.copy()
    oc.run_layer(DIMS_15B, layer, x, k2, v2, ctx, 1)
    np.testing.assert_array_equal(kc, k2)
    np.testing.assert_array_equal(vc, v2)
    forget(L, layer, tiles)


@pytest.mark.parametrize("prefix,ntok", [(0, 1), (5, 24), (40, 9)])
def test_pf_run_batch_vs_sequential_decode(si_ctx, oc, prefix, ntok):
    L = bind(si_ctx.L)
    layer = xs_layer(oc, DIMS_15B, 77)
    tiles = colsoa_tiles(oc, layer)
    total = prefix + ntok
    kc, vc = xs_kv_history(oc, 78, prefix + 1, 256, total=total)
    x = stream(oc, 79, ntok * 1536).reshape(ntok, 1536)
    lt, fw = layer_t(layer), fused_t(tiles)
    ws = PfWorkspaceT()
    L.si_ref_pf_workspace_open(C.addressof(ws), ntok + 3, 1536)
    assert ws.capacity == ntok + 3 and ws.xin
    y = np.zeros((ntok, 1536), np.float32)
    kg, vg = kc.copy(), vc.copy()
    L.si_ref_pf_run_batch(C.addressof(lt), C.addressof(fw), None, C.addressof(ws), x.ctypes.data,
                          ntok, prefix, kg.ctypes.data, vg.ctypes.data, y.ctypes.data,
                          1536, 12, 2, 128, 1e6, 1e-6)
    L.pf_workspace_close(C.addressof(ws))
    assert ws.capacity == 0 and not ws.xin
    dims = dict(DIMS_15B, rope_theta=1e6, rms_eps=1e-6, intermediate=0)
    k2, v2 = kc.copy(), vc.copy()
    want = oc.prefill_sequential(dims, layer, x, prefix, k2, v2)
    assert_layer_close(want, y, LAYER_RTOL, "prefill output")
    np.testing.assert_array_equal(kg, k2)
    np.testing.assert_array_equal(vg, v2)
    forget(L, layer, tiles)
