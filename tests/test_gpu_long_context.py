"""Long-context parity: decode and prefill attention at 8192 and 32768 positions.

The reference accepts contexts up to 32768 (qwen_one_layer.c:608, the
`context` argument's range check).  These cases run the CUDA path there, at the
reference's own attention-layer dims (1536 hidden, 12 Q / 2 KV heads,
head_dim 128) with its fp16 cache and with fp32, against the oracle's
attention_flash (attention_kernels.h:80-164) to the reference's attention bar
(1e-5 + 1e-4 |x|, audit_fusion_timing.c:108), and the drop-in run_layer
against the oracle's run_layer (qwen_one_layer.c:237-281) -- and against the
reference's own run_layer where oracle/_ref is built -- to the layer bar 1e-3.
Each case prints the largest attention error relative to the output's scale
so growth with the context shows in the log.
"""
import ctypes as C

import numpy as np
import pytest

from common import DIMS_15B, assert_close, assert_layer_close, stream, xs_kv_history, xs_layer
from golden.make_golden import LAYER_SEED

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

ATT_ATOL, ATT_RTOL = 1e-5, 1e-4
LAYER_RTOL = 1e-3
ATT15 = dict(DIMS_15B, intermediate=0, rope_theta=1e6, rms_eps=1e-6)


def _scale_err(want, got):
    want = np.asarray(want, np.float64)
    return float(np.max(np.abs(np.asarray(got, np.float64) - want)) / np.max(np.abs(want)))


def _history(rng, L, kvd, f32):
    k = rng.standard_normal((L, kvd)).astype(np.float32)
    v = rng.standard_normal((L, kvd)).astype(np.float32)
    if not f32:
        k, v = k.astype(np.float16).view(np.uint16), v.astype(np.float16).view(np.uint16)
    return k, v


@pytest.mark.parametrize("kv_f32", [False, True])
def test_decode_attention_long_context(si_ctx, oc, kv_f32):
    """Three sequences at 8192, 20000 and 32768 positions in one decode launch."""
    ctxs = [8192, 20000, 32768]
    B, L = len(ctxs), max(ctxs)
    D, Hq, Hkv = ATT15["head_dim"], ATT15["n_q_heads"], ATT15["n_kv_heads"]
    rng = np.random.default_rng(8192 + int(kv_f32))
    kv = si_ctx.kv(ATT15, B, L, kv_f32)
    hist = []
    for b, n in enumerate(ctxs):
        k, v = _history(rng, n, Hkv * D, kv_f32)
        kv.write(b, 0, k, v)
        hist.append((k, v))
    q = (rng.standard_normal((B, Hq * D)) * 2).astype(np.float32)
    qd = torch.from_numpy(q).cuda()
    out = torch.zeros(B * Hq * D, device="cuda")
    torch.cuda.synchronize()
    si_ctx.attention_decode(kv, ATT15, qd, B, ctxs, out)
    si_ctx.status()
    got = out.cpu().numpy().reshape(B, -1)
    for b, n in enumerate(ctxs):
        k, v = hist[b]
        want = oc.attention(ATT15, q[b], k.reshape(-1), v.reshape(-1), n, 1)
        print(f"\ndecode attention ctx {n} ({'fp32' if kv_f32 else 'fp16'} KV): "
              f"max err / scale {_scale_err(want, got[b]):.3g}")
        assert_close(want, got[b], ATT_ATOL, ATT_RTOL, f"decode attention ctx={n}")
    kv.free()


@pytest.mark.parametrize("exact", [False, True], ids=["tcgen05", "exact"])
@pytest.mark.parametrize("kv_f32", [False, True])
def test_prefill_attention_long_prefix(si_ctx, oc, kv_f32, exact):
    """A 96-token prefill chunk whose last token sits at position 32767 (prefix
    32672, mid-tile for both kernels), every checked token against the oracle
    at context prefix + t + 1."""
    D, Hq, Hkv = ATT15["head_dim"], ATT15["n_q_heads"], ATT15["n_kv_heads"]
    L, ntok = 32768, 96
    prefix = L - ntok
    rng = np.random.default_rng(32768 + 2 * int(kv_f32) + int(exact))
    k, v = _history(rng, L, Hkv * D, kv_f32)
    kv = si_ctx.kv(ATT15, 1, L, kv_f32)
    kv.write(0, 0, k, v)
    q = (rng.standard_normal((ntok, Hq * D)) * 2).astype(np.float32)
    qd = torch.from_numpy(q).cuda()
    out = torch.zeros(ntok * Hq * D, device="cuda")
    torch.cuda.synchronize()
    si_ctx.set_exact_attention(exact)
    try:
        si_ctx.attention_prefill(kv, ATT15, qd, ntok, 0, prefix, out)
    finally:
        si_ctx.set_exact_attention(False)
    si_ctx.status()
    got = out.cpu().numpy().reshape(ntok, -1)
    worst = 0.0
    for t in (0, 1, 31, 32, 63, 64, ntok - 1):
        n = prefix + t + 1
        want = oc.attention(ATT15, q[t], k[:n].reshape(-1), v[:n].reshape(-1), n, 1)
        worst = max(worst, _scale_err(want, got[t]))
        assert_close(want, got[t], ATT_ATOL, ATT_RTOL, f"prefill token {t} ctx {n}")
    print(f"\nprefill attention at prefix {prefix} ({'exact' if exact else 'tcgen05'}, "
          f"{'fp32' if kv_f32 else 'fp16'} KV): max err / scale {worst:.3g}")
    kv.free()


class _LayerT(C.Structure):  # layer_t, qwen_one_layer.c:75-86
    _fields_ = [(n, C.c_void_p) for n in ("wq", "wk", "wv", "wo", "norm", "bq", "bk", "bv")]


class _PhaseT(C.Structure):  # phase_t, defines.h:35-37, returned by value
    _fields_ = [(n, C.c_float) for n in ("rms", "q8_input", "q_proj", "k_proj", "v_proj",
                                         "rope_cache", "attention", "q8_output", "out_proj")]


@pytest.mark.parametrize("context", [8192, 32768])
def test_run_layer_long_context(si_ctx, oc, request, context):
    """The drop-in run_layer (host buffers, fp16 KV, flash attention) at the
    reference's largest contexts: against the oracle's run_layer, and against
    the reference's own run_layer when oracle/_ref is built."""
    layer = xs_layer(oc, DIMS_15B, LAYER_SEED)
    x = stream(oc, 0x1000 + context, 1536, 1.0)
    kc, vc = xs_kv_history(oc, 0x2000 + context, context, 256)
    k0, v0 = kc.copy(), vc.copy()
    lt = _LayerT(*[layer[k].ctypes.data for k in ("wq", "wk", "wv", "wo", "norm", "bq", "bk",
                                                  "bv")])
    y = np.zeros(1536, np.float32)
    att = np.zeros(1536, np.float32)
    q8 = np.zeros(48 * 34, np.uint8)
    L = si_ctx.L
    L.si_ref_run_layer.restype = _PhaseT
    L.si_ref_run_layer.argtypes = ([C.c_void_p] * 4 + [C.c_int, C.c_void_p, C.c_int] +
                                   [C.c_void_p] * 3 + [C.c_int] * 4 + [C.c_float] * 2)
    try:
        L.si_ref_run_layer(C.addressof(lt), x.ctypes.data, kc.ctypes.data, vc.ctypes.data,
                           context, y.ctypes.data, 1, None, att.ctypes.data, q8.ctypes.data,
                           1536, 12, 2, 128, 1e6, 1e-6)
    finally:
        for k in ("wq", "wk", "wv", "wo"):
            L.si_forget_host_weights(layer[k].ctypes.data)
    ko, vo = k0.copy(), v0.copy()
    want = oc.run_layer(ATT15, layer, x, ko, vo, context)
    # the appended K/V row (RoPE'd, fp16) is bit-identical to the oracle's
    np.testing.assert_array_equal(kc, ko)
    np.testing.assert_array_equal(vc, vo)
    print(f"\nrun_layer ctx {context}: max err / scale vs oracle {_scale_err(want, y):.3g}")
    assert_layer_close(want, y, LAYER_RTOL, f"run_layer ctx={context} vs oracle")
    import os
    import oracle as oracle_mod
    if os.path.exists(oracle_mod.LIB_REF):
        ref = request.getfixturevalue("ref")
        kr, vr = k0.copy(), v0.copy()
        yr, attr, _ = ref.run_layer(layer, x, kr, vr, context)
        print(f"run_layer ctx {context}: max err / scale vs reference {_scale_err(yr, y):.3g}, "
              f"attention {_scale_err(attr, att):.3g}")
        assert_close(attr, att, ATT_ATOL, ATT_RTOL, f"attention ctx={context} vs reference")
        assert_layer_close(yr, y, LAYER_RTOL, f"run_layer ctx={context} vs reference")
