"""CPU tests: the oracle restatement is pinned to the reference.

Two anchors: (1) golden vectors produced by the reference's own code
(tests/golden/make_golden.py), checked bit-for-bit; (2) where the reference
checkout exists, the reference translation unit itself (oracle/_ref) on fresh
inputs.  Only after these pass is the oracle used to check the CUDA path.
"""
import hashlib

import numpy as np
import pytest

from common import DIMS_15B, stream, xs_kv_history, xs_layer, synth
from golden.make_golden import LAYER_SEED, RUN_CASES, q8_inputs, x_pattern


def test_f16_conversions_match_golden(oc, golden):
    f32 = np.array([oc.lib.oc_f16_to_f32(int(h)) for h in range(65536)], np.float32)
    digest = hashlib.sha256(f32.view(np.uint32).tobytes()).digest()
    assert digest == golden["f16_to_f32_sha256"].tobytes()
    bits = golden["f32_bits"]
    got = np.array([oc.lib.oc_f32_to_f16(float(v)) for v in bits.view(np.float32)], np.uint16)
    np.testing.assert_array_equal(got, golden["f32_to_f16"])


def test_numpy_f16_rounding_matches_reference(golden):
    """numpy's float32->float16 (used to build fixtures) rounds like f32_to_f16 for finite values."""
    bits = golden["f32_bits"]
    vals = bits.view(np.float32)
    fin = np.isfinite(vals)
    with np.errstate(over="ignore"):
        got = vals[fin].astype(np.float16).view(np.uint16)
    np.testing.assert_array_equal(got, golden["f32_to_f16"][fin])


def test_q8_quantizer_matches_golden(oc, golden):
    qx = q8_inputs(oc)
    np.testing.assert_array_equal(qx, golden["q8_x"])
    for r in range(qx.shape[0]):
        np.testing.assert_array_equal(oc.quantize_q8(qx[r]), golden["q8_out"][r])


def test_q8_rejects_ragged_length(oc):
    with pytest.raises(ValueError):
        oc.quantize_q8(np.zeros(33, np.float32))


def test_matvec_and_block_sums_match_golden(oc, golden):
    layer = xs_layer(oc, DIMS_15B, LAYER_SEED)
    q8 = oc.quantize_q8(stream(oc, 21, 1536))
    w = layer["wq"][:256]
    np.testing.assert_array_equal(oc.matvec(w, q8, 1536, 256, layer["bq"][:256]),
                                  golden["mv_out_bias"])
    np.testing.assert_array_equal(oc.matvec(w, q8, 1536, 256), golden["mv_out"])
    np.testing.assert_array_equal(oc.block_isums(w, q8, 1536, 256), golden["mv_isum"])


def test_rmsnorm_rope_match_golden(oc, golden):
    layer = xs_layer(oc, DIMS_15B, LAYER_SEED)
    rx = stream(oc, 31, 1536, 2.0)
    np.testing.assert_array_equal(oc.rmsnorm(rx, layer["norm"]), golden["rms_out"])
    np.testing.assert_array_equal(oc.rmsnorm(rx, None), golden["rms_out_noweight"])
    heads = stream(oc, 41, 12 * 128)
    for i, p in enumerate(golden["rope_pos"]):
        np.testing.assert_array_equal(oc.rope(heads, 12, int(p), 128), golden["rope_out"][i])


def test_rope_table_matches_rope(oc):
    heads = stream(oc, 42, 4 * 64)
    c, s = oc.rope_table(0, 300, 64)
    for p in (0, 7, 299):
        want = oc.rope(heads, 4, p, 64)
        h = heads.reshape(4, 64)
        got = np.empty_like(h)
        with np.errstate(all="ignore"):
            a, b = h[:, :32], h[:, 32:]
            got[:, :32] = (a * c[p]).astype(np.float32) - (b * s[p]).astype(np.float32)
            got[:, 32:] = (b * c[p]).astype(np.float32) + (a * s[p]).astype(np.float32)
        np.testing.assert_array_equal(got.reshape(-1), want)


def test_attention_matches_golden(oc, golden):
    qa = stream(oc, 0x91BE2145, 1536, 1.5)
    kc = stream(oc, 0x91BE2146, 64 * 256, 1.5).astype(np.float16).view(np.uint16)
    vc = stream(oc, 0x91BE2147, 64 * 256, 1.5).astype(np.float16).view(np.uint16)
    for i, c in enumerate(golden["attn_ctx"]):
        np.testing.assert_array_equal(oc.attention(DIMS_15B, qa, kc, vc, int(c), 1),
                                      golden["attn_flash"][i])
        np.testing.assert_array_equal(oc.attention(DIMS_15B, qa, kc, vc, int(c), 0),
                                      golden["attn_standard"][i])


@pytest.mark.parametrize("case", range(len(RUN_CASES)))
def test_run_layer_matches_golden(oc, golden, case):
    ctx, kscale, kind = RUN_CASES[case]
    layer = xs_layer(oc, DIMS_15B, LAYER_SEED)
    x = x_pattern(oc, kind, 100 + case)
    for method in (1, 0):
        kc, vc = xs_kv_history(oc, 200 + case, ctx, 256, kscale=kscale)
        y, att, q8 = oc.run_layer(DIMS_15B, layer, x, kc, vc, ctx, method, captures=True)
        tag = f"run{case}_{'flash' if method else 'standard'}"
        np.testing.assert_array_equal(y, golden[tag + "_y"])
        np.testing.assert_array_equal(att, golden[tag + "_attn"])
        np.testing.assert_array_equal(q8, golden[tag + "_q8"])
        np.testing.assert_array_equal(kc[(ctx - 1) * 256:], golden[tag + "_knew"])
        np.testing.assert_array_equal(vc[(ctx - 1) * 256:], golden[tag + "_vnew"])


def test_colsoa_pack_matches_reference_repack(oc, golden):
    layer = xs_layer(oc, DIMS_15B, LAYER_SEED)
    q = np.concatenate([oc.pack_colsoa_tile(layer["wq"], layer["wq"], 1536, p * 256,
                                            p * 256 + 128, 0, 48) for p in range(6)])
    kv = np.concatenate([oc.pack_colsoa_tile(layer["wk"], layer["wv"], 1536, g * 128, g * 128,
                                             0, 48) for g in range(2)])
    o = np.concatenate([oc.pack_colsoa_tile(layer["wo"], layer["wo"], 1536, t * 256,
                                            t * 256 + 128, p * 256, 8)
                        for p in range(6) for t in range(6)])
    for name, t in (("q", q), ("kv", kv), ("o", o)):
        assert hashlib.sha256(t.tobytes()).digest() == golden[f"colsoa_{name}_sha256"].tobytes()
    q8 = oc.quantize_q8(stream(oc, 21, 1536))
    np.testing.assert_array_equal(
        oc.fused_column_matvec(q[:245760], q8, 48, layer["bq"][:128], layer["bq"][128:256]),
        golden["fcm_q_tile0"])


def test_numpy_q4_quantizer_matches_oracle(oc):
    rng = np.random.default_rng(7)
    w = rng.normal(0, 0.02, size=(64, 256)).astype(np.float32)
    w[0, :32] = 0.0                  # all-zero block: d = 0
    w[1, 5] = -0.5                   # negative signed max
    w[2, :32] = 1e-9                 # subnormal-fp16 scale
    np.testing.assert_array_equal(synth.q4_0_quantize(w), oc.quantize_q4_0(w))


def test_prefill_sequential_is_decode_loop(oc):
    dims = dict(hidden=256, n_q_heads=4, n_kv_heads=2, head_dim=64, intermediate=0)
    layer = xs_layer(oc, dims, 9)
    x = stream(oc, 10, 5 * 256).reshape(5, 256)
    kc, vc = xs_kv_history(oc, 11, 4, 128, total=8)
    k2, v2 = kc.copy(), vc.copy()
    y = oc.prefill_sequential(dims, layer, x, 3, kc, vc)
    for t in range(5):
        np.testing.assert_array_equal(oc.run_layer(dims, layer, x[t], k2, v2, 3 + t + 1), y[t])
    np.testing.assert_array_equal(kc, k2)


# ---- live reference (only where the reference checkout was built) -----------

def test_oracle_equals_reference_on_fresh_inputs(oc, ref):
    for seed in range(3):
        x = stream(oc, 1000 + seed, 1536, 4.0)
        np.testing.assert_array_equal(oc.quantize_q8(x), ref.quantize_q8(x))
        layer = xs_layer(oc, DIMS_15B, 77 + seed)
        q8 = ref.quantize_q8(x)
        np.testing.assert_array_equal(oc.matvec(layer["wk"], q8, 1536, 256, layer["bk"]),
                                      ref.matvec(layer["wk"], q8, 1536, 256, layer["bk"]))
        np.testing.assert_array_equal(oc.rmsnorm(x, layer["norm"]),
                                      ref.rmsnorm(x, layer["norm"]))
        ctx = 33 + seed
        k0, v0 = xs_kv_history(oc, 5 + seed, ctx, 256)
        ka, va = k0.copy(), v0.copy()
        kb, vb = k0.copy(), v0.copy()
        y0, a0, q0 = oc.run_layer(DIMS_15B, layer, x, ka, va, ctx, 1, captures=True)
        y1, a1, q1 = ref.run_layer(layer, x, kb, vb, ctx, 1)
        np.testing.assert_array_equal(y0, y1)
        np.testing.assert_array_equal(a0, a1)
        np.testing.assert_array_equal(q0, q1)
        np.testing.assert_array_equal(ka, kb)


def test_reference_rng_is_restated(oc, ref):
    ref.seed(0x5217AC8B)
    oc.seed(0x5217AC8B)
    np.testing.assert_array_equal(ref.random_floats(1000), oc.random_floats(1000))
