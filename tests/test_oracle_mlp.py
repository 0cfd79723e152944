"""The parts of the decoder layer the reference does not have (north_star MLP
and residuals) are pinned only by the oracle's restatement.  This checks the
restatement's wiring independently: numpy rebuilds the MLP and the full layer
from the oracle pieces the reference pins (RMSNorm, Q8_0 quantiser,
matvec_q4q8, run_layer's attention sublayer) -- norm2 on the residual stream,
gate and up from the same Q8 input, SiLU(g)*u in float32, its Q8, the down
projection, and the two residual adds.  numpy's float32 exp may differ from
C's expf by an ulp, which can move one Q8 rounding, hence the tolerances.
"""
from __future__ import annotations

import numpy as np

from common import synth

DIMS = dict(hidden=896, n_q_heads=14, n_kv_heads=2, head_dim=64, intermediate=4864,
            rope_theta=1e6, rms_eps=1e-6)


def _mlp_numpy(oc, layer, h):
    H, I = DIMS["hidden"], DIMS["intermediate"]
    normed = oc.rmsnorm(h, layer["norm2"], DIMS["rms_eps"])
    q = oc.quantize_q8(normed)
    gate = oc.matvec(layer["w_gate"], q, H, I)
    up = oc.matvec(layer["w_up"], q, H, I)
    g = gate.astype(np.float32)
    act = (g / (np.float32(1.0) + np.exp(-g, dtype=np.float32))).astype(np.float32) * up
    return oc.matvec(layer["w_down"], oc.quantize_q8(act.astype(np.float32)), I, H)


def test_mlp_wiring(oc):
    rng = np.random.default_rng(9)
    layer = synth.random_layer(DIMS, 9)
    for scale in (0.5, 1.0, 4.0):
        h = (rng.standard_normal(DIMS["hidden"]) * scale).astype(np.float32)
        got = oc.mlp(DIMS, layer, h)
        want = _mlp_numpy(oc, layer, h)
        assert np.all(np.isfinite(got))
        err = np.abs(got - want).max() / np.abs(want).max()
        assert err < 1e-3, err


def test_decoder_layer_residuals(oc):
    rng = np.random.default_rng(10)
    layer = synth.random_layer(DIMS, 10)
    H, KVD, ctx = DIMS["hidden"], DIMS["n_kv_heads"] * DIMS["head_dim"], 9
    kc = rng.standard_normal(ctx * KVD).astype(np.float32)
    vc = rng.standard_normal(ctx * KVD).astype(np.float32)
    x = rng.standard_normal(H).astype(np.float32)
    y = oc.decoder_layer(DIMS, layer, x, kc.copy(), vc.copy(), ctx)
    attn = oc.run_layer(DIMS, layer, x, kc.copy(), vc.copy(), ctx)
    attn = attn[0] if isinstance(attn, tuple) else attn
    h = x + attn
    want = h + oc.mlp(DIMS, layer, h)
    np.testing.assert_array_equal(y, want)
    # and with an independent MLP, within the exp tolerance
    want_np = h + _mlp_numpy(oc, layer, h)
    assert np.abs(y - want_np).max() / np.abs(want_np).max() < 1e-3
