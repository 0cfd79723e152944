"""Parity at the full sizes of the BASELINE configurations, through properties
that do not depend on size plus oracle checks on sampled tokens.

* config 1 (1.5B projection sweep, M in {1, 16, 128, 512, 2048}): both GEMMs
  (tcgen05, mma.sync) equal the in-order GEMV element for element at M = 16, 128, 512
  (M = 2048 is in test_gpu_gemm.py, M = 1 is the GEMV itself).
* config 2 (7B layer, 2048-token prefill, then decode): with the exact
  attention kernel the prefill equals 2048 sequential decode steps (the
  reference's prefill oracle, bench_ai_dma_prefill.c:104-108) bit for bit --
  outputs and KV cache: the projections keep the reference's block order in
  both kernels and a token's attention splits depend only on its own context
  length; the decode steps after it match the oracle's decoder layer.  The
  tensor-core prefill attention (the default) is checked in
  test_gpu_attention_tc.py.
* config 3 (7B, batch 64, fp32 KV of 4096 positions): the batched decode step
  (GEMM gate/up projection) equals single-sequence decode steps (GEMV) bit
  for bit, and matches the oracle's decoder layer on sampled sequences.
"""
import numpy as np
import pytest

from common import assert_layer_close

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

DIMS_7B = dict(hidden=3584, n_q_heads=28, n_kv_heads=4, head_dim=128, intermediate=18944,
               rope_theta=1e6, rms_eps=1e-6)
LAYER_RTOL = 1e-3


def z(n, dt=torch.float32):
    t = torch.zeros(n, dtype=dt, device="cuda")
    torch.cuda.synchronize()  # the fill runs on torch's stream, the kernels on the library's
    return t


@pytest.mark.parametrize("kernel", [1, 4], ids=["tcgen05", "mma"])
@pytest.mark.parametrize("M", [16, 128, 512])
@pytest.mark.parametrize("name,N,K", [("qkv", 2048, 1536), ("o", 1536, 1536),
                                      ("gate", 8960, 1536), ("down", 1536, 8960)])
def test_config1_sweep_gemm_equals_gemv(si_ctx, name, N, K, M, kernel):
    m = si_ctx.matrix_synth(N, K, seed=1000 + N + K)
    x = torch.randn(M, K, device="cuda", generator=torch.Generator("cuda").manual_seed(M))
    torch.cuda.synchronize()
    qs, d = z(M * K, torch.int8), z(M * K // 32, torch.int16)
    si_ctx.q8_quantize(x, M, K, qs, d)
    a, b = z(M * N), z(M * N)
    si_ctx.matmul(m, qs, d, M, None, a, kernel=kernel)
    si_ctx.matmul(m, qs, d, M, None, b, kernel=0)
    si_ctx.status()
    assert torch.isfinite(a).all() and torch.equal(a, b)
    m.free()


def test_config2_prefill_then_decode(si_ctx, oc):
    si_ctx.set_exact_attention(True)
    try:
        _config2_prefill_then_decode(si_ctx, oc)
    finally:
        si_ctx.set_exact_attention(False)


def _config2_prefill_then_decode(si_ctx, oc):
    import sib200
    ntok, ndec = 2048, 4
    L = ntok + ndec
    layer = si_ctx.layer_synth(DIMS_7B, 2)
    g = torch.Generator("cuda").manual_seed(2)
    X = torch.randn(ntok + ndec, DIMS_7B["hidden"], device="cuda", generator=g)
    torch.cuda.synchronize()
    # Prefill all 2048 tokens at once ...
    kva = si_ctx.kv(DIMS_7B, 1, L, False)
    ya = torch.zeros(ntok, DIMS_7B["hidden"], device="cuda")
    torch.cuda.synchronize()
    layer.prefill_dev(kva, 0, X[:ntok], ntok, 0, ya, sib200.SI_LAYER_FULL)
    # ... and token by token.
    kvb = si_ctx.kv(DIMS_7B, 1, L, False)
    yb = torch.zeros_like(ya)
    torch.cuda.synchronize()
    for t in range(ntok):
        layer.decode_dev(kvb, X[t], [t + 1], yb[t], sib200.SI_LAYER_FULL)
    si_ctx.status()
    assert torch.isfinite(ya).all()
    assert torch.equal(ya, yb)
    kvd = DIMS_7B["n_kv_heads"] * DIMS_7B["head_dim"]
    ka, va = np.zeros((ntok, kvd), np.uint16), np.zeros((ntok, kvd), np.uint16)
    kb, vb = np.zeros_like(ka), np.zeros_like(va)
    kva.read(0, 0, ntok, ka, va)
    kvb.read(0, 0, ntok, kb, vb)
    np.testing.assert_array_equal(ka, kb)
    np.testing.assert_array_equal(va, vb)
    # Decode after the prefill, checked against the oracle on the last step.
    yd = torch.zeros(ndec, DIMS_7B["hidden"], device="cuda")
    torch.cuda.synchronize()
    for i in range(ndec):
        layer.decode_dev(kva, X[ntok + i], [ntok + i + 1], yd[i], sib200.SI_LAYER_FULL)
    si_ctx.status()
    host = layer.host()
    n = ntok + ndec
    kh, vh = np.zeros((n, kvd), np.uint16), np.zeros((n, kvd), np.uint16)
    kva.read(0, 0, n - 1, kh[:n - 1], vh[:n - 1])
    want = oc.decoder_layer(DIMS_7B, host, X[n - 1].cpu().numpy(), kh.reshape(-1),
                            vh.reshape(-1), n)
    assert_layer_close(want, yd[ndec - 1].cpu().numpy(), LAYER_RTOL, "decode after prefill")
    for o in (kva, kvb, layer):
        o.free()


def test_config3_batched_decode(si_ctx, oc):
    import sib200
    B, ctx_len = 64, 4096
    layer = si_ctx.layer_synth(DIMS_7B, 3)
    kv = si_ctx.kv(DIMS_7B, B, ctx_len, True)
    kv.fill_synth(3, 1.0, ctx_len - 1)
    g = torch.Generator("cuda").manual_seed(3)
    X = torch.randn(B, DIMS_7B["hidden"], device="cuda", generator=g)
    Y = torch.zeros_like(X)
    torch.cuda.synchronize()
    layer.decode_dev(kv, X, [ctx_len] * B, Y, sib200.SI_LAYER_FULL)
    si_ctx.status()
    assert torch.isfinite(Y).all()
    host = layer.host()
    kvd = DIMS_7B["n_kv_heads"] * DIMS_7B["head_dim"]
    for b in (0, 37, B - 1):
        k = np.zeros((ctx_len, kvd), np.float32)
        v = np.zeros_like(k)
        kv.read(b, 0, ctx_len - 1, k[:ctx_len - 1], v[:ctx_len - 1])
        one = si_ctx.kv(DIMS_7B, 1, ctx_len, True)
        one.write(0, 0, k[:ctx_len - 1], v[:ctx_len - 1])
        y1 = torch.zeros(DIMS_7B["hidden"], device="cuda")
        torch.cuda.synchronize()
        layer.decode_dev(one, X[b], [ctx_len], y1, sib200.SI_LAYER_FULL)
        si_ctx.status()
        assert torch.equal(y1, Y[b]), f"sequence {b}: batched != single"
        one.free()
        want = oc.decoder_layer(DIMS_7B, host, X[b].cpu().numpy(), k.reshape(-1),
                                v.reshape(-1), ctx_len)
        assert_layer_close(want, Y[b].cpu().numpy(), LAYER_RTOL, f"sequence {b}")
    kv.free()
    layer.free()


@pytest.mark.parametrize("hq,hkv,hd", [(14, 2, 64), (12, 2, 128), (8, 8, 128), (16, 2, 128)])
@pytest.mark.parametrize("kv_f32", [False, True])
def test_prefill_kernel_equals_decode_kernel(hq, hkv, hd, kv_f32):
    """The flash-style prefill attention (contiguous tokens, splits walked in one
    CTA) and the split decode attention (one token per step) evaluate a token by
    the same procedure: a 150-token prefill after a 130-position history (three
    splits, ragged last query tile) equals 150 decode steps bit for bit, for
    group sizes 7, 6, 1 and 8, head_dim 64 and 128, fp16 and fp32 caches."""
    import sib200
    dims = dict(hidden=hq * hd, n_q_heads=hq, n_kv_heads=hkv, head_dim=hd, intermediate=0,
                rope_theta=1e6, rms_eps=1e-6)
    prefix, ntok = 130, 150
    L = prefix + ntok
    ctx = sib200.Context(0, 4096, 1e6, hd)
    ctx.set_exact_attention(True)
    try:
        layer = ctx.layer_synth(dims, 11 + hq)
        g = torch.Generator("cuda").manual_seed(hq + hkv)
        X = torch.randn(ntok, dims["hidden"], device="cuda", generator=g)
        ya, yb = torch.zeros_like(X), torch.zeros_like(X)
        kva, kvb = ctx.kv(dims, 1, L, kv_f32), ctx.kv(dims, 1, L, kv_f32)
        kva.fill_synth(7, 1.0, prefix)
        kvb.fill_synth(7, 1.0, prefix)
        torch.cuda.synchronize()
        layer.prefill_dev(kva, 0, X, ntok, prefix, ya, sib200.SI_LAYER_ATTN)
        for t in range(ntok):
            layer.decode_dev(kvb, X[t], [prefix + t + 1], yb[t], sib200.SI_LAYER_ATTN)
        ctx.status()
        assert torch.isfinite(ya).all()
        assert torch.equal(ya, yb)
        for o in (kva, kvb, layer):
            o.free()
    finally:
        ctx.close()
