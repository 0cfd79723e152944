"""GPU parity: the CUDA path through the C ABI against the oracle and the golden vectors.

Bars (north_star): Q8_0 activations and per-block int32 sums bit-exact; projection
outputs bit-exact here (the kernels keep the reference's block order), and in any
case within 1e-5 relative; attention within the reference's own standard-vs-flash
bar |a-b| <= 1e-5 + 1e-4*|x| (audit_fusion_timing.c:108); layer outputs within
1e-3 relative.
"""
import numpy as np
import pytest

from common import (DIMS_15B, assert_close, assert_layer_close, stream, synth, xs_kv_history,
                    xs_layer)
from golden.make_golden import LAYER_SEED, RUN_CASES, q8_inputs, x_pattern

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

ATT_ATOL, ATT_RTOL = 1e-5, 1e-4
LAYER_RTOL = 1e-3


def dev(a):
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    torch.cuda.synchronize()
    return t


def empty(n, dtype):
    """A zeroed device buffer; the fill runs on torch's stream, so wait for it
    before a library call on the library's stream writes the buffer."""
    t = torch.zeros(n, dtype=dtype, device="cuda")
    torch.cuda.synchronize()
    return t


def host(ctx, t):
    ctx.sync()
    return t.cpu().numpy()


def gpu_q8(ctx, x2d):
    M, K = x2d.shape
    x = dev(x2d.astype(np.float32))
    qs, d = empty(M * K, torch.int8), empty(M * K // 32, torch.int16)
    ctx.q8_quantize(x, M, K, qs, d)
    blocks = empty(M * K // 32 * 34, torch.uint8)
    ctx.q8_to_blocks(qs, d, M, K, blocks)
    return qs, d, host(ctx, blocks).reshape(M, -1)


def test_q8_bit_exact_golden(si_ctx, golden, oc):
    qx = q8_inputs(oc)
    _, _, blocks = gpu_q8(si_ctx, qx)
    np.testing.assert_array_equal(blocks, golden["q8_out"])


@pytest.mark.parametrize("M,K", [(1, 32), (7, 896), (64, 8960), (3, 29568)])
def test_q8_bit_exact_random(si_ctx, oc, M, K):
    x = (np.random.default_rng(M * K).standard_normal((M, K)) *
         np.random.default_rng(1).uniform(1e-3, 10, (M, 1))).astype(np.float32)
    _, _, blocks = gpu_q8(si_ctx, x)
    for m in range(M):
        np.testing.assert_array_equal(blocks[m], oc.quantize_q8(x[m]))


def test_matrix_roundtrip(si_ctx):
    w = synth.random_q4(np.random.default_rng(3), 96, 320)
    m = si_ctx.matrix(w, 96, 320)
    back = np.zeros_like(w)
    m.download(back)
    np.testing.assert_array_equal(back, w)


def test_gemv_golden_bit_exact(si_ctx, golden, oc):
    layer = xs_layer(oc, DIMS_15B, LAYER_SEED)
    q8 = oc.quantize_q8(stream(oc, 21, 1536))
    m = si_ctx.matrix(layer["wq"][:256], 256, 1536)
    qs, d = (dev(a) for a in synth.q8_split(q8, 1536))
    out = empty(256, torch.float32)
    si_ctx.matmul(m, qs, d, 1, dev(layer["bq"][:256]), out, kernel=0)
    np.testing.assert_array_equal(host(si_ctx, out), golden["mv_out_bias"])
    si_ctx.matmul(m, qs, d, 1, None, out, kernel=0)
    np.testing.assert_array_equal(host(si_ctx, out), golden["mv_out"])
    isum = empty(256 * 48, torch.int32)
    si_ctx.block_isums(m, qs, 1, isum)
    np.testing.assert_array_equal(host(si_ctx, isum).reshape(256, 48), golden["mv_isum"])


@pytest.mark.parametrize("kernel", [0, 2, 3], ids=["auto", "mma", "dp4a"])
@pytest.mark.parametrize("N,K,M", [(2048, 1536, 1), (1536, 8960, 2), (256, 896, 3),
                                   (128, 4864, 5), (512, 3584, 8), (96, 1536, 13),
                                   (5120, 512, 2), (10240, 256, 3), (32, 32, 1),
                                   (3072, 640, 4), (2368, 320, 1), (256, 1536, 16),
                                   (160, 544, 21)])
def test_gemv_bit_exact_vs_oracle(si_ctx, oc, N, K, M, kernel):
    """Both GEMV forms (dp4a; mma.sync with tokens as the 16 M-rows) against the
    oracle's matvec_q4q8, element for element; K = 544 and 32 exercise a ragged
    last chunk of the 17-block ring, M = 21 two token groups of 16."""
    rng = np.random.default_rng(N + K + M)
    w = synth.random_q4(rng, N, K)
    x = rng.standard_normal((M, K)).astype(np.float32)
    bias = rng.normal(0, 0.02, N).astype(np.float32)
    m = si_ctx.matrix(w, N, K)
    qs, d, blocks = gpu_q8(si_ctx, x)
    out = empty(M * N, torch.float32)
    si_ctx.matmul(m, qs, d, M, dev(bias), out, kernel=kernel)
    got = host(si_ctx, out).reshape(M, N)
    for t in range(M):
        np.testing.assert_array_equal(got[t], oc.matvec(w, blocks[t], K, N, bias))


@pytest.mark.parametrize("N,K", [(8192, 8192), (10240, 8192), (8192, 29568), (4608, 3584),
                                 (1280, 8192), (2560, 8192)])
@pytest.mark.parametrize("M", [1, 2, 3, 8, 16])
def test_gemv_mma_equals_dp4a_large(si_ctx, N, K, M):
    """At the 7B/72B decode shapes -- whole-tile CTAs at two or three per SM
    (10240 rows: 320 tiles; the dp4a form then streams two tiles in some
    CTAs) and half-tile CTAs for the tensor-parallel QKV shards (1280, 2560
    rows) -- the two GEMV forms return the same bits."""
    m = si_ctx.matrix_synth(N, K, seed=N + K + M)
    x = torch.randn(M, K, device="cuda", generator=torch.Generator("cuda").manual_seed(M))
    torch.cuda.synchronize()
    qs, d = empty(M * K, torch.int8), empty(M * K // 32, torch.int16)
    si_ctx.q8_quantize(x, M, K, qs, d)
    a, b = empty(M * N, torch.float32), empty(M * N, torch.float32)
    si_ctx.matmul(m, qs, d, M, None, a, kernel=2)
    si_ctx.matmul(m, qs, d, M, None, b, kernel=3)
    si_ctx.status()
    assert torch.isfinite(a).all() and torch.equal(a, b)
    m.free()


@pytest.mark.parametrize("kernel,M", [(None, 3), (2, 3), (3, 3), (2, 8), (3, 8), (2, 11),
                                      (3, 11), (2, 1)])
def test_gateup_silu_q8(si_ctx, oc, kernel, M):
    rng = np.random.default_rng(5)
    H, I = 896, 4864
    g, u = synth.random_q4(rng, I, H), synth.random_q4(rng, I, H)
    x = rng.standard_normal((M, H)).astype(np.float32)
    mg, mu = si_ctx.matrix(g, I, H), si_ctx.matrix(u, I, H)
    qs, d, blocks = gpu_q8(si_ctx, x)
    aq, ad, af = empty(M * I, torch.int8), empty(M * I // 32, torch.int16), empty(M * I, torch.float32)
    si_ctx.gateup_q8(mg, mu, qs, d, M, aq, ad, af, kernel=kernel)
    act = host(si_ctx, af).reshape(M, I)
    ablk = torch.zeros(M * I // 32 * 34, dtype=torch.uint8, device="cuda")
    torch.cuda.synchronize()
    si_ctx.q8_to_blocks(aq, ad, M, I, ablk)
    ablk = host(si_ctx, ablk).reshape(M, -1)
    for t in range(M):
        gate = oc.matvec(g, blocks[t], H, I)
        up = oc.matvec(u, blocks[t], H, I)
        want = (gate / (np.float32(1) + np.exp(-gate))).astype(np.float32) * up
        assert_close(want, act[t], 1e-7, 1e-6, "silu(gate)*up")
        # The fused Q8 equals quantising the kernel's own fp32 activation.
        np.testing.assert_array_equal(ablk[t], oc.quantize_q8(act[t]))


def test_rmsnorm_golden_and_fused_q8(si_ctx, golden, oc):
    layer = xs_layer(oc, DIMS_15B, LAYER_SEED)
    rx = stream(oc, 31, 1536, 2.0)
    x, w = dev(rx), dev(layer["norm"])
    out = empty(1536, torch.float32)
    qs, d = empty(1536, torch.int8), empty(48, torch.int16)
    si_ctx.rmsnorm_q8(x, w, 1, 1536, 1e-6, out, qs, d)
    np.testing.assert_array_equal(host(si_ctx, out), golden["rms_out"])
    blk = empty(48 * 34, torch.uint8)
    si_ctx.q8_to_blocks(qs, d, 1, 1536, blk)
    np.testing.assert_array_equal(host(si_ctx, blk), oc.quantize_q8(golden["rms_out"]))
    si_ctx.rmsnorm_q8(x, None, 1, 1536, 1e-6, out)
    np.testing.assert_array_equal(host(si_ctx, out), golden["rms_out_noweight"])


def test_reference_shaped_calls_golden(si_ctx, golden, oc):
    """quantize_q8 / matvec_q4q8 / rope / rmsnorm with the reference's signatures."""
    import ctypes as C
    L = si_ctx.L
    qx = q8_inputs(oc)
    out = np.zeros(48 * 34, np.uint8)
    L.quantize_q8(qx[0].ctypes.data, out.ctypes.data, 1536)
    np.testing.assert_array_equal(out, golden["q8_out"][0])
    layer = xs_layer(oc, DIMS_15B, LAYER_SEED)
    q8 = oc.quantize_q8(stream(oc, 21, 1536))
    w = np.ascontiguousarray(layer["wq"][:256])
    bias = np.ascontiguousarray(layer["bq"][:256])
    y = np.zeros(256, np.float32)
    L.matvec_q4q8(w.ctypes.data, q8.ctypes.data, 1536, 256, bias.ctypes.data, y.ctypes.data)
    np.testing.assert_array_equal(y, golden["mv_out_bias"])
    L.si_forget_host_weights(w.ctypes.data)
    heads = stream(oc, 41, 12 * 128)
    for i, p in enumerate(golden["rope_pos"]):
        h = heads.copy()
        L.si_ref_rope(h.ctypes.data, 12, int(p), 128, C.c_float(1e6))
        np.testing.assert_array_equal(h, golden["rope_out"][i])
    rx = stream(oc, 31, 1536, 2.0)
    o = np.zeros(1536, np.float32)
    L.si_ref_rmsnorm(rx.ctypes.data, layer["norm"].ctypes.data, o.ctypes.data, 1536, C.c_float(1e-6))
    np.testing.assert_array_equal(o, golden["rms_out"])


def test_attention_golden(si_ctx, golden, oc):
    qa = stream(oc, 0x91BE2145, 1536, 1.5)
    kc = stream(oc, 0x91BE2146, 64 * 256, 1.5).astype(np.float16).view(np.uint16)
    vc = stream(oc, 0x91BE2147, 64 * 256, 1.5).astype(np.float16).view(np.uint16)
    L = si_ctx.L
    for i, c in enumerate(golden["attn_ctx"]):
        out = np.zeros(1536, np.float32)
        L.si_ref_attention(1, qa.ctypes.data, kc.ctypes.data, vc.ctypes.data, int(c),
                           out.ctypes.data, None, 12, 2, 128)
        assert_close(golden["attn_flash"][i], out, ATT_ATOL, ATT_RTOL, f"attention ctx={c}")
        assert_close(golden["attn_standard"][i], out, ATT_ATOL, ATT_RTOL, f"attention ctx={c}")


@pytest.mark.parametrize("kv_f32", [False, True])
@pytest.mark.parametrize("dims,ctxs", [
    (dict(hidden=896, n_q_heads=14, n_kv_heads=2, head_dim=64), [1, 64, 300]),
    (dict(hidden=3584, n_q_heads=28, n_kv_heads=4, head_dim=128), [5, 1000, 4096]),
])
def test_attention_batched_vs_oracle(si_ctx, oc, dims, ctxs, kv_f32):
    B, L = len(ctxs), max(ctxs)
    D, Hq, Hkv = dims["head_dim"], dims["n_q_heads"], dims["n_kv_heads"]
    rng = np.random.default_rng(L)
    kv = si_ctx.kv(dims, B, L, kv_f32)
    ks, vs = [], []
    for b in range(B):
        k = rng.standard_normal((L, Hkv * D)).astype(np.float32)
        v = rng.standard_normal((L, Hkv * D)).astype(np.float32)
        if not kv_f32:
            k, v = k.astype(np.float16).view(np.uint16), v.astype(np.float16).view(np.uint16)
        kv.write(b, 0, k, v)
        ks.append(k)
        vs.append(v)
    q = rng.standard_normal((B, Hq * D)).astype(np.float32)
    out = empty(B * Hq * D, torch.float32)
    si_ctx.attention_decode(kv, dims, dev(q), B, ctxs, out)
    got = host(si_ctx, out).reshape(B, -1)
    for b in range(B):
        want = oc.attention(dims, q[b], ks[b].reshape(-1), vs[b].reshape(-1), ctxs[b], 1)
        assert_close(want, got[b], ATT_ATOL, ATT_RTOL, f"attention b={b} ctx={ctxs[b]}")


def test_attention_decode_rejects_empty_context(si_ctx):
    """A context length of 0 has no key to attend to: the entry point returns
    SI_ERR_INVALID instead of launching (the decode step requires >= 1 too)."""
    import sib200
    dims = dict(hidden=896, n_q_heads=14, n_kv_heads=2, head_dim=64)
    kv = si_ctx.kv(dims, 2, 16, True)
    q = empty(2 * 14 * 64, torch.float32)
    out = empty(2 * 14 * 64, torch.float32)
    with pytest.raises(sib200.SiError) as e:
        si_ctx.attention_decode(kv, dims, q, 2, [3, 0], out)
    assert e.value.status == sib200.SI_ERR_INVALID
    si_ctx.status()
    kv.free()


@pytest.mark.parametrize("case", range(len(RUN_CASES)))
def test_run_layer_golden(si_ctx, golden, oc, case):
    """run_layer with the reference's signature against the reference's own outputs."""
    import ctypes as C
    ctx, kscale, kind = RUN_CASES[case]
    layer = xs_layer(oc, DIMS_15B, LAYER_SEED)
    x = x_pattern(oc, kind, 100 + case)
    kc, vc = xs_kv_history(oc, 200 + case, ctx, 256, kscale=kscale)

    class LayerT(C.Structure):
        _fields_ = [(n, C.c_void_p) for n in ("wq", "wk", "wv", "wo", "norm", "bq", "bk", "bv")]

    lt = LayerT(*[layer[k].ctypes.data for k in ("wq", "wk", "wv", "wo", "norm", "bq", "bk", "bv")])
    y = np.zeros(1536, np.float32)
    att = np.zeros(1536, np.float32)
    q8 = np.zeros(48 * 34, np.uint8)
    class PhaseT(C.Structure):  # defines.h:35-37, returned by value
        _fields_ = [(n, C.c_float) for n in ("rms", "q8_input", "q_proj", "k_proj", "v_proj",
                                             "rope_cache", "attention", "q8_output", "out_proj")]

    L = si_ctx.L
    L.si_ref_run_layer.restype = PhaseT
    L.si_ref_run_layer.argtypes = ([C.c_void_p] * 4 + [C.c_int, C.c_void_p, C.c_int] +
                                   [C.c_void_p] * 3 + [C.c_int] * 4 + [C.c_float] * 2)
    ph = L.si_ref_run_layer(C.addressof(lt), x.ctypes.data, kc.ctypes.data, vc.ctypes.data, ctx,
                            y.ctypes.data, 1, None, att.ctypes.data, q8.ctypes.data,
                            1536, 12, 2, 128, 1e6, 1e-6)
    assert ph.q_proj > 0 and ph.attention > 0 and ph.out_proj > 0
    tag = f"run{case}_flash"
    np.testing.assert_array_equal(kc[(ctx - 1) * 256:], golden[tag + "_knew"])
    np.testing.assert_array_equal(vc[(ctx - 1) * 256:], golden[tag + "_vnew"])
    assert_close(golden[tag + "_attn"], att, ATT_ATOL, ATT_RTOL, "attention output")
    ref_blocks = golden[tag + "_q8"].reshape(48, 34)
    diff = int((q8.reshape(48, 34) != ref_blocks).any(axis=1).sum())
    assert diff <= 2, f"{diff}/48 Q8 blocks differ"
    if diff == 0:
        np.testing.assert_array_equal(y, golden[tag + "_y"])
    assert_layer_close(golden[tag + "_y"], y, LAYER_RTOL, "layer output")
    for k in ("wq", "wk", "wv", "wo"):
        L.si_forget_host_weights(layer[k].ctypes.data)


def _layer_case(oc, dims, seed, mlp):
    d = dict(dims, rope_theta=1e6, rms_eps=1e-6)
    if not mlp:
        d["intermediate"] = 0
    return d, xs_layer(oc, d, seed, mlp=mlp)


@pytest.mark.parametrize("mode", [0, 1])
def test_decode_batched_vs_oracle(si_ctx, oc, mode):
    dims, layer = _layer_case(oc, dict(hidden=896, n_q_heads=14, n_kv_heads=2, head_dim=64,
                                       intermediate=4864), 31, mlp=True)
    import sib200
    ctx64 = sib200.Context(0, 4096, 1e6, 64)
    try:
        gl = ctx64.layer(dims, layer)
        lens = [1, 9, 64, 130]
        B, L = len(lens), 160
        kv = ctx64.kv(dims, B, L, True)
        hist = []
        for b, n in enumerate(lens):
            k, v = xs_kv_history(oc, 40 + b, n, 128, f32=True, total=L)
            kv.write(b, 0, k.reshape(L, 128), v.reshape(L, 128))
            hist.append((k, v))
        x = stream(oc, 77, B * 896).reshape(B, 896)
        y = np.zeros_like(x)
        gl.decode(kv, x, lens, y, mode)
        for b, n in enumerate(lens):
            k, v = hist[b]
            want = (oc.decoder_layer(dims, layer, x[b], k, v, n) if mode else
                    oc.run_layer(dims, layer, x[b], k, v, n))
            assert_layer_close(want, y[b], LAYER_RTOL, f"decode b={b} ctx={n}")
            kn = np.zeros((1, 128), np.float32)
            vn = np.zeros((1, 128), np.float32)
            kv.read(b, n - 1, 1, kn, vn)
            np.testing.assert_array_equal(kn.reshape(-1), k[(n - 1) * 128:n * 128])
            np.testing.assert_array_equal(vn.reshape(-1), v[(n - 1) * 128:n * 128])
    finally:
        ctx64.close()


@pytest.mark.parametrize("exact", [True, False], ids=["exact-attention", "tcgen05-attention"])
@pytest.mark.parametrize("kv_f32", [False, True])
def test_prefill_vs_sequential_decode(si_ctx, oc, kv_f32, exact):
    """Causal prefill equals the reference's prefill oracle: decode token by token
    with context prefix+t+1 (bench_ai_dma_prefill.c:104-108), with either
    prefill attention kernel, to the layer bar."""
    dims, layer = _layer_case(oc, DIMS_15B, 55, mlp=False)
    prefix, ntok, L = 7, 24, 64
    k, v = xs_kv_history(oc, 56, prefix + 1, 256, f32=kv_f32, total=L)
    x = stream(oc, 57, ntok * 1536).reshape(ntok, 1536)
    kv = si_ctx.kv(dims, 1, L, kv_f32)
    kv.write(0, 0, k.reshape(L, 256), v.reshape(L, 256))
    gl = si_ctx.layer(dims, layer)
    y = np.zeros_like(x)
    si_ctx.set_exact_attention(exact)
    try:
        gl.prefill(kv, 0, x, ntok, prefix, y, 0)
    finally:
        si_ctx.set_exact_attention(False)
    k2, v2 = k.copy(), v.copy()
    want = oc.prefill_sequential(dims, layer, x, prefix, k2, v2)
    assert_layer_close(want, y, LAYER_RTOL, "prefill output")
    kg = np.zeros((L, 256), k.dtype)
    vg = np.zeros((L, 256), v.dtype)
    kv.read(0, 0, L, kg, vg)
    np.testing.assert_array_equal(kg.reshape(-1), k2)
    np.testing.assert_array_equal(vg.reshape(-1), v2)


def test_bad_context_is_rejected_cleanly(si_ctx, oc):
    import sib200
    dims, layer = _layer_case(oc, DIMS_15B, 60, mlp=False)
    gl = si_ctx.layer(dims, layer)
    kv = si_ctx.kv(dims, 1, 16, False)
    x = np.zeros(1536, np.float32)
    y = np.zeros(1536, np.float32)
    with pytest.raises(sib200.SiError) as e:
        gl.decode(kv, x, [17], y)        # beyond the cache
    assert e.value.status == 1
    with pytest.raises(sib200.SiError):
        gl.decode(kv, x, [0], y)         # no slot for the new token
    si_ctx.status()                      # device error word is clean; context still usable
    gl.decode(kv, x, [3], y)
    assert np.all(np.isfinite(y))


@pytest.mark.parametrize("I,H", [(18944, 3584), (3712, 8192), (14784, 8192)])
@pytest.mark.parametrize("M", [1, 2, 3, 8, 16])
def test_gateup_mma_equals_dp4a(si_ctx, I, H, M):
    """SwiGLU + Q8 epilogue: both GEMV forms return the same activation bits
    (the 7B pair's 592 tiles and the TP = 2 shard's 462: the dp4a form streams
    two tiles per CTA)."""
    mg, mu = si_ctx.matrix_synth(I, H, seed=I + M), si_ctx.matrix_synth(I, H, seed=H + M)
    x = torch.randn(M, H, device="cuda", generator=torch.Generator("cuda").manual_seed(M))
    torch.cuda.synchronize()
    qs, d = empty(M * H, torch.int8), empty(M * H // 32, torch.int16)
    si_ctx.q8_quantize(x, M, H, qs, d)
    out = []
    for kernel in (2, 3):
        aq, ad = empty(M * I, torch.int8), empty(M * I // 32, torch.int16)
        af = empty(M * I, torch.float32)
        si_ctx.gateup_q8(mg, mu, qs, d, M, aq, ad, af, kernel=kernel)
        out.append((aq, ad, af))
    si_ctx.status()
    for p, q in zip(*out):
        assert torch.equal(p, q)
    mg.free()
    mu.free()
