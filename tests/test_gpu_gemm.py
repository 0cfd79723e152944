"""GPU parity of the Q4_0 x Q8_0 GEMMs (prefill / batched decode path): the
tcgen05 kernel (kernel=1) and the mma.sync kernel (kernel=4).

The kernel keeps the reference's per-block order (bias, then
out += ((float)isum*dw)*dx for b = 0..KB-1), so its outputs are compared
bit-for-bit: with the oracle on sampled tokens, and with the CUDA-core GEMV
(itself bit-exact) on whole full-size matrices -- a size-independent check.
"""
import numpy as np
import pytest

from common import assert_close, synth

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def dev(a):
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    torch.cuda.synchronize()
    return t


def z(n, dt):
    t = torch.zeros(n, dtype=dt, device="cuda")
    torch.cuda.synchronize()  # the fill runs on torch's stream, the kernels on the library's
    return t


def q8_dev(ctx, x):
    M, K = x.shape
    qs, d = z(M * K, torch.int8), z(M * K // 32, torch.int16)
    ctx.q8_quantize(dev(x), M, K, qs, d)
    blk = z(M * K // 32 * 34, torch.uint8)
    ctx.q8_to_blocks(qs, d, M, K, blk)
    ctx.sync()
    return qs, d, blk.cpu().numpy().reshape(M, -1)


@pytest.mark.parametrize("kernel", [1, 4], ids=["tcgen05", "mma"])
@pytest.mark.parametrize("N,K,M", [(128, 128, 1), (256, 1536, 16), (2048, 1536, 130),
                                   (128, 8960, 64), (1536, 3584, 257), (896, 4864, 9),
                                   (384, 896, 300)])
def test_gemm_bit_exact_vs_oracle(si_ctx, oc, N, K, M, kernel):
    if kernel == 1 and (N % 128 or K % 128):
        pytest.skip("tcgen05 GEMM needs rows and cols % 128")
    rng = np.random.default_rng(N * 7 + K + M)
    w = synth.random_q4(rng, N, K)
    x = rng.standard_normal((M, K)).astype(np.float32)
    bias = rng.normal(0, 0.02, N).astype(np.float32)
    m = si_ctx.matrix(w, N, K)
    qs, d, blocks = q8_dev(si_ctx, x)
    out = z(M * N, torch.float32)
    si_ctx.matmul(m, qs, d, M, dev(bias), out, kernel=kernel)
    si_ctx.status()
    got = out.cpu().numpy().reshape(M, N)
    for t in sorted({0, M // 2, M - 1}):
        np.testing.assert_array_equal(got[t], oc.matvec(w, blocks[t], K, N, bias), f"token {t}")
    ref = z(M * N, torch.float32)
    si_ctx.matmul(m, qs, d, M, dev(bias), ref, kernel=0)
    si_ctx.sync()
    np.testing.assert_array_equal(got, ref.cpu().numpy().reshape(M, N))


@pytest.mark.parametrize("kernel", [1, 4], ids=["tcgen05", "mma"])
@pytest.mark.parametrize("name,N,K", [("qkv", 2048, 1536), ("o", 1536, 1536),
                                      ("gate", 8960, 1536), ("down", 1536, 8960)])
def test_gemm_config1_full_size_equals_gemv(si_ctx, name, N, K, kernel):
    """Config-1 shapes at M = 2048: GEMM == in-order GEMV, every element."""
    M = 2048
    m = si_ctx.matrix_synth(N, K, seed=hash(name) & 0xFFFF)
    x = torch.randn(M, K, device="cuda")
    torch.cuda.synchronize()
    qs, d = z(M * K, torch.int8), z(M * K // 32, torch.int16)
    si_ctx.q8_quantize(x, M, K, qs, d)
    a, b = z(M * N, torch.float32), z(M * N, torch.float32)
    si_ctx.matmul(m, qs, d, M, None, a, kernel=kernel)
    si_ctx.matmul(m, qs, d, M, None, b, kernel=0)
    si_ctx.status()
    assert torch.isfinite(a).all()
    assert torch.equal(a, b)


@pytest.mark.parametrize("kernel", [1, 4], ids=["tcgen05", "mma"])
@pytest.mark.parametrize("M", [16, 200])
def test_gemm_swiglu_epilogue(si_ctx, oc, M, kernel):
    rng = np.random.default_rng(M)
    H, I = 1536, 8960
    g, u = synth.random_q4(rng, I, H), synth.random_q4(rng, I, H)
    x = rng.standard_normal((M, H)).astype(np.float32)
    mg, mu = si_ctx.matrix(g, I, H), si_ctx.matrix(u, I, H)
    qs, d, blocks = q8_dev(si_ctx, x)
    aq, ad, af = z(M * I, torch.int8), z(M * I // 32, torch.int16), z(M * I, torch.float32)
    si_ctx.gateup_q8(mg, mu, qs, d, M, aq, ad, af, kernel=kernel)
    si_ctx.status()
    # the same bits as the GEMV's SwiGLU epilogue
    aq2, ad2, af2 = z(M * I, torch.int8), z(M * I // 32, torch.int16), z(M * I, torch.float32)
    si_ctx.gateup_q8(mg, mu, qs, d, M, aq2, ad2, af2, kernel=0)
    si_ctx.status()
    assert torch.equal(aq, aq2) and torch.equal(ad, ad2) and torch.equal(af, af2)
    act = af.cpu().numpy().reshape(M, I)
    blk = z(M * I // 32 * 34, torch.uint8)
    si_ctx.q8_to_blocks(aq, ad, M, I, blk)
    si_ctx.sync()
    blk = blk.cpu().numpy().reshape(M, -1)
    for t in (0, M - 1):
        gate = oc.matvec(g, blocks[t], H, I)
        up = oc.matvec(u, blocks[t], H, I)
        want = (gate / (np.float32(1) + np.exp(-gate))).astype(np.float32) * up
        assert_close(want, act[t], 1e-7, 1e-6, f"silu(gate)*up token {t}")
        np.testing.assert_array_equal(blk[t], oc.quantize_q8(act[t]))


@pytest.mark.parametrize("n", [128, 256])
def test_int8_tensor_core_probe(si_ctx, n):
    """The int8 throughput probe that supplies the prefill roofline's
    denominator: it completes (its bounded wait does not expire), reports the
    operation count it performs, and its measured rate is a plausible B200
    dense int8 rate (between 1 and 6 POPS; the data sheet gives 4.5)."""
    stream = torch.cuda.ExternalStream(si_ctx.stream)
    iters = 8192
    ops = si_ctx.tc_i8_peak(n, iters)
    si_ctx.sync()
    si_ctx.status()
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    assert ops == sms * iters * 4 * 2 * 128 * n * 32
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        start.record()
        for _ in range(3):
            si_ctx.tc_i8_peak(n, iters)
        end.record()
    end.synchronize()
    si_ctx.status()
    tops = 3 * ops / (start.elapsed_time(end) / 1e3) / 1e12
    assert 1000 < tops < 6000, tops


# The fused-rescale mode (kernel 5) drops one rounding per block term, so it is
# held to the projection bar of the north star, 1e-5 relative: every output
# within 1e-5 of the row's largest magnitude and the whole matrix within 1e-6
# relative L2 of the exact kernel's bits (which the tests above pin to the
# reference).
FUSED_MAX_REL, FUSED_L2_REL = 1e-5, 1e-6


@pytest.mark.parametrize("N,K,M", [(256, 1536, 16), (2048, 1536, 130), (1536, 8960, 257),
                                   (8192, 29568, 64)])
def test_gemm_fused_rescale_within_projection_bar(si_ctx, oc, N, K, M):
    m = si_ctx.matrix_synth(N, K, seed=N + K + M)
    x = torch.randn(M, K, device="cuda")
    bias = torch.randn(N, device="cuda") * 0.02
    torch.cuda.synchronize()
    qs, d = z(M * K, torch.int8), z(M * K // 32, torch.int16)
    si_ctx.q8_quantize(x, M, K, qs, d)
    exact, fused = z(M * N, torch.float32), z(M * N, torch.float32)
    si_ctx.matmul(m, qs, d, M, bias, exact, kernel=1)
    si_ctx.matmul(m, qs, d, M, bias, fused, kernel=5)
    si_ctx.status()
    e = exact.double().reshape(M, N)
    f = fused.double().reshape(M, N)
    assert torch.isfinite(f).all()
    scale = e.abs().amax(dim=1, keepdim=True)
    assert float(((f - e).abs() / scale).max()) <= FUSED_MAX_REL
    assert float((f - e).norm() / e.norm()) <= FUSED_L2_REL


@pytest.mark.parametrize("M", [64, 300])
def test_gemm_swiglu_fused_rescale_within_projection_bar(si_ctx, M):
    H, I = 1536, 8960
    mg, mu = si_ctx.matrix_synth(I, H, seed=31), si_ctx.matrix_synth(I, H, seed=32)
    x = torch.randn(M, H, device="cuda")
    torch.cuda.synchronize()
    qs, d = z(M * H, torch.int8), z(M * H // 32, torch.int16)
    si_ctx.q8_quantize(x, M, H, qs, d)
    outs = {}
    for k in (1, 5):
        aq, ad, af = z(M * I, torch.int8), z(M * I // 32, torch.int16), z(M * I, torch.float32)
        si_ctx.gateup_q8(mg, mu, qs, d, M, aq, ad, af, kernel=k)
        si_ctx.status()
        outs[k] = (aq, ad, af)
    e, f = outs[1][2].double().reshape(M, I), outs[5][2].double().reshape(M, I)
    scale = e.abs().amax(dim=1, keepdim=True)
    # silu(g)*u amplifies the gate and up terms' relative differences at most 2x
    assert float(((f - e).abs() / scale).max()) <= 2 * FUSED_MAX_REL
    # Q8 of the activation: codes move by at most one step, and rarely
    dq = (outs[5][0].int() - outs[1][0].int()).abs()
    assert int(dq.max()) <= 1 and float((dq > 0).float().mean()) < 1e-3
