"""GPU parity of the GEMV that reads row-major GGUF Q4_0 blocks directly (no
repack; the reference's own layout, qwen_one_layer.c:148-162): bit for bit
against the oracle's matvec_q4q8 and against the repacked GEMV, for rows
16-byte aligned (K % 256 == 0) and only 8-byte aligned (the 72B down
projection's 924 blocks per row), 1 to 8 tokens, ragged row counts."""
import numpy as np
import pytest

from common import synth

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def dev(a):
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    torch.cuda.synchronize()
    return t


@pytest.mark.parametrize("N,K,M", [(256, 1536, 1), (4608, 3584, 3), (100, 896, 8),
                                   (1000, 29568, 2), (8192, 29568, 1)])
def test_gguf_gemv_bit_exact(si_ctx, oc, N, K, M):
    rng = np.random.default_rng(N + K + M)
    if N * K > 64 * 1024 * 1024:  # full 72B down matrix: seeded device synthesis
        m = si_ctx.matrix_synth(N, K, seed=77)
        w = m.download_gguf()
    else:
        w = synth.random_q4(rng, N, K)
        # the repacked layout needs whole 32-row tiles; the GGUF GEMV does not
        m = si_ctx.matrix(w, N, K) if N % 32 == 0 else None
    x = rng.standard_normal((M, K)).astype(np.float32)
    bias = rng.normal(0, 0.02, N).astype(np.float32)
    xd = dev(x)
    qs = torch.zeros(M * K, dtype=torch.int8, device="cuda")
    d = torch.zeros(M * K // 32, dtype=torch.int16, device="cuda")
    torch.cuda.synchronize()
    si_ctx.q8_quantize(xd, M, K, qs, d)
    wg = dev(w.reshape(-1))
    got = torch.zeros(M * N, device="cuda")
    want = torch.zeros(M * N, device="cuda")
    b = dev(bias)
    torch.cuda.synchronize()
    si_ctx.matvec_gguf(wg, N, K, qs, d, M, b, got)
    if m is not None:
        si_ctx.matmul(m, qs, d, M, b, want, kernel=0)
    si_ctx.status()
    if m is not None:
        assert torch.equal(got, want)
    blk = torch.zeros(M * K // 32 * 34, dtype=torch.uint8, device="cuda")
    torch.cuda.synchronize()
    si_ctx.q8_to_blocks(qs, d, M, K, blk)
    si_ctx.sync()
    blk = blk.cpu().numpy().reshape(M, -1)
    g = got.cpu().numpy().reshape(M, N)
    rows = slice(0, min(N, 512))
    for t in sorted({0, M - 1}):
        np.testing.assert_array_equal(
            g[t, rows], oc.matvec(w.reshape(N, -1)[rows], blk[t], K, rows.stop, bias[rows]),
            f"token {t}")
    if m is not None:
        m.free()


def test_gguf_gemv_rejects_unsupported(si_ctx):
    import sib200
    qs = torch.zeros(160, dtype=torch.int8, device="cuda")
    d = torch.zeros(5, dtype=torch.int16, device="cuda")
    w = torch.zeros(18 * 5, dtype=torch.uint8, device="cuda")
    out = torch.zeros(1, device="cuda")
    with pytest.raises(sib200.SiError) as e:
        si_ctx.matvec_gguf(w, 1, 160, qs, d, 1, None, out)  # K % 128 != 0
    assert e.value.status == sib200.SI_ERR_UNSUPPORTED
    si_ctx.status()
