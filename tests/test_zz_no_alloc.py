"""GPU test of si_matmul_tc_static_dev, the tcgen05 GEMM entry point that
allocates nothing per call (its scratch is a fixed array inside the library).

Called through the C ABI; every output must equal, bit for bit, the output of
the existing tcgen05 entry point si_matmul_dev_kernel(..., kernel=1) on the
same inputs.  Consecutive calls with different shapes check that the shared
array's leftover contents never leak into a result.  Kept in its own file,
collected last, so it runs both alone in a fresh process and after the rest.
"""
import numpy as np
import pytest

import sib200
from sib200 import _p

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

SI_ERR_INVALID = 1
LIMIT = 4 * 1024 * 1024  # SI_STATIC_GEMM_SCRATCH_BYTES


def scratch_bytes(K, M):
    return (K // 32) * ((M + 3) // 4 * 4) * 4


def run_case(ctx, N, K, M, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    w = ctx.matrix_synth(N, K, seed=seed)
    x = torch.randn(M, K, device="cuda", generator=g)
    bias = torch.randn(N, device="cuda", generator=g) * 0.02
    qs = torch.zeros(M * K, dtype=torch.int8, device="cuda")
    d = torch.zeros(M * K // 32, dtype=torch.int16, device="cuda")
    torch.cuda.synchronize()
    ctx.q8_quantize(x, M, K, qs, d)
    want = torch.zeros(M * N, device="cuda")
    got = torch.full((M * N,), float("nan"), device="cuda")
    torch.cuda.synchronize()
    ctx.matmul(w, qs, d, M, bias, want, kernel=1)
    ctx.sync()
    st = ctx.L.si_matmul_tc_static_dev(ctx.h, w.h, _p(qs), _p(d), M, _p(bias), _p(got))
    sib200.check(st, "si_matmul_tc_static_dev")
    ctx.status()
    assert torch.isfinite(got).all()
    assert torch.equal(got, want), f"N={N} K={K} M={M}"
    w.free()


def test_static_scratch_gemm_allocates_nothing():
    """On a fresh context the static entry point runs before anything has sized
    the context's GEMM scratch, and it must leave the context's on-demand
    buffers empty; a second call at a larger size must not change the device's
    free memory either.  Only then is its output compared with the allocating
    tcgen05 entry point's."""
    ctx = sib200.Context(0, max_positions=256, rope_theta=1e6, head_dim=128)
    try:
        N, K = 256, 1536
        w = ctx.matrix_synth(N, K, seed=21)
        g = torch.Generator(device="cuda").manual_seed(21)
        M1, M2 = 64, 1024
        x = torch.randn(M2, K, device="cuda", generator=g)
        qs = torch.zeros(M2 * K, dtype=torch.int8, device="cuda")
        d = torch.zeros(M2 * K // 32, dtype=torch.int16, device="cuda")
        got1 = torch.full((M1 * N,), float("nan"), device="cuda")
        got2 = torch.full((M2 * N,), float("nan"), device="cuda")
        torch.cuda.synchronize()
        ctx.q8_quantize(x, M2, K, qs, d)
        ctx.sync()
        held = ctx.scratch_bytes()
        # First call on this device resolves the array's address (set-up).
        sib200.check(ctx.L.si_matmul_tc_static_dev(ctx.h, w.h, _p(qs), _p(d), M1, None,
                                                   _p(got1)), "si_matmul_tc_static_dev")
        ctx.sync()
        assert ctx.scratch_bytes() == held, "the static entry point grew the context's buffers"
        free0 = torch.cuda.mem_get_info()[0]
        sib200.check(ctx.L.si_matmul_tc_static_dev(ctx.h, w.h, _p(qs), _p(d), M2, None,
                                                   _p(got2)), "si_matmul_tc_static_dev")
        ctx.sync()
        assert torch.cuda.mem_get_info()[0] == free0, "device memory was allocated"
        assert ctx.scratch_bytes() == held
        ctx.status()
        for M, got in ((M1, got1), (M2, got2)):
            want = torch.zeros(M * N, device="cuda")
            torch.cuda.synchronize()
            ctx.matmul(w, qs, d, M, None, want, kernel=1)
            ctx.sync()
            assert torch.equal(got, want), f"M={M}"
        w.free()
    finally:
        ctx.close()


def test_static_scratch_gemm_matches_tcgen05_entry_point(si_ctx):
    assert scratch_bytes(8960, 3744) <= LIMIT
    # Large scratch use first, then smaller shapes over its leftovers, then the
    # largest M that fits for K = 8960.
    run_case(si_ctx, 2048, 1536, 2048, seed=11)
    run_case(si_ctx, 1536, 8960, 130, seed=12)
    run_case(si_ctx, 256, 1536, 9, seed=13)
    run_case(si_ctx, 128, 8960, 3744, seed=14)


def test_static_scratch_gemm_rejects_oversize(si_ctx):
    K, M, N = 8960, 3748, 128
    assert scratch_bytes(K, M) > LIMIT
    w = si_ctx.matrix_synth(N, K, seed=5)
    qs = torch.zeros(M * K, dtype=torch.int8, device="cuda")
    d = torch.zeros(M * K // 32, dtype=torch.int16, device="cuda")
    out = torch.zeros(M * N, device="cuda")
    torch.cuda.synchronize()
    st = si_ctx.L.si_matmul_tc_static_dev(si_ctx.h, w.h, _p(qs), _p(d), M, None, _p(out))
    assert st == SI_ERR_INVALID
    assert b"static GEMM scratch too small" in si_ctx.L.si_last_error()
    si_ctx.status()
    assert int(torch.count_nonzero(out)) == 0
    w.free()
