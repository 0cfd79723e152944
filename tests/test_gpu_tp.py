"""Tensor parallelism on two, four and eight GPUs (where the host has them):
the sharded layer (one process per GPU) against the same layer on one GPU, for
decode steps (GEMV path) and a prefill (40 tokens at two and four ranks: the
GEMV, then an NCCL all-reduce; 300 tokens at eight ranks: the GEMM, then NCCL).
At eight ranks the layer has the Qwen2.5-72B dimensions, so the MLP splits
unevenly (231 units of 128 intermediate rows: 29 on seven ranks, 28 on the
last) exactly as in the 72B tensor-parallel stack.  Decode runs both ways the group can
add the row-parallel partial sums: fused into the projection (peer stores over
NVLink plus a flag-gated combine kernel) and through NCCL's all-reduce.
Five consecutive decode steps exercise both receive-slot parities and the
flag epochs, eagerly and as replays of one captured step whose exchange epochs
come from a device counter (same bits required).  Cross-rank summation reorders the fp32 sums, so at two and four
ranks the bar is the layer bar, 1e-3; every rank must hold identical outputs.

At eight ranks and 72B dimensions a reordered sum cannot be held to 1e-3
against the one-GPU layer: when a last-bit difference flips one Q8 rounding of
the MLP input, the 72B layer output moves by about 2e-3 (some 350 of the
activation's Q8 codes follow it; measured with the oracle), in the reference's
arithmetic as much as here, and a reordered sum causes such a flip for some
tokens.  So at eight ranks: the attention sublayer alone (no Q8 after the
row-parallel sum) must match one GPU within 1e-5, decode through NCCL and
prefill; and the full layer must stay within the bound of a few such flips,
5e-3, with most tokens (where nothing flipped) inside 1e-3.  Skipped on hosts
with fewer GPUs than ranks.
"""
import numpy as np
import pytest

from common import assert_layer_close

torch = pytest.importorskip("torch")
pytestmark = [pytest.mark.gpu, pytest.mark.timeout(600)]

FULLS = {2: dict(hidden=1024, n_q_heads=8, n_kv_heads=2, head_dim=128, intermediate=2816,
                 rope_theta=1e6, rms_eps=1e-6),
         4: dict(hidden=1024, n_q_heads=8, n_kv_heads=4, head_dim=128, intermediate=2816,
                 rope_theta=1e6, rms_eps=1e-6),
         8: dict(hidden=8192, n_q_heads=64, n_kv_heads=8, head_dim=128, intermediate=29568,
                 rope_theta=1e6, rms_eps=1e-6)}
SEED, CTX, PREFIX, STEPS, BATCH = 5, 37, 11, 5, 3
NTOKS = {2: 40, 4: 40, 8: 300}   # prefill tokens per world size
L = 320                          # cache positions: PREFIX + the longest prefill fits


def _inputs(FULL, NTOK):
    rng = np.random.default_rng(17)
    kvd = FULL["n_kv_heads"] * FULL["head_dim"]
    k = (rng.standard_normal((L, kvd)) * 0.5).astype(np.float32)
    v = (rng.standard_normal((L, kvd)) * 0.5).astype(np.float32)
    x = rng.standard_normal((STEPS, BATCH, FULL["hidden"])).astype(np.float32)
    X = rng.standard_normal((NTOK, FULL["hidden"])).astype(np.float32)
    return k, v, x, X


def _decode(ctx, step, dims, k, v, x):
    """STEPS decode steps of BATCH sequences from context CTX on."""
    kvd = dims["n_kv_heads"] * dims["head_dim"]
    kv = ctx.kv(dims, BATCH, L, True)
    for b in range(BATCH):
        kv.write(b, 0, np.ascontiguousarray(k[:CTX - 1, :kvd]), np.ascontiguousarray(v[:CTX - 1, :kvd]))
    out = []
    for s in range(STEPS):
        xin = torch.from_numpy(x[s]).cuda()
        y = torch.zeros_like(xin)
        torch.cuda.synchronize()
        step(kv, xin, [CTX + s] * BATCH, y)
        ctx.status()
        out.append(y.cpu().numpy())
    kv.free()
    return np.stack(out)


def _decode_graph(ctx, tp, layer, dims, k, v, x):
    """The fused decode steps again, with device-resident lengths: the first
    step eager, the rest replays of one captured step (input copied into the
    captured input buffer before each replay)."""
    import sib200
    kvd = dims["n_kv_heads"] * dims["head_dim"]
    kv = ctx.kv(dims, BATCH, L, True)
    for b in range(BATCH):
        kv.write(b, 0, np.ascontiguousarray(k[:CTX - 1, :kvd]), np.ascontiguousarray(v[:CTX - 1, :kvd]))
    st = ctx.decode_state([CTX] * BATCH, L)
    stream = torch.cuda.ExternalStream(ctx.stream)
    xin = torch.from_numpy(x[0]).cuda()
    y = torch.zeros_like(xin)
    xs = [torch.from_numpy(x[s]).cuda() for s in range(STEPS)]
    torch.cuda.synchronize()

    def step():
        tp.decode_state_dev(layer, kv, xin, st, y, sib200.SI_LAYER_FULL)
        st.advance()
    out = []
    step()
    ctx.sync()
    out.append(y.cpu().numpy())
    graph = ctx.capture(step)
    for s in range(1, STEPS):
        with torch.cuda.stream(stream):
            xin.copy_(xs[s])
        graph.launch()
        ctx.sync()
        out.append(y.cpu().numpy())
    ctx.status()
    graph.free()
    st.free()
    kv.free()
    return np.stack(out)


def _prefill(ctx, step, dims, k, v, X):
    kvd = dims["n_kv_heads"] * dims["head_dim"]
    kv = ctx.kv(dims, 1, L, True)
    kv.write(0, 0, np.ascontiguousarray(k[:PREFIX, :kvd]), np.ascontiguousarray(v[:PREFIX, :kvd]))
    xin = torch.from_numpy(X).cuda()
    y = torch.zeros_like(xin)
    torch.cuda.synchronize()
    step(kv, xin, y)
    ctx.status()
    kv.free()
    return y.cpu().numpy()


def _rank(rank, world, uid, path):
    import sib200
    FULL, NTOK = FULLS[world], NTOKS[world]
    torch.cuda.set_device(rank)
    ctx = sib200.Context(rank, 4096, 1e6, 128)
    k, v, x, X = _inputs(FULL, NTOK)
    d, _ = sib200.tp_local_dims(FULL, rank, world)
    kvd = d["n_kv_heads"] * d["head_dim"]
    sl = slice(rank * kvd, (rank + 1) * kvd)
    ks, vs = np.ascontiguousarray(k[:, sl]), np.ascontiguousarray(v[:, sl])
    tp = ctx.tp(uid, rank, world)
    layer = ctx.layer_tp_synth(FULL, SEED, rank, world)
    dec = lambda kv, xin, lens, y: tp.decode_dev(layer, kv, xin, lens, y)
    fused = _decode(ctx, dec, d, ks, vs, x)
    graphed = _decode_graph(ctx, tp, layer, d, ks, vs, x)
    # device-counted epochs and graph replays: the same bits as the eager steps
    np.testing.assert_array_equal(graphed, fused)
    tp.set_options(fused=False)
    nccl = _decode(ctx, dec, d, ks, vs, x)
    tp.set_options(fused=True)
    pre = _prefill(ctx, lambda kv, xin, y: tp.prefill_dev(layer, kv, 0, xin, NTOK, PREFIX, y), d,
                   ks, vs, X)
    np.save(f"{path}.rank{rank}.npy", fused)
    attn = {}
    if world == 8:  # NCCL on the attention sublayer alone (see the module docstring)
        tp.set_options(fused=False)
        attn["nccl_dec"] = _decode(ctx, lambda kv, xin, lens, y: tp.decode_dev(
            layer, kv, xin, lens, y, sib200.SI_LAYER_ATTN), d, ks, vs, x)
        tp.set_options(fused=True)
        attn["pre"] = _prefill(ctx, lambda kv, xin, y: tp.prefill_dev(
            layer, kv, 0, xin, NTOK, PREFIX, y, sib200.SI_LAYER_ATTN), d, ks, vs, X)
    if rank == 0:
        full = ctx.layer_synth(FULL, SEED)
        one_dec = _decode(ctx, lambda kv, xin, lens, y: full.decode_dev(kv, xin, lens, y,
                                                                        sib200.SI_LAYER_FULL),
                          FULL, k, v, x)
        one_pre = _prefill(ctx, lambda kv, xin, y: full.prefill_dev(kv, 0, xin, NTOK, PREFIX, y,
                                                                    sib200.SI_LAYER_FULL),
                           FULL, k, v, X)
        extra = {}
        if world == 8:
            extra["one_attn_dec"] = _decode(ctx, lambda kv, xin, lens, y: full.decode_dev(
                kv, xin, lens, y, sib200.SI_LAYER_ATTN), FULL, k, v, x)
            extra["one_attn_pre"] = _prefill(ctx, lambda kv, xin, y: full.prefill_dev(
                kv, 0, xin, NTOK, PREFIX, y, sib200.SI_LAYER_ATTN), FULL, k, v, X)
            extra.update({f"attn_{k_}": v_ for k_, v_ in attn.items()})
        np.savez(path, one_dec=one_dec, fused=fused, nccl=nccl, one_pre=one_pre, pre=pre, **extra)
        full.free()
    layer.free()
    tp.free()
    ctx.close()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tp_layer_matches_one_gpu(tmp_path, world):
    import sib200
    import torch.multiprocessing as mp
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    uid = sib200.tp_unique_id()
    path = str(tmp_path / "tp")
    mp.spawn(_rank, args=(world, uid, path), nprocs=world, join=True)
    r = np.load(path + ".npz")
    # every rank sums the slots in the same order: identical hidden states
    for rk in range(1, world):
        np.testing.assert_array_equal(np.load(path + ".rank0.npy"),
                                      np.load(path + f".rank{rk}.npy"))
    if world == 8:
        _check_world8(r, path)
        return
    for s in range(STEPS):
        for b in range(BATCH):
            assert_layer_close(r["one_dec"][s, b], r["fused"][s, b], 1e-3, f"fused step {s} seq {b}")
            assert_layer_close(r["one_dec"][s, b], r["nccl"][s, b], 1e-3, f"NCCL step {s} seq {b}")
    for t in range(NTOKS[world]):
        assert_layer_close(r["one_pre"][t], r["pre"][t], 1e-3, f"TP={world} prefill token {t}")


def _check_world8(r, path):
    """Eight ranks, 72B dimensions (see the module docstring for the bars)."""
    errs = []
    for s in range(STEPS):
        for b in range(BATCH):
            assert_layer_close(r["one_attn_dec"][s, b], r["attn_nccl_dec"][s, b], 1e-5,
                               f"NCCL attention sublayer step {s} seq {b}")
            for mode in ("fused", "nccl"):
                assert_layer_close(r["one_dec"][s, b], r[mode][s, b], 5e-3, f"{mode} step {s} seq {b}")
                d = r[mode][s, b].astype(np.float64) - r["one_dec"][s, b]
                errs.append(np.linalg.norm(d) / np.linalg.norm(r["one_dec"][s, b]))
    for t in range(NTOKS[8]):
        assert_layer_close(r["one_attn_pre"][t], r["attn_pre"][t], 1e-5,
                           f"NCCL attention sublayer prefill token {t}")
        assert_layer_close(r["one_pre"][t], r["pre"][t], 5e-3, f"TP=8 prefill token {t}")
        d = r["pre"][t].astype(np.float64) - r["one_pre"][t]
        errs.append(np.linalg.norm(d) / np.linalg.norm(r["one_pre"][t]))
    errs = np.array(errs)
    assert np.mean(errs <= 1e-3) >= 0.5, f"most tokens should see no Q8 flip: {np.sort(errs)[-10:]}"


def test_fused_reduction_wait_times_out(si_ctx):
    """The fused reduction's wait for other ranks is bounded: against a flag
    that nothing sets it returns SI_ERR_TIMEOUT, and the context stays usable."""
    import sib200
    assert si_ctx.tp_probe_wait(20000) == sib200.SI_ERR_TIMEOUT
    si_ctx.status()
    x = torch.randn(64, device="cuda")
    qs = torch.zeros(64, dtype=torch.int8, device="cuda")
    d = torch.zeros(2, dtype=torch.int16, device="cuda")
    torch.cuda.synchronize()
    si_ctx.q8_quantize(x, 1, 64, qs, d)
    si_ctx.status()
