"""Tensor parallelism over NCCL on two GPUs: the sharded layer (one process per
GPU, all-reduce after the O and down projections) against the same layer on
one GPU, for a batch-1 decode step (GEMV path) and a 40-token prefill
(tcgen05 GEMM path).  Cross-rank summation reorders the fp32 sums, so the bar
is the layer bar, 1e-3.  Skipped on hosts with fewer than two GPUs.
"""
import os

import numpy as np
import pytest

from common import assert_layer_close

torch = pytest.importorskip("torch")
pytestmark = [pytest.mark.gpu, pytest.mark.timeout(600)]

FULL = dict(hidden=1024, n_q_heads=8, n_kv_heads=2, head_dim=128, intermediate=2816,
            rope_theta=1e6, rms_eps=1e-6)
SEED, CTX, PREFIX, NTOK, L = 5, 37, 11, 40, 64


def _inputs():
    rng = np.random.default_rng(17)
    kvd = FULL["n_kv_heads"] * FULL["head_dim"]
    k = (rng.standard_normal((L, kvd)) * 0.5).astype(np.float32)
    v = (rng.standard_normal((L, kvd)) * 0.5).astype(np.float32)
    x = rng.standard_normal(FULL["hidden"]).astype(np.float32)
    X = rng.standard_normal((NTOK, FULL["hidden"])).astype(np.float32)
    return k, v, x, X


def _run(ctx, step, dims, k, v, x, X):
    """Decode at context CTX (history CTX-1) and prefill NTOK tokens after PREFIX."""
    import sib200
    kvd = dims["n_kv_heads"] * dims["head_dim"]
    out = []
    for kind in ("decode", "prefill"):
        kv = ctx.kv(dims, 1, L, True)
        hist = CTX - 1 if kind == "decode" else PREFIX
        kv.write(0, 0, np.ascontiguousarray(k[:hist, :kvd]), np.ascontiguousarray(v[:hist, :kvd]))
        xin = torch.from_numpy(x if kind == "decode" else X).cuda()
        y = torch.zeros_like(xin)
        torch.cuda.synchronize()
        step(kind, kv, xin, y)
        ctx.status()
        out.append(y.cpu().numpy())
        kv.free()
    return out


def _rank(rank, world, uid, path):
    import sib200
    torch.cuda.set_device(rank)
    ctx = sib200.Context(rank, 4096, 1e6, 128)
    k, v, x, X = _inputs()
    d, _ = sib200.tp_local_dims(FULL, rank, world)
    kvd = d["n_kv_heads"] * d["head_dim"]
    sl = slice(rank * kvd, (rank + 1) * kvd)
    tp = ctx.tp(uid, rank, world)
    layer = ctx.layer_tp_synth(FULL, SEED, rank, world)

    def tp_step(kind, kv, xin, y):
        if kind == "decode":
            tp.decode_dev(layer, kv, xin, [CTX], y)
        else:
            tp.prefill_dev(layer, kv, 0, xin, NTOK, PREFIX, y)

    got = _run(ctx, tp_step, d, np.ascontiguousarray(k[:, sl]), np.ascontiguousarray(v[:, sl]),
               x, X)
    if rank == 0:
        full = ctx.layer_synth(FULL, SEED)

        def one_step(kind, kv, xin, y):
            if kind == "decode":
                full.decode_dev(kv, xin, [CTX], y, sib200.SI_LAYER_FULL)
            else:
                full.prefill_dev(kv, 0, xin, NTOK, PREFIX, y, sib200.SI_LAYER_FULL)

        want = _run(ctx, one_step, FULL, k, v, x, X)
        np.save(path, np.concatenate([want[0][None], got[0][None]]))
        np.save(path + ".prefill.npy", np.stack([want[1], got[1]]))
        full.free()
    layer.free()
    tp.free()
    ctx.close()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs two GPUs")
def test_tp2_layer_matches_one_gpu(tmp_path):
    import sib200
    import torch.multiprocessing as mp
    uid = sib200.tp_unique_id()
    path = str(tmp_path / "decode.npy")
    mp.spawn(_rank, args=(2, uid, path), nprocs=2, join=True)
    want, got = np.load(path)
    assert_layer_close(want, got, 1e-3, "TP=2 decode step")
    pw, pg = np.load(path + ".prefill.npy")
    for t in range(NTOK):
        assert_layer_close(pw[t], pg[t], 1e-3, f"TP=2 prefill token {t}")
