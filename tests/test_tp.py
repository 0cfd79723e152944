"""Tensor-parallel sharding (the 72B configuration over 2/4/8 GPUs), host side.

The shard boundaries come from the C library's si_tp_split / si_tp_local_dims
(host-only functions, callable without a GPU).  The world-size-2 case runs the
sharded decoder layer as two gloo ranks on CPU with the oracle: each rank runs
its heads' attention sublayer and its slice of the MLP, the row-parallel
partial sums are all-reduced, and the result must match the unsharded layer
within the layer bar -- the same scheme the GPU path runs over NCCL.
"""
import os
import socket

import numpy as np
import pytest

from common import assert_layer_close, stream, xs_kv_history, xs_layer

DIMS = dict(hidden=512, n_q_heads=4, n_kv_heads=2, head_dim=128, intermediate=1408,
            rope_theta=1e6, rms_eps=1e-6)
CONFIG4 = dict(hidden=8192, n_q_heads=64, n_kv_heads=8, head_dim=128, intermediate=29568,
               rope_theta=1e6, rms_eps=1e-6)


def sib():
    import sib200
    return sib200


@pytest.mark.parametrize("units", [1, 7, 22, 231, 924])
@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_split_covers_and_balances(units, world):
    s = sib()
    parts = [s.tp_split(units, r, world) for r in range(world)]
    pos = 0
    for first, count in parts:
        assert first == pos
        pos += count
    assert pos == units
    counts = [c for _, c in parts]
    assert max(counts) - min(counts) <= 1


def test_config4_shards():
    s = sib()
    for world, (q, kv) in {1: (64, 8), 2: (32, 4), 4: (16, 2), 8: (8, 1)}.items():
        rows = []
        for r in range(world):
            d, first = s.tp_local_dims(CONFIG4, r, world)
            assert (d["n_q_heads"], d["n_kv_heads"], d["hidden"]) == (q, kv, 8192)
            assert d["intermediate"] % 128 == 0 and first % 128 == 0
            rows.append((first, d["intermediate"]))
        assert sum(c for _, c in rows) == 29568
        assert all(rows[i][0] + rows[i][1] == rows[i + 1][0] for i in range(world - 1))
    with pytest.raises(s.SiError):
        s.tp_local_dims(CONFIG4, 0, 3)  # 64 heads do not split over 3 ranks


def shard(layer, d, rank, world, first):
    """This rank's slices of a host layer in GGUF row-major Q4_0 (18 B blocks)."""
    H, D = d["hidden"], d["head_dim"]
    qd, kvd = d["n_q_heads"] * D, d["n_kv_heads"] * D
    QD = qd * world
    q0, kv0, I = rank * qd, rank * kvd, d["intermediate"]

    def rows(w, cols, r0, n):
        return np.ascontiguousarray(w.reshape(-1, cols // 32 * 18)[r0:r0 + n]).reshape(-1)

    def cols(w, ncols, c0, n):
        m = w.reshape(-1, ncols // 32, 18)[:, c0 // 32:(c0 + n) // 32]
        return np.ascontiguousarray(m).reshape(-1)

    Ifull = layer["w_gate"].size // (H // 32 * 18)
    return {"wq": rows(layer["wq"], H, q0, qd), "wk": rows(layer["wk"], H, kv0, kvd),
            "wv": rows(layer["wv"], H, kv0, kvd), "wo": cols(layer["wo"], QD, q0, qd),
            "bq": layer["bq"][q0:q0 + qd].copy(), "bk": layer["bk"][kv0:kv0 + kvd].copy(),
            "bv": layer["bv"][kv0:kv0 + kvd].copy(), "norm": layer["norm"],
            "w_gate": rows(layer["w_gate"], H, first, I), "w_up": rows(layer["w_up"], H, first, I),
            "w_down": cols(layer["w_down"], Ifull, first, I), "norm2": layer["norm2"]}


def _rank(rank, world, port, ctx_len, out):
    import torch.distributed as dist
    from oracle import Oracle
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import torch
        oc = Oracle()
        s = sib()
        layer = xs_layer(oc, DIMS, 91, mlp=True)
        kc, vc = xs_kv_history(oc, 92, ctx_len, 256, f32=True)
        x = stream(oc, 93, DIMS["hidden"])
        d, first = s.tp_local_dims(DIMS, rank, world)
        loc = shard(layer, d, rank, world, first)
        kvd = d["n_kv_heads"] * d["head_dim"]
        sl = slice(rank * kvd, (rank + 1) * kvd)
        kl = np.ascontiguousarray(kc.reshape(ctx_len, 256)[:, sl]).reshape(-1)
        vl = np.ascontiguousarray(vc.reshape(ctx_len, 256)[:, sl]).reshape(-1)
        part = oc.run_layer(d, loc, x, kl, vl, ctx_len)           # o-proj partial sum
        t = torch.from_numpy(part)
        dist.all_reduce(t)
        h = (x + t.numpy()).astype(np.float32)
        m = torch.from_numpy(oc.mlp(d, loc, h))                   # down-proj partial sum
        dist.all_reduce(m)
        y = (h + m.numpy()).astype(np.float32)
        if rank == 0:
            full_k, full_v = kc.copy(), vc.copy()
            want = oc.decoder_layer(DIMS, layer, x, full_k, full_v, ctx_len)
            np.save(out, np.stack([want, y]))
            # each rank's appended K/V slot is the same slice of the unsharded one
            nk = full_k.reshape(ctx_len, 256)[ctx_len - 1, sl]
            assert np.array_equal(kl.reshape(ctx_len, kvd)[ctx_len - 1], nk)
    finally:
        dist.destroy_process_group()


def test_sharded_layer_two_gloo_ranks(tmp_path):
    import torch.multiprocessing as mp
    with socket.socket() as so:
        so.bind(("127.0.0.1", 0))
        port = so.getsockname()[1]
    out = str(tmp_path / "y.npy")
    mp.spawn(_rank, args=(2, port, 21, out), nprocs=2, join=True)
    want, got = np.load(out)
    assert_layer_close(want, got, 1e-3, "TP=2 decoder layer")
