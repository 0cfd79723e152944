#!/usr/bin/env python3
"""Benchmark of the Qwen decoder-layer hot path (BASELINE metric: layer prefill
tok/s + decode us/token, as fractions of the HBM / int8 tensor-core rooflines).

Headline workload, the same at every GPU count so the 1 -> 8 GPU curve measures
tensor parallelism: BASELINE.json configs[4], a stack of 8 Qwen2.5-72B-shaped
layers (hidden 8192, 64 Q / 8 KV heads, intermediate 29568, Q4_0 weights, fp32
KV), tensor-parallel over the N ranks of `bench.py --gpus N` (column-sharded
QKV/gate/up, row-sharded o/down; one rank per GPU).

* step   = one 4096-token prefill of sequence 0 through the 8 layers;
* value  = prefill tok/s of the whole job (the same 4096 tokens at every N:
           strong scaling), device-timed with CUDA events on the library's
           stream, inputs resident in HBM, max over ranks;
* decode = 256 decode steps of a batch of 8 (contexts 4097..4352), us per step
           and per token, beside the headline;
* e2e    = the headline through the C ABI with host buffers: every step copies
           its 128 MiB fp32 input in from rank 0's pinned host memory (with
           several ranks, broadcast from rank 0 over NVLink inside the step) and
           its 128 MiB output back to rank 0 (two buffer sets, so the copies of
           neighbouring steps overlap the compute on their own streams);
* roofline: the prefill's dominant kernel (the gate/up GEMM at 4096 tokens)
           against the int8 tensor-core rate measured here by a tcgen05
           kind::i8 probe; `layer_roofline` adds the whole prefill (int8 ops)
           and the decode step (weight + KV bytes) per rank;
* cpu_baseline: the reference's CPU path on the host cores -- its own
           quantize_q8 / matvec_q4q8 (oracle/_ref, rows split over the threads)
           with the oracle's restatement of rmsnorm / rope / attention_flash at
           the 72B dimensions -- on a bounded token sample, extrapolated
           linearly to the 4096-token x 8-layer prefill (rank 0, N = 1).

At N = 1 the line also carries the other BASELINE configurations, each with its
own measurement: config2 (one 7B layer: 2048-token prefill, 128 decode steps;
e2e through the host-pointer C ABI; CPU baseline on the same dims), config3
(batch-64 7B decode over 4096-position fp32 caches), config1 (the 1.5B
projection set and its token sweep), decode_gemv_roofline, gemm_schemes (the
prefill GEMM's exact int8 kernels beside bf16/fp16-dequant cuBLAS GEMMs, with
their errors) and reference_layer (the reference's own attention layer timed
on the host against this library).
`--impl reference` times the reference's CPU path on the headline workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "simple-inference_b200"))

METRIC = "Qwen layer prefill tok/s + decode µs/token; % of HBM / int8-TC roofline"
INT8_SPEC_TOPS = 4500.0  # B200 dense int8 data-sheet figure, shown beside the measured one

CONFIG4 = dict(hidden=8192, n_q_heads=64, n_kv_heads=8, head_dim=128, intermediate=29568,
               rope_theta=1e6, rms_eps=1e-6)
TP_LAYERS, TP_PREFILL, TP_BATCH, TP_DECODE = 8, 4096, 8, 256
# Cache capacity: the prefill and 256 decode positions, plus the slot a
# device-side length reaches after the last step's advance.
TP_MAX_CTX = TP_PREFILL + TP_DECODE + 1
DIMS_7B = dict(hidden=3584, n_q_heads=28, n_kv_heads=4, head_dim=128, intermediate=18944,
               rope_theta=1e6, rms_eps=1e-6)
C2_PREFILL, C2_DECODE = 2048, 128
DIMS_05B = dict(hidden=896, n_q_heads=14, n_kv_heads=2, head_dim=64, intermediate=4864,
                rope_theta=1e6, rms_eps=1e-6)
C0_PREFILL = 64
C3_BATCH, C3_CTX = 64, 4096
H1, I1, QKV1 = 1536, 8960, 2048          # config 1: the 1.5B projection set
C1_COPIES, C1_M = 10, 2048
SWEEP_M = (1, 16, 128, 512, 2048)
# DRAM bytes (read + write) of one launch of the headline's dominant kernel,
# from an `ncu --set full -k regex:k_gemm_q4q8 -s 1 -c 1` capture of
# `bench.py --probe gateup-72b` (its gate/up GEMM at 4096 tokens on one 72B
# layer): 324.2 MB read + 126.3 MB written.  Re-measure when the kernel changes.
NCU_TRAFFIC_GATEUP_72B = 450505728


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return {"hbm_gbs": d["hbm_gbs"], "src": "measured"}
    return {"hbm_gbs": 6650.0, "src": "fallback"}


def q4_bytes(n, k):
    return n * k // 32 * 18


def layer_weight_bytes(d):
    H, D = d["hidden"], d["head_dim"]
    QD, KVD, I = d["n_q_heads"] * D, d["n_kv_heads"] * D, d["intermediate"]
    return q4_bytes(QD + 2 * KVD, H) + q4_bytes(H, QD) + q4_bytes(2 * I, H) + q4_bytes(H, I)


def layer_int8_ops(d, M):
    """int8 operations (2 per multiply-add) of a layer's projections over M tokens."""
    H, D = d["hidden"], d["head_dim"]
    QD, KVD, I = d["n_q_heads"] * D, d["n_kv_heads"] * D, d["intermediate"]
    return 2 * M * H * (QD + 2 * KVD + 2 * I) + 2 * M * QD * H + 2 * M * I * H


class Clocks:
    """nvidia-smi sampling during the timed region."""

    def __init__(self, index: int):
        self.index = index
        self.samples = []
        self._stop = threading.Event()
        self._t = None

    def __enter__(self):
        q = ("clocks.sm,clocks.max.sm,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

        def run():
            while not self._stop.is_set():
                try:
                    out = subprocess.run(["nvidia-smi", "-i", str(self.index), f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits"], capture_output=True,
                                         text=True, timeout=5).stdout.strip()
                    if out:
                        self.samples.append([s.strip() for s in out.split(",")])
                except Exception:
                    pass
                self._stop.wait(0.2)
        self._t = threading.Thread(target=run, daemon=True)
        self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        self._t.join(timeout=10)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(s[0]) for s in self.samples if s[0].replace(".", "").isdigit()]
        mx = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in self.samples for i in range(4)
                          if len(s) > 3 + i and s[3 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(self.samples)}


def time_region(torch, stream, fn, steps):
    """Seconds for `steps` calls of fn(i), CUDA events on `stream`."""
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        start.record()
        for i in range(steps):
            fn(i)
        end.record()
    end.synchronize()
    return start.elapsed_time(end) / 1e3


def log(msg):
    if os.environ.get("SI_BENCH_VERBOSE"):
        print(f"[bench] {msg}", file=sys.stderr, flush=True)


# ---------------------------------------------------------------------------
# the reference's CPU path (reference arm, cpu_baseline legs)
# ---------------------------------------------------------------------------
class CpuLayer:
    """One decoder layer on the host cores, the reference's way: per token
    rmsnorm -> quantize_q8 -> matvec_q4q8 (QKV + bias) -> rope -> KV append ->
    attention_flash -> quantize_q8 -> matvec_q4q8 (o) -> residual, then the
    MLP (rmsnorm, gate/up matvec, SiLU*mul, quantize_q8, down matvec,
    residual).  quantize_q8 and matvec_q4q8 are the reference's own functions
    (oracle/_ref; the oracle's restatement where the reference was not built
    here), matvec rows split over the threads (each row's arithmetic is the
    reference's); rmsnorm, rope and attention_flash are the oracle's
    restatement at these dimensions (the reference compiles them for 1.5B
    only), attention heads split over the threads.  Weights are seeded random
    Q4_0 bytes: the time of this code does not depend on their values."""

    def __init__(self, dims, seed, ctx_cap, threads, kv_f32):
        import ctypes as C
        from concurrent.futures import ThreadPoolExecutor
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle
        self.C, self.oracle = C, oracle
        self.oc = oracle.Oracle()
        if os.path.exists(oracle.LIB_REF):
            r = oracle.Reference()
            self.kind, self._mv, self._q8 = "reference", r.lib.ref_matvec_q4q8, r.lib.ref_quantize_q8
        else:
            self.kind = "port"
            self._mv, self._q8 = self.oc.lib.oc_matvec_q4q8, self.oc.lib.oc_quantize_q8
        self.d = dims
        H, D = dims["hidden"], dims["head_dim"]
        self.H, self.D, self.Hq, self.Hkv = H, D, dims["n_q_heads"], dims["n_kv_heads"]
        self.QD, self.KVD, self.I = self.Hq * D, self.Hkv * D, dims["intermediate"]
        rng = np.random.default_rng(seed)

        def q4(rows, k):
            w = rng.integers(0, 256, size=(rows, k // 32, 18), dtype=np.uint8)
            sc = (rng.uniform(0.5, 1.5, size=(rows, k // 32)) * 0.006).astype(np.float16)
            w[:, :, 0:2] = sc.view(np.uint8).reshape(rows, k // 32, 2)
            return np.ascontiguousarray(w.reshape(rows, -1))
        self.wqkv = q4(self.QD + 2 * self.KVD, H)
        self.wo = q4(H, self.QD)
        self.wg, self.wu, self.wd = q4(self.I, H), q4(self.I, H), q4(H, self.I)
        self.bqkv = rng.normal(0, 0.02, self.QD + 2 * self.KVD).astype(np.float32)
        self.norm = (1 + rng.normal(0, 0.02, H)).astype(np.float32)
        self.norm2 = (1 + rng.normal(0, 0.02, H)).astype(np.float32)
        kvt = np.float32 if kv_f32 else np.float16
        self.kc = rng.standard_normal((ctx_cap, self.KVD), dtype=np.float32).astype(kvt)
        self.vc = rng.standard_normal((ctx_cap, self.KVD), dtype=np.float32).astype(kvt)
        if not kv_f32:
            self.kc, self.vc = self.kc.view(np.uint16), self.vc.view(np.uint16)
        self.kv_f32 = kv_f32
        self.threads = threads
        self.pool = ThreadPoolExecutor(threads)
        self.dm = oracle.make_dims(dims)

    def close(self):
        self.pool.shutdown()

    def q8(self, x):
        out = np.zeros(x.size // 32 * 34, np.uint8)
        self._q8(np.ascontiguousarray(x, np.float32), out, x.size)
        return out

    def mv(self, w, q8, K, N, bias=None):
        C = self.C
        out = np.zeros(N, np.float32)
        rows = -(-N // self.threads)

        def part(t):  # row slices: each row's arithmetic is the reference's
            r0, r1 = t * rows, min(N, (t + 1) * rows)
            if r0 < r1:
                self._mv(w[r0:r1], q8, K, r1 - r0,
                         None if bias is None else bias[r0:r1].ctypes.data_as(C.c_void_p),
                         out[r0:r1])
        list(self.pool.map(part, range(self.threads)))
        return out

    def attention(self, q, ctx):
        C = self.C
        out = np.zeros(self.QD, np.float32)
        per = -(-self.Hq // self.threads)
        kp, vp = self.kc.ctypes.data_as(C.c_void_p), self.vc.ctypes.data_as(C.c_void_p)

        def part(t):
            h0, h1 = t * per, min(self.Hq, (t + 1) * per)
            if h0 < h1:
                self.oc.lib.oc_attention_flash_heads(C.byref(self.dm), q, kp, vp,
                                                     int(self.kv_f32), ctx, out, h0, h1)
        list(self.pool.map(part, range(self.threads)))
        return out

    def token(self, x, ctx):
        """One token of the layer at context length ctx (its K/V go to slot ctx-1)."""
        H, QD, KVD, I = self.H, self.QD, self.KVD, self.I
        xn = self.oc.rmsnorm(x, self.norm)
        qkv = self.mv(self.wqkv, self.q8(xn), H, QD + 2 * KVD, self.bqkv)
        q = self.oc.rope(qkv[:QD], self.Hq, ctx - 1, self.D)
        k = self.oc.rope(qkv[QD:QD + KVD], self.Hkv, ctx - 1, self.D)
        v = qkv[QD + KVD:]
        if self.kv_f32:
            self.kc[ctx - 1], self.vc[ctx - 1] = k, v
        else:
            self.kc[ctx - 1] = k.astype(np.float16).view(np.uint16)
            self.vc[ctx - 1] = v.astype(np.float16).view(np.uint16)
        attn = self.attention(q, ctx)
        h = (x + self.mv(self.wo, self.q8(attn), QD, H)).astype(np.float32)
        hq = self.q8(self.oc.rmsnorm(h, self.norm2))
        g, u = self.mv(self.wg, hq, H, I), self.mv(self.wu, hq, H, I)
        a = ((g / (np.float32(1) + np.exp(-g))) * u).astype(np.float32)
        return (h + self.mv(self.wd, self.q8(a), I, H)).astype(np.float32)


def cpu_layer_rounds(cl, prefill, decode_ctx, rounds=None, seconds=None, per_round=4):
    """Times per-token layer steps on the host: each round runs `per_round`
    prefill tokens at the midpoint contexts of `per_round` equal slices of
    [1, prefill] and one decode token at context `decode_ctx`.  A token's cost
    is linear in its context (projections constant, attention proportional),
    so the midpoints' mean is the mean over the whole prefill.  Runs `rounds`
    rounds, or rounds until `seconds` have passed (at least one)."""
    rng = np.random.default_rng(7)
    ctxs = [int((i + 0.5) * prefill / per_round) + 1 for i in range(per_round)]
    x = rng.standard_normal((per_round + 1, cl.H)).astype(np.float32)
    cl.token(x[0], 2)  # warm the pool and the caches' pages
    tp, td, n = [], [], 0
    t_start = time.perf_counter()
    while True:
        for i, c in enumerate(ctxs):
            t0 = time.perf_counter()
            cl.token(x[i], c)
            tp.append(time.perf_counter() - t0)
        t0 = time.perf_counter()
        cl.token(x[-1], decode_ctx)
        td.append(time.perf_counter() - t0)
        n += 1
        if rounds is not None and n >= rounds:
            break
        if seconds is not None and time.perf_counter() - t_start >= seconds:
            break
    return {"prefill_s_per_token_layer": statistics.mean(tp),
            "decode_s_per_token_layer": statistics.mean(td),
            "prefill_tokens": len(tp), "decode_tokens": len(td), "contexts": ctxs,
            "decode_context": decode_ctx, "wall_s": time.perf_counter() - t_start}


def cpu_layer_baseline(dims, layers, prefill, decode_ctx, kv_f32, seconds, seed, label):
    threads = len(os.sched_getaffinity(0))
    cl = CpuLayer(dims, seed, max(prefill, decode_ctx) + 1, threads, kv_f32)
    try:
        r = cpu_layer_rounds(cl, prefill, decode_ctx, seconds=seconds)
    finally:
        cl.close()
    t_prefill = layers * prefill * r["prefill_s_per_token_layer"]
    return {"value": round(prefill / t_prefill, 4), "unit": "tok/s", "cores": threads,
            "kind": cl.kind,
            "decode_us_per_token": round(layers * r["decode_s_per_token_layer"] * 1e6, 1),
            "sample": (f"{label}: {r['prefill_tokens']} prefill tokens at contexts "
                       f"{r['contexts']} and {r['decode_tokens']} decode tokens at context "
                       f"{decode_ctx} through one layer ({r['wall_s']:.1f} s on {threads} "
                       f"threads), extrapolated linearly to {prefill} tokens x {layers} "
                       f"layer(s); matvec/quantize_q8 {cl.kind}, rmsnorm/rope/attention the "
                       f"oracle's restatement")}


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def int8_peak(ctx, torch, stream):
    """Dense int8 tensor-core rate of this GPU: the tcgen05 kind::i8 probe
    (128 x n x 32 MMAs from shared memory, one CTA per SM), CUDA events."""
    out = {}
    for n in (256, 128):
        iters = 65536
        ops = ctx.tc_i8_peak(n, iters)
        for _ in range(2):
            ctx.tc_i8_peak(n, iters)
        t = time_region(torch, stream, lambda i: ctx.tc_i8_peak(n, iters), 5) / 5
        ctx.status()
        out[f"128x{n}x32"] = round(ops / t / 1e12, 1)
    return {"tops": max(out.values()), "per_shape": out,
            "how": "tcgen05.mma kind::i8, operands resident in shared memory, one CTA per SM, "
                   "5 launches of 65536 x 4 MMAs per CTA, CUDA events (burst)",
            "spec_tops": INT8_SPEC_TOPS}


def run_config4(args, rank, world, local_rank, ctx, torch, barrier_sync, max_over_ranks, peak):
    """The headline: 8 Qwen2.5-72B layers at TP = world."""
    import sib200
    stream = torch.cuda.ExternalStream(ctx.stream)
    if world > 1:
        import torch.distributed as tdist
        box = [sib200.tp_unique_id() if rank == 0 else None]
        tdist.broadcast_object_list(box, src=0)
        uid = box[0]
    else:
        uid = sib200.tp_unique_id()
    tp = ctx.tp(uid, rank, world)
    d, _ = sib200.tp_local_dims(CONFIG4, rank, world)
    layers = [ctx.layer_tp_synth(CONFIG4, 4 + 1000 * i, rank, world) for i in range(TP_LAYERS)]
    kvs = [ctx.kv(d, TP_BATCH, TP_MAX_CTX, True) for _ in range(TP_LAYERS)]
    for i, kv in enumerate(kvs):
        kv.fill_synth(4 + 1000 * i, 1.0, TP_PREFILL)
    Hd = CONFIG4["hidden"]
    g = torch.Generator(device="cuda").manual_seed(4)
    x_in = torch.randn(TP_PREFILL, Hd, device="cuda", generator=g)
    sets = [(torch.empty(TP_PREFILL, Hd, device="cuda"), torch.empty(TP_PREFILL, Hd, device="cuda"))
            for _ in range(2)]
    xd = [torch.randn(TP_BATCH, Hd, device="cuda", generator=g), torch.empty(TP_BATCH, Hd, device="cuda")]
    x0 = xd[0].clone()
    torch.cuda.synchronize()

    def prefill_on(a, b):
        """8 layers, ping-ponging a -> b -> a ...; the output ends in a."""
        for j, (layer, kv) in enumerate(zip(layers, kvs)):
            src, dst = (a, b) if j % 2 == 0 else (b, a)
            tp.prefill_dev(layer, kv, 0, src, TP_PREFILL, 0, dst)

    def step(i):
        a, b = sets[i % 2]
        a.copy_(x_in)
        prefill_on(a, b)

    # The copy of the resident input into the step's buffer is a device copy
    # (0.27 GB of HBM traffic against the step's ~4 GB / TP of weights).
    with torch.cuda.stream(stream):
        for i in range(args.warmup):
            step(i)
    barrier_sync()
    n0 = sib200.kernel_launches()
    with Clocks(local_rank) as clk:
        t = time_region(torch, stream, step, args.steps)
    launches = sib200.kernel_launches() - n0
    barrier_sync()
    t = max_over_ranks(t)
    log(f"config4 prefill {t / args.steps * 1e3:.2f} ms/step")

    # ---- e2e: pinned host input in, prefill, pinned host output out --------
    # One process serves the request: rank 0 copies the input in from its
    # pinned host buffer and the output (identical on every rank after the
    # last all-reduce) back out; with several ranks the input reaches the
    # others by an NCCL broadcast over NVLink inside the timed step.
    host_io = rank == 0
    if world > 1:
        import torch.distributed as tdist
    hx = torch.randn(TP_PREFILL, Hd, generator=torch.Generator().manual_seed(4)).pin_memory()
    hy = [torch.empty(TP_PREFILL, Hd).pin_memory() for _ in range(2)]
    s_in, s_out = torch.cuda.Stream(), torch.cuda.Stream()
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_comp = [torch.cuda.Event() for _ in range(2)]
    ev_out = [torch.cuda.Event() for _ in range(2)]
    for e in ev_comp + ev_out:
        e.record(stream)

    def e2e_step(i):
        k = i % 2
        a, b = sets[k]
        if host_io:
            s_in.wait_event(ev_comp[k])       # step i-2 has finished with this set
            with torch.cuda.stream(s_in):
                a.copy_(hx, non_blocking=True)
                ev_in[k].record(s_in)
            stream.wait_event(ev_in[k])
            stream.wait_event(ev_out[k])      # step i-2's output has left this set
        if world > 1:
            with torch.cuda.stream(stream):
                tdist.broadcast(a, src=0)
        prefill_on(a, b)
        ev_comp[k].record(stream)
        if host_io:
            s_out.wait_event(ev_comp[k])
            with torch.cuda.stream(s_out):
                hy[k].copy_(a, non_blocking=True)
                ev_out[k].record(s_out)

    for i in range(2):
        e2e_step(i)
    torch.cuda.synchronize()
    barrier_sync()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s_in if host_io else stream)
    for i in range(args.steps):
        e2e_step(i)
    e1.record(s_out if host_io else stream)
    e1.synchronize()
    te = max_over_ranks(e0.elapsed_time(e1) / 1e3)
    barrier_sync()
    log(f"config4 e2e {te / args.steps * 1e3:.2f} ms/step")

    # ---- decode: 256 steps of a batch of 8 -----------------------------------
    # The 8-layer step is captured once as a CUDA graph with the context
    # lengths on the device (si_decode_state) and replayed step after step; on
    # several ranks the fused exchanges' epochs come from a device counter the
    # step's advance moves on.  The NCCL variant runs eagerly.
    def decode(s):
        lens = [TP_PREFILL + s + 1] * TP_BATCH
        for j, (layer, kv) in enumerate(zip(layers, kvs)):
            tp.decode_dev(layer, kv, xd[j % 2], lens, xd[(j + 1) % 2])

    def time_decode():
        for s in range(3):
            decode(s)
        with torch.cuda.stream(stream):
            xd[0].copy_(x0)
        barrier_sync()
        return max_over_ranks(time_region(torch, stream, decode, TP_DECODE)) / TP_DECODE

    def time_decode_graph():
        lens0 = [TP_PREFILL + 1] * TP_BATCH
        st = ctx.decode_state(lens0, TP_MAX_CTX)

        def step():
            for j, (layer, kv) in enumerate(zip(layers, kvs)):
                if world > 1:
                    tp.decode_state_dev(layer, kv, xd[j % 2], st, xd[(j + 1) % 2])
                else:
                    layer.decode_state_dev(kv, xd[j % 2], st, xd[(j + 1) % 2],
                                           sib200.SI_LAYER_FULL)
            st.advance()
        step()  # sizes the context's buffers before the capture
        ctx.sync()
        gph = ctx.capture(step)
        for _ in range(3):
            gph.launch()
        st.set(lens0)
        with torch.cuda.stream(stream):
            xd[0].copy_(x0)
        barrier_sync()
        t_ = time_region(torch, stream, lambda i: gph.launch(), TP_DECODE) / TP_DECODE
        ctx.status()
        gph.free()
        st.free()
        return t_

    tdec = time_decode_graph()
    tdec_nccl = None
    if world > 1:
        tp.set_options(fused=False)
        tdec_nccl = time_decode()
        tp.set_options(fused=True)
    ctx.status()
    finite = bool(torch.isfinite(xd[0]).all().item()) and bool(torch.isfinite(sets[0][0]).all().item())

    # ---- the prefill's dominant kernel: the gate/up GEMM at 4096 tokens -------
    Il = d["intermediate"]
    xq = torch.empty(TP_PREFILL * Hd, dtype=torch.int8, device="cuda")
    xdd = torch.empty(TP_PREFILL * Hd // 32, dtype=torch.int16, device="cuda")
    aq = torch.empty(TP_PREFILL * Il, dtype=torch.int8, device="cuda")
    ad = torch.empty(TP_PREFILL * Il // 32, dtype=torch.int16, device="cuda")
    torch.cuda.synchronize()
    ctx.q8_quantize(x_in, TP_PREFILL, Hd, xq, xdd)
    mats = [(layer.matrix(2), layer.matrix(3)) for layer in layers]
    gu = lambda i: ctx.gateup_q8(mats[i % TP_LAYERS][0], mats[i % TP_LAYERS][1], xq, xdd,
                                 TP_PREFILL, aq, ad)
    for i in range(3):
        gu(i)
    barrier_sync()
    tg = max_over_ranks(time_region(torch, stream, gu, 2 * TP_LAYERS)) / (2 * TP_LAYERS)
    gu_ops = 2 * TP_PREFILL * 2 * Il * Hd
    ctx.status()

    D = CONFIG4["head_dim"]
    KVD = d["n_kv_heads"] * D
    wlayer = layer_weight_bytes(d)
    mean_ctx = TP_PREFILL + (TP_DECODE + 1) / 2
    kv_read = TP_BATCH * mean_ctx * KVD * 2 * 4
    dec_bytes = TP_LAYERS * (wlayer + kv_read)
    pk = peaks()
    tstep = t / args.steps
    pf_ops = TP_LAYERS * layer_int8_ops(d, TP_PREFILL)
    res = {
        "value": round(TP_PREFILL * args.steps / t, 1),
        "ms_per_step": round(tstep * 1e3, 3),
        "gpu_launches": int(launches),
        "clocks": clk.summary(),
        "e2e": {"value": round(TP_PREFILL * args.steps / te, 1), "unit": "tok/s",
                "h2d_bytes_per_step": TP_PREFILL * Hd * 4, "d2h_bytes_per_step": TP_PREFILL * Hd * 4,
                "how": "per step: the 4096 x 8192 fp32 input from rank 0's pinned host memory "
                       "(with several ranks, broadcast from rank 0 over NVLink by NCCL inside "
                       "the step), the 8-layer prefill through si_prefill_tp_dev, the output "
                       "(identical on every rank) back to rank 0's pinned host memory; copies of "
                       "neighbouring steps overlap on two copy streams; time = max over ranks"},
        "decode": {"batch": TP_BATCH, "steps": TP_DECODE,
                   "context": f"{TP_PREFILL + 1}..{TP_PREFILL + TP_DECODE}",
                   "launch": "one 8-layer step captured as a CUDA graph (device-resident "
                             "context lengths and exchange epochs), replayed per step",
                   "us_per_step": round(tdec * 1e6, 2),
                   "us_per_token": round(tdec * 1e6 / TP_BATCH, 3),
                   "tok_s": round(TP_BATCH / tdec, 1),
                   "reduction": ("fused into the projection (epoch-tagged NVLink peer stores)"
                                 if world > 1 else "none (one rank)"),
                   "us_per_step_nccl_allreduce_eager": round(tdec_nccl * 1e6, 2) if tdec_nccl else None},
        "roofline": {"bound": "tensor", "kernel": "gate/up GEMM + SiLU*mul + Q8 (4096 tokens, "
                                                  f"2x{Il}x{Hd} per rank)",
                     "achieved": round(gu_ops / tg / 1e12, 2),
                     "peak": peak["tops"], "unit": "TOP/s",
                     "frac": round(gu_ops / tg / 1e12 / peak["tops"], 4),
                     "peak_src": "measured here (tcgen05 kind::i8 probe, burst)",
                     "frac_of_spec": round(gu_ops / tg / 1e12 / INT8_SPEC_TOPS, 4),
                     "us_per_launch": round(tg * 1e6, 2),
                     "algorithmic_ops_per_launch": gu_ops,
                     "traffic": NCU_TRAFFIC_GATEUP_72B},
        "layer_roofline": {
            "prefill": {"int8_ops_per_step_per_rank": pf_ops,
                        "achieved_tops": round(pf_ops / tstep / 1e12, 2),
                        "frac_of_int8_peak": round(pf_ops / tstep / 1e12 / peak["tops"], 4)},
            "decode": {"bytes_per_step_per_rank": int(dec_bytes),
                       "achieved_gbs": round(dec_bytes / tdec / 1e9, 1), "peak_gbs": pk["hbm_gbs"],
                       "frac_of_hbm": round(dec_bytes / tdec / 1e9 / pk["hbm_gbs"], 4),
                       "peak_src": pk["src"]}},
        "finite": finite,
    }
    del xd, x_in, xq, xdd, aq, ad, sets, hx, hy
    for o in kvs + layers:
        o.free()
    tp.free()
    return res


def run_config0(torch):
    """BASELINE config 0 (the reference's own CPU-runnable scale): one
    Qwen2.5-0.5B layer (hidden 896, 14 Q / 2 KV heads, head_dim 64,
    intermediate 4864), a 64-token prefill then one decode step at context 65,
    fp32 KV.  Device time of each with CUDA events (the prefill re-run over the
    same positions), on its own context (RoPE tables for head_dim 64)."""
    import sib200
    c0 = sib200.Context(0, max_positions=256, rope_theta=1e6, head_dim=64)
    stream = torch.cuda.ExternalStream(c0.stream)
    try:
        layer = c0.layer_synth(DIMS_05B, 0)
        kv = c0.kv(DIMS_05B, 1, C0_PREFILL + 2, True)
        g = torch.Generator(device="cuda").manual_seed(0)
        X = torch.randn(C0_PREFILL, DIMS_05B["hidden"], device="cuda", generator=g)
        Y = torch.empty_like(X)
        xd = torch.randn(1, DIMS_05B["hidden"], device="cuda", generator=g)
        yd = torch.empty_like(xd)
        torch.cuda.synchronize()
        pf = lambda _=0: layer.prefill_dev(kv, 0, X, C0_PREFILL, 0, Y, sib200.SI_LAYER_FULL)
        dec = lambda _=0: layer.decode_dev(kv, xd, [C0_PREFILL + 1], yd, sib200.SI_LAYER_FULL)
        for _ in range(3):
            pf()
            dec()
        reps = 50
        tpf = time_region(torch, stream, pf, reps) / reps
        tdec = time_region(torch, stream, dec, reps) / reps
        c0.status()
        out = {"workload": "BASELINE config 0: one Qwen2.5-0.5B layer (hidden 896, 14 Q / 2 KV "
                           "heads, head_dim 64, intermediate 4864), 64-token prefill then one "
                           "decode step (context 65), fp32 KV",
               "prefill_us": round(tpf * 1e6, 1), "prefill_tok_s": round(C0_PREFILL / tpf, 1),
               "decode_us_per_token": round(tdec * 1e6, 2),
               "timing": "CUDA events, eager launches, 50 repetitions"}
        kv.free()
        layer.free()
        return out
    finally:
        c0.sync()
        c0.close()


def run_config2(ctx, torch, stream, args, peak):
    """one Qwen2.5-7B layer, a 2048-token prefill (fp16 KV)
    then 128 decode steps at batch 1; and config 3: one decode step of 64
    sequences over fp32 KV histories of 4096 positions."""
    import sib200
    layer = ctx.layer_synth(DIMS_7B, 2)
    H = DIMS_7B["hidden"]
    g = torch.Generator(device="cuda").manual_seed(2)
    kv = ctx.kv(DIMS_7B, 1, C2_PREFILL + C2_DECODE + 1, False)
    X = torch.randn(C2_PREFILL, H, device="cuda", generator=g)
    Y = torch.empty_like(X)
    xd = torch.randn(C2_DECODE, H, device="cuda", generator=g)
    yd = torch.empty_like(xd)
    torch.cuda.synchronize()
    pf = lambda _=0: layer.prefill_dev(kv, 0, X, C2_PREFILL, 0, Y, sib200.SI_LAYER_FULL)
    for _ in range(3):
        pf()
    tpf = time_region(torch, stream, pf, 5) / 5
    # Decode: two steps (x -> y -> x) captured with device context lengths and
    # replayed, 128 steps in all.
    st = ctx.decode_state([C2_PREFILL + 1], C2_PREFILL + C2_DECODE + 1)
    xa, ya = xd[0:1].clone(), torch.empty_like(xd[0:1])

    def two_steps():
        layer.decode_state_dev(kv, xa, st, ya, sib200.SI_LAYER_FULL)
        st.advance()
        layer.decode_state_dev(kv, ya, st, xa, sib200.SI_LAYER_FULL)
        st.advance()
    two_steps()
    ctx.sync()
    gph = ctx.capture(two_steps)
    gph.launch()
    st.set([C2_PREFILL + 1])
    tdec = time_region(torch, stream, lambda i: gph.launch(), C2_DECODE // 2) / C2_DECODE
    ctx.status()
    gph.free()
    st.free()
    dec = lambda i: layer.decode_dev(kv, xd[i], [C2_PREFILL + i + 1], yd[i], sib200.SI_LAYER_FULL)
    for i in range(3):
        dec(i)
    tdec_eager = time_region(torch, stream, dec, C2_DECODE) / C2_DECODE
    # e2e: the host-pointer C ABI (si_prefill / si_decode_step), pinned numpy buffers
    hx = torch.randn(C2_PREFILL, H).pin_memory().numpy()
    hy = torch.empty(C2_PREFILL, H).pin_memory().numpy()
    layer.prefill(kv, 0, hx, C2_PREFILL, 0, hy, sib200.SI_LAYER_FULL)
    reps = 5
    t0 = time.perf_counter()
    for _ in range(reps):
        layer.prefill(kv, 0, hx, C2_PREFILL, 0, hy, sib200.SI_LAYER_FULL)
    te = (time.perf_counter() - t0) / reps
    hxd, hyd = hx[:1].copy(), hy[:1].copy()
    t0 = time.perf_counter()
    for i in range(C2_DECODE):
        layer.decode(kv, hxd, [C2_PREFILL + i + 1], hyd, sib200.SI_LAYER_FULL)
    ted = (time.perf_counter() - t0) / C2_DECODE
    # the prefill's dominant kernel at 2048 tokens
    I = DIMS_7B["intermediate"]
    xq = torch.empty(C2_PREFILL * H, dtype=torch.int8, device="cuda")
    xdd = torch.empty(C2_PREFILL * H // 32, dtype=torch.int16, device="cuda")
    aq = torch.empty(C2_PREFILL * I, dtype=torch.int8, device="cuda")
    ad = torch.empty(C2_PREFILL * I // 32, dtype=torch.int16, device="cuda")
    torch.cuda.synchronize()
    ctx.q8_quantize(X, C2_PREFILL, H, xq, xdd)
    gm, um = layer.matrix(2), layer.matrix(3)
    gu = lambda i: ctx.gateup_q8(gm, um, xq, xdd, C2_PREFILL, aq, ad)
    gu(0)
    tg = time_region(torch, stream, gu, 10) / 10
    gu_ops = 2 * C2_PREFILL * 2 * I * H
    ctx.status()
    kv.free()
    pk = peaks()
    wb = layer_weight_bytes(DIMS_7B)
    mean_ctx = C2_PREFILL + (C2_DECODE + 1) / 2
    dbytes = wb + mean_ctx * DIMS_7B["n_kv_heads"] * 128 * 2 * 2
    out2 = {"workload": "BASELINE config 2: one Qwen2.5-7B layer (hidden 3584, 28 Q / 4 KV "
                        "heads, intermediate 18944), 2048-token prefill (fp16 KV), then 128 "
                        "decode steps at batch 1",
            "prefill_ms": round(tpf * 1e3, 3), "prefill_tok_s": round(C2_PREFILL / tpf, 1),
            "decode_us_per_token": round(tdec * 1e6, 2),
            "decode_launch": "CUDA graph of two steps with device-resident context lengths",
            "decode_us_per_token_eager": round(tdec_eager * 1e6, 2),
            "e2e": {"prefill_tok_s": round(C2_PREFILL / te, 1),
                    "decode_us_per_token": round(ted * 1e6, 2),
                    "h2d_bytes_per_step": C2_PREFILL * H * 4, "d2h_bytes_per_step": C2_PREFILL * H * 4,
                    "how": "si_prefill / si_decode_step (host pointers, pinned), wall clock "
                           "around each synchronous call"},
            "roofline": {"prefill_gateup": {"achieved_tops": round(gu_ops / tg / 1e12, 2),
                                            "us": round(tg * 1e6, 2), "peak_tops": peak["tops"],
                                            "frac": round(gu_ops / tg / 1e12 / peak["tops"], 4)},
                         "prefill_layer": {"achieved_tops": round(layer_int8_ops(DIMS_7B, C2_PREFILL) / tpf / 1e12, 2),
                                           "frac": round(layer_int8_ops(DIMS_7B, C2_PREFILL) / tpf / 1e12 / peak["tops"], 4)},
                         "decode_step": {"bytes": int(dbytes),
                                         "achieved_gbs": round(dbytes / tdec / 1e9, 1),
                                         "frac": round(dbytes / tdec / 1e9 / pk["hbm_gbs"], 4),
                                         "peak_gbs": pk["hbm_gbs"]}},
            "timing": "CUDA events on the library stream; decode steps launched eagerly"}
    del X, Y, xd, yd, xq, xdd, aq, ad
    # ---- config 3 ----
    B, L = C3_BATCH, C3_CTX
    kv3 = ctx.kv(DIMS_7B, B, L, True)
    kv3.fill_synth(3, 1.0, L - 1)
    X3 = torch.randn(B, H, device="cuda", generator=g)
    Y3 = torch.empty_like(X3)
    torch.cuda.synchronize()
    d3 = lambda _=0: layer.decode_dev(kv3, X3, [L] * B, Y3, sib200.SI_LAYER_FULL)
    for _ in range(3):
        d3()
    t3 = time_region(torch, stream, d3, 20) / 20
    ctx.status()
    kv3.free()
    layer.free()
    kvb = B * L * DIMS_7B["n_kv_heads"] * DIMS_7B["head_dim"] * 2 * 4
    b3 = kvb + wb
    out3 = {"workload": "BASELINE config 3: one Qwen2.5-7B layer, one decode step of 64 "
                        "sequences over fp32 KV histories of 4096 positions",
            "us_per_step": round(t3 * 1e6, 2), "us_per_token": round(t3 * 1e6 / B, 3),
            "tok_s": round(B / t3, 1), "kv_bytes_per_step": kvb,
            "roofline": {"bytes": b3, "achieved_gbs": round(b3 / t3 / 1e9, 1),
                         "frac": round(b3 / t3 / 1e9 / pk["hbm_gbs"], 4)}}
    return out2, out3


class ProjectionSet:
    """the 1.5B projection set, ten weight copies (263 MB)."""

    def __init__(self, ctx, torch, copies, seed=1):
        self.ctx, self.torch = ctx, torch
        self.sets = []
        for c in range(copies):
            s = seed * 1000 + 10 * c
            self.sets.append(dict(
                qkv=ctx.matrix_synth(QKV1, H1, s + 1), o=ctx.matrix_synth(H1, H1, s + 2),
                gate=ctx.matrix_synth(I1, H1, s + 3), up=ctx.matrix_synth(I1, H1, s + 4),
                down=ctx.matrix_synth(H1, I1, s + 5)))
        g = torch.Generator(device="cuda").manual_seed(seed)
        self.bias = (torch.randn(QKV1, device="cuda", generator=g) * 0.02).contiguous()
        ctx.sync()

    def buffers(self, M):
        t, dev = self.torch, "cuda"
        return dict(
            x=t.randn(M, H1, device=dev), oin=t.randn(M, H1, device=dev),
            xq=t.empty(M * H1, dtype=t.int8, device=dev), xd=t.empty(M * H1 // 32, dtype=t.int16, device=dev),
            oq=t.empty(M * H1, dtype=t.int8, device=dev), od=t.empty(M * H1 // 32, dtype=t.int16, device=dev),
            aq=t.empty(M * I1, dtype=t.int8, device=dev), ad=t.empty(M * I1 // 32, dtype=t.int16, device=dev),
            qkv=t.empty(M, QKV1, device=dev), yo=t.empty(M, H1, device=dev), yd=t.empty(M, H1, device=dev))

    def step(self, b, M, i):
        ctx, w = self.ctx, self.sets[i % len(self.sets)]
        ctx.q8_quantize(b["x"], M, H1, b["xq"], b["xd"])
        ctx.matmul(w["qkv"], b["xq"], b["xd"], M, self.bias, b["qkv"])
        ctx.q8_quantize(b["oin"], M, H1, b["oq"], b["od"])
        ctx.matmul(w["o"], b["oq"], b["od"], M, None, b["yo"])
        ctx.gateup_q8(w["gate"], w["up"], b["xq"], b["xd"], M, b["aq"], b["ad"])
        ctx.matmul(w["down"], b["aq"], b["ad"], M, None, b["yd"])

    def free(self):
        for s in self.sets:
            for m in s.values():
                m.free()
        self.sets = []


def run_config1(ctx, torch, stream):
    """The 1.5B projection set over BASELINE config 1's token counts, CUDA graph
    replays over ten weight copies (more than twice L2)."""
    ps = ProjectionSet(ctx, torch, C1_COPIES)
    sweep = {}
    for M in SWEEP_M:
        b = ps.buffers(M)
        ps.step(b, M, 0)
        ctx.sync()
        gph = ctx.capture(lambda: [ps.step(b, M, c) for c in range(C1_COPIES)])
        gph.launch()
        reps = 20 if M <= 16 else 3
        ts = time_region(torch, stream, lambda i: gph.launch(), reps) / (reps * C1_COPIES)
        sweep[str(M)] = {"ms_per_step": round(ts * 1e3, 4), "tok_s": round(M / ts, 1)}
        gph.free()
        del b
    ps.free()
    return {"workload": "BASELINE config 1: Qwen2.5-1.5B projection set (QKV 2048x1536 +bias, "
                        "o 1536^2, gate+up 2x8960x1536 +SiLU*mul+Q8, down 1536x8960), each "
                        "behind its Q8_0 quantiser",
            "sweep": sweep,
            "timing": "CUDA graph replays over 10 weight copies (263 MB), CUDA events"}


def decode_gemv_roofline(ctx, torch, stream):
    """Kernel-level decode roofline where the GEMV is HBM-bound: the 72B down
    projection (8192 x 29568, 136 MB of Q4_0) at 1 token (dp4a form) and at 8
    tokens (tensor-core form, config 4's batch), and the 7B down projection at
    1 token, each also from row-major GGUF blocks without the repack; weight
    copies (272-305 MB) rotate so every launch streams from HBM; CUDA graph
    replays timed with CUDA events."""
    pk = peaks()
    out = {}
    for label, N, K, M, ncopy in (("72B down, 1 token", 8192, 29568, 1, 2),
                                  ("72B down, 8 tokens", 8192, 29568, 8, 2),
                                  ("7B down, 1 token", 3584, 18944, 1, 8)):
        mats = [ctx.matrix_synth(N, K, seed=90 + i) for i in range(ncopy)]
        x = torch.randn(M, K, device="cuda")
        qs = torch.empty(M * K, dtype=torch.int8, device="cuda")
        d = torch.empty(M * K // 32, dtype=torch.int16, device="cuda")
        y = torch.empty(M * N, device="cuda")
        torch.cuda.synchronize()
        ctx.q8_quantize(x, M, K, qs, d)
        ctx.sync()
        gph = ctx.capture(lambda: [ctx.matmul(m, qs, d, M, None, y) for m in mats])
        for _ in range(3):
            gph.launch()
        reps = 20
        t = time_region(torch, stream, lambda i: gph.launch(), reps) / (reps * ncopy)
        wb = N * K * 18 // 32
        out[label] = {"kernel": "k_gemv (dp4a form)" if M <= 2 else "k_gemv_mma (tensor-core form)",
                      "shape": f"{N}x{K}", "tokens": M, "us": round(t * 1e6, 2),
                      "weight_bytes": wb, "achieved_gbs": round(wb / t / 1e9, 1),
                      "peak_gbs": pk["hbm_gbs"], "peak_src": pk["src"],
                      "frac": round(wb / t / 1e9 / pk["hbm_gbs"], 4)}
        gph.free()
        if M <= 8:
            # The same projection from row-major GGUF blocks (no repack).
            gg = [torch.from_numpy(m.download_gguf()).cuda() for m in mats]
            torch.cuda.synchronize()
            gph = ctx.capture(lambda: [ctx.matvec_gguf(w_, N, K, qs, d, M, None, y) for w_ in gg])
            for _ in range(3):
                gph.launch()
            t = time_region(torch, stream, lambda i: gph.launch(), reps) / (reps * ncopy)
            out[label + ", row-major GGUF (no repack)"] = {
                "kernel": "k_gemv_gguf", "shape": f"{N}x{K}", "tokens": M,
                "us": round(t * 1e6, 2), "weight_bytes": wb,
                "achieved_gbs": round(wb / t / 1e9, 1), "peak_gbs": pk["hbm_gbs"],
                "frac": round(wb / t / 1e9 / pk["hbm_gbs"], 4)}
            gph.free()
            del gg
        for m in mats:
            m.free()
    return out


def gemm_schemes(ctx, torch, stream, int8_peak_tops):
    """The prefill projection's schemes side by side on the 72B o shape (8192 x
    8192 Q4_0, 4096 tokens): this library's exact tcgen05 kind::i8 GEMM (the
    dispatched prefill path from K = 4096), its fused-rescale form (one FMA per
    block, within 1e-6), the mma.sync GEMM, and the bf16 / fp16-dequant
    alternative -- weights dequantised once to bf16 / fp16 ((q - 8) * dw,
    stored as such), activations (qx * dx) likewise, a cuBLAS GEMM with fp32
    accumulation through torch.matmul.  Per scheme: time, int8-equivalent
    TOP/s (2*M*N*K), that against its own measured peak (the int8 tcgen05
    probe; MEASURED_PEAKS' bf16 figure for cuBLAS), and the largest difference
    from the exact scheme relative to the output's largest element."""
    import numpy as np
    N = K = 8192
    M = 4096
    m = ctx.matrix_synth(N, K, seed=21)
    g = torch.Generator(device="cuda").manual_seed(21)
    x = torch.randn(M, K, device="cuda", generator=g)
    qs = torch.empty(M * K, dtype=torch.int8, device="cuda")
    d = torch.empty(M * K // 32, dtype=torch.int16, device="cuda")
    torch.cuda.synchronize()
    ctx.q8_quantize(x, M, K, qs, d)
    ctx.sync()
    ops = 2.0 * M * N * K
    out, ys = {}, {}
    for name, kern in (("tcgen05 i8, exact", 1), ("tcgen05 i8, fused rescale", 5),
                       ("mma.sync i8, exact", 4)):
        y = torch.empty(M * N, device="cuda")
        ctx.matmul(m, qs, d, M, None, y, kernel=kern)
        ctx.sync()
        reps = 5
        t = time_region(torch, stream, lambda i: ctx.matmul(m, qs, d, M, None, y, kernel=kern),
                        reps) / reps
        ctx.status()
        ys[name] = y.view(M, N)
        out[name] = {"us": round(t * 1e6, 1), "tops": round(ops / t / 1e12, 1),
                     "frac_of_peak": round(ops / t / 1e12 / int8_peak_tops, 4) if int8_peak_tops else None,
                     "peak": "int8 tcgen05 probe"}
    ref = ys["tcgen05 i8, exact"].double()
    scale = float(ref.abs().max())
    # Dequantised operands: W[n][k] = (q - 8) * dw from the GGUF rows.
    raw = m.download_gguf().reshape(N, K // 32, 18)
    dw = raw[:, :, :2].copy().view(np.float16).astype(np.float32)          # [N][KB][1]
    nib = raw[:, :, 2:]
    q = np.concatenate([nib & 15, nib >> 4], axis=2).astype(np.float32) - 8.0
    w32 = torch.from_numpy((q * dw).reshape(N, K)).cuda()
    xq = qs.view(M, K // 32, 32).float() * d.view(M, K // 32, 1).view(torch.float16).float()
    xq = xq.view(M, K)
    pk = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json"))) if os.path.exists(
        os.path.join(ROOT, "MEASURED_PEAKS.json")) else {}
    for name, dt in (("bf16-dequant, cuBLAS", torch.bfloat16), ("fp16-dequant, cuBLAS", torch.float16)):
        wd, xd = w32.to(dt), xq.to(dt)
        torch.cuda.synchronize()
        yd = torch.matmul(xd, wd.t())
        torch.cuda.synchronize()
        reps = 5
        t = time_region(torch, stream, lambda i: torch.matmul(xd, wd.t()), reps) / reps
        err = float((yd.double() - ref).abs().max()) / scale
        out[name] = {"us": round(t * 1e6, 1), "tops": round(ops / t / 1e12, 1),
                     "frac_of_peak": round(ops / t / 1e12 / pk["bf16_tflops"], 4) if pk.get("bf16_tflops") else None,
                     "peak": "MEASURED_PEAKS bf16 (cuBLAS)", "max_err_vs_exact": err}
        del wd, xd, yd
    for name in ("tcgen05 i8, fused rescale", "mma.sync i8, exact"):
        out[name]["max_err_vs_exact"] = float((ys[name].double() - ref).abs().max()) / scale
    out["shape"] = f"{N}x{K} Q4_0, {M} tokens"
    out["bar"] = "projection outputs within 1e-5 relative of the reference (bit-exact for the exact schemes)"
    m.free()
    return out


def reference_layer_decode(ctx, torch, stream, n_tokens=32, context0=512):
    """The reference's own workload, apples to apples: its attention layer
    (RMSNorm, QKV + bias, RoPE, fp16 KV append, flash attention, o-projection;
    qwen_one_layer.c:237-281) at its compiled 1.5B dims, decoding n_tokens
    after a context0-position fp16 history.  Timed three ways: the reference's
    run_layer on one host core; this library's drop-in run_layer (host
    buffers, si_ref_run_layer: the call a reference caller makes); and the
    device-resident decode step (si_decode_step_dev, CUDA events).  Reports
    the largest output difference against the reference, over the outputs'
    largest magnitude."""
    import ctypes as C
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    import sib200
    from sib200 import synth
    dims = dict(hidden=1536, n_q_heads=12, n_kv_heads=2, head_dim=128, intermediate=0,
                rope_theta=1e6, rms_eps=1e-6)
    H, KVD, L = 1536, 256, context0 + n_tokens
    rng = np.random.default_rng(5)
    layer = synth.random_layer(dims, 5, mlp=False)
    kc0 = (rng.standard_normal(L * KVD) * 0.5).astype(np.float16).view(np.uint16)
    vc0 = (rng.standard_normal(L * KVD) * 0.5).astype(np.float16).view(np.uint16)
    xs = rng.standard_normal((n_tokens, H)).astype(np.float32)
    ctxs = [context0 + i + 1 for i in range(n_tokens)]
    res = {"workload": f"reference attention layer (1536 hidden, 12 Q / 2 KV heads, fp16 KV), "
                       f"{n_tokens} decode steps after {context0} positions",
           "tokens": n_tokens}
    ys_ref = None
    if os.path.exists(oracle.LIB_REF):
        ref = oracle.Reference()
        kr, vr = kc0.copy(), vc0.copy()
        ys_ref = np.zeros((n_tokens, H), np.float32)
        t0 = time.perf_counter()
        for i in range(n_tokens):
            ys_ref[i] = ref.run_layer(layer, xs[i], kr, vr, ctxs[i])[0]
        res["reference_host_us_per_token"] = round((time.perf_counter() - t0) / n_tokens * 1e6, 1)
        res["reference_cores"] = 1

    class LayerT(C.Structure):
        _fields_ = [(n, C.c_void_p) for n in ("wq", "wk", "wv", "wo", "norm", "bq", "bk", "bv")]

    class PhaseT(C.Structure):
        _fields_ = [(n, C.c_float) for n in ("rms", "q8_input", "q_proj", "k_proj", "v_proj",
                                             "rope_cache", "attention", "q8_output", "out_proj")]
    Lb = ctx.L
    Lb.si_ref_run_layer.restype = PhaseT
    Lb.si_ref_run_layer.argtypes = ([C.c_void_p] * 4 + [C.c_int, C.c_void_p, C.c_int] +
                                    [C.c_void_p] * 3 + [C.c_int] * 4 + [C.c_float] * 2)
    lt = LayerT(*[layer[k].ctypes.data for k in ("wq", "wk", "wv", "wo", "norm", "bq", "bk", "bv")])
    kd, vd = kc0.copy(), vc0.copy()
    y = np.zeros(H, np.float32)
    ys_drop = np.zeros((n_tokens, H), np.float32)
    call = lambda i: Lb.si_ref_run_layer(C.addressof(lt), xs[i].ctypes.data, kd.ctypes.data,
                                         vd.ctypes.data, ctxs[i], y.ctypes.data, 1, None, None,
                                         None, H, 12, 2, 128, 1e6, 1e-6)
    call(0)  # uploads and caches the weights
    kd[:], vd[:] = kc0, vc0
    t0 = time.perf_counter()
    for i in range(n_tokens):
        call(i)
        ys_drop[i] = y
    res["dropin_run_layer_us_per_token"] = round((time.perf_counter() - t0) / n_tokens * 1e6, 1)
    for k in ("wq", "wk", "wv", "wo"):
        Lb.si_forget_host_weights(layer[k].ctypes.data)
    gl = ctx.layer(dims, layer)
    kv = ctx.kv(dims, 1, L, False)
    kv.write(0, 0, kc0[: context0 * KVD].reshape(context0, KVD),
             vc0[: context0 * KVD].reshape(context0, KVD))
    xd = torch.from_numpy(xs).cuda()
    yd = torch.zeros_like(xd)
    torch.cuda.synchronize()
    t = time_region(torch, stream, lambda i: gl.decode_dev(kv, xd[i], [ctxs[i]], yd[i],
                                                           sib200.SI_LAYER_ATTN), n_tokens)
    res["device_us_per_token"] = round(t / n_tokens * 1e6, 2)
    ys_dev = yd.cpu().numpy()
    if ys_ref is not None:
        scale = float(np.abs(ys_ref).max())
        res["max_err_vs_reference"] = {
            "dropin": float(np.abs(ys_drop - ys_ref).max() / scale),
            "device": float(np.abs(ys_dev - ys_ref).max() / scale)}
    kv.free()
    gl.free()
    return res


def extra(result, key, fn):
    """A failed extra measurement must not lose the bench line."""
    try:
        result[key] = fn()
        log(f"{key}: {result[key]}")
    except Exception as exc:
        result[key] = {"error": f"{type(exc).__name__}: {str(exc)[:300]}"}
        log(f"{key} failed: {exc}")


def run_ours(args, rank, world, local_rank):
    import gc
    import torch
    import sib200
    torch.cuda.set_device(local_rank)
    ctx = sib200.Context(local_rank, max_positions=TP_MAX_CTX, rope_theta=1e6, head_dim=128)
    stream = torch.cuda.ExternalStream(ctx.stream)
    dist = world > 1
    if dist:
        import torch.distributed as tdist

    def barrier_sync():
        torch.cuda.synchronize()
        ctx.sync()
        if dist:
            tdist.barrier()

    def max_over_ranks(v):
        if not dist:
            return v
        t = torch.tensor([v], device="cuda", dtype=torch.float64)
        tdist.all_reduce(t, op=tdist.ReduceOp.MAX)
        return float(t.item())

    peak = int8_peak(ctx, torch, stream)
    log(f"int8 peak {peak}")
    c4 = run_config4(args, rank, world, local_rank, ctx, torch, barrier_sync, max_over_ranks, peak)
    result = {
        "metric": METRIC, "value": c4["value"], "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": c4["ms_per_step"],
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "i8",
        "data": "synthetic (seeded Q4_0 N(0,0.02) weights, N(0,1) activations and KV)",
        "config": {"workload": "BASELINE config 4: 8 Qwen2.5-72B layers (hidden 8192, 64 Q / 8 KV "
                               "heads, intermediate 29568), Q4_0 x Q8_0, fp32 KV; one step = a "
                               "4096-token prefill through the 8 layers",
                   "prefill_tokens_per_step": TP_PREFILL, "layers": TP_LAYERS,
                   "parallelism": f"tp{world} (column-sharded QKV/gate/up, row-sharded o/down)",
                   "l2": f"inputs larger than L2: {TP_LAYERS * layer_weight_bytes(CONFIG4) / 1e9 / world:.2f} "
                         "GB of weights per rank per step",
                   "timing": "CUDA events on the library stream, max over ranks; eager launches"},
        "decode_us_per_token": c4["decode"]["us_per_token"],
        "decode": c4["decode"],
        "roofline": c4["roofline"],
        "layer_roofline": c4["layer_roofline"],
        "int8_peak": peak,
        "e2e": c4["e2e"],
        "gpu_launches": c4["gpu_launches"],
        "clocks": c4["clocks"],
        "finite": c4["finite"],
    }
    gc.collect()
    if world == 1:
        def cfg23():
            c2, c3 = run_config2(ctx, torch, stream, args, peak)
            result["config3"] = c3
            return c2
        extra(result, "config2", cfg23)
        extra(result, "config1", lambda: run_config1(ctx, torch, stream))
        extra(result, "config0", lambda: run_config0(torch))
        extra(result, "decode_gemv_roofline", lambda: decode_gemv_roofline(ctx, torch, stream))
        extra(result, "gemm_schemes", lambda: gemm_schemes(
            ctx, torch, stream, (result.get("int8_peak") or {}).get("tops")))
        extra(result, "reference_layer", lambda: reference_layer_decode(ctx, torch, stream))
        if not args.no_cpu_baseline:
            log("cpu baselines")
            extra(result, "cpu_baseline", lambda: cpu_layer_baseline(
                CONFIG4, TP_LAYERS, TP_PREFILL, TP_PREFILL + TP_DECODE // 2 + 1, True,
                args.cpu_seconds, 4, "config 4 (72B dims, fp32 KV)"))
            if isinstance(result.get("config2"), dict) and "error" not in result["config2"]:
                extra(result["config2"], "cpu_baseline", lambda: cpu_layer_baseline(
                    DIMS_7B, 1, C2_PREFILL, C2_PREFILL + C2_DECODE // 2 + 1, False,
                    args.cpu_seconds / 2, 2, "config 2 (7B dims, fp16 KV)"))
            if isinstance(result.get("config3"), dict):
                extra(result["config3"], "cpu_baseline", lambda: cpu_config3(args.cpu_seconds / 3))
            if isinstance(result.get("config0"), dict) and "error" not in result["config0"]:
                extra(result["config0"], "cpu_baseline", lambda: cpu_layer_baseline(
                    DIMS_05B, 1, C0_PREFILL, C0_PREFILL + 1, True, min(3.0, args.cpu_seconds),
                    0, "config 0 (0.5B dims, fp32 KV)"))
    torch.cuda.synchronize()
    ctx.sync()
    gc.collect()
    ctx.h = None  # the stream is left to process exit (torch events may reference it)
    return result


def cpu_config3(seconds):
    """Config 3 on the host: 64 sequences x one token at context 4096 through
    one 7B layer (fp32 KV) = 64 per-token layer steps; timed on a sample."""
    threads = len(os.sched_getaffinity(0))
    cl = CpuLayer(DIMS_7B, 3, C3_CTX + 1, threads, True)
    try:
        x = np.random.default_rng(3).standard_normal(DIMS_7B["hidden"]).astype(np.float32)
        cl.token(x, C3_CTX)
        n, t0 = 0, time.perf_counter()
        while n < 1 or time.perf_counter() - t0 < seconds:
            cl.token(x, C3_CTX)
            n += 1
        per = (time.perf_counter() - t0) / n
    finally:
        cl.close()
    return {"value": round(C3_BATCH * per * 1e6, 1), "unit": "us/step", "cores": threads,
            "kind": cl.kind,
            "sample": f"{n} tokens at context {C3_CTX} through one 7B layer on {threads} "
                      f"threads, x {C3_BATCH} sequences per step"}


# ---------------------------------------------------------------------------
# reference arm
# ---------------------------------------------------------------------------
def run_reference(args, rank):
    if rank != 0:
        return None
    threads = len(os.sched_getaffinity(0))
    cl = CpuLayer(CONFIG4, 4, TP_MAX_CTX + 1, threads, True)
    dctx = TP_PREFILL + TP_DECODE // 2 + 1
    try:
        cpu_layer_rounds(cl, TP_PREFILL, dctx, rounds=args.warmup)
        r = cpu_layer_rounds(cl, TP_PREFILL, dctx, rounds=args.steps)
    finally:
        cl.close()
    t_prefill = TP_LAYERS * TP_PREFILL * r["prefill_s_per_token_layer"]
    v = TP_PREFILL / t_prefill
    sample = (f"{r['prefill_tokens']} prefill tokens at contexts {r['contexts']} and "
              f"{r['decode_tokens']} decode tokens at context {dctx} through one 72B layer on "
              f"{threads} threads ({args.steps} steps of one round each), extrapolated "
              f"linearly to {TP_PREFILL} tokens x {TP_LAYERS} layers; matvec/quantize_q8 "
              f"{cl.kind}, rmsnorm/rope/attention the oracle's restatement")
    return {"impl": "reference", "metric": METRIC, "value": round(v, 4), "unit": "tok/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(t_prefill * 1e3, 1), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "i8", "data": "synthetic",
            "config": {"workload": "BASELINE config 4: 8 Qwen2.5-72B layers, 4096-token prefill "
                                   "(the reference's prefill on a CPU is its per-token decode "
                                   "loop, bench_ai_dma_prefill.c:104-108)",
                       "parallelism": f"host cores ({threads} threads)"},
            "decode_us_per_token": round(TP_LAYERS * r["decode_s_per_token_layer"] * 1e6, 1),
            "cpu_baseline": {"value": round(v, 4), "unit": "tok/s", "cores": threads,
                             "kind": cl.kind, "sample": sample},
            "e2e": {"value": round(v, 4), "unit": "tok/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}


# ---------------------------------------------------------------------------
# untimed workloads for profilers
# ---------------------------------------------------------------------------
def probe_config4_layer():
    """One Qwen2.5-72B layer on GPU 0 (TP = 1): three decode steps of a batch
    of 8 at context 4097.. and one 4096-token prefill, no timing."""
    import torch
    import sib200
    torch.cuda.set_device(0)
    ctx = sib200.Context(0, max_positions=TP_MAX_CTX, rope_theta=1e6, head_dim=128)
    layer = ctx.layer_synth(CONFIG4, 4)
    kv = ctx.kv(CONFIG4, TP_BATCH, TP_MAX_CTX, True)
    kv.fill_synth(4, 1.0, TP_PREFILL)
    g = torch.Generator(device="cuda").manual_seed(4)
    x = torch.randn(TP_BATCH, CONFIG4["hidden"], device="cuda", generator=g)
    xp = torch.randn(TP_PREFILL, CONFIG4["hidden"], device="cuda", generator=g)
    y, yp = torch.empty_like(x), torch.empty_like(xp)
    torch.cuda.synchronize()
    for i in range(3):
        layer.decode_dev(kv, x, [TP_PREFILL + 1 + i] * TP_BATCH, y, sib200.SI_LAYER_FULL)
    layer.prefill_dev(kv, 0, xp, TP_PREFILL, 0, yp, sib200.SI_LAYER_FULL)
    ctx.sync()
    ctx.status()
    print("ok")


def probe_gateup_72b():
    """The headline's dominant kernel alone: the gate/up GEMM (+SiLU*mul, Q8) of
    one 72B layer at 4096 tokens, three launches, no timing."""
    import torch
    import sib200
    torch.cuda.set_device(0)
    ctx = sib200.Context(0, max_positions=256, rope_theta=1e6, head_dim=128)
    H, I, M = CONFIG4["hidden"], CONFIG4["intermediate"], TP_PREFILL
    gm, um = ctx.matrix_synth(I, H, 5), ctx.matrix_synth(I, H, 6)
    x = torch.randn(M, H, device="cuda")
    xq = torch.empty(M * H, dtype=torch.int8, device="cuda")
    xd = torch.empty(M * H // 32, dtype=torch.int16, device="cuda")
    aq = torch.empty(M * I, dtype=torch.int8, device="cuda")
    ad = torch.empty(M * I // 32, dtype=torch.int16, device="cuda")
    torch.cuda.synchronize()
    ctx.q8_quantize(x, M, H, xq, xd)
    for _ in range(3):
        ctx.gateup_q8(gm, um, xq, xd, M, aq, ad)
    ctx.sync()
    ctx.status()
    print("ok")


def probe_config2_decode():
    """One Qwen2.5-7B layer on GPU 0: three decode steps at batch 1 after a
    2048-position fp16 history, no timing."""
    import torch
    import sib200
    torch.cuda.set_device(0)
    ctx = sib200.Context(0, max_positions=TP_MAX_CTX, rope_theta=1e6, head_dim=128)
    layer = ctx.layer_synth(DIMS_7B, 2)
    kv = ctx.kv(DIMS_7B, 1, 2176, False)
    kv.fill_synth(2, 1.0, 2048)
    g = torch.Generator(device="cuda").manual_seed(2)
    x = torch.randn(3, DIMS_7B["hidden"], device="cuda", generator=g)
    y = torch.empty_like(x)
    torch.cuda.synchronize()
    for i in range(3):
        layer.decode_dev(kv, x[i], [2049 + i], y[i], sib200.SI_LAYER_FULL)
    ctx.sync()
    ctx.status()
    print("ok")


def probe_attn_prefill_72b():
    """The prefill attention of one 72B layer (4096 causal tokens, 64 Q / 8 KV
    heads, fp32 KV) through the default (tcgen05) kernel, three launches, no
    timing."""
    import torch
    import sib200
    torch.cuda.set_device(0)
    ctx = sib200.Context(0, max_positions=TP_PREFILL, rope_theta=1e6, head_dim=128)
    dims = dict(CONFIG4, intermediate=0)
    kv = ctx.kv(dims, 1, TP_PREFILL, True)
    kv.fill_synth(4, 1.0, TP_PREFILL)
    q = torch.randn(TP_PREFILL * CONFIG4["n_q_heads"] * 128, device="cuda")
    out = torch.empty_like(q)
    torch.cuda.synchronize()
    for _ in range(3):
        ctx.attention_prefill(kv, dims, q, TP_PREFILL, 0, 0, out)
    ctx.sync()
    ctx.status()
    print("ok")


PROBES = {"config4-layer": probe_config4_layer, "config2-decode": probe_config2_decode,
          "gateup-72b": probe_gateup_72b, "attn-prefill-72b": probe_attn_prefill_72b}


def main():
    import faulthandler
    faulthandler.enable()
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--probe", choices=sorted(PROBES),
                    help="run one untimed workload for a profiler and exit")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.probe:
        PROBES[args.probe]()
        return
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        res = run_reference(args, rank)
        if res is not None:
            print(json.dumps(res), flush=True)
        return
    if world > 1:
        import datetime
        import torch
        import torch.distributed as tdist
        torch.cuda.set_device(local_rank)
        tdist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                 device_id=torch.device("cuda", local_rank))
    res = run_ours(args, rank, world, local_rank)
    if world > 1:
        import torch.distributed as tdist
        tdist.barrier()
        tdist.destroy_process_group()
    if rank == 0:
        print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
