#!/usr/bin/env python3
"""Benchmark of the Q4_0 x Q8_0 projection hot path.

Workload: the Qwen2.5-1.5B projection set -- fused
QKV 2048x1536 (+bias), o 1536x1536, gate+up 2x8960x1536 (+SiLU*mul, Q8 epilogue),
down 1536x8960 -- each behind its Q8_0 activation quantiser.  One step = one pass
of the whole set over M tokens of synthetic activations.

* value  = prefill tokens/s at M = 2048 (whole job, all ranks), device-timed with
           CUDA events on the library's stream, inputs resident in HBM;
* e2e    = the same through the C ABI with pinned host buffers: host->device copy
           of the step's two fp32 inputs and device->host copy of its three fp32
           outputs inside the timed region, steps pipelined over two buffer sets
           (copies of neighbouring steps overlap the compute on their own streams);
* decode = the same set at M = 1 (microseconds per token) in `decode`;
* roofline: the dominant kernel's algorithmic throughput against MEASURED_PEAKS.json;
* cpu_baseline: the reference's own matvec_q4q8/quantize_q8 (oracle/_ref when built
  here, else the oracle restatement) on the host cores, on a bounded token sample;
* config2 / config3 / tp_config4: the other BASELINE configurations' layer steps;
* decode_gemv_roofline: the decode GEMV at shapes where it is HBM-bound (72B and
  7B down projections, 1 and 8 tokens) against the measured HBM bandwidth;
* reference_layer: the reference's own attention layer (1.5B dims, fp16 KV)
  timed as its run_layer on one host core, this library's drop-in run_layer
  and the device decode step, with the error against the reference.

Weights are seeded synthetic Q4_0 (N(0, 0.02)); ten weight copies (263 MB, over
twice the 126 MB L2) are rotated across steps so every step streams from HBM.
`--impl reference` times the reference's CPU implementation on this workload.
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

H, I = 1536, 8960
QKV_N = 2048
PREFILL_M = 2048
COPIES = 10
METRIC = "Qwen layer prefill tok/s + decode µs/token; % of HBM / int8-TC roofline"
INT8_SPEC_TOPS = 4500.0  # B200 dense int8 tensor-core spec; not in MEASURED_PEAKS.json
SWEEP_M = (1, 16, 128, 512, 2048)  # BASELINE config 1 token counts
# DRAM bytes (read + write) per launch of the gate/up GEMM at M = 2048, from one
# `ncu --set full -k regex:k_gemm_mma -s 2 -c 1` capture of
# `bench.py --steps 2 --warmup 3 --no-tp --no-cpu-baseline` (its first, cold
# step); re-measure when the kernel changes.
NCU_TRAFFIC = {"gateup": 19091456}


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return {"hbm_gbs": d["hbm_gbs"], "src": "measured"}
    return {"hbm_gbs": 6650.0, "src": "fallback"}


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


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
class ProjectionSet:
    """Device weights (several copies) and activation buffers for one M."""

    def __init__(self, ctx, torch, copies: int, seed: int = 1):
        self.ctx, self.torch = ctx, torch
        self.sets = []
        for c in range(copies):
            s = seed * 1000 + 10 * c
            self.sets.append(dict(
                qkv=ctx.matrix_synth(QKV_N, H, s + 1), o=ctx.matrix_synth(H, H, s + 2),
                gate=ctx.matrix_synth(I, H, s + 3), up=ctx.matrix_synth(I, H, s + 4),
                down=ctx.matrix_synth(H, I, s + 5)))
        g = torch.Generator(device="cuda").manual_seed(seed)
        self.bias = (torch.randn(QKV_N, device="cuda", generator=g) * 0.02).contiguous()
        ctx.sync()

    def buffers(self, M):
        t = self.torch
        dev = "cuda"
        return dict(
            x=t.randn(M, H, device=dev), oin=t.randn(M, H, device=dev),
            xq=t.empty(M * H, dtype=t.int8, device=dev), xd=t.empty(M * H // 32, dtype=t.int16, device=dev),
            oq=t.empty(M * H, dtype=t.int8, device=dev), od=t.empty(M * H // 32, dtype=t.int16, device=dev),
            aq=t.empty(M * I, dtype=t.int8, device=dev), ad=t.empty(M * I // 32, dtype=t.int16, device=dev),
            qkv=t.empty(M, QKV_N, device=dev), yo=t.empty(M, H, device=dev), yd=t.empty(M, H, device=dev))

    def step(self, b, M, i, timers=None):
        """One pass of the projection set; returns the number of kernels launched."""
        ctx, w = self.ctx, self.sets[i % len(self.sets)]
        ev = timers
        if ev: ev[0].record()
        ctx.q8_quantize(b["x"], M, H, b["xq"], b["xd"])
        if ev: ev[1].record()
        ctx.matmul(w["qkv"], b["xq"], b["xd"], M, self.bias, b["qkv"])
        if ev: ev[2].record()
        ctx.q8_quantize(b["oin"], M, H, b["oq"], b["od"])
        if ev: ev[3].record()
        ctx.matmul(w["o"], b["oq"], b["od"], M, None, b["yo"])
        if ev: ev[4].record()
        ctx.gateup_q8(w["gate"], w["up"], b["xq"], b["xd"], M, b["aq"], b["ad"])
        if ev: ev[5].record()
        ctx.matmul(w["down"], b["aq"], b["ad"], M, None, b["yd"])
        if ev: ev[6].record()
        return 6

    def kernel(self, b, M, i, name):
        """Launch one kernel of the step (for per-kernel timing)."""
        ctx, w = self.ctx, self.sets[i % len(self.sets)]
        if name == "q8_x":
            ctx.q8_quantize(b["x"], M, H, b["xq"], b["xd"])
        elif name == "qkv":
            ctx.matmul(w["qkv"], b["xq"], b["xd"], M, self.bias, b["qkv"])
        elif name == "q8_o":
            ctx.q8_quantize(b["oin"], M, H, b["oq"], b["od"])
        elif name == "o":
            ctx.matmul(w["o"], b["oq"], b["od"], M, None, b["yo"])
        elif name == "gateup":
            ctx.gateup_q8(w["gate"], w["up"], b["xq"], b["xd"], M, b["aq"], b["ad"])
        else:
            ctx.matmul(w["down"], b["aq"], b["ad"], M, None, b["yd"])

    def free(self):
        for s in self.sets:
            for m in s.values():
                m.free()
        self.sets = []


def weight_bytes(M):
    """Algorithmic HBM bytes of each projection kernel (weights 18 B/32, Q8 input
    34 B/32 per token, fp32 outputs)."""
    def mm(N, K, out_elem=4):
        return N * K * 18 // 32 + M * K * 34 // 32 + M * N * out_elem
    return {"qkv": mm(QKV_N, H) + QKV_N * 4, "o": mm(H, H),
            "gateup": 2 * I * H * 18 // 32 + M * H * 34 // 32 + M * I * 34 // 32,
            "down": mm(H, I)}


def flops(M):
    return {"qkv": 2 * M * QKV_N * H, "o": 2 * M * H * H, "gateup": 2 * M * 2 * I * H,
            "down": 2 * M * H * I}


def time_region(torch, stream, fn, steps):
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        start.record()
        for i in range(steps):
            fn(i)
        end.record()
    end.synchronize()
    return start.elapsed_time(end) / 1e3


# ---------------------------------------------------------------------------
# 8 Qwen2.5-72B layers, tensor-parallel over the ranks
# ---------------------------------------------------------------------------
CONFIG4 = dict(hidden=8192, n_q_heads=64, n_kv_heads=8, head_dim=128, intermediate=29568,
               rope_theta=1e6, rms_eps=1e-6)
TP_LAYERS, TP_PREFILL, TP_BATCH, TP_DECODE = 8, 4096, 8, 256
TP_MAX_CTX = TP_PREFILL + TP_DECODE


def q4_bytes(n, k):
    return n * k // 32 * 18


DIMS_7B = dict(hidden=3584, n_q_heads=28, n_kv_heads=4, head_dim=128, intermediate=18944,
               rope_theta=1e6, rms_eps=1e-6)


def decode_gemv_roofline(ctx, torch, stream, max_over_ranks):
    """Kernel-level decode roofline where the GEMV is HBM-bound.  The config-1
    matrices (1.3-15.5 MB) are too small for that -- launch and first-byte
    latency dominate them -- so this times the 72B down projection (8192 x
    29568, 136 MB of Q4_0 weights) at 1 token (dp4a form) and at 8 tokens
    (tensor-core form, config 4's decode batch), and the 7B down projection
    (3584 x 18944, config 2) at 1 token.  Weight copies rotate (272-305 MB,
    more than twice L2) so every launch streams from HBM; launches are CUDA
    graph replays timed with CUDA events on the library's stream."""
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
        g = ctx.capture(lambda: [ctx.matmul(m, qs, d, M, None, y) for m in mats])
        for _ in range(3):
            g.launch()
        reps = 20
        t = max_over_ranks(time_region(torch, stream, lambda i: g.launch(), reps)) / (reps * ncopy)
        wb = N * K * 18 // 32
        out[label] = {"kernel": "k_gemv (dp4a form)" if M <= 2 else "k_gemv_mma (tensor-core form)",
                      "shape": f"{N}x{K}", "tokens": M, "us": round(t * 1e6, 2),
                      "weight_bytes": wb, "achieved_gbs": round(wb / t / 1e9, 1),
                      "peak_gbs": pk["hbm_gbs"], "peak_src": pk["src"],
                      "frac": round(wb / t / 1e9 / pk["hbm_gbs"], 4)}
        g.free()
        for m in mats:
            m.free()
        del x, qs, d, y
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

    # The reference on the host (single-threaded, as it is written).
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

    # This library's drop-in run_layer: host weights (cached on the device by
    # address), host KV, host x and y per call.
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

    # Device-resident decode of the same layer.
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


def run_layers_7b(args, rank, world, ctx, torch, barrier_sync, max_over_ranks):
    """BASELINE configs 2 and 3 on each rank (replicas): one Qwen2.5-7B layer.
    Config 2: a 2048-token prefill (fp16 KV), then 128 sequential decode steps
    at batch 1.  Config 3: one decode step of 64 sequences with fp32 KV
    histories of 4096 positions.  Device time, CUDA events on the library
    stream, max over ranks; decode steps are eager launches."""
    import sib200
    stream = torch.cuda.ExternalStream(ctx.stream)
    layer = ctx.layer_synth(DIMS_7B, 2)
    H = DIMS_7B["hidden"]
    g = torch.Generator(device="cuda").manual_seed(2)
    # config 2
    ntok, ndec = 2048, 128
    kv = ctx.kv(DIMS_7B, 1, ntok + ndec, False)
    X = torch.randn(ntok, H, device="cuda", generator=g)
    Y = torch.empty_like(X)
    xd = torch.randn(ndec, H, device="cuda", generator=g)
    yd = torch.empty_like(xd)
    torch.cuda.synchronize()
    pf = lambda _=0: layer.prefill_dev(kv, 0, X, ntok, 0, Y, sib200.SI_LAYER_FULL)
    pf()
    barrier_sync()
    tpf = max_over_ranks(time_region(torch, stream, pf, 3)) / 3
    dec = lambda i: layer.decode_dev(kv, xd[i], [ntok + i + 1], yd[i], sib200.SI_LAYER_FULL)
    for i in range(3):
        dec(i)
    barrier_sync()
    tdec = max_over_ranks(time_region(torch, stream, dec, ndec)) / ndec
    kv.free()
    # config 3
    B, L = 64, 4096
    kv3 = ctx.kv(DIMS_7B, B, L, True)
    kv3.fill_synth(3, 1.0, L - 1)
    X3 = torch.randn(B, H, device="cuda", generator=g)
    Y3 = torch.empty_like(X3)
    torch.cuda.synchronize()
    d3 = lambda _=0: layer.decode_dev(kv3, X3, [L] * B, Y3, sib200.SI_LAYER_FULL)
    for _ in range(3):
        d3()
    barrier_sync()
    t3 = max_over_ranks(time_region(torch, stream, d3, 20)) / 20
    ctx.status()
    kv3.free()
    layer.free()
    kvb = B * L * DIMS_7B["n_kv_heads"] * DIMS_7B["head_dim"] * 2 * 4
    return {
        "config2": {"workload": "BASELINE config 2: one Qwen2.5-7B layer, 2048-token prefill "
                                "(fp16 KV), then 128 decode steps at batch 1",
                    "prefill_ms": round(tpf * 1e3, 3),
                    "prefill_tok_s": round(world * ntok / tpf, 1),
                    "decode_us_per_token": round(tdec * 1e6, 2)},
        "config3": {"workload": "BASELINE config 3: one Qwen2.5-7B layer, one decode step of "
                                "64 sequences with fp32 KV histories of 4096 positions",
                    "us_per_step": round(t3 * 1e6, 2),
                    "us_per_token": round(t3 * 1e6 / B, 3),
                    "tok_s": round(world * B / t3, 1),
                    "kv_bytes_per_step": kvb},
        "timing": "CUDA events on the library stream, max over ranks; eager launches",
    }


def run_tp_config4(args, rank, world, ctx, torch, barrier_sync, max_over_ranks):
    """The layer stack at TP = world: a 4096-token prefill of sequence 0, then 256
    decode steps of a batch of 8 (sequence 0 continues its prefill; the other 7
    hold seeded N(0,1) fp32 histories of 4096 positions).  Each rank holds its
    heads and its slice of the MLP; the O and down partial sums are all-reduced
    over NCCL.  Times are device times on the library stream, max over ranks;
    decode steps are launched eagerly (host context lengths every step)."""
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
    xp = [torch.randn(TP_PREFILL, Hd, device="cuda", generator=g), torch.empty(TP_PREFILL, Hd, device="cuda")]
    xd = [torch.randn(TP_BATCH, Hd, device="cuda", generator=g), torch.empty(TP_BATCH, Hd, device="cuda")]
    x0 = xd[0].clone()
    torch.cuda.synchronize()

    def prefill(_=0):
        for j, (layer, kv) in enumerate(zip(layers, kvs)):
            tp.prefill_dev(layer, kv, 0, xp[j % 2], TP_PREFILL, 0, xp[(j + 1) % 2])

    def decode(step):
        lens = [TP_PREFILL + step + 1] * TP_BATCH
        for j, (layer, kv) in enumerate(zip(layers, kvs)):
            tp.decode_dev(layer, kv, xd[j % 2], lens, xd[(j + 1) % 2])

    prefill()
    barrier_sync()
    reps = 2
    tpf = max_over_ranks(time_region(torch, stream, prefill, reps)) / reps
    def time_decode():
        for s in range(3):
            decode(s)
        xd[0].copy_(x0)
        barrier_sync()
        return max_over_ranks(time_region(torch, stream, decode, TP_DECODE)) / TP_DECODE

    tdec = time_decode()  # row-parallel sums fused into the projections (world > 1)
    tdec_nccl = None
    if world > 1:
        tp.set_options(fused=False)
        tdec_nccl = time_decode()
        tp.set_options(fused=True)
    ctx.status()
    ok = bool(torch.isfinite(xd[0]).all().item()) and bool(torch.isfinite(xp[0]).all().item())

    D, QD, KVD = CONFIG4["head_dim"], d["n_q_heads"] * CONFIG4["head_dim"], d["n_kv_heads"] * CONFIG4["head_dim"]
    Il = d["intermediate"]
    wlayer = q4_bytes(QD + 2 * KVD, Hd) + q4_bytes(Hd, QD) + q4_bytes(2 * Il, Hd) + q4_bytes(Hd, Il)
    mean_ctx = TP_PREFILL + (TP_DECODE + 1) / 2
    kv_read = TP_BATCH * mean_ctx * KVD * 2 * 4
    per_step = TP_LAYERS * (wlayer + kv_read)
    res = {
        "workload": "BASELINE config 4: 8 Qwen2.5-72B layers (hidden 8192, 64 Q / 8 KV heads, "
                    "intermediate 29568), Q4_0 weights, fp32 KV; column-sharded QKV/gate/up, "
                    "row-sharded o/down; decode adds the row-parallel partial sums through "
                    "NVLink peer stores fused into the projection, prefill through NCCL",
        "tp": world, "finite": ok,
        "prefill": {"tokens": TP_PREFILL, "ms": round(tpf * 1e3, 3),
                    "tok_s": round(TP_PREFILL / tpf, 1)},
        "decode": {"batch": TP_BATCH, "steps": TP_DECODE,
                   "context": f"{TP_PREFILL + 1}..{TP_MAX_CTX}",
                   "us_per_step": round(tdec * 1e6, 2),
                   "us_per_token": round(tdec * 1e6 / TP_BATCH, 3),
                   "tok_s": round(TP_BATCH / tdec, 1),
                   "hbm_bytes_per_step_per_rank": int(per_step),
                   "achieved_gbs_per_rank": round(per_step / tdec / 1e9, 1),
                   "reduction": "fused into the projection (epoch-tagged peer stores)" if world > 1
                                else "none (one rank)",
                   "us_per_step_nccl_allreduce": round(tdec_nccl * 1e6, 2) if tdec_nccl else None},
        "timing": "CUDA events on the library stream, max over ranks; eager launches",
    }
    for o in kvs + layers:
        o.free()
    tp.free()
    return res


def run_ours(args, rank, world, local_rank):
    import gc
    import torch
    import sib200
    torch.cuda.set_device(local_rank)
    ctx = sib200.Context(local_rank, max_positions=TP_MAX_CTX, rope_theta=1e6, head_dim=128)
    stream = torch.cuda.ExternalStream(ctx.stream)
    ps = ProjectionSet(ctx, torch, COPIES)
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

    names = ["q8_x", "qkv", "q8_o", "o", "gateup", "down"]

    def graphs_for(M, b):
        """One CUDA graph per weight copy (one step each), and per kernel one graph
        launching that kernel on every copy, so per-kernel device time is measured
        without host launch gaps."""
        ps.step(b, M, 0)  # one eager pass sizes the library's scratch before capture
        ctx.sync()
        steps = [ctx.capture(lambda c=c: ps.step(b, M, c)) for c in range(COPIES)]
        per_kernel = {n: ctx.capture(lambda n=n: [ps.kernel(b, M, c, n) for c in range(COPIES)])
                      for n in names}
        return steps, per_kernel

    def kernel_times(per_kernel, reps):
        out = {}
        for n, g in per_kernel.items():
            g.launch()
            t = time_region(torch, stream, lambda i: g.launch(), reps)
            out[n] = t / (reps * COPIES)
        return out

    # ---- prefill, M = 2048 -------------------------------------------------
    M = PREFILL_M
    b = ps.buffers(M)
    steps, per_kernel = graphs_for(M, b)
    kernels_per_step = steps[0].kernels()  # counted from the captured graph
    log(f"graphs captured ({kernels_per_step} kernels per step)")
    for i in range(args.warmup):
        steps[i % COPIES].launch()
    barrier_sync()
    with Clocks(local_rank) as clk:
        t = time_region(torch, stream, lambda i: steps[(i + args.warmup) % COPIES].launch(),
                        args.steps)
    barrier_sync()
    t = max_over_ranks(t)
    log(f"prefill timed {t:.4f}s")
    value = world * M * args.steps / t
    ms_per_step = t / args.steps * 1e3
    kt = kernel_times(per_kernel, 3)
    log(f"prefill kernels {kt}")

    # ---- decode, M = 1 -----------------------------------------------------
    bd = ps.buffers(1)
    dsteps_g, dper_kernel = graphs_for(1, bd)
    for i in range(max(args.warmup, COPIES)):
        dsteps_g[i % COPIES].launch()
    barrier_sync()
    dsteps = max(args.steps, 100)
    td = time_region(torch, stream, lambda i: dsteps_g[i % COPIES].launch(), dsteps)
    td = max_over_ranks(td)
    kd = kernel_times(dper_kernel, 20)
    log(f"decode kernels {kd}")

    # ---- the config-1 token sweep (device time per step, 10 weight copies) ----
    sweep = {1: td / dsteps, M: t / args.steps}
    for Ms in SWEEP_M:
        if Ms in sweep:
            continue
        bs = ps.buffers(Ms)
        ps.step(bs, Ms, 0)
        ctx.sync()
        g = ctx.capture(lambda: [ps.step(bs, Ms, c) for c in range(COPIES)])
        g.launch()
        ts = time_region(torch, stream, lambda i: g.launch(), 3) / (3 * COPIES)
        sweep[Ms] = max_over_ranks(ts)
        g.free()
        del bs
    log(f"sweep {sweep}")

    # ---- end to end through the C ABI with pinned host buffers ---------------
    # Each step copies its two fp32 inputs in from pinned host memory, runs the
    # projection set and copies its three fp32 outputs back.  Steps are
    # pipelined over two buffer sets: the host->device copy of step i+1 and the
    # device->host copy of step i-1 run on their own streams (their own copy
    # engines) while step i computes; events order every reuse of a buffer.
    hx = torch.randn(M, H).pin_memory()
    ho = torch.randn(M, H).pin_memory()
    outs = [(torch.empty(M, QKV_N).pin_memory(), torch.empty(M, H).pin_memory(),
             torch.empty(M, H).pin_memory()) for _ in range(2)]
    b2 = ps.buffers(M)
    ps.step(b2, M, 0)
    ctx.sync()
    steps2 = [ctx.capture(lambda c=c: ps.step(b2, M, c)) for c in range(COPIES)]
    sets = [(b, steps), (b2, steps2)]
    s_in, s_out = torch.cuda.Stream(), torch.cuda.Stream()
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_comp = [torch.cuda.Event() for _ in range(2)]
    ev_out = [torch.cuda.Event() for _ in range(2)]

    def e2e_step(i):
        k = i % 2
        bb, gs = sets[k]
        s_in.wait_event(ev_comp[k])          # step i-2 has read this set's inputs
        with torch.cuda.stream(s_in):
            bb["x"].copy_(hx, non_blocking=True)
            bb["oin"].copy_(ho, non_blocking=True)
            ev_in[k].record(s_in)
        stream.wait_event(ev_in[k])
        stream.wait_event(ev_out[k])         # step i-2's outputs have left this set
        gs[i % COPIES].launch()
        ev_comp[k].record(stream)
        s_out.wait_event(ev_comp[k])
        with torch.cuda.stream(s_out):
            oq, oo, od = outs[k]
            oq.copy_(bb["qkv"], non_blocking=True)
            oo.copy_(bb["yo"], non_blocking=True)
            od.copy_(bb["yd"], non_blocking=True)
            ev_out[k].record(s_out)

    for i in range(2):
        e2e_step(i)
    torch.cuda.synchronize()
    barrier_sync()
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e_start.record(s_in)
    for i in range(args.steps):
        e2e_step(i)
    e_end.record(s_out)
    e_end.synchronize()
    te = max_over_ranks(e_start.elapsed_time(e_end) / 1e3)
    log(f"e2e {te:.4f}s")
    for g_ in steps2:
        g_.free()
    h2d = 2 * M * H * 4
    d2h = M * (QKV_N + 2 * H) * 4

    pk = peaks()
    wb = weight_bytes(1)
    dom_d = max(wb, key=lambda n: kd[n])
    fl = flops(M)
    dom_p = max(fl, key=lambda n: kt[n])
    result = {
        "metric": METRIC, "value": round(value, 1), "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "i8",
        "data": "synthetic (seeded Q4_0 N(0,0.02) weights, N(0,1) activations)",
        "config": {"workload": "BASELINE config 1: Qwen2.5-1.5B projection set (QKV 2048x1536"
                               " +bias, o 1536^2, gate+up 2x8960x1536 +SiLU*mul+Q8, down "
                               "1536x8960), Q4_0 x Q8_0",
                   "prefill_tokens_per_step": M, "parallelism": f"replicas x{world}",
                   "l2": f"{COPIES} weight copies ({COPIES * 26.3:.0f} MB > 2x L2) rotated per step",
                   "timing": "CUDA graph replays, CUDA events on the library stream",
                   "e2e": "pinned host buffers; host->device, compute and device->host of "
                          "neighbouring steps overlap on three streams"},
        "decode": {"us_per_token": round(td / dsteps * 1e6, 3),
                   "kernel_us": {n: round(kd[n] * 1e6, 3) for n in names},
                   "roofline": {"bound": "hbm", "kernel": dom_d,
                                "achieved": round(wb[dom_d] / kd[dom_d] / 1e9, 1),
                                "peak": pk["hbm_gbs"], "unit": "GB/s",
                                "frac": round(wb[dom_d] / kd[dom_d] / 1e9 / pk["hbm_gbs"], 4),
                                "peak_src": pk["src"],
                                "all": {n: round(wb[n] / kd[n] / 1e9, 1) for n in wb}}},
        "prefill_kernel_ms": {n: round(kt[n] * 1e3, 4) for n in names},
        "roofline": {"bound": "tensor", "kernel": dom_p,
                     "achieved": round(fl[dom_p] / kt[dom_p] / 1e12, 2),
                     "peak": INT8_SPEC_TOPS, "unit": "TOP/s",
                     "frac": round(fl[dom_p] / kt[dom_p] / 1e12 / INT8_SPEC_TOPS, 4),
                     "peak_src": "spec (dense int8; MEASURED_PEAKS.json has no int8 figure)",
                     "all": {n: round(fl[n] / kt[n] / 1e12, 2) for n in fl},
                     "traffic": NCU_TRAFFIC.get(dom_p)},
        "e2e": {"value": round(world * M * args.steps / te, 1), "unit": "tok/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "gpu_launches": kernels_per_step * args.steps,
        "sweep": {str(m): {"ms_per_step": round(sweep[m] * 1e3, 4),
                           "tok_s": round(world * m / sweep[m], 1)} for m in SWEEP_M},
        "clocks": clk.summary(),
    }
    log("configs 2 and 3")
    result.update(run_layers_7b(args, rank, world, ctx, torch, barrier_sync, max_over_ranks))
    log(f"configs 2/3 {result['config2']} {result['config3']}")
    try:
        result["decode_gemv_roofline"] = decode_gemv_roofline(ctx, torch, stream, max_over_ranks)
        log(f"decode GEMV roofline {result['decode_gemv_roofline']}")
    except Exception as exc:  # a failed extra measurement must not lose the bench line
        result["decode_gemv_roofline"] = {"error": str(exc)[:200]}
        log(f"decode GEMV roofline failed: {exc}")
    if rank == 0:
        try:
            result["reference_layer"] = reference_layer_decode(ctx, torch, stream)
            log(f"reference layer {result['reference_layer']}")
        except Exception as exc:  # a failed extra measurement must not lose the bench line
            result["reference_layer"] = {"error": str(exc)[:200]}
            log(f"reference layer failed: {exc}")
    if not args.no_tp:
        log("tp config 4")
        result["tp_config4"] = run_tp_config4(args, rank, world, ctx, torch, barrier_sync,
                                              max_over_ranks)
        log(f"tp {result['tp_config4']}")
    if rank == 0 and not args.no_cpu_baseline:
        log("cpu baseline")
        result["cpu_baseline"] = cpu_baseline(args.cpu_seconds)
    # torch's allocators keep events recorded on the library's stream (pinned
    # copies ran on it), so the stream is left to process exit rather than
    # destroyed under them; graphs and weights are released explicitly.
    torch.cuda.synchronize()
    ctx.sync()
    del steps, per_kernel, dsteps_g, dper_kernel
    gc.collect()
    ps.free()
    ctx.h = None
    return result


# ---------------------------------------------------------------------------
# CPU: the reference's own functions on the host cores
# ---------------------------------------------------------------------------
def cpu_impl():
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    if os.path.exists(oracle.LIB_REF):
        r = oracle.Reference()
        return "reference", r.lib.ref_matvec_q4q8, r.lib.ref_quantize_q8
    o = oracle.Oracle()
    return "port", o.lib.oc_matvec_q4q8, o.lib.oc_quantize_q8


def cpu_projection_tokens(seconds: float, threads: int):
    """Tokens/s of the projection set on the host: each token runs quantize_q8 +
    matvec_q4q8 for QKV/o/gate/up/down (+SiLU*mul), rows split over threads."""
    import ctypes as C
    from concurrent.futures import ThreadPoolExecutor
    from sib200 import synth
    kind, matvec, quant = cpu_impl()
    rng = np.random.default_rng(1)
    W = {"qkv": synth.random_q4(rng, QKV_N, H), "o": synth.random_q4(rng, H, H),
         "gate": synth.random_q4(rng, I, H), "up": synth.random_q4(rng, I, H),
         "down": synth.random_q4(rng, H, I)}
    bias = rng.normal(0, 0.02, QKV_N).astype(np.float32)
    pool = ThreadPoolExecutor(threads)

    def mv(w, q8, K, N, b, out):
        rows = -(-N // threads)

        def part(t):  # row slices: the same arithmetic per row, so results are unchanged
            r0, r1 = t * rows, min(N, (t + 1) * rows)
            if r0 < r1:
                matvec(w[r0:r1], q8, K, r1 - r0,
                       None if b is None else b[r0:r1].ctypes.data_as(C.c_void_p), out[r0:r1])
        list(pool.map(part, range(threads)))

    def token(x, o_in):
        q8 = np.zeros(H // 32 * 34, np.uint8)
        quant(x, q8, H)
        qkv = np.zeros(QKV_N, np.float32)
        mv(W["qkv"], q8, H, QKV_N, bias, qkv)
        oq = np.zeros(H // 32 * 34, np.uint8)
        quant(o_in, oq, H)
        yo = np.zeros(H, np.float32)
        mv(W["o"], oq, H, H, None, yo)
        g = np.zeros(I, np.float32)
        u = np.zeros(I, np.float32)
        mv(W["gate"], q8, H, I, None, g)
        mv(W["up"], q8, H, I, None, u)
        a = ((g / (np.float32(1) + np.exp(-g))) * u).astype(np.float32)
        aq = np.zeros(I // 32 * 34, np.uint8)
        quant(a, aq, I)
        yd = np.zeros(H, np.float32)
        mv(W["down"], aq, I, H, None, yd)

    x = rng.standard_normal((64, H)).astype(np.float32)
    token(x[0], x[1])  # warm
    n, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < seconds:
        token(x[n % 64], x[(n + 1) % 64])
        n += 1
    dt = time.perf_counter() - t0
    pool.shutdown()
    return kind, n, dt


def cpu_baseline(seconds):
    threads = len(os.sched_getaffinity(0))
    kind, n, dt = cpu_projection_tokens(seconds, threads)
    return {"value": round(n / dt, 3), "unit": "tok/s", "cores": threads, "kind": kind,
            "sample": f"{n} tokens of the config-1 projection set (quantize_q8 + matvec_q4q8 "
                      f"x5 + SiLU*mul), rows split over {threads} threads, {dt:.1f} s"}


def run_reference(args, rank):
    if rank != 0:
        return None
    per_step = []
    threads = len(os.sched_getaffinity(0))
    kind = None
    for i in range(args.warmup + args.steps):
        kind, n, dt = cpu_projection_tokens(args.cpu_seconds / max(1, args.steps), threads)
        if i >= args.warmup:
            per_step.append((n, dt))
    toks = sum(n for n, _ in per_step)
    secs = sum(dt for _, dt in per_step)
    v = toks / secs
    return {"impl": "reference", "metric": METRIC, "value": round(v, 3), "unit": "tok/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(secs / args.steps * 1e3, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "i8", "data": "synthetic",
            "config": {"workload": "BASELINE config 1 projection set, per-token (the reference "
                                   "has no batched prefill on CPU)", "parallelism": "host cores"},
            "cpu_baseline": {"value": round(v, 3), "unit": "tok/s", "cores": threads,
                             "kind": kind, "sample": f"{toks} tokens over {args.steps} steps"},
            "e2e": {"value": round(v, 3), "unit": "tok/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}


def probe_config4_layer():
    """One Qwen2.5-72B layer on GPU 0 (TP = 1): three decode steps of a batch
    of 8 at context 4097.. and one 4096-token prefill, no timing -- the
    workload the config-4 ncu summaries capture."""
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


def probe_config2_decode():
    """One Qwen2.5-7B layer on GPU 0: three decode steps at batch 1 after a
    2048-position fp16 history, no timing -- the workload of the config-2
    decode ncu summaries."""
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


def log(msg):
    if os.environ.get("SI_BENCH_VERBOSE"):
        print(f"[bench] {msg}", file=sys.stderr, flush=True)


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
    ap.add_argument("--no-tp", action="store_true", help="skip the config-4 tensor-parallel stack")
    ap.add_argument("--probe", choices=["config4-layer", "config2-decode"],
                    help="run one untimed workload for a profiler and exit")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.probe == "config4-layer":
        probe_config4_layer()
        return
    if args.probe == "config2-decode":
        probe_config2_decode()
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
