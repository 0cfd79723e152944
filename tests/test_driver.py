"""The C driver si_qwen_one_layer (the reference's qwen_one_layer.c main on
libsi_b200): command line and errors on CPU, results on the GPU.

The GPU cases write a synthetic 1.5B layer in the reference's file formats
(q/k/v/o.q4_0, norm and bias .f32, q/kv/o.colsoa), run the driver, and check
its printed output checksum against the oracle's run_layer on the same inputs:
the driver draws them from the reference's xorshift32 stream
(qwen_one_layer.c:88-96, 228-235), regenerated here with the oracle's copy.
"""
import os
import re
import subprocess

import numpy as np
import pytest

from common import DIMS_15B, ROOT, xs_layer

DRIVER = os.path.join(ROOT, "simple-inference_b200", "lib", "si_qwen_one_layer")

needs_driver = pytest.mark.skipif(not os.path.exists(DRIVER), reason="driver not built")


def run(*args, timeout=300):
    return subprocess.run([DRIVER, *map(str, args)], capture_output=True, text=True,
                          timeout=timeout)


@needs_driver
def test_usage_and_argument_errors():
    r = run()
    assert r.returncode == 2 and "Usage:" in r.stderr
    r = run("/nonexistent", "abc")
    assert r.returncode == 1 and "error: Invalid context argument" in r.stderr
    r = run("/nonexistent", "0")
    assert r.returncode == 1 and "Context must be 1..32768" in r.stderr
    r = run("/nonexistent", "16", "1", "bogus")
    assert r.returncode == 1 and "Attention mode must be" in r.stderr


def write_layer(oc, d):
    layer = xs_layer(oc, DIMS_15B, 0x4242)
    for key, name in (("wq", "q.q4_0"), ("wk", "k.q4_0"), ("wv", "v.q4_0"), ("wo", "o.q4_0"),
                      ("norm", "norm.f32"), ("bq", "q_bias.f32"), ("bk", "k_bias.f32"),
                      ("bv", "v_bias.f32")):
        layer[key].tofile(os.path.join(d, name))
    q = np.concatenate([oc.pack_colsoa_tile(layer["wq"], layer["wq"], 1536, p * 256,
                                            p * 256 + 128, 0, 48) for p in range(6)])
    kv = np.concatenate([oc.pack_colsoa_tile(layer["wk"], layer["wv"], 1536, g * 128, g * 128,
                                             0, 48) for g in range(2)])
    o = np.concatenate([oc.pack_colsoa_tile(layer["wo"], layer["wo"], 1536, t * 256,
                                            t * 256 + 128, p * 256, 8)
                        for p in range(6) for t in range(6)])
    q.tofile(os.path.join(d, "q.colsoa"))
    kv.tofile(os.path.join(d, "kv.colsoa"))
    o.tofile(os.path.join(d, "o.colsoa"))
    return layer


def driver_inputs(oc, context):
    """x, then the fp16 history k/v interleaved per element, from one stream."""
    oc.seed(0x5217AC8B)
    x = oc.random_floats(1536)
    n = (context - 1) * 256
    r = oc.random_floats(2 * n)
    kc = np.zeros(context * 256, np.uint16)
    vc = np.zeros(context * 256, np.uint16)
    kc[:n] = (r[0::2] * np.float32(0.25)).astype(np.float16).view(np.uint16)
    vc[:n] = (r[1::2] * np.float32(0.25)).astype(np.float16).view(np.uint16)
    return x, kc, vc


@needs_driver
@pytest.mark.gpu
@pytest.mark.parametrize("mode,context", [("flash", 17), ("standard", 64), ("compare", 33),
                                          ("fused", 40), ("soa-staged", 5),
                                          ("fused-compare", 9)])
def test_driver_checksum_vs_oracle(oc, tmp_path, mode, context):
    layer = write_layer(oc, str(tmp_path))
    r = run(str(tmp_path), context, 2, mode)
    assert r.returncode == 0, r.stderr
    m = re.search(r"Output checksum:? ([-+0-9.eE]+)", r.stdout)
    assert m, r.stdout
    got = float(m.group(1))
    x, kc, vc = driver_inputs(oc, context)
    y = oc.run_layer(DIMS_15B, layer, x, kc, vc, context, 0 if mode == "standard" else 1)
    want = float(np.sum(y.astype(np.float64)))
    assert abs(got - want) <= 1e-3 * float(np.sum(np.abs(y))) + 1e-6, (got, want)
    if "compare" in mode:
        m = re.search(r"Q8 blocks differing (\d+)/48", r.stdout)
        assert m and int(m.group(1)) <= 2, r.stdout
