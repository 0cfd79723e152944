"""Decode steps with device-resident context lengths (si_decode_state), the
form a multi-layer step is captured in once and replayed as a CUDA graph: the
graph replays must equal the eager steps with host lengths bit for bit --
outputs and KV cache -- over several steps of a two-layer stack, for a batch
with different context lengths and for fp16 and fp32 caches; lengths advance
on the device and an advance past the cache records SI_ERR_INVALID."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

DIMS = dict(hidden=3584, n_q_heads=28, n_kv_heads=4, head_dim=128, intermediate=18944,
            rope_theta=1e6, rms_eps=1e-6)


@pytest.mark.parametrize("kv_f32", [False, True])
def test_graph_replayed_decode_equals_eager(si_ctx, kv_f32):
    import sib200
    B, L, STEPS = 3, 400, 5
    lens0 = [100, 257, 130]
    layers = [si_ctx.layer_synth(DIMS, 40 + i) for i in range(2)]
    H = DIMS["hidden"]
    g = torch.Generator("cuda").manual_seed(9)
    x0 = torch.randn(B, H, device="cuda", generator=g)

    def caches():
        kvs = [si_ctx.kv(DIMS, B, L, kv_f32) for _ in layers]
        for i, kv in enumerate(kvs):
            kv.fill_synth(70 + i, 1.0, L)
        return kvs

    # eager, host lengths
    kva = caches()
    xa = [x0.clone(), torch.empty_like(x0)]
    outs_a = []
    torch.cuda.synchronize()
    for s in range(STEPS):
        lens = [c + s for c in lens0]
        for j, (layer, kv) in enumerate(zip(layers, kva)):
            layer.decode_dev(kv, xa[j % 2], lens, xa[(j + 1) % 2], sib200.SI_LAYER_FULL)
        si_ctx.sync()  # the copy below runs on torch's stream
        outs_a.append(xa[0].clone())
    si_ctx.status()

    # one step captured with device lengths, replayed
    kvb = caches()
    xb = [x0.clone(), torch.empty_like(x0)]
    st = si_ctx.decode_state(lens0, L)
    torch.cuda.synchronize()

    def step():
        for j, (layer, kv) in enumerate(zip(layers, kvb)):
            layer.decode_state_dev(kv, xb[j % 2], st, xb[(j + 1) % 2], sib200.SI_LAYER_FULL)
        st.advance()

    # an eager first step sizes the context's buffers before capture
    step()
    si_ctx.sync()
    graph = si_ctx.capture(step)
    outs_b = [xb[0].clone()]
    for s in range(1, STEPS):
        graph.launch()
        si_ctx.sync()
        outs_b.append(xb[0].clone())
    si_ctx.sync()
    si_ctx.status()
    assert st.lens() == [c + STEPS for c in lens0]
    for s in range(STEPS):
        assert torch.equal(outs_a[s], outs_b[s]), f"step {s}"
    kvd = DIMS["n_kv_heads"] * DIMS["head_dim"]
    dt = np.float32 if kv_f32 else np.uint16
    for kv1, kv2 in zip(kva, kvb):
        for b in range(B):
            n = lens0[b] + STEPS - 1
            k1, v1 = np.zeros((n, kvd), dt), np.zeros((n, kvd), dt)
            k2, v2 = np.zeros_like(k1), np.zeros_like(v1)
            kv1.read(b, 0, n, k1, v1)
            kv2.read(b, 0, n, k2, v2)
            np.testing.assert_array_equal(k1, k2)
            np.testing.assert_array_equal(v1, v2)
    graph.free()
    st.free()
    for o in kva + kvb + layers:
        o.free()


def test_decode_state_advance_stops_at_the_cache(si_ctx):
    import sib200
    st = si_ctx.decode_state([7, 9], 10)
    st.advance()
    si_ctx.status()
    assert st.lens() == [8, 10]
    st.advance()  # 10 + 1 would pass the cache: that length stays, error recorded
    with pytest.raises(sib200.SiError) as e:
        si_ctx.status()
    assert e.value.status == sib200.SI_ERR_INVALID
    assert st.lens() == [9, 10]
    st.set([1, 1])
    assert st.lens() == [1, 1]
    si_ctx.status()
    st.free()
