"""The arithmetic identities behind the projection kernels' exact rescale,
checked on the CPU in IEEE single precision.

Reference arithmetic (qwen_one_layer.c:148-162): per block,
term = ((float)isum * dw) * dx with two roundings, isum the int32 sum of 32
products of (q - 8) in [-8, 7] with int8 activations in [-127, 127], dw and dx
fp16 values (dx = amax/127 >= 0), and the terms added to the output one block
at a time.  The GPU kernels never form (float)isum directly:

* the dp4a and mma forms see 16*isum (the nibbles sit in the high half of each
  byte) and use ((float)(16*isum) * dw) * (dx/16);
* the tensor-core kernels take the integer 0x4B400000 as the mma accumulator
  input, so the result's bits are the float f = 1.5*2^23 + 16*isum, and form
  fma(f, dw, -1.5*2^23*dw) -- one rounding of 16*isum*dw -- instead of an
  int-to-float conversion followed by a multiply.

numpy float32 arithmetic rounds every operation to nearest-even, like the
kernels' explicit .rn operations; a fused multiply-add is modelled as the
float64 value rounded once to float32, which is exact here because every
product and sum involved fits in 53 bits.
"""
import numpy as np

MAGIC = 12582912.0  # 1.5 * 2**23, the float whose bits are 0x4B400000
N = 1_000_000


def _f16(rng, n, nonneg=False):
    """Random finite fp16 values (normals and subnormals) as float32."""
    bits = rng.integers(0, 0x7C00, n, dtype=np.uint16)  # exponent < 31: finite
    if not nonneg:
        bits |= (rng.integers(0, 2, n).astype(np.uint16) << 15)
    return bits.view(np.float16).astype(np.float32)


def _isum(rng, n):
    # The full range of a block sum, with the extremes and zero forced in.
    s = rng.integers(-32 * 8 * 127, 32 * 8 * 127 + 1, n).astype(np.int32)
    s[:6] = [0, 1, -1, 32 * 8 * 127, -32 * 8 * 127, -32 * 7 * 127]
    return s


def _bits(x):
    return np.ascontiguousarray(x, np.float32).view(np.uint32)


def test_power_of_two_scaling_keeps_both_roundings():
    """((float)(16*isum) * dw) * (dx/16) == ((float)isum * dw) * dx, bit for bit."""
    rng = np.random.default_rng(1)
    isum, dw, dx = _isum(rng, N), _f16(rng, N), _f16(rng, N, nonneg=True)
    want = (isum.astype(np.float32) * dw) * dx
    got = ((16 * isum).astype(np.float32) * dw) * (dx * np.float32(0.0625))
    np.testing.assert_array_equal(_bits(got), _bits(want))


def test_magic_constant_fma_is_the_rounded_product():
    """fma(f, dw, -1.5*2^23*dw) with f = bits(0x4B400000 + d) equals (float)d * dw."""
    rng = np.random.default_rng(2)
    d = 16 * _isum(rng, N).astype(np.int64)
    dw = _f16(rng, N)
    # The integer add the mma accumulator performs, read back as a float.
    f = (np.int64(0x4B400000) + d).astype(np.uint32).view(np.float32)
    assert np.all(f.astype(np.float64) == MAGIC + d)  # exact: |d| < 2^22
    nk = dw * np.float32(-MAGIC)
    assert np.all(nk.astype(np.float64) == -MAGIC * dw.astype(np.float64))  # exact
    got = (f.astype(np.float64) * dw.astype(np.float64) + nk.astype(np.float64)).astype(np.float32)
    want = d.astype(np.float32) * dw
    # Equal as values everywhere; as bits wherever the product is not zero.
    # (A zero product -- isum = 0 or a zero scale -- comes out +0.0 where the
    # reference may have -0.0; that can change an output only if it is
    # exactly zero and its bias is -0.0.)
    np.testing.assert_array_equal(got, want)
    nz = (d != 0) & (dw != 0)
    np.testing.assert_array_equal(_bits(got[nz]), _bits(want[nz]))


def test_magic_constant_with_prescaled_scale():
    """The GEMM's variant: fma(f, dw/16, -1.5*2^23*dw/16) * dx == ((float)isum*dw)*dx."""
    rng = np.random.default_rng(3)
    isum = _isum(rng, N).astype(np.int64)
    dw, dx = _f16(rng, N), _f16(rng, N, nonneg=True)
    f = (np.int64(0x4B400000) + 16 * isum).astype(np.uint32).view(np.float32)
    dw16 = dw * np.float32(0.0625)
    nk = np.float32(-MAGIC) * dw16
    p = (f.astype(np.float64) * dw16.astype(np.float64) + nk.astype(np.float64)).astype(np.float32)
    got = p * dx
    want = (isum.astype(np.float32) * dw) * dx
    np.testing.assert_array_equal(got, want)
    nz = (isum != 0) & (dw != 0)
    np.testing.assert_array_equal(_bits(got[nz]), _bits(want[nz]))
