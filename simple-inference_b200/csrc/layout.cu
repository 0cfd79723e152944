// layout.cu -- weight and activation layout conversions on the device.
//
// The reference repacks GGUF Q4_0 rows offline into 256-output column-SoA tiles
// with fp32 scales (repack_weights.py:55-75, fused_layer.h:11-21).  Here the
// repack runs on the GPU into a row-tile SoA layout shaped for 128-bit
// coalesced loads and TMA boxes:
//   nib[rows/32][KB][32 rows][16 bytes]  GGUF nibble order, each byte ^ 0x88
//   scl[rows/32][KB][32 rows]            the unchanged fp16 block scale
// so a warp reading block b of a 32-row tile reads 512 contiguous bytes, one
// 16-byte vector per lane (lane = row).  Scales stay fp16 (4.5 bits/weight).
#include "si_common.cuh"
#include "si_kernels.cuh"

namespace si {

__global__ void k_repack_gguf(const uint8_t *__restrict__ src, int rows, int KB,
                              uint8_t *__restrict__ nib, uint16_t *__restrict__ scl) {
  size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (size_t)rows * KB) return;
  int row = (int)(i / KB), b = (int)(i % KB);
  const uint16_t *p = reinterpret_cast<const uint16_t *>(src + i * 18);  // 18-byte blocks: 2-aligned
  uint32_t w[4];
#pragma unroll
  for (int j = 0; j < 4; ++j)
    w[j] = ((uint32_t)p[1 + 2 * j] | ((uint32_t)p[2 + 2 * j] << 16)) ^ 0x88888888u;
  size_t slot = ((size_t)(row / SI_RT) * KB + b) * SI_RT + (row % SI_RT);
  reinterpret_cast<uint4 *>(nib)[slot] = make_uint4(w[0], w[1], w[2], w[3]);
  scl[slot] = p[0];
}

__global__ void k_unpack_to_gguf(const uint8_t *__restrict__ nib, const uint16_t *__restrict__ scl,
                                 int rows, int KB, uint8_t *__restrict__ dst) {
  size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (size_t)rows * KB) return;
  int row = (int)(i / KB), b = (int)(i % KB);
  size_t slot = ((size_t)(row / SI_RT) * KB + b) * SI_RT + (row % SI_RT);
  uint4 v = reinterpret_cast<const uint4 *>(nib)[slot];
  uint16_t *p = reinterpret_cast<uint16_t *>(dst + i * 18);
  p[0] = scl[slot];
  uint32_t w[4] = {v.x ^ 0x88888888u, v.y ^ 0x88888888u, v.z ^ 0x88888888u, v.w ^ 0x88888888u};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    p[1 + 2 * j] = (uint16_t)w[j];
    p[2 + 2 * j] = (uint16_t)(w[j] >> 16);
  }
}

// Counter-based generator: splitmix64 finaliser of (seed, index).
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
// Standard normal by Box-Muller from one 64-bit draw.
__device__ __forceinline__ float normal_from(uint64_t h) {
  float u1 = ((float)(uint32_t)(h >> 40) + 0.5f) * (1.0f / 16777216.0f);
  float u2 = (float)(uint32_t)(h & 0xFFFFFFu) * (1.0f / 16777216.0f);
  return sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);
}

// Seeded synthetic Q4_0 weights written straight into the SoA layout.  Values
// ~N(0, std) are quantised with the GGUF Q4_0 rule: d = (signed value of
// max|x|) / -8 stored fp16, q = min(15, (int)(x/d + 8.5)).
// Rows [row0, row0+rows) x blocks [cb0, cb0+KB) of a seeded matrix with
// full_KB blocks per row: every block's values depend only on (seed, its index
// in the full matrix), so a shard generated alone equals the same slice of the
// whole matrix.
__global__ void k_synth_q4(int rows, int KB, uint64_t seed, float stdv, uint8_t *__restrict__ nib,
                           uint16_t *__restrict__ scl, int row0, int cb0, int full_KB) {
  size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (size_t)rows * KB) return;
  int row = (int)(i / KB), b = (int)(i % KB);
  const size_t gi = (size_t)(row0 + row) * full_KB + cb0 + b;
  float x[32];
  float amax = 0.0f, smax = 0.0f;
  uint64_t base = mix64(seed) ^ ((uint64_t)gi << 5);
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    x[j] = normal_from(mix64(base + j)) * stdv;
    float a = fabsf(x[j]);
    if (a > amax) { amax = a; smax = x[j]; }
  }
  float d = __fdiv_rn(smax, -8.0f);
  float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
  uint32_t w[4] = {0, 0, 0, 0};
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    int lo = (int)__fadd_rn(__fmul_rn(x[j], id), 8.5f);
    int hi = (int)__fadd_rn(__fmul_rn(x[j + 16], id), 8.5f);
    lo = lo > 15 ? 15 : lo;
    hi = hi > 15 ? 15 : hi;
    uint32_t byte = (uint32_t)(lo | (hi << 4)) ^ 0x88u;
    w[j >> 2] |= byte << (8 * (j & 3));
  }
  size_t slot = ((size_t)(row / SI_RT) * KB + b) * SI_RT + (row % SI_RT);
  reinterpret_cast<uint4 *>(nib)[slot] = make_uint4(w[0], w[1], w[2], w[3]);
  scl[slot] = f32_to_f16(d);
}

// Elements [i0, i0+n) of a seeded vector.
__global__ void k_synth_f32(float *dst, size_t n, uint64_t seed, float mean, float stdv,
                            size_t i0) {
  size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) dst[i] = mean + stdv * normal_from(mix64(mix64(seed) + i0 + i));
}

__global__ void k_synth_kv(void *dst, size_t n, int f32, uint64_t seed, float stdv) {
  size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float v = stdv * normal_from(mix64(mix64(seed) + i));
  if (f32) static_cast<float *>(dst)[i] = v;
  else static_cast<uint16_t *>(dst)[i] = f32_to_f16(v);
}

__global__ void k_q8_to_blocks(const int8_t *__restrict__ qs, const uint16_t *__restrict__ d,
                               size_t nblocks, uint8_t *__restrict__ blocks) {
  size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= nblocks) return;
  uint8_t *o = blocks + i * 34;
  uint16_t dv = d[i];
  o[0] = (uint8_t)dv;
  o[1] = (uint8_t)(dv >> 8);
  const int8_t *q = qs + i * 32;
#pragma unroll
  for (int j = 0; j < 32; ++j) o[2 + j] = (uint8_t)q[j];
}

__global__ void k_q8_from_blocks(const uint8_t *__restrict__ blocks, size_t nblocks,
                                 int8_t *__restrict__ qs, uint16_t *__restrict__ d) {
  size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= nblocks) return;
  const uint8_t *b = blocks + i * 34;
  d[i] = (uint16_t)(b[0] | (b[1] << 8));
#pragma unroll
  for (int j = 0; j < 32; ++j) qs[i * 32 + j] = (int8_t)b[2 + j];
}

static inline unsigned nblk(size_t n, int t) { return (unsigned)((n + t - 1) / t); }

cudaError_t launch_repack_gguf(const uint8_t *gguf, int rows, int KB, uint8_t *nib,
                               uint16_t *scl, cudaStream_t s) {
  size_t n = (size_t)rows * KB;
  count_launch();
  k_repack_gguf<<<nblk(n, 256), 256, 0, s>>>(gguf, rows, KB, nib, scl);
  return cudaGetLastError();
}
cudaError_t launch_unpack_to_gguf(const uint8_t *nib, const uint16_t *scl, int rows, int KB,
                                  uint8_t *gguf, cudaStream_t s) {
  size_t n = (size_t)rows * KB;
  count_launch();
  k_unpack_to_gguf<<<nblk(n, 256), 256, 0, s>>>(nib, scl, rows, KB, gguf);
  return cudaGetLastError();
}
cudaError_t launch_synth_q4(int rows, int KB, uint64_t seed, float stdv, uint8_t *nib,
                            uint16_t *scl, cudaStream_t s, int row0, int cb0, int full_KB) {
  size_t n = (size_t)rows * KB;
  count_launch();
  k_synth_q4<<<nblk(n, 128), 128, 0, s>>>(rows, KB, seed, stdv, nib, scl, row0, cb0,
                                          full_KB > 0 ? full_KB : KB);
  return cudaGetLastError();
}
cudaError_t launch_synth_f32(float *dst, size_t n, uint64_t seed, float mean, float stdv,
                             cudaStream_t s, size_t i0) {
  if (n == 0) return cudaSuccess;
  count_launch();
  k_synth_f32<<<nblk(n, 256), 256, 0, s>>>(dst, n, seed, mean, stdv, i0);
  return cudaGetLastError();
}
cudaError_t launch_synth_kv(void *dst, size_t n, int f32, uint64_t seed, float stdv,
                            cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  count_launch();
  k_synth_kv<<<nblk(n, 256), 256, 0, s>>>(dst, n, f32, seed, stdv);
  return cudaGetLastError();
}
cudaError_t launch_q8_to_blocks(const int8_t *qs, const uint16_t *d, int M, int K,
                                uint8_t *blocks, cudaStream_t s) {
  size_t n = (size_t)M * (K / 32);
  if (n == 0) return cudaSuccess;
  count_launch();
  k_q8_to_blocks<<<nblk(n, 128), 128, 0, s>>>(qs, d, n, blocks);
  return cudaGetLastError();
}
cudaError_t launch_q8_from_blocks(const uint8_t *blocks, int M, int K, int8_t *qs, uint16_t *d,
                                  cudaStream_t s) {
  size_t n = (size_t)M * (K / 32);
  if (n == 0) return cudaSuccess;
  count_launch();
  k_q8_from_blocks<<<nblk(n, 128), 128, 0, s>>>(blocks, n, qs, d);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Column-SoA tiles (the reference's repack_weights.py output, read by
// fused_column_matvec, fused_layer.h:169-245).  A tile is one 32-input group
// per Q4_0 block: 32 columns of 128 bytes (byte j of column k holds output j in
// its low nibble and output j+128 in its high nibble, input k of the block),
// then 256 fp32 scales -- 5120 bytes per group.
// ---------------------------------------------------------------------------
constexpr int kGroupBytes = 5120;

__device__ __forceinline__ uint32_t colsoa_nib(const uint8_t *g, int k, int j, int half) {
  return (g[k * 128 + j] >> (4 * half)) & 15u;
}

// Destination row r (of the rows this launch fills) and block b -> the group
// that holds them, the byte column j and the nibble half.
//   kind 0 (Q):   tile p covers rows [256p, 256p+256) over all KB blocks.
//   kind 1 (K|V): tile g holds K rows [128g, 128g+128) low and V rows high;
//                 the destination has all K rows, then all V rows (kv_rows each).
//   kind 2 (O):   pair p, output subtile yt (8 groups each, p-major) covers
//                 rows [256yt, 256yt+256) for input blocks [8p, 8p+8).
__global__ void k_colsoa_to_rt(const uint8_t *__restrict__ tiles, int kind, int nrows, int row0,
                               int KB, int hidden, size_t tile_bytes, int kv_rows,
                               uint8_t *__restrict__ nib, uint16_t *__restrict__ scl) {
  const size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (size_t)nrows * KB) return;
  const int r = (int)(idx / KB), b = (int)(idx % KB);
  int j, half;
  size_t off;
  if (kind == 0) {
    half = (r % 256) / 128;
    j = r % 128;
    off = (size_t)(r / 256) * tile_bytes + (size_t)b * kGroupBytes;
  } else if (kind == 1) {
    half = r >= kv_rows;
    const int rr = half ? r - kv_rows : r;
    j = rr % 128;
    off = (size_t)(rr / 128) * tile_bytes + (size_t)b * kGroupBytes;
  } else {
    half = (r % 256) / 128;
    j = r % 128;
    off = ((size_t)(b / 8) * (hidden / 256) + r / 256) * 8 * kGroupBytes +
          (size_t)(b % 8) * kGroupBytes;
  }
  const uint8_t *g = tiles + off;
  const int n = row0 + r;
  uint8_t *dst = nib + (((size_t)(n / SI_RT) * KB + b) * SI_RT + n % SI_RT) * 16;
#pragma unroll
  for (int i = 0; i < 16; ++i)
    dst[i] = (uint8_t)((colsoa_nib(g, i, j, half) | colsoa_nib(g, i + 16, j, half) << 4) ^ 0x88u);
  const float sc = *reinterpret_cast<const float *>(g + 4096 + 4 * (j + 128 * half));
  scl[((size_t)(n / SI_RT) * KB + b) * SI_RT + n % SI_RT] = f32_to_f16(sc);
}

// fused_column_matvec (fused_layer.h:169-245) on one tile: thread j owns output
// j (low nibbles for j < 128, high for j >= 128); blocks in order with the
// reference's roundings, ((float)isum * scale) * dx.
__global__ void __launch_bounds__(256) k_colsoa_matvec(const uint8_t *__restrict__ tile,
                                                      const uint8_t *__restrict__ xb, int nblocks,
                                                      const float *__restrict__ bias_lo,
                                                      const float *__restrict__ bias_hi,
                                                      float *__restrict__ out, int add) {
  const int jo = threadIdx.x, half = jo / 128, j = jo % 128;
  float acc;
  if (add) acc = out[jo];
  else if (half) acc = bias_hi ? bias_hi[j] : 0.0f;
  else acc = bias_lo ? bias_lo[j] : 0.0f;
  for (int b = 0; b < nblocks; ++b) {
    const uint8_t *g = tile + (size_t)b * kGroupBytes;
    const uint8_t *x = xb + (size_t)b * 34;
    int isum = 0;
#pragma unroll
    for (int k = 0; k < 32; ++k) isum += ((int)colsoa_nib(g, k, j, half) - 8) * (int8_t)x[2 + k];
    const float sc = *reinterpret_cast<const float *>(g + 4096 + 4 * jo);
    const float dx = f16_to_f32((uint16_t)(x[0] | x[1] << 8));
    acc = __fadd_rn(acc, __fmul_rn(__fmul_rn((float)isum, sc), dx));
  }
  out[jo] = acc;
}

cudaError_t launch_colsoa_to_rt(const uint8_t *tiles, int kind, int nrows, int row0, int KB,
                                int hidden, size_t tile_bytes, int kv_rows, uint8_t *nib,
                                uint16_t *scl, cudaStream_t s) {
  size_t n = (size_t)nrows * KB;
  if (n == 0) return cudaSuccess;
  count_launch();
  k_colsoa_to_rt<<<nblk(n, 256), 256, 0, s>>>(tiles, kind, nrows, row0, KB, hidden, tile_bytes,
                                             kv_rows, nib, scl);
  return cudaGetLastError();
}

cudaError_t launch_colsoa_matvec(const uint8_t *tile, const uint8_t *x_blocks, int nblocks,
                                 const float *bias_lo, const float *bias_hi, float *out, int add,
                                 cudaStream_t s) {
  count_launch();
  k_colsoa_matvec<<<1, 256, 0, s>>>(tile, x_blocks, nblocks, bias_lo, bias_hi, out, add);
  return cudaGetLastError();
}

}  // namespace si
