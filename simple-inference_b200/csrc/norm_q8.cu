// norm_q8.cu -- Q8_0 activation quantiser and RMSNorm (+ fused Q8).
//
// Q8_0 (qwen_one_layer.c:98-116): one warp per 32-element block, lane = element.
// RMSNorm (qwen_one_layer.c:164-169): sum of squares in fp64, then
// inv = 1 / sqrtf((float)(ss / n) + eps) and out = (x * inv) * w, each product
// rounded separately.  The fp64 tree sum differs from the reference's serial
// fp64 sum only in the last bits of a double, far below the float rounding.
#include "si_common.cuh"
#include "si_kernels.cuh"
#include "si_peer.cuh"
#include "si_tma.cuh"

namespace si {

// Row counts up to this take the cluster form of the RMSNorm.
constexpr int kRmsClusterMaxRows = 64;

// Eight lanes per Q8 block, four elements per lane (one 16-byte load and one
// 4-byte store each); the block's amax is reduced over the eight lanes.  Same
// per-element arithmetic as q8_lane.  Warp-strided over x [M][K] contiguous
// (so the block index is global); every lane of a warp runs every iteration.
__global__ void k_q8_quantize(const float *__restrict__ x, size_t nblocks,
                              int8_t *__restrict__ qs, uint16_t *__restrict__ d) {
  pdl_trigger();
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const size_t nwarp = (nblocks + 3) / 4;
  const size_t stride = (size_t)gridDim.x * (blockDim.x >> 5);
  for (size_t w = ((size_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; w < nwarp; w += stride) {
    const size_t i = w * 32 + lane;  // float4 index
    const bool ok = i < nblocks * 8;
    const float4 v = ok ? reinterpret_cast<const float4 *>(x)[i] : make_float4(0, 0, 0, 0);
    unsigned m = max(max(__float_as_uint(fabsf(v.x)), __float_as_uint(fabsf(v.y))),
                     max(__float_as_uint(fabsf(v.z)), __float_as_uint(fabsf(v.w))));
    m = max(m, __shfl_xor_sync(0xffffffffu, m, 4));
    m = max(m, __shfl_xor_sync(0xffffffffu, m, 2));
    m = max(m, __shfl_xor_sync(0xffffffffu, m, 1));
    if (!ok) continue;
    const float dd = __fdiv_rn(__uint_as_float(m), 127.0f);
    const float inv = dd == 0.0f ? 0.0f : __fdiv_rn(1.0f, dd);
    auto q = [&](float e) {
      int t = __float2int_rn(__fmul_rn(e, inv));
      t = t > 127 ? 127 : (t < -127 ? -127 : t);
      return (uint32_t)(t & 0xFF);
    };
    reinterpret_cast<uint32_t *>(qs)[i] = q(v.x) | q(v.y) << 8 | q(v.z) << 16 | q(v.w) << 24;
    if ((lane & 7) == 0) d[i >> 3] = f32_to_f16(dd);
  }
}

// One CTA per row, the row held in registers (VPT float4 per thread) so it is
// read once; thread t holds float4 t + j*blockDim, so the eight float4 of a
// Q8 block sit in eight adjacent lanes.  out (fp32) and the Q8 pair are each
// optional.
template <int VPT, bool PEER>
__global__ void __launch_bounds__(512) k_rmsnorm_q8(const float *__restrict__ x,
                                                     const float *__restrict__ w, int n, float eps,
                                                     float *__restrict__ out,
                                                     int8_t *__restrict__ qs,
                                                     uint16_t *__restrict__ d, const RmsPeer rp) {
  pdl_trigger();
  pdl_wait();
  const int row = blockIdx.x, n4 = n / 4;
  const float4 *xr = reinterpret_cast<const float4 *>(x + (size_t)row * n);
  float4 v[VPT];
  double ss = 0.0;
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int i = threadIdx.x + j * blockDim.x;
    v[j] = i < n4 ? xr[i] : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  if (PEER) {
    // h = x + the ranks' partial sums, added in rank order (tp_peer.cu's order),
    // each word waited for until it carries this call's epoch.
    const unsigned long long deadline = globaltimer() + rp.timeout_ns;
    const unsigned long long ep64 = peer_epoch(rp.p);
    const unsigned ep = (unsigned)ep64;
    bool bad = false;
    const unsigned long long *slot[kPeerMaxWorld];
#pragma unroll
    for (int r = 0; r < kPeerMaxWorld; ++r)
      slot[r] = peer_slot(rp.p, ep64, r < rp.p.world ? r : 0);
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int i = threadIdx.x + j * blockDim.x;
      if (i < n4) {
        const size_t e0 = (size_t)row * n + 4 * i;
        float sum[4];
        peer_sum4(slot, rp.p.world, e0, ep, deadline, rp.err, bad, sum);
        v[j] = make_float4(__fadd_rn(v[j].x, sum[0]), __fadd_rn(v[j].y, sum[1]),
                           __fadd_rn(v[j].z, sum[2]), __fadd_rn(v[j].w, sum[3]));
        if (!bad) reinterpret_cast<float4 *>(rp.h_out + (size_t)row * n)[i] = v[j];
      }
    }
    // A timed-out row is left unwritten; the block's reductions below still
    // run (every thread reaches them) on whatever the row holds.
  }
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const double a = v[j].x, b = v[j].y, c = v[j].z, e = v[j].w;
    ss = __dadd_rn(ss, __dmul_rn(a, a));
    ss = __dadd_rn(ss, __dmul_rn(b, b));
    ss = __dadd_rn(ss, __dmul_rn(c, c));
    ss = __dadd_rn(ss, __dmul_rn(e, e));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss = __dadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
  __shared__ double part[32];
  __shared__ float s_inv;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) part[warp] = ss;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) t = __dadd_rn(t, part[i]);
    const float mean = (float)__ddiv_rn(t, (double)n);
    s_inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
  }
  __syncthreads();
  const float inv = s_inv;
  const float4 *wr = reinterpret_cast<const float4 *>(w);
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int i = threadIdx.x + j * blockDim.x;
    const bool ok = i < n4;  // uniform over each 8-lane Q8 group (n4 % 8 == 0)
    float4 y = make_float4(__fmul_rn(v[j].x, inv), __fmul_rn(v[j].y, inv),
                           __fmul_rn(v[j].z, inv), __fmul_rn(v[j].w, inv));
    if (w && ok) {
      const float4 g = wr[i];
      y = make_float4(__fmul_rn(y.x, g.x), __fmul_rn(y.y, g.y), __fmul_rn(y.z, g.z),
                      __fmul_rn(y.w, g.w));
    }
    if (out && ok) reinterpret_cast<float4 *>(out + (size_t)row * n)[i] = y;
    if (qs) {
      unsigned m = max(max(__float_as_uint(fabsf(y.x)), __float_as_uint(fabsf(y.y))),
                       max(__float_as_uint(fabsf(y.z)), __float_as_uint(fabsf(y.w))));
      m = max(m, __shfl_xor_sync(0xffffffffu, m, 4));
      m = max(m, __shfl_xor_sync(0xffffffffu, m, 2));
      m = max(m, __shfl_xor_sync(0xffffffffu, m, 1));
      if (ok) {
        const float dd = __fdiv_rn(__uint_as_float(m), 127.0f);
        const float qi = dd == 0.0f ? 0.0f : __fdiv_rn(1.0f, dd);
        auto q = [&](float e) {
          int t = __float2int_rn(__fmul_rn(e, qi));
          t = t > 127 ? 127 : (t < -127 ? -127 : t);
          return (uint32_t)(t & 0xFF);
        };
        const size_t gi = (size_t)row * n4 + i;
        reinterpret_cast<uint32_t *>(qs)[gi] = q(y.x) | q(y.y) << 8 | q(y.z) << 16 | q(y.w) << 24;
        if ((i & 7) == 0) d[gi >> 3] = f32_to_f16(dd);
      }
    }
  }
}

// Few rows (decode steps): C CTAs per row in one thread-block cluster, CTA c
// holding the row's c-th slice of n/C elements in registers.  Same
// per-element arithmetic as k_rmsnorm_q8; the fp64 sum of squares is summed
// per CTA, then the C partial sums are added in CTA order by reading each
// CTA's shared memory through the cluster (distributed shared memory).  In
// the peer form each CTA waits for and adds only its slice of the ranks'
// words, so the exchange is read by C x M CTAs instead of M.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;"
               ::: "memory");
}
__device__ __forceinline__ double cluster_ld_f64(const double *p, int cta) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_u32(p)), "r"(cta));
  double v;
  asm volatile("ld.shared::cluster.f64 %0, [%1];" : "=d"(v) : "r"(remote) : "memory");
  return v;
}

template <int VPT, bool PEER>
__global__ void __launch_bounds__(256) k_rmsnorm_q8c(const float *__restrict__ x,
                                                      const float *__restrict__ w, int n, float eps,
                                                      float *__restrict__ out,
                                                      int8_t *__restrict__ qs,
                                                      uint16_t *__restrict__ d, const RmsPeer rp) {
  pdl_trigger();
  pdl_wait();
  const int C = gridDim.x, c = blockIdx.x, row = blockIdx.y;
  const int s4 = n / 4 / C;                                    // float4 per CTA
  const size_t f0 = (size_t)row * (n / 4) + (size_t)c * s4;    // first float4 of the slice
  const float4 *xr = reinterpret_cast<const float4 *>(x) + f0;
  float4 v[VPT];
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int i = threadIdx.x + j * blockDim.x;
    v[j] = i < s4 ? xr[i] : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  if (PEER) {
    const unsigned long long deadline = globaltimer() + rp.timeout_ns;
    const unsigned long long ep64 = peer_epoch(rp.p);
    const unsigned ep = (unsigned)ep64;
    bool bad = false;
    const unsigned long long *slot[kPeerMaxWorld];
#pragma unroll
    for (int r = 0; r < kPeerMaxWorld; ++r)
      slot[r] = peer_slot(rp.p, ep64, r < rp.p.world ? r : 0);
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int i = threadIdx.x + j * blockDim.x;
      if (i < s4) {
        float sum[4];
        peer_sum4(slot, rp.p.world, 4 * (f0 + i), ep, deadline, rp.err, bad, sum);
        v[j] = make_float4(__fadd_rn(v[j].x, sum[0]), __fadd_rn(v[j].y, sum[1]),
                           __fadd_rn(v[j].z, sum[2]), __fadd_rn(v[j].w, sum[3]));
        if (!bad) reinterpret_cast<float4 *>(rp.h_out)[f0 + i] = v[j];
      }
    }
  }
  double ss = 0.0;
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const double a = v[j].x, b = v[j].y, cc = v[j].z, e = v[j].w;
    ss = __dadd_rn(ss, __dmul_rn(a, a));
    ss = __dadd_rn(ss, __dmul_rn(b, b));
    ss = __dadd_rn(ss, __dmul_rn(cc, cc));
    ss = __dadd_rn(ss, __dmul_rn(e, e));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss = __dadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
  __shared__ double part[8];
  __shared__ double cta_ss;
  __shared__ float s_inv;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) part[warp] = ss;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) t = __dadd_rn(t, part[i]);
    cta_ss = t;
  }
  cluster_sync_all();  // every CTA's partial sum is in its shared memory
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int r = 0; r < C; ++r) t = __dadd_rn(t, cluster_ld_f64(&cta_ss, r));
    const float mean = (float)__ddiv_rn(t, (double)n);
    s_inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
  }
  __syncthreads();
  const float inv = s_inv;
  const float4 *wr = reinterpret_cast<const float4 *>(w) + (size_t)c * s4;
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int i = threadIdx.x + j * blockDim.x;
    const bool ok = i < s4;  // uniform over each 8-lane Q8 group (s4 % 8 == 0)
    float4 y = make_float4(__fmul_rn(v[j].x, inv), __fmul_rn(v[j].y, inv),
                           __fmul_rn(v[j].z, inv), __fmul_rn(v[j].w, inv));
    if (w && ok) {
      const float4 g = wr[i];
      y = make_float4(__fmul_rn(y.x, g.x), __fmul_rn(y.y, g.y), __fmul_rn(y.z, g.z),
                      __fmul_rn(y.w, g.w));
    }
    if (out && ok) reinterpret_cast<float4 *>(out)[f0 + i] = y;
    if (qs) {
      unsigned m = max(max(__float_as_uint(fabsf(y.x)), __float_as_uint(fabsf(y.y))),
                       max(__float_as_uint(fabsf(y.z)), __float_as_uint(fabsf(y.w))));
      m = max(m, __shfl_xor_sync(0xffffffffu, m, 4));
      m = max(m, __shfl_xor_sync(0xffffffffu, m, 2));
      m = max(m, __shfl_xor_sync(0xffffffffu, m, 1));
      if (ok) {
        const float dd = __fdiv_rn(__uint_as_float(m), 127.0f);
        const float qi = dd == 0.0f ? 0.0f : __fdiv_rn(1.0f, dd);
        auto q = [&](float e) {
          int t = __float2int_rn(__fmul_rn(e, qi));
          t = t > 127 ? 127 : (t < -127 ? -127 : t);
          return (uint32_t)(t & 0xFF);
        };
        const size_t gi = f0 + i;
        reinterpret_cast<uint32_t *>(qs)[gi] = q(y.x) | q(y.y) << 8 | q(y.z) << 16 | q(y.w) << 24;
        if ((gi & 7) == 0) d[gi >> 3] = f32_to_f16(dd);
      }
    }
  }
  cluster_sync_all();  // no CTA leaves while another may still read its partial sum
}

template <int VPT, bool PEER>
cudaError_t launch_rms_cluster(int C, int M, int threads, const float *x, const float *w, int n,
                               float eps, float *out, int8_t *qs, uint16_t *d, const RmsPeer &rp,
                               cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(C, M);
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = C;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  count_launch();
  return cudaLaunchKernelEx(&cfg, k_rmsnorm_q8c<VPT, PEER>, x, w, n, eps, out, qs, d, rp);
}

__global__ void k_add(const float *__restrict__ a, const float *__restrict__ b,
                      float *__restrict__ y, size_t n) {
  pdl_trigger();
  pdl_wait();
  size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) y[i] = __fadd_rn(a[i], b[i]);
}

cudaError_t launch_q8_quantize(const float *x, int M, int K, int8_t *qs, uint16_t *d,
                               cudaStream_t s) {
  size_t nblocks = (size_t)M * (K / 32);
  if (nblocks == 0) return cudaSuccess;
  if ((reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(qs) & 3) ||
      (reinterpret_cast<uintptr_t>(d) & 1))
    return cudaErrorMisalignedAddress;
  // 4 blocks per warp, 8 warps per CTA; at most 8 CTAs per SM's worth of grid.
  const size_t ctas = (nblocks + 31) / 32;
  const unsigned grid = (unsigned)(ctas < 148 * 8 ? ctas : 148 * 8);
  return launch_pdl(k_q8_quantize, dim3(grid), dim3(256), 0, s, x, nblocks, qs, d);
}

cudaError_t launch_rmsnorm_q8(const float *x, const float *w, int M, int n, float eps,
                              float *out, int8_t *qs, uint16_t *d, cudaStream_t s,
                              const RmsPeer *rpp) {
  RmsPeer rp{};
  if (rpp) {
    rp = *rpp;
    if (rp.p.world < 1 || rp.p.world > kPeerMaxWorld || (size_t)M * n > (size_t)rp.p.slot ||
        !rp.h_out || (reinterpret_cast<uintptr_t>(rp.h_out) & 15) || rp.p.slot % 4)
      return cudaErrorInvalidValue;
  }
  if (M == 0) return cudaSuccess;
  if (n % 4 || (qs && n % 32) || (reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(w) & 15) ||
      (reinterpret_cast<uintptr_t>(out) & 15) || (reinterpret_cast<uintptr_t>(qs) & 3) ||
      (reinterpret_cast<uintptr_t>(d) & 1))
    return cudaErrorMisalignedAddress;
  const int n4 = n / 4;
  const bool peer = rpp != nullptr;
  // Decode-sized row counts: split each row over a cluster of 8, 4 or 2 CTAs
  // (each slice a whole number of Q8 blocks), at most 4 float4 per thread.
  if (M <= kRmsClusterMaxRows) {
    int C = 8;
    while (C > 1 && n4 % (C * 8)) C >>= 1;
    if (C > 1) {
      const int s4 = n4 / C;
      int threads = (s4 + 31) / 32 * 32;
      if (threads > 256) threads = 256;
      const int vpt = (s4 + threads - 1) / threads;
      if (vpt == 1)
        return peer ? launch_rms_cluster<1, true>(C, M, threads, x, w, n, eps, out, qs, d, rp, s)
                    : launch_rms_cluster<1, false>(C, M, threads, x, w, n, eps, out, qs, d, rp, s);
      if (vpt == 2)
        return peer ? launch_rms_cluster<2, true>(C, M, threads, x, w, n, eps, out, qs, d, rp, s)
                    : launch_rms_cluster<2, false>(C, M, threads, x, w, n, eps, out, qs, d, rp, s);
      if (vpt <= 4)
        return peer ? launch_rms_cluster<4, true>(C, M, threads, x, w, n, eps, out, qs, d, rp, s)
                    : launch_rms_cluster<4, false>(C, M, threads, x, w, n, eps, out, qs, d, rp, s);
    }
  }
  // Threads: a multiple of 32 with at most 4 float4 each up to 512 threads.
  int threads = ((n4 + 3) / 4 + 31) / 32 * 32;
  threads = threads < 128 ? 128 : (threads > 512 ? 512 : threads);
  const int vpt = (n4 + threads - 1) / threads;
  const dim3 g(M), b(threads);
  switch (vpt) {
    case 1: return peer ? launch_pdl(k_rmsnorm_q8<1, true>, g, b, 0, s, x, w, n, eps, out, qs, d, rp)
                        : launch_pdl(k_rmsnorm_q8<1, false>, g, b, 0, s, x, w, n, eps, out, qs, d, rp);
    case 2: return peer ? launch_pdl(k_rmsnorm_q8<2, true>, g, b, 0, s, x, w, n, eps, out, qs, d, rp)
                        : launch_pdl(k_rmsnorm_q8<2, false>, g, b, 0, s, x, w, n, eps, out, qs, d, rp);
    case 3: return peer ? launch_pdl(k_rmsnorm_q8<3, true>, g, b, 0, s, x, w, n, eps, out, qs, d, rp)
                        : launch_pdl(k_rmsnorm_q8<3, false>, g, b, 0, s, x, w, n, eps, out, qs, d, rp);
    case 4: return peer ? launch_pdl(k_rmsnorm_q8<4, true>, g, b, 0, s, x, w, n, eps, out, qs, d, rp)
                        : launch_pdl(k_rmsnorm_q8<4, false>, g, b, 0, s, x, w, n, eps, out, qs, d, rp);
    case 5: case 6: case 7: case 8:
      return peer ? launch_pdl(k_rmsnorm_q8<8, true>, g, b, 0, s, x, w, n, eps, out, qs, d, rp)
                  : launch_pdl(k_rmsnorm_q8<8, false>, g, b, 0, s, x, w, n, eps, out, qs, d, rp);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_add(const float *a, const float *b, float *y, size_t n, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  return launch_pdl(k_add, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, s, a, b, y, n);
}

}  // namespace si
