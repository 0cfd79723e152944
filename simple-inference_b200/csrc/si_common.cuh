// si_common.cuh -- shared device helpers for the sm_100a kernels.
//
// Numerics follow the reference's portable C path, which is built with
// -ffp-contract=off (reference Makefile:7): every product and sum below is an
// explicitly rounded __f*_rn intrinsic so nvcc cannot contract it into an FMA.
#pragma once
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>

#define SI_QK 32
#define SI_RT 32  // rows per row-tile of the SoA weight layout

#include <utility>

namespace si {

// Programmatic dependent launch.  A decode step is a chain of small kernels,
// each shorter than its own launch latency plus the latency of its first
// loads.  Kernels launched with launch_pdl() may start while the previous
// kernel of the stream is still running: they call pdl_trigger() first (so
// their own successor may be scheduled early too), may then read data no
// earlier kernel writes (weights), and call pdl_wait() -- which returns once
// every grid they depend on has completed and its writes are visible --
// before they read or write anything else.  Both are no-ops in a launch
// without the attribute.
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Grids larger than this many CTAs gain nothing from an early start (most of
// their CTAs cannot be resident before the previous grid ends) and are
// launched without the attribute.
constexpr unsigned kPdlMaxCtas = 4096;

// Process-wide count of kernels this library has queued (all devices and
// contexts), read through si_kernel_launches(); every launch site bumps it.
extern unsigned long long g_kernel_launches;
inline void count_launch() { __atomic_fetch_add(&g_kernel_launches, 1ull, __ATOMIC_RELAXED); }

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t s, Args &&...args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = (unsigned long long)grid.x * grid.y * grid.z <= kPdlMaxCtas ? 1 : 0;
  count_launch();
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// Kernels that detect bad input or a bounded wait that ran out record a
// si_status code in the context's device error word (first error wins); the
// host reads and clears it in si_ctx_status().
__device__ __forceinline__ void raise_error(int *err, int code) {
  if (err) atomicCAS(err, 0, code);
}

// Exact fp16 -> fp32 of the reference (qwen_one_layer.c:42-59); the hardware
// conversion is exact for every half including subnormals.
__device__ __forceinline__ float f16_to_f32(uint16_t h) {
  return __half2float(__ushort_as_half(h));
}
// Round-to-nearest-even fp32 -> fp16 with subnormals and overflow to inf, the
// rounding of qwen_one_layer.c:61-86 for every finite input.
__device__ __forceinline__ uint16_t f32_to_f16(float x) {
  return __half_as_ushort(__float2half_rn(x));
}

// One Q8_0 block from 32 values held one per lane of a full warp
// (qwen_one_layer.c:98-116): amax -> d = amax/127 (fp32) -> store fp16(d) ->
// inv = d==0 ? 0 : 1/d -> q = rint(x*inv) clamped to +-127.
__device__ __forceinline__ int8_t q8_lane(float x, uint16_t &d16) {
  float a = fabsf(x);
  unsigned amax_bits = __reduce_max_sync(0xffffffffu, __float_as_uint(a));
  float amax = __uint_as_float(amax_bits);
  float d = __fdiv_rn(amax, 127.0f);
  d16 = f32_to_f16(d);
  float inv = d == 0.0f ? 0.0f : __fdiv_rn(1.0f, d);
  int q = __float2int_rn(__fmul_rn(x, inv));
  q = q > 127 ? 127 : (q < -127 ? -127 : q);
  return (int8_t)q;
}

// Q4 nibble words stored with every byte XOR 0x88, so each nibble is the
// 4-bit two's complement of (q - 8).  Placing a nibble in the high half of a
// byte gives the signed byte 16*(q-8); the dp4a sums are therefore 16*isum.
__device__ __forceinline__ int lo_nib_s8x16(uint32_t w) { return (int)((w << 4) & 0xF0F0F0F0u); }
__device__ __forceinline__ int hi_nib_s8x16(uint32_t w) { return (int)(w & 0xF0F0F0F0u); }

}  // namespace si
