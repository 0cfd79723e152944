// si_peer.cuh -- the bounded wait for every rank's flag of a fused
// row-parallel projection (see tp_peer.cu), shared by the kernels that
// consume the receive slots.
#pragma once
#include "si_common.cuh"
#include "si_kernels.cuh"
#include "si_tma.cuh"

namespace si {

__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long *p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Called by every thread of the CTA.  Thread 0 polls this rank's flags until
// each rank has published p.epoch; past timeout_ns it records SI_ERR_TIMEOUT
// (6) in err and every thread gets false.
__device__ __forceinline__ bool tp_wait_flags(const PeerOut &p, unsigned long long timeout_ns,
                                              int *err) {
  __shared__ int bad;
  if (threadIdx.x == 0) {
    bad = 0;
    const char *own = p.base[p.rank];
    const unsigned long long t0 = globaltimer();
    for (int src = 0; src < p.world && !bad; ++src) {
      const unsigned long long *f =
          reinterpret_cast<const unsigned long long *>(own + kPeerFlags + src * 128);
      while (ld_acquire_sys(f) < p.epoch) {
        if (globaltimer() - t0 > timeout_ns) {
          bad = 1;
          raise_error(err, 6 /* SI_ERR_TIMEOUT */);
          break;
        }
        __nanosleep(64);
      }
    }
  }
  __syncthreads();
  return !bad;
}

}  // namespace si
