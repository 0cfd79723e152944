// si_peer.cuh -- reading the receive slots of a fused row-parallel
// projection (see tp_peer.cu): each 8-byte word is (float bits | epoch << 32),
// written by its producer in one store; a reader polls a word until it carries
// the expected epoch, with a time bound.
#pragma once
#include "si_common.cuh"
#include "si_kernels.cuh"
#include "si_tma.cuh"

namespace si {

// Value of word p once it carries `epoch` (low 32 bits).  Past the deadline
// the thread records SI_ERR_TIMEOUT (6) once, sets *bad and returns 0.
__device__ __forceinline__ float peer_word(const unsigned long long *p, unsigned epoch,
                                           unsigned long long deadline, int *err, bool &bad) {
  unsigned long long w;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
  if (bad) return 0.0f;
  while ((unsigned)(w >> 32) != epoch) {
    if (globaltimer() > deadline) {
      bad = true;
      raise_error(err, 6 /* SI_ERR_TIMEOUT */);
      return 0.0f;
    }
    __nanosleep(32);
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
  }
  return __uint_as_float((unsigned)w);
}

// Word 0 of source rank src's slot for the call of effective epoch ep, on this rank.
__device__ __forceinline__ const unsigned long long *peer_slot(const PeerOut &p,
                                                               unsigned long long ep, int src) {
  return reinterpret_cast<const unsigned long long *>(p.base[p.rank] + kPeerData) +
         ((size_t)(ep & 1) * p.world + src) * p.slot;
}

}  // namespace si
