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

__device__ __forceinline__ unsigned long long peer_ld(const unsigned long long *p) {
  unsigned long long w;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
  return w;
}

// The sum over ranks, in rank order, of word i of every source's slot, each
// word waited for until it carries `epoch`.  All the ranks' loads are issued
// before any is waited on (a system-scope load takes a round trip to L2; one
// after another they would serialise), then only the words not yet written
// are polled again.  Past the deadline: SI_ERR_TIMEOUT, *bad set, 0 returned.
template <int MAXW>
__device__ __forceinline__ float peer_sum(const unsigned long long *const (&slot)[MAXW],
                                          int world, size_t i, unsigned epoch,
                                          unsigned long long deadline, int *err, bool &bad) {
  unsigned long long w[MAXW];
#pragma unroll
  for (int r = 0; r < MAXW; ++r)
    if (r < world) w[r] = peer_ld(slot[r] + i);
  float s = 0.0f;
#pragma unroll
  for (int r = 0; r < MAXW; ++r) {
    if (r >= world) break;
    while (!bad && (unsigned)(w[r] >> 32) != epoch) {
      if (globaltimer() > deadline) {
        bad = true;
        raise_error(err, 6 /* SI_ERR_TIMEOUT */);
        break;
      }
      __nanosleep(32);
      w[r] = peer_ld(slot[r] + i);
    }
    const float v = __uint_as_float((unsigned)w[r]);
    s = r == 0 ? v : __fadd_rn(s, v);
  }
  return bad ? 0.0f : s;
}

__device__ __forceinline__ void peer_ld2(const unsigned long long *p, unsigned long long &a,
                                         unsigned long long &b) {
  asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p)
               : "memory");
}

// peer_sum for the four words i .. i+3 (i a multiple of 4): two 16-byte loads
// per rank, all ranks' in flight together.
template <int MAXW>
__device__ __forceinline__ void peer_sum4(const unsigned long long *const (&slot)[MAXW],
                                          int world, size_t i, unsigned epoch,
                                          unsigned long long deadline, int *err, bool &bad,
                                          float (&out)[4]) {
  unsigned long long w[MAXW][4];
#pragma unroll
  for (int r = 0; r < MAXW; ++r)
    if (r < world) {
      peer_ld2(slot[r] + i, w[r][0], w[r][1]);
      peer_ld2(slot[r] + i + 2, w[r][2], w[r][3]);
    }
#pragma unroll
  for (int r = 0; r < MAXW; ++r) {
    if (r >= world) break;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      while (!bad && (unsigned)(w[r][c] >> 32) != epoch) {
        if (globaltimer() > deadline) {
          bad = true;
          raise_error(err, 6 /* SI_ERR_TIMEOUT */);
          break;
        }
        __nanosleep(32);
        w[r][c] = peer_ld(slot[r] + i + c);
      }
      const float v = __uint_as_float((unsigned)w[r][c]);
      out[c] = r == 0 ? v : __fadd_rn(out[c], v);
    }
  }
  if (bad) out[0] = out[1] = out[2] = out[3] = 0.0f;
}

// Word 0 of source rank src's slot for the call of effective epoch ep, on this rank.
__device__ __forceinline__ const unsigned long long *peer_slot(const PeerOut &p,
                                                               unsigned long long ep, int src) {
  return reinterpret_cast<const unsigned long long *>(p.base[p.rank] + kPeerData) +
         ((size_t)(ep & 1) * p.world + src) * p.slot;
}

}  // namespace si
