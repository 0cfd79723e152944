// tp_peer.cu -- the reduction half of the fused row-parallel projection.
//
// Tensor parallelism (no counterpart in the single-core reference; its layer
// is qwen_one_layer.c:245-280) splits QKV/gate/up by output rows and O/down
// by input rows, so the O and down projections leave partial sums that every
// rank must add.  Instead of a separate all-reduce, the projection's own GEMV
// writes its partial sums straight into every rank's receive slot over NVLink
// (peer stores from the tensor-core GEMV's epilogue, tile by tile as the
// tiles finish), each value in one 8-byte word together with the call's
// epoch; this kernel polls the words until they carry the epoch -- the data
// is its own flag, so no fence or flag hop sits on the critical path -- and
// adds the slots in rank order and the residual.  Every rank sums in the same
// order, so all ranks hold bit-identical hidden states.
//
// The wait is bounded: past timeout_ns a thread records SI_ERR_TIMEOUT in the
// context's error word and stops without writing its outputs, so a rank that
// never arrives ends in an error on the host instead of a hung GPU.
#include "si_common.cuh"
#include "si_kernels.cuh"
#include "si_peer.cuh"
#include "si_tma.cuh"

namespace si {

namespace {
__global__ void __launch_bounds__(256) k_tp_combine(const PeerOut p, const float *resid,
                                                    float *y, size_t n,
                                                    unsigned long long timeout_ns, int *err) {
  pdl_trigger();
  pdl_wait();
  const unsigned long long deadline = globaltimer() + timeout_ns;
  const unsigned long long ep64 = peer_epoch(p);
  const unsigned ep = (unsigned)ep64;
  bool bad = false;
  const unsigned long long *slot[kPeerMaxWorld];
#pragma unroll
  for (int r = 0; r < kPeerMaxWorld; ++r) slot[r] = peer_slot(p, ep64, r < p.world ? r : 0);
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x) {
    const float s = peer_sum(slot, p.world, i, ep, deadline, err, bad);
    if (bad) return;
    y[i] = resid ? __fadd_rn(resid[i], s) : s;
  }
}
__global__ void k_epoch_advance(unsigned long long *counter, unsigned n) {
  pdl_trigger();
  pdl_wait();
  if (threadIdx.x == 0) *counter += n;
}
}  // namespace

cudaError_t launch_epoch_advance(unsigned long long *counter, unsigned n, cudaStream_t s) {
  return launch_pdl(k_epoch_advance, dim3(1), dim3(32), 0, s, counter, n);
}

cudaError_t launch_tp_combine(const PeerOut &p, const float *resid, float *y, size_t n,
                              unsigned long long timeout_ns, int *err, cudaStream_t s) {
  if (p.world < 1 || p.world > kPeerMaxWorld || p.rank < 0 || p.rank >= p.world ||
      n > (size_t)p.slot)
    return cudaErrorInvalidValue;
  const unsigned blocks = (unsigned)((n + 1023) / 1024);
  return launch_pdl(k_tp_combine, dim3(blocks < 1 ? 1 : blocks), dim3(256), 0, s, p, resid, y, n,
                    timeout_ns, err);
}

}  // namespace si
