// gemm_tc.cu -- tcgen05 (sm_100a) Q4_0 x Q8_0 GEMM for prefill and batched decode.
// Placeholder until the tensor-core kernel lands: reports itself unsupported so
// the dispatcher keeps every shape on the CUDA-core path.
#include "si_kernels.cuh"

namespace si {
bool gemm_tc_supported(int, int, int) { return false; }
cudaError_t launch_gemm_tc(const GemvArgs &, bool, cudaStream_t) { return cudaErrorNotSupported; }
}  // namespace si
