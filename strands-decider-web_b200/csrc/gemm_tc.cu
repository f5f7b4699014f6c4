// tcgen05 GEMM family (placeholder until the kernel lands).
#include "common.cuh"

namespace s4 {
bool tc_available() { return false; }
cudaError_t launch_tc_gemm(const uint8_t*, const uint8_t*, const __half*, __half*, uint32_t*, int, int, int, int, int,
                           int, int, cudaStream_t) {
  return cudaErrorNotSupported;
}
}  // namespace s4
