// Chunked tensor-core WKV-7 ClampW path (placeholder until the kernels land).
#include "wkv7_common.cuh"

namespace camoe {
namespace chunked {
cudaError_t launch_fwd(const FwdArgs&, cudaStream_t) { return cudaErrorNotSupported; }
cudaError_t launch_bwd(const BwdArgs&, cudaStream_t) { return cudaErrorNotSupported; }
size_t ckpt_bytes(int64_t chains, int64_t T) {
  return static_cast<size_t>(chains * ((T + kChunk - 1) / kChunk)) * kN * kN * sizeof(float);
}
}  // namespace chunked
}  // namespace camoe
