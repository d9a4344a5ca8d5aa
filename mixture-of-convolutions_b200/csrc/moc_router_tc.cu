// Tensor-core router kernels (bf16).  Placeholder until the kernels land.
#include "moc_common.cuh"
#include "moc_internal.h"

namespace moc {
bool tc_router_supported(int64_t, int64_t, int, int) { return false; }
int tc_router_forward(int64_t, int64_t, int, int, const void*, const void*, void*, cudaStream_t) {
  return MOC_ERR_UNSUPPORTED_SHAPE;
}
size_t tc_router_backward_ws(int64_t, int64_t, int) { return 0; }
int tc_router_backward(int64_t, int64_t, int, int, const void*, const void*, const void*, const void*, int, void*,
                       void*, void*, size_t, cudaStream_t) {
  return MOC_ERR_UNSUPPORTED_SHAPE;
}
}  // namespace moc
