// Tensor-core MoC convolution kernels (bf16).  Placeholder until the kernels land.
#include "moc_common.cuh"
#include "moc_internal.h"

namespace moc {
bool tc_conv_supported(const moc_problem&) { return false; }
int tc_forward(const moc_problem&, const void*, const void*, const void*, void*, cudaStream_t) {
  return MOC_ERR_UNSUPPORTED_SHAPE;
}
size_t tc_backward_ws(const moc_problem&) { return 0; }
int tc_backward(const moc_problem&, const void*, const void*, const void*, const void*, void*, void*, void*, void*,
                size_t, cudaStream_t) {
  return MOC_ERR_UNSUPPORTED_SHAPE;
}
}  // namespace moc
