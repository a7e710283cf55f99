// Tensor-core (tcgen05) convolution paths.  Until a shape is claimed here
// the exact SIMT implicit GEMM in conv.cu runs it.
#include "common.cuh"

namespace pvb2 {

size_t conv_tc_workspace(const pvb2_conv2d_desc*, int) { return 0; }

int conv_tc_fwd(const pvb2_conv2d_desc*, const float*, const float*, const float*, float*, void*, size_t,
                cudaStream_t, bool* handled) {
  *handled = false;
  return PVB2_OK;
}

int conv_tc_bwd_data(const pvb2_conv2d_desc*, const float*, const float*, float*, void*, size_t, cudaStream_t,
                     bool* handled) {
  *handled = false;
  return PVB2_OK;
}

int conv_tc_bwd_filter(const pvb2_conv2d_desc*, const float*, const float*, float*, void*, size_t, cudaStream_t,
                       bool* handled) {
  *handled = false;
  return PVB2_OK;
}

}  // namespace pvb2
