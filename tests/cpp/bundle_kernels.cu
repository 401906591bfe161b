// Test kernels for the lrrt::bundle device test: built into a cubin that the
// committed manifest tests/cpp/bundle_manifest.json describes.
#include <cstdint>

// out[i] = x[i] * factor (+ bias[i] when bias is bound), i < n.
extern "C" __global__ void bundle_scale_kernel(const float *x, float *out, const float *bias,
                                               float factor, uint32_t n) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) {
    out[i] = x[i] * factor + (bias != nullptr ? bias[i] : 0.0f);
  }
}

// out[i] = i + offset for i < n (a second kernel of the same bundle).
extern "C" __global__ void bundle_iota_kernel(uint32_t *out, uint32_t offset, uint32_t n) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) {
    out[i] = i + offset;
  }
}
