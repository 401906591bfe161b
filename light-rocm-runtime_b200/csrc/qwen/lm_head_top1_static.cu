// Greedy LM-head top-1 whose scratch is file-scope device memory, so the call
// allocates nothing.
//
// It is a variant of the LM-head partition and reduce kernels
// (reference benchmarks/qwen_stateful_graph_kernel.cpp lm_head_top1_partition
// :231-272 and reduce_top1 :339-356, restated in qwen_stateful_graph.cu as
// generic_lm_head / generic_reduce_top1): those write one candidate per
// partition into partial_max_values / partial_max_indices, buffers the caller
// allocates. Here the per-block candidates live in the static array below.
//
// Every row's dot product uses the reference order (lane l accumulates
// columns l, l+32, ... with fmaf, then a shfl_down tree), and candidates are
// merged with better_top1 (larger value, ties to the lower row), so the token
// and logit equal those of the partitioned path bit for bit.
#include "lm_head_top1_static.hpp"

#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <mutex>

namespace lrq_static {
namespace {

constexpr uint32_t kThreads = 256;
constexpr uint32_t kWarps = kThreads / 32u;
constexpr unsigned kFullMask = 0xffffffffu;
constexpr uint32_t kMaxDevices = 64;

struct Top1Scratch {
  float values[kMaxBlocks];      // one candidate per block
  uint32_t indices[kMaxBlocks];
  uint32_t arrivals;             // blocks done; must be 0 when a launch starts
  float result_value;            // written by the last block
  uint32_t result_index;
};

// 8 KB of device memory per process and device, zero at module load.
static __device__ __align__(256) Top1Scratch g_top1_scratch;

__device__ __forceinline__ bool better_top1(float value, uint32_t index, float best_value,
                                            uint32_t best_index) {
  return value > best_value || (value == best_value && index < best_index);
}

__global__ void __launch_bounds__(kThreads)
lm_head_top1_kernel(const float *__restrict__ lm_head, const float *__restrict__ hidden,
                    uint32_t rows, uint32_t columns, Top1Scratch *scratch) {
  __shared__ float warp_values[kWarps];
  __shared__ uint32_t warp_indices[kWarps];
  __shared__ uint32_t last_block;
  const uint32_t lane = threadIdx.x & 31u;
  const uint32_t warp = threadIdx.x >> 5u;
  float best_value = -INFINITY;
  uint32_t best_index = UINT32_MAX;
  for (uint32_t row = blockIdx.x * kWarps + warp; row < rows; row += gridDim.x * kWarps) {
    const float *weights = lm_head + size_t{row} * columns;
    float sum = 0.0f;
    for (uint32_t column = lane; column < columns; column += 32u) {
      sum = fmaf(__ldg(hidden + column), __ldg(weights + column), sum);
    }
    for (uint32_t offset = 16; offset != 0; offset >>= 1u) {
      sum += __shfl_down_sync(kFullMask, sum, offset);
    }
    if (lane == 0 && better_top1(sum, row, best_value, best_index)) {
      best_value = sum;
      best_index = row;
    }
  }
  if (lane == 0) {
    warp_values[warp] = best_value;
    warp_indices[warp] = best_index;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (uint32_t w = 1; w < kWarps; ++w) {
      if (better_top1(warp_values[w], warp_indices[w], warp_values[0], warp_indices[0])) {
        warp_values[0] = warp_values[w];
        warp_indices[0] = warp_indices[w];
      }
    }
    scratch->values[blockIdx.x] = warp_values[0];
    scratch->indices[blockIdx.x] = warp_indices[0];
    __threadfence(); // candidate before the arrival
    last_block = atomicAdd(&scratch->arrivals, 1u) + 1u == gridDim.x ? 1u : 0u;
  }
  __syncthreads();
  if (last_block != 0u && threadIdx.x == 0) {
    __threadfence(); // every block's candidate is visible after its arrival
    float value = __ldcg(&scratch->values[0]);
    uint32_t index = __ldcg(&scratch->indices[0]);
    for (uint32_t b = 1; b < gridDim.x; ++b) {
      const float other = __ldcg(&scratch->values[b]);
      const uint32_t other_index = __ldcg(&scratch->indices[b]);
      if (better_top1(other, other_index, value, index)) {
        value = other;
        index = other_index;
      }
    }
    scratch->result_value = value;
    scratch->result_index = index;
    scratch->arrivals = 0; // ready for the next launch
  }
}

struct DeviceSetUp {
  bool done = false;
  Top1Scratch *scratch = nullptr;
  uint32_t default_blocks = 0;
};

std::mutex g_set_up_mutex;
DeviceSetUp g_set_up[kMaxDevices];

bool fail(std::string &error, const char *what, cudaError_t status) {
  error = std::string(what) + ": " + cudaGetErrorString(status);
  return false;
}

// Once per device: the scratch's device address and the default grid.
bool set_up(uint32_t device, DeviceSetUp &out, std::string &error) {
  std::lock_guard<std::mutex> lock(g_set_up_mutex);
  DeviceSetUp &entry = g_set_up[device];
  if (!entry.done) {
    void *address = nullptr;
    cudaError_t status = cudaGetSymbolAddress(&address, g_top1_scratch);
    if (status != cudaSuccess) {
      return fail(error, "cudaGetSymbolAddress", status);
    }
    int sms = 0;
    status = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount,
                                    static_cast<int>(device));
    if (status != cudaSuccess) {
      return fail(error, "cudaDeviceGetAttribute", status);
    }
    entry.scratch = static_cast<Top1Scratch *>(address);
    entry.default_blocks = std::min<uint32_t>(2u * static_cast<uint32_t>(sms), kMaxBlocks);
    entry.done = true;
  }
  out = entry;
  return true;
}

} // namespace

lr_status_t lm_head_top1(uint32_t device, void *stream, const float *lm_head,
                         const float *hidden, uint32_t rows, uint32_t columns,
                         uint32_t blocks, uint32_t *token, float *logit,
                         std::string &error) {
  if (lm_head == nullptr || hidden == nullptr || token == nullptr || logit == nullptr ||
      rows == 0 || columns == 0 || device >= kMaxDevices) {
    error = "null pointer, zero rows or columns, or device index out of range";
    return LR_ERROR_INVALID_ARGUMENT;
  }
  if (blocks > kMaxBlocks) {
    char text[160];
    std::snprintf(text, sizeof(text),
                  "%u blocks requested; the static scratch holds %u block candidates",
                  blocks, kMaxBlocks);
    error = text;
    return LR_ERROR_INVALID_ARGUMENT;
  }
  // The caller's current device is restored on every return path.
  int previous = 0;
  cudaError_t status = cudaGetDevice(&previous);
  if (status != cudaSuccess) {
    fail(error, "cudaGetDevice", status);
    return LR_ERROR_RUNTIME;
  }
  struct RestoreDevice {
    int device;
    ~RestoreDevice() { cudaSetDevice(device); }
  } restore{previous};
  status = cudaSetDevice(static_cast<int>(device));
  if (status != cudaSuccess) {
    fail(error, "cudaSetDevice", status);
    return LR_ERROR_RUNTIME;
  }
  DeviceSetUp setup;
  if (!set_up(device, setup, error)) {
    return LR_ERROR_RUNTIME;
  }
  const uint32_t grid = blocks != 0 ? blocks : setup.default_blocks;
  cudaStream_t queue = static_cast<cudaStream_t>(stream);
  // The arrival counter must start at zero; a launch that never finished
  // (an earlier device error) may have left it set.
  status = cudaMemsetAsync(&setup.scratch->arrivals, 0, sizeof(uint32_t), queue);
  if (status != cudaSuccess) {
    fail(error, "cudaMemsetAsync", status);
    return LR_ERROR_RUNTIME;
  }
  lm_head_top1_kernel<<<grid, kThreads, 0, queue>>>(lm_head, hidden, rows, columns,
                                                    setup.scratch);
  status = cudaGetLastError();
  if (status != cudaSuccess) {
    fail(error, "lm_head_top1_kernel launch", status);
    return LR_ERROR_RUNTIME;
  }
  status = cudaMemcpyAsync(token, &setup.scratch->result_index, sizeof(uint32_t),
                           cudaMemcpyDeviceToHost, queue);
  if (status == cudaSuccess) {
    status = cudaMemcpyAsync(logit, &setup.scratch->result_value, sizeof(float),
                             cudaMemcpyDeviceToHost, queue);
  }
  if (status == cudaSuccess) {
    status = cudaStreamSynchronize(queue);
  }
  if (status != cudaSuccess) {
    fail(error, "lm_head_top1 result copy", status);
    return LR_ERROR_DEVICE_FAULT;
  }
  return LR_SUCCESS;
}

} // namespace lrq_static
