// Constants and host helpers shared by the prefill and batched-decode
// drivers (prefill.cpp, batch.cpp): model widths, tensor-core tile widths,
// TMA tensor-map encoding and launch shapes.
#ifndef LRRT_B200_QWEN_PREFILL_COMMON_HPP_
#define LRRT_B200_QWEN_PREFILL_COMMON_HPP_

#include "lrrt/lrrt.hpp"
#include "lrrt/qwen/prefill.hpp"
#include "lrrt/qwen/stateful_graph_context.hpp"

#include <cuda.h>
#include <cuda_runtime_api.h>

#include <cstring>
#include <stdexcept>
#include <string>

namespace lrrt::qwen::prefill::detail {

namespace qd = lrrt::qwen::stateful_graph;

constexpr uint32_t kHidden = qd::kHiddenSize;
constexpr uint32_t kQkv = qd::kPackedQkvSize;
constexpr uint32_t kIntermediate = qd::kIntermediateSize;
constexpr uint32_t kSms = 148;           // B200 SM count: one TC GEMM CTA per SM
constexpr uint32_t kWaitLimitMs = 2000;  // per mbarrier wait of the TC GEMM
// Accumulator columns per tensor-core tile of each GEMM: output widths 1152
// (QKV) = 6 x 192, 896 (o_proj, down) = 4 x 224, gate/up = 38 x (128 gate +
// 128 up); the LM head uses 256.
constexpr uint32_t kQkvTile = 192, kHiddenTile = 224, kGateUpTile = 256;

// Floats of one layer's GEMM weights: QKV, o_proj, gate/up, down.
constexpr size_t kQkvFloats = size_t{kQkv} * kHidden;
constexpr size_t kOFloats = size_t{kHidden} * kHidden;
constexpr size_t kGateUpFloats = size_t{2} * kIntermediate * kHidden;
constexpr size_t kDownFloats = size_t{kHidden} * kIntermediate;
constexpr size_t kLayerFloats = kQkvFloats + kOFloats + kGateUpFloats + kDownFloats;

static_assert(sizeof(CUtensorMap) == sizeof(TensorMap), "TensorMap must hold a CUtensorMap");

using EncodeTiled = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                 const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                 const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                 CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiled encode_tiled() {
  static const EncodeTiled function = [] {
    void *entry = nullptr;
    cudaDriverEntryPointQueryResult found{};
    const cudaError_t status = cudaGetDriverEntryPointByVersion(
        "cuTensorMapEncodeTiled", &entry, 12000, cudaEnableDefault, &found);
    if (status != cudaSuccess || found != cudaDriverEntryPointSuccess || entry == nullptr) {
      throw std::runtime_error("cuTensorMapEncodeTiled is not available");
    }
    return reinterpret_cast<EncodeTiled>(entry);
  }();
  return function;
}

// 2-D fp32 map over a row-major [rows][columns] array: box of 16 columns
// (one 64-byte swizzle row) x box_rows rows, 64-byte swizzle, zero fill
// outside the array.
inline TensorMap map_2d(const float *base, uint64_t rows, uint64_t columns, uint32_t box_rows) {
  CUtensorMap map{};
  const cuuint64_t dims[2] = {columns, rows};
  const cuuint64_t strides[1] = {columns * sizeof(float)};
  const cuuint32_t box[2] = {kTcTileK, box_rows};
  const cuuint32_t element_strides[2] = {1, 1};
  const CUresult status = encode_tiled()(
      &map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float *>(base), dims, strides, box,
      element_strides, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (status != CUDA_SUCCESS) {
    throw std::runtime_error("cuTensorMapEncodeTiled failed (" + std::to_string(status) + ")");
  }
  TensorMap out{};
  std::memcpy(&out, &map, sizeof(out));
  return out;
}

inline lr_launch_config_t rows_config(uint32_t blocks, uint32_t threads, uint32_t shared = 0) {
  return lr_launch_config_t{{blocks * threads, 1, 1}, {threads, 1, 1}, shared};
}

// Dynamic shared memory of a row kernel that stages `columns` partial sums
// per split of a deferred GEMM (none when the GEMM wrote its output).
inline uint32_t staged_bytes(const PartialTiles &partials, uint32_t columns) {
  return partials.partials != nullptr ? partials.splits * columns * 4u : 0u;
}

inline uint32_t ceil_div(uint64_t a, uint64_t b) { return static_cast<uint32_t>((a + b - 1) / b); }

// Threads per block of the one-block-per-row kernels (RoPE, residual finish):
// wide blocks when a few rows must use the whole GPU (batched decode), 256
// when there are enough rows to fill the SMs several times (prefill).
inline uint32_t row_threads(uint32_t rows) { return rows >= kSms ? 256u : kRowThreads; }

} // namespace lrrt::qwen::prefill::detail

#endif // LRRT_B200_QWEN_PREFILL_COMMON_HPP_
