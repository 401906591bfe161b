// Shared-memory layout of the fused resident decode path, shared by the
// sm_100a kernel (which carves its dynamic shared memory with it) and the host
// driver (which sizes the launch's dynamic shared memory from it).
#ifndef LRRT_QWEN_RESIDENT_LAYOUT_HPP_
#define LRRT_QWEN_RESIDENT_LAYOUT_HPP_

#include "lrrt/persistent_graph/abi.hpp"
#include "lrrt/qwen/stateful_graph_context.hpp"

#include <cstdint>

namespace lrrt::qwen::stateful_graph::resident {

constexpr uint32_t kSlots = 7;                                       // ring depth
constexpr uint32_t kSlotRows = 8;                                    // rows of 896 per slot
constexpr uint32_t kRowBytes = kHiddenSize * sizeof(float);          // 3584
constexpr uint32_t kSlotBytes = kSlotRows * kRowBytes;               // 28672
constexpr uint32_t kDownRowBytes = kIntermediateSize * sizeof(float); // 19456
constexpr uint32_t kRingBytes = kSlots * kSlotBytes;
constexpr uint32_t kInputFloats = kIntermediateSize; // largest GEMV input vector
constexpr uint32_t kBlockThreads = lrrt::persistent_graph::kWorkerThreads;

struct FusedShared {
  unsigned char ring[kRingBytes];
  float input[kInputFloats];   // GEMV input vector; attention scratch
  float hidden[kHiddenSize];
  float results[2][kSlotRows]; // per-slot row results, double-buffered
  float reduce[kBlockThreads];
  uint64_t full[kSlots];       // one mbarrier per ring slot
  uint32_t tags[kSlots];       // (kind, layer, unit) of the unit in each slot
  uint32_t flag;
  uint32_t broadcast;
};

// Dynamic shared memory a compiled launch needs for the fused path.
constexpr uint32_t kFusedSharedBytes = sizeof(FusedShared);
static_assert(kDownRowBytes <= kSlotBytes);
static_assert(kFusedSharedBytes + 2048u <= 232448u,
              "fused path plus static shared memory exceeds 227 KB");

} // namespace lrrt::qwen::stateful_graph::resident

#endif // LRRT_QWEN_RESIDENT_LAYOUT_HPP_
