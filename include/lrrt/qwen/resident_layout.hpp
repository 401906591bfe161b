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

constexpr uint32_t kMaxFusedLayers = 48;  // layers covered by the pointer table
constexpr uint32_t kLayerMatrices = 7;    // q, k, v, o, gate, up, down

struct FusedShared {
  unsigned char ring[kRingBytes];
  float input[kInputFloats];   // GEMV input vector; attention and LM-head scratch
  float reduce[kBlockThreads]; // block reductions, softmax running state
  const float *layer_weights[kMaxFusedLayers][kLayerMatrices];
  uint64_t full[kSlots];       // one mbarrier per ring slot (bytes landed)
  uint32_t sequence[kSlots];   // stream sequence number of the unit in each slot
  uint32_t unit_tag[kSlots];   // (kind, layer, unit) of that unit
  uint32_t pair_done[kSlots];  // warps done with a unit shared by four warps (mod 4)
  uint32_t flag;
  uint32_t broadcast;
};

// Dynamic shared memory a compiled launch needs for the fused path.
constexpr uint32_t kFusedSharedBytes = sizeof(FusedShared);
static_assert(kDownRowBytes <= kSlotBytes);
static_assert(kFusedSharedBytes + 4096u <= 232448u,
              "fused path plus static shared memory exceeds 227 KB");

} // namespace lrrt::qwen::stateful_graph::resident

#endif // LRRT_QWEN_RESIDENT_LAYOUT_HPP_
