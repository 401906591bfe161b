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
constexpr uint32_t kGroupColumns = kQueriesPerKvHead * kHeadSize;    // 448
constexpr uint32_t kHalfRowBytes = kGroupColumns * sizeof(float);    // 1792
constexpr uint32_t kORows = kSlotBytes / kHalfRowBytes;              // 16 o_proj rows per unit
constexpr uint32_t kOBoxColumns = kGroupColumns / 2u;                // 224: two boxes per unit
constexpr uint32_t kRingBytes = kSlots * kSlotBytes;
constexpr uint32_t kBlockThreads = lrrt::persistent_graph::kWorkerThreads;

constexpr uint32_t kMaxFusedLayers = 48;  // layers covered by the pointer table
constexpr uint32_t kLayerMatrices = 7;    // q, k, v, o, gate, up, down
static_assert(kMaxFusedLayers <= kWorkspaceMapLayers);

// Decode attention computed per block from shared memory (one KV group, all
// of its cached positions) covers contexts up to this many positions; longer
// contexts split positions over blocks. The cached rows arrive as three ring
// units of 56 positions (see resident_schedule.hpp), the current position's
// K/V and the group's queries through the qkv exchange.
constexpr uint32_t kLocalAttentionLimit = 169;
constexpr uint32_t kLocalQuery = 0;                                          // [448]
constexpr uint32_t kLocalScores = kLocalQuery + kGroupColumns;               // [7][limit]
constexpr uint32_t kLocalCurrent =                                           // K [64], V [64]
    (kLocalScores + kQueriesPerKvHead * kLocalAttentionLimit + 3u) / 4u * 4u;
constexpr uint32_t kLocalPartial = kLocalCurrent + 2u * kHeadSize;           // [448]
constexpr uint32_t kWorkFloats = kLocalPartial + kGroupColumns;
static_assert(kWorkFloats >= 1120, "top-1 reduce scratch must fit the work area");

// The ring comes first and is 1024-byte aligned: KV units are 2-D TMA boxes
// with 128-byte swizzle, whose destination must be aligned to the 1024-byte
// swizzle atom (every slot is 28 x 1024 bytes).
struct FusedShared {
  unsigned char ring[kRingBytes];
  float input[kHiddenSize];    // GEMV input vector (normalised hidden, attention output)
  float hidden[kHiddenSize];   // this block's copy of the residual stream
  float reduce[kBlockThreads]; // block reductions, softmax running state
  float work[kWorkFloats];     // local attention, LM-head and top-1 scratch
  const float *layer_weights[kMaxFusedLayers][kLayerMatrices];
  uint64_t full[kSlots];       // one mbarrier per ring slot (bytes landed)
  uint32_t sequence[kSlots];   // stream sequence number of the unit in each slot
  uint32_t unit_tag[kSlots];   // (kind, layer, unit) of that unit
  uint32_t pair_done[kSlots];  // warps done with a unit shared by four warps (mod 4)
  uint32_t rows_done[kSlots];  // warps done with an o_proj unit (mod 8)
  uint32_t flag;
  uint32_t broadcast;
};

// Dynamic shared memory a compiled launch needs for the fused path (the
// kernel rounds the start of its dynamic shared memory up to 1024 bytes).
constexpr uint32_t kFusedSharedAlign = 1024;
constexpr uint32_t kFusedSharedBytes = sizeof(FusedShared) + kFusedSharedAlign;
static_assert(kSlotBytes % kFusedSharedAlign == 0);
static_assert(kDownRowBytes <= kSlotBytes);
static_assert(kFusedSharedBytes + 4096u <= 232448u,
              "fused path plus static shared memory exceeds 227 KB");

} // namespace lrrt::qwen::stateful_graph::resident

#endif // LRRT_QWEN_RESIDENT_LAYOUT_HPP_
