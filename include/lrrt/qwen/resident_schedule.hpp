// Work partition and weight-stream order of the fused resident decode path,
// shared by the sm_100a kernel and host-side tests.
//
// Every block (worker w of W) owns a contiguous range of "units" of each
// weight matrix; a unit is what one shared-memory ring slot holds:
//   QKV   144 units: 8 rows = rows f..f+3 of one head and their rotary
//                    partners f+32..f+35 (Q heads 0-13, K heads, then V)
//   KV      3 units per block (not partitioned: every block reads its own
//                    KV group): cached K and V rows of positions 56j..56j+55,
//                    loaded only for the positions the step attends to
//   OUT   112 units: 16 consecutive o_proj rows restricted to the 448 input
//                    columns of one KV group (units 0-55 group 0, 56-111
//                    group 1), copied as two 224-column 2-D tensor boxes;
//                    o_proj is split along its input over the groups
//   GU   1216 units: gate rows 4u..4u+3 followed by up rows 4u..4u+3
//   DOWN  896 units: one 4864-float down_proj row
//   LM   ceil(V/8) units: 8 LM-head rows (the last may be shorter)
// QKV, DOWN and LM units are split evenly. OUT units follow the attention
// split: the first ceil(W/2) blocks compute the attention of KV group 0 and
// own group 0's OUT units (split evenly among them), the others group 1's
// (one block owns both when W == 1). Gate/up units are assigned so that each
// block's bytes per layer (all four matrices) are balanced.
//
// A block's weight stream is the cyclic sequence
//   [QKV(l), KV(l), OUT(l), GU(l), DOWN(l)] for l = 0..L-1, then LM(0), repeat,
// restricted to its own units. The producer issues it in this order; the
// consumer walks the compiled stages, which visit the same units in the same
// order, and checks each slot's tag.
#ifndef LRRT_QWEN_RESIDENT_SCHEDULE_HPP_
#define LRRT_QWEN_RESIDENT_SCHEDULE_HPP_

#include "lrrt/persistent_graph/abi.hpp"
#include "lrrt/qwen/resident_layout.hpp"
#include "lrrt/qwen/stateful_graph_context.hpp"

#include <cstdint>

namespace lrrt::qwen::stateful_graph::resident {

// Kinds in stream order within a layer (the cursor walks them in sequence).
enum StreamKind : uint32_t { kNoKind = 0, kQkv = 1, kKv = 2, kOut = 3, kGateUp = 4,
                             kDown = 5, kLmHead = 6 };
constexpr uint32_t kKinds = 7;
constexpr uint32_t kKvUnits = 3;                               // per block and layer
constexpr uint32_t kKvUnitPositions = kSlotBytes / (2u * kKvSize / kKvHeads * 4u); // 56
static_assert(kKvUnits * kKvUnitPositions + 1u >= kLocalAttentionLimit,
              "KV units cover every cached position of a local-attention step");

constexpr uint32_t kQkvUnits = kPackedQkvSize / kSlotRows;     // 144
constexpr uint32_t kQUnits = kQuerySize / kSlotRows;           // 112
constexpr uint32_t kKUnits = kKvSize / kSlotRows;              // 16
constexpr uint32_t kOGroupUnits = kHiddenSize / kORows;        // 56 per KV group
constexpr uint32_t kOUnits = kKvHeads * kOGroupUnits;          // 112
constexpr uint32_t kOUnitBytes = kORows * kHalfRowBytes;       // 28672
static_assert(kHiddenSize % kORows == 0 && kOUnitBytes <= kSlotBytes);
constexpr uint32_t kGuRowsPerUnit = kSlotRows / 2u;            // 4
constexpr uint32_t kGuUnits = kIntermediateSize / kGuRowsPerUnit; // 1216
constexpr uint32_t kDownUnits = kHiddenSize;                   // 896
static_assert(kPackedQkvSize % kSlotRows == 0);
static_assert(kIntermediateSize % kGuRowsPerUnit == 0);

struct UnitRange {
  uint32_t begin, end;
};

LRRT_HOST_DEVICE constexpr uint32_t lm_units_for(uint32_t vocab) {
  return (vocab + kSlotRows - 1u) / kSlotRows;
}

// [w*U/W, (w+1)*U/W): contiguous, disjoint, covering [0, U).
LRRT_HOST_DEVICE inline UnitRange even_range(uint32_t units, uint32_t worker,
                                             uint32_t workers) {
  return {static_cast<uint32_t>(uint64_t{units} * worker / workers),
          static_cast<uint32_t>(uint64_t{units} * (worker + 1u) / workers)};
}

// Block holding unit `unit` of an even_range split (its inverse).
LRRT_HOST_DEVICE inline uint32_t even_owner(uint32_t unit, uint32_t units,
                                            uint32_t workers) {
  return static_cast<uint32_t>((uint64_t{unit + 1u} * workers - 1u) / units);
}

// Blocks [0, attention_split(W)) attend KV group 0, the rest group 1.
LRRT_HOST_DEVICE constexpr uint32_t attention_split(uint32_t workers) {
  return (workers + 1u) / 2u;
}

LRRT_HOST_DEVICE constexpr uint32_t attention_group(uint32_t worker, uint32_t workers) {
  return worker < attention_split(workers) ? 0u : 1u;
}

// Blocks of a KV group, and a block's index within its group.
LRRT_HOST_DEVICE constexpr uint32_t group_size(uint32_t group, uint32_t workers) {
  return group == 0u ? attention_split(workers) : workers - attention_split(workers);
}

LRRT_HOST_DEVICE constexpr uint32_t group_rank(uint32_t worker, uint32_t workers) {
  return worker < attention_split(workers) ? worker : worker - attention_split(workers);
}

// How a decode step with `positions` KV positions (cached rows + the current
// one) computes attention:
//   local   every block attends its KV group over all positions by itself
//           (the cached rows as its three KV units);
//   spread  the blocks of a group split the positions into contiguous slices
//           of at most three KV units, publish per-head partial softmax
//           states through the exchange, and a few warps per group merge
//           them into the attention output;
//   split   longer contexts: items over all blocks between grid barriers.
enum class AttentionMode : uint32_t { local = 0, spread = 1, split = 2 };

LRRT_HOST_DEVICE constexpr AttentionMode attention_mode(uint32_t positions, uint32_t workers) {
  return positions <= kLocalAttentionLimit ? AttentionMode::local
         : positions <= kKvUnits * kKvUnitPositions * (workers / 2u) ? AttentionMode::spread
                                                                     : AttentionMode::split;
}

// Spread attention: the slice of block `rank` of a group of `size` blocks is
// positions [first, first + rows) read from the cache, plus the current
// position (index positions - 1, which is not yet in the cache when the KV
// units are issued) when `current`. rows <= kKvUnits * kKvUnitPositions
// whenever attention_mode() is spread.
struct SpreadSlice {
  uint32_t first;
  uint32_t rows;
  bool current;
};

LRRT_HOST_DEVICE constexpr SpreadSlice spread_slice(uint32_t positions, uint32_t rank,
                                                    uint32_t size) {
  const uint32_t per = (positions + size - 1u) / size;
  const uint32_t first = rank * per < positions ? rank * per : positions;
  const uint32_t last = first + per < positions ? first + per : positions;
  const bool current = last == positions && first < positions;
  return {first, last - first - (current ? 1u : 0u), current};
}

LRRT_HOST_DEVICE inline UnitRange out_range(uint32_t worker, uint32_t workers) {
  if (workers == 1u) {
    return {0, kOUnits};
  }
  const uint32_t split = attention_split(workers);
  if (worker < split) {
    return even_range(kOGroupUnits, worker, split);
  }
  const UnitRange r = even_range(kOGroupUnits, worker - split, workers - split);
  return {kOGroupUnits + r.begin, kOGroupUnits + r.end};
}

LRRT_HOST_DEVICE inline uint64_t fixed_layer_bytes(uint32_t worker, uint32_t workers) {
  const UnitRange q = even_range(kQkvUnits, worker, workers);
  const UnitRange o = out_range(worker, workers);
  const UnitRange d = even_range(kDownUnits, worker, workers);
  return uint64_t{q.end - q.begin} * kSlotBytes + uint64_t{o.end - o.begin} * kOUnitBytes +
         uint64_t{d.end - d.begin} * kDownRowBytes;
}

// Gate/up split by cumulative rounding of each block's remaining byte budget
// (total layer bytes / W minus its QKV + OUT + DOWN bytes). Non-decreasing
// boundaries, first block starts at 0, last ends at kGuUnits.
LRRT_HOST_DEVICE inline uint32_t gate_up_boundary(uint32_t worker, uint32_t workers,
                                                  uint64_t fixed_prefix) {
  if (worker + 1u >= workers) {
    return kGuUnits;
  }
  const uint64_t total = uint64_t{kQkvUnits + kGuUnits} * kSlotBytes +
                         uint64_t{kOUnits} * kOUnitBytes +
                         uint64_t{kDownUnits} * kDownRowBytes;
  const int64_t want = static_cast<int64_t>(total * (worker + 1u) / workers) -
                       static_cast<int64_t>(fixed_prefix);
  const int64_t units = want <= 0 ? 0 : (want + kSlotBytes / 2) / kSlotBytes;
  return units > static_cast<int64_t>(kGuUnits) ? kGuUnits : static_cast<uint32_t>(units);
}

LRRT_HOST_DEVICE inline UnitRange balanced_gate_up(uint32_t worker, uint32_t workers) {
  uint64_t fixed_prefix = 0;
  uint32_t previous = 0, current = 0;
  for (uint32_t w = 0; w <= worker; ++w) {
    fixed_prefix += fixed_layer_bytes(w, workers);
    uint32_t boundary = gate_up_boundary(w, workers, fixed_prefix);
    boundary = boundary < current ? current : boundary; // keep boundaries monotone
    previous = current;
    current = boundary;
  }
  return {previous, current};
}

struct UnitRanges {
  UnitRange of[kKinds];
};

LRRT_HOST_DEVICE inline UnitRanges unit_ranges(uint32_t worker, uint32_t workers,
                                               uint32_t vocab) {
  UnitRanges r{};
  r.of[kNoKind] = {0, 0};
  r.of[kQkv] = even_range(kQkvUnits, worker, workers);
  r.of[kKv] = {0, kKvUnits};
  r.of[kOut] = out_range(worker, workers);
  r.of[kGateUp] = balanced_gate_up(worker, workers);
  r.of[kDown] = even_range(kDownUnits, worker, workers);
  r.of[kLmHead] = even_range(lm_units_for(vocab), worker, workers);
  return r;
}

// Tag of a unit in a ring slot: kind, layer (LM head uses layer 0), unit.
LRRT_HOST_DEVICE constexpr uint32_t make_tag(uint32_t kind, uint32_t layer, uint32_t unit) {
  return (kind << 28) | ((layer & 0xffu) << 20) | (unit & 0xfffffu);
}

struct StreamCursor {
  uint32_t layer;
  uint32_t kind;
  uint32_t unit;
};

// Moves the cursor to the first existing unit at or after it, wrapping
// layers and decode steps. `layers` >= 1; at least one unit must exist per
// cycle (the caller checks) or the cursor stops after a bounded search.
LRRT_HOST_DEVICE inline void normalize_cursor(const UnitRanges &r, uint32_t layers,
                                              StreamCursor &c) {
  for (uint32_t guard = 0; guard < 8u * (layers + 2u); ++guard) {
    if (c.unit < r.of[c.kind].end) {
      return;
    }
    if (c.kind == kLmHead) {
      c.kind = kQkv;
      c.layer = 0;
    } else if (c.kind == kDown) {
      if (c.layer + 1u >= layers) {
        c.kind = kLmHead;
        c.layer = 0;
      } else {
        c.kind = kQkv;
        ++c.layer;
      }
    } else {
      ++c.kind;
    }
    c.unit = r.of[c.kind].begin;
  }
}

LRRT_HOST_DEVICE inline void advance_cursor(const UnitRanges &r, uint32_t layers,
                                            StreamCursor &c) {
  ++c.unit;
  normalize_cursor(r, layers, c);
}

// Cursor at the start of the Program the launch begins with: program 0 at the
// QKV units of layer `layer`, program 1 at its gate/up units, program 2 at the
// LM head.
LRRT_HOST_DEVICE inline StreamCursor start_cursor(const UnitRanges &r, uint32_t layers,
                                                  uint32_t program, uint32_t layer) {
  StreamCursor c{program == 2 ? 0u : layer,
                 program == 0 ? kQkv : (program == 1 ? kGateUp : kLmHead), 0};
  c.unit = r.of[c.kind].begin;
  normalize_cursor(r, layers, c);
  return c;
}

LRRT_HOST_DEVICE inline uint32_t units_per_cycle(const UnitRanges &r, uint32_t layers) {
  uint32_t units = r.of[kLmHead].end - r.of[kLmHead].begin;
  for (uint32_t k = kQkv; k <= kDown; ++k) {
    units += layers * (r.of[k].end - r.of[k].begin);
  }
  return units;
}

// Random access into the stream: the unit at sequence number `n` of a launch
// whose stream starts at cycle offset `start` (see stream_start_offset).
struct StreamMap {
  uint32_t layers;
  uint32_t per_layer;  // this block's QKV + OUT + GU + DOWN units per layer
  uint32_t cycle;      // layers * per_layer + LM units
  uint32_t start;      // cycle offset of sequence number 0
  uint32_t first[kKinds];
  uint32_t count[kKinds];
};

LRRT_HOST_DEVICE inline StreamMap make_stream_map(const UnitRanges &r, uint32_t layers,
                                                  uint32_t program, uint32_t layer) {
  StreamMap m{};
  m.layers = layers;
  for (uint32_t k = 0; k < kKinds; ++k) {
    m.first[k] = r.of[k].begin;
    m.count[k] = r.of[k].end - r.of[k].begin;
  }
  m.per_layer =
      m.count[kQkv] + m.count[kKv] + m.count[kOut] + m.count[kGateUp] + m.count[kDown];
  m.cycle = layers * m.per_layer + m.count[kLmHead];
  // program 0 starts at the QKV units of `layer`, program 1 at its gate/up
  // units, program 2 at the LM head.
  const uint32_t layer_offset = layer * m.per_layer;
  m.start = program == 0   ? layer_offset
            : program == 1 ? layer_offset + m.count[kQkv] + m.count[kKv] + m.count[kOut]
                           : layers * m.per_layer;
  return m;
}

LRRT_HOST_DEVICE inline StreamCursor stream_unit(const StreamMap &m, uint32_t n) {
  uint32_t at = static_cast<uint32_t>((uint64_t{m.start} + n) % m.cycle);
  const uint32_t decoder = m.layers * m.per_layer;
  if (at >= decoder) {
    return {0, kLmHead, m.first[kLmHead] + (at - decoder)};
  }
  const uint32_t layer = at / m.per_layer;
  at -= layer * m.per_layer;
  uint32_t kind = kQkv;
  while (at >= m.count[kind]) {
    at -= m.count[kind];
    ++kind;
  }
  return {layer, kind, m.first[kind] + at};
}

// Incremental form of stream_unit for the lane that refills a ring slot:
// (layer, index) with layer == layers meaning the LM-head region, and the
// number of whole cycles (decode tokens) since the launch's stream start;
// advancing by a ring's depth costs a compare and a subtraction per region
// crossed instead of a division.
struct StreamPosition {
  uint32_t layer;
  uint32_t index;
  uint32_t cycle;
};

LRRT_HOST_DEVICE inline uint32_t region_units(const StreamMap &m, uint32_t layer) {
  return layer < m.layers ? m.per_layer : m.count[kLmHead];
}

LRRT_HOST_DEVICE inline StreamPosition stream_position(const StreamMap &m, uint32_t n) {
  const uint64_t absolute = uint64_t{m.start} + n;
  const uint32_t at = static_cast<uint32_t>(absolute % m.cycle);
  const uint32_t cycle = static_cast<uint32_t>(absolute / m.cycle);
  const uint32_t decoder = m.layers * m.per_layer;
  if (at >= decoder) {
    return {m.layers, at - decoder, cycle};
  }
  return {at / m.per_layer, at % m.per_layer, cycle};
}

// Moves `p` forward by `by` units (the stream must not be empty).
LRRT_HOST_DEVICE inline void advance_position(const StreamMap &m, StreamPosition &p,
                                              uint32_t by) {
  p.index += by;
  // Each pass leaves a region; m.layers + 1 regions form a cycle, and `by`
  // is smaller than a cycle for every caller.
  for (uint32_t guard = 0; guard < 2u * (m.layers + 1u) + by; ++guard) {
    const uint32_t size = region_units(m, p.layer);
    if (p.index < size) {
      return;
    }
    p.index -= size;
    if (p.layer >= m.layers) {
      p.layer = 0;
      ++p.cycle;
    } else {
      ++p.layer;
    }
  }
}

LRRT_HOST_DEVICE inline StreamCursor position_cursor(const StreamMap &m, StreamPosition p) {
  if (p.layer >= m.layers) {
    return {0, kLmHead, m.first[kLmHead] + p.index};
  }
  uint32_t at = p.index;
  uint32_t kind = kQkv;
  while (kind < kDown && at >= m.count[kind]) {
    at -= m.count[kind];
    ++kind;
  }
  return {p.layer, kind, m.first[kind] + at};
}

} // namespace lrrt::qwen::stateful_graph::resident

#endif // LRRT_QWEN_RESIDENT_SCHEDULE_HPP_
