// Host checks of the fused path's work partition and weight-stream order
// (include/lrrt/qwen/resident_schedule.hpp): every unit of every matrix has
// exactly one owner, gate/up balancing keeps per-block layer bytes close to the
// mean, even_owner inverts even_range, and the producer's cyclic stream visits
// exactly the units the compiled stages consume, in the same order (also when
// each ring slot advances its own stream position by the ring depth), and
// spread attention's position slices tile each KV group's cache.
#include "lrrt/qwen/resident_schedule.hpp"

#include <algorithm>
#include <cstdio>
#include <vector>

namespace r = lrrt::qwen::stateful_graph::resident;

static int failures = 0;

static void expect(bool condition, const char *what, uint32_t a = 0, uint32_t b = 0,
                   uint32_t c = 0) {
  if (!condition) {
    std::fprintf(stderr, "FAILED: %s (%u %u %u)\n", what, a, b, c);
    ++failures;
  }
}

static uint32_t units_of(uint32_t kind, uint32_t vocab) {
  switch (kind) {
  case r::kQkv: return r::kQkvUnits;
  case r::kKv: return r::kKvUnits;
  case r::kOut: return r::kOUnits;
  case r::kGateUp: return r::kGuUnits;
  case r::kDown: return r::kDownUnits;
  default: return r::lm_units_for(vocab);
  }
}

// Units in consumption order for `tokens` decode steps starting at `program`.
static std::vector<uint32_t> consumer_tags(const r::UnitRanges &ranges, uint32_t layers,
                                           uint32_t program, uint32_t tokens) {
  std::vector<uint32_t> tags;
  auto visit = [&](uint32_t kind, uint32_t layer) {
    for (uint32_t u = ranges.of[kind].begin; u < ranges.of[kind].end; ++u) {
      tags.push_back(r::make_tag(kind, layer, u));
    }
  };
  bool first = true;
  for (uint32_t t = 0; t < tokens; ++t) {
    for (uint32_t l = 0; l < layers; ++l) {
      if (!(first && program == 2)) {
        if (!(first && program == 1 && l == 0)) {
          visit(r::kQkv, l);
          visit(r::kKv, l);
          visit(r::kOut, l);
        }
        visit(r::kGateUp, l);
        visit(r::kDown, l);
      }
    }
    visit(r::kLmHead, 0);
    first = false;
  }
  return tags;
}

// Spread attention: for every worker count and context length the mode
// picks, each group's slices tile the cached rows [0, positions - 1) in block
// order, exactly one block takes the current position, and no slice needs
// more than the three KV units of a layer.
static void check_spread_slices() {
  for (uint32_t workers : {2u, 3u, 7u, 64u, 147u, 148u, 256u}) {
    const uint32_t limit = r::kKvUnits * r::kKvUnitPositions * (workers / 2u);
    expect(r::attention_mode(r::kLocalAttentionLimit, workers) == r::AttentionMode::local,
           "local up to the limit", workers);
    for (uint32_t positions = r::kLocalAttentionLimit + 1u; positions <= limit + 2u;
         positions += positions < 400u ? 1u : 97u) {
      const r::AttentionMode mode = r::attention_mode(positions, workers);
      expect(mode == (positions <= limit ? r::AttentionMode::spread : r::AttentionMode::split),
             "spread up to three units per block", workers, positions);
      if (mode != r::AttentionMode::spread) {
        continue;
      }
      for (uint32_t group = 0; group < 2; ++group) {
        const uint32_t size = r::group_size(group, workers);
        uint32_t next = 0, owners = 0;
        for (uint32_t rank = 0; rank < size; ++rank) {
          const r::SpreadSlice slice = r::spread_slice(positions, rank, size);
          expect(slice.first == next || slice.rows == 0, "slices contiguous", workers,
                 positions, rank);
          expect(slice.rows <= r::kKvUnits * r::kKvUnitPositions, "three units", workers,
                 positions, rank);
          next = slice.rows != 0 ? slice.first + slice.rows : next;
          owners += slice.current ? 1u : 0u;
          expect(!slice.current || slice.first + slice.rows == positions - 1u,
                 "current position ends the slice", workers, positions, rank);
        }
        expect(next == positions - 1u, "slices cover the cached rows", workers, positions);
        expect(owners == 1u, "one block takes the current position", workers, positions);
      }
    }
  }
  for (uint32_t workers = 2; workers <= 300; ++workers) {
    for (uint32_t worker = 0; worker < workers; ++worker) {
      const uint32_t group = r::attention_group(worker, workers);
      const uint32_t rank = r::group_rank(worker, workers);
      expect(rank < r::group_size(group, workers), "rank inside its group", workers, worker);
      expect(worker == (group == 0 ? rank : r::attention_split(workers) + rank),
             "rank inverts", workers, worker);
    }
  }
}

int main() {
  check_spread_slices();
  const uint32_t worker_counts[] = {1, 2, 3, 7, 64, 147, 148, 256};
  const uint32_t vocabs[] = {1, 7, 64, 4096, 151936};
  for (uint32_t workers : worker_counts) {
    for (uint32_t vocab : vocabs) {
      for (uint32_t kind = r::kQkv; kind <= r::kLmHead; ++kind) {
        const uint32_t units = units_of(kind, vocab);
        if (kind == r::kKv) {
          // Not partitioned: every block streams its own KV group's rows.
          for (uint32_t w = 0; w < workers; ++w) {
            const r::UnitRange range = r::unit_ranges(w, workers, vocab).of[kind];
            expect(range.begin == 0 && range.end == r::kKvUnits, "KV units per block", w);
          }
          continue;
        }
        std::vector<uint32_t> owners(units, 0);
        uint32_t next = 0;
        for (uint32_t w = 0; w < workers; ++w) {
          const r::UnitRange range = r::unit_ranges(w, workers, vocab).of[kind];
          expect(range.begin == next && range.begin <= range.end, "contiguous ranges",
                 workers, kind, w);
          for (uint32_t u = range.begin; u < range.end && u < units; ++u) {
            ++owners[u];
            if (kind != r::kGateUp && kind != r::kOut) {
              expect(r::even_owner(u, units, workers) == w, "even_owner inverts",
                     workers, kind, u);
            }
          }
          next = range.end;
        }
        expect(next == units, "ranges cover all units", workers, kind, next);
        if (kind == r::kOut && workers >= 2) {
          for (uint32_t w = 0; w < workers; ++w) {
            const r::UnitRange range = r::unit_ranges(w, workers, vocab).of[kind];
            const uint32_t group = r::attention_group(w, workers);
            expect(range.begin == range.end ||
                       (range.begin / r::kOGroupUnits == group &&
                        (range.end - 1u) / r::kOGroupUnits == group),
                   "out units in the block's attention group", workers, w);
          }
        }
        expect(std::all_of(owners.begin(), owners.end(), [](uint32_t n) { return n == 1; }),
               "each unit owned once", workers, kind);
      }
    }
    // Per-block decoder bytes stay within two slots of the mean.
    const double mean =
        (double(r::kQkvUnits + r::kGuUnits) * r::kSlotBytes +
         double(r::kOUnits) * r::kOUnitBytes + double(r::kDownUnits) * r::kDownRowBytes) /
        workers;
    for (uint32_t w = 0; w < workers; ++w) {
      const r::UnitRanges ranges = r::unit_ranges(w, workers, 4096);
      const double bytes = double(r::fixed_layer_bytes(w, workers)) +
                           double(ranges.of[r::kGateUp].end - ranges.of[r::kGateUp].begin) *
                               r::kSlotBytes;
      expect(bytes <= mean + 2.0 * r::kSlotBytes || workers > 1216, "balanced layer bytes",
             workers, w);
    }
  }
  // Producer stream == consumer order, three decode steps, every start program.
  for (uint32_t workers : {1u, 5u, 148u}) {
    for (uint32_t layers : {1u, 2u, 24u}) {
      for (uint32_t vocab : {7u, 4096u, 151936u}) {
        for (uint32_t program = 0; program < 3; ++program) {
          for (uint32_t w = 0; w < workers; w += std::max(1u, workers / 7u)) {
            const r::UnitRanges ranges = r::unit_ranges(w, workers, vocab);
            const std::vector<uint32_t> want = consumer_tags(ranges, layers, program, 3);
            if (want.empty()) {
              expect(r::units_per_cycle(ranges, layers) == 0, "empty stream");
              continue;
            }
            r::StreamCursor c = r::start_cursor(ranges, layers, program, 0);
            const r::StreamMap map = r::make_stream_map(ranges, layers, program, 0);
            // Ring slots advance their position by the ring depth.
            const uint32_t depth = r::kSlots;
            std::vector<r::StreamPosition> slots;
            for (uint32_t k = 0; k < depth; ++k) {
              slots.push_back(r::stream_position(map, k));
            }
            for (size_t i = 0; i < want.size(); ++i) {
              const uint32_t got = r::make_tag(c.kind, c.layer, c.unit);
              const r::StreamCursor random = r::stream_unit(map, static_cast<uint32_t>(i));
              r::StreamPosition &slot = slots[i % depth];
              const r::StreamCursor ring = r::position_cursor(map, slot);
              if (got != want[i] ||
                  r::make_tag(random.kind, random.layer, random.unit) != want[i] ||
                  r::make_tag(ring.kind, ring.layer, ring.unit) != want[i]) {
                expect(false, "stream order", workers, w, static_cast<uint32_t>(i));
                break;
              }
              const r::StreamPosition direct = r::stream_position(map, static_cast<uint32_t>(i));
              expect(direct.cycle == slot.cycle && direct.layer == slot.layer &&
                         direct.index == slot.index,
                     "stream position cycle", workers, w, static_cast<uint32_t>(i));
              r::advance_cursor(ranges, layers, c);
              r::advance_position(map, slot, depth);
            }
          }
        }
      }
    }
  }
  if (failures == 0) {
    std::printf("resident schedule checks: ok\n");
  }
  return failures == 0 ? 0 : 1;
}
