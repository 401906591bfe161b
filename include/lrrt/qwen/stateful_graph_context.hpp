// Qwen2 decode workload ABI consumed by the resident megakernel
// (light-rocm-runtime executor/qwen/stateful_graph_context.hpp:11-178).
//
// Shapes, opcodes 1-13, DecodeState (32 B), TailContext (96 B) and Context
// (224 B) keep the reference byte layouts, pinned by the static_asserts below.
// One B200 addition sits in TailContext's tail padding (bytes 88-95, zero in a
// value-initialised reference struct): `workspace`, a device scratch block the
// sm_100a fast path needs for split-context attention and the LM-head top-1
// candidates. A null workspace makes the kernel use its generic task path.
#ifndef LRRT_QWEN_STATEFUL_GRAPH_CONTEXT_HPP_
#define LRRT_QWEN_STATEFUL_GRAPH_CONTEXT_HPP_

#include "lrrt/persistent_graph/abi.hpp"

#include <cstddef>
#include <cstdint>
#include <type_traits>

namespace lrrt::qwen::stateful_graph {

constexpr uint32_t kHiddenSize = 896;
constexpr uint32_t kAttentionHeads = 14;
constexpr uint32_t kKvHeads = 2;
constexpr uint32_t kHeadSize = 64;
constexpr uint32_t kRotarySize = kHeadSize / 2u;
constexpr uint32_t kRotaryHeads = kAttentionHeads + kKvHeads;
constexpr uint32_t kQuerySize = kAttentionHeads * kHeadSize;
constexpr uint32_t kKvSize = kKvHeads * kHeadSize;
constexpr uint32_t kPackedQkvSize = kQuerySize + 2u * kKvSize;
constexpr uint32_t kIntermediateSize = 4864;
constexpr uint32_t kAttentionProjectionPartitions = 8;
constexpr uint32_t kAttentionTaskPartitions = 7;
constexpr uint32_t kAttentionOutputPartitions = 8;
constexpr uint32_t kFfnProjectionPartitions = 20;
constexpr uint32_t kDownProjectionPartitions = 32;
constexpr uint32_t kMaximumLmHeadPartitions = 32;
constexpr uint32_t kAttentionTaskCount = 2u + kAttentionProjectionPartitions +
                                         kAttentionTaskPartitions +
                                         kAttentionOutputPartitions;
constexpr uint32_t kFfnTaskCount =
    2u + kFfnProjectionPartitions + kDownProjectionPartitions;
constexpr uint32_t kDecoderTaskCount = kAttentionTaskCount + kFfnTaskCount;
constexpr uint32_t kMaximumTailTaskCount = 3u + kMaximumLmHeadPartitions;
constexpr uint32_t kQueriesPerKvHead = kAttentionHeads / kKvHeads;

enum class ProfileStage : uint32_t {
  attention_norm,
  qkv_projection,
  rope_kv_cache,
  attention,
  attention_output,
  mlp_norm,
  gate_up_silu,
  down_projection,
  residual_advance,
  final_norm,
  lm_head_top1,
  top1_reduce,
  embedding_feedback,
  count,
};

constexpr uint32_t kProfileStageCount = static_cast<uint32_t>(ProfileStage::count);

struct StageProfileEntry {
  uint64_t begin_tick;
  uint64_t end_tick;
};

// Filled only by the stage-profile kernels. On B200 ticks are %globaltimer
// nanoseconds.
struct alignas(16) StageProfile {
  uint64_t previous_tick;
  uint64_t stage_ticks[kProfileStageCount];
  uint64_t stage_counts[kProfileStageCount];
  StageProfileEntry *entries;
  uint32_t entry_count;
  uint32_t reserved;
};

enum class Opcode : uint32_t {
  attention_rmsnorm_f32 = 1,
  qkv_projection_f32 = 2,
  rope_kv_cache_f32 = 3,
  grouped_query_attention_f32 = 4,
  attention_output_residual_f32 = 5,
  mlp_rmsnorm_f32 = 6,
  gate_up_silu_f32 = 7,
  down_matvec_f32 = 8,
  residual_advance = 9,
  final_rmsnorm_f32 = 10,
  lm_head_top1_partition_f32 = 11,
  top1_reduce = 12,
  embedding_feedback_f32 = 13,
};

enum class StopReason : uint32_t {
  none = 0,
  maximum_tokens = 1,
  eos_token = 2,
};

// Per-stream decode progress; the scheduler itself only sees predicate_value.
struct alignas(16) DecodeState {
  uint32_t token_position;
  uint32_t kv_length;
  uint32_t sampled_token;
  uint32_t eos_token;
  uint32_t generated_tokens;
  uint32_t maximum_tokens;
  uint32_t stop_reason;
  float sampled_logit;
};

constexpr uint32_t kWorkspaceMagic = 0x51573231u; // "QW21"
constexpr uint32_t kAttentionPartialStride = kHeadSize + 2u; // acc[64], max, sum

// Exchange words of the fused path: every value one block produces for the
// others within a decoder layer travels as one 64-bit word, tag << 32 | float
// bits, with tag = graph step + 1. A consumer polls the words it needs until
// each carries the step's tag, so the wait and the data read are the same
// loads. Arrays alternate by step parity; offsets in words:
//   qkv  [2][kPackedQkvSize]          rotated q, rotated k, v of the step
//   out  [2][kKvHeads][kHiddenSize]   o_proj split over the two KV groups
//   act  [2][kIntermediateSize]       silu(gate) * up
//   down [2][kHiddenSize]             down projection
//   attention [2][kQuerySize]         attention output of a spread step
// All words are zero when no launch is running (a launch clears the words it
// wrote before it returns; zero never matches a tag).
constexpr uint32_t kExchangeQkv = 0;
constexpr uint32_t kExchangeOut = kExchangeQkv + 2u * kPackedQkvSize;
constexpr uint32_t kExchangeAct = kExchangeOut + 2u * kKvHeads * kHiddenSize;
constexpr uint32_t kExchangeDown = kExchangeAct + 2u * kIntermediateSize;
constexpr uint32_t kExchangeAttention = kExchangeDown + 2u * kHiddenSize;
constexpr uint32_t kExchangeWords = kExchangeAttention + 2u * kQuerySize;
// Spread-attention partial state of one block: per query head of its group,
// the unnormalised weighted value sum [64], the score maximum and the sum of
// exp(score - maximum), as exchange words.
constexpr uint32_t kSpreadWords = kQueriesPerKvHead * kAttentionPartialStride; // 462

// B200 scratch for the fused resident path (no reference counterpart). One
// zero-filled allocation: this header, then
//  attention_partials: [worker_capacity][kQueriesPerKvHead][kAttentionPartialStride]
//  attention_arrivals: [kKvHeads], zero whenever no attention stage is running
//  top1_values/top1_indices: [worker_capacity + kMaximumLmHeadPartitions]
//  exchange: [kExchangeWords] 64-bit words (see above)
//  attention_words: [2][worker_capacity][kSpreadWords] exchange words, by step
//    parity and block (spread attention partial states)
//  kv_maps: [kWorkspaceMapLayers][3] CUtensorMap (128 B each: key cache,
//    value cache of each layer, dims {kKvSize, cache_capacity}, box 32
//    columns x 56 rows, 128-byte swizzle, for the fused path's KV ring
//    units; o_proj weight, dims {kHiddenSize, kHiddenSize}, box 224 columns x
//    16 rows, no swizzle, for its OUT units)
constexpr uint32_t kWorkspaceMapLayers = 48;
constexpr uint32_t kWorkspaceMapsPerLayer = 3; // key cache, value cache, o_proj
constexpr uint32_t kTensorMapBytes = 128;
struct alignas(16) Workspace {
  uint32_t magic;
  uint32_t worker_capacity;
  uint32_t reserved[2];
  float *attention_partials;
  uint32_t *attention_arrivals;
  float *top1_values;
  uint32_t *top1_indices;
  uint64_t *exchange;
  const void *kv_maps;
  float *logits; // optional [vocab_size]: every LM-head row of the last step (test capture)
  uint64_t *attention_words;
};

// Bytes of one allocation holding a Workspace header followed by its arrays.
constexpr size_t workspace_bytes(uint32_t worker_capacity) {
  return 256u +
         size_t{worker_capacity} * kQueriesPerKvHead * kAttentionPartialStride *
             sizeof(float) +
         256u + 2u * (size_t{worker_capacity} + kMaximumLmHeadPartitions) *
                    sizeof(uint32_t) +
         256u + size_t{kExchangeWords} * sizeof(uint64_t) + 256u +
         2u * size_t{worker_capacity} * kSpreadWords * sizeof(uint64_t) + 256u +
         size_t{kWorkspaceMapLayers} * kWorkspaceMapsPerLayer * kTensorMapBytes + 256u;
}

// Model tail shared by every layer Context.
struct alignas(16) TailContext {
  const float *final_norm_weight;
  const float *lm_head_weight;
  const float *token_embeddings;
  float *final_normalized;
  float *partial_max_values;
  uint32_t *partial_max_indices;
  DecodeState *decode_state;
  uint32_t *output_tokens;
  uint32_t vocab_size;
  uint32_t partition_count;
  uint32_t embedding_count;
  uint32_t reserved;
  StageProfile *stage_profile;
  Workspace *workspace; // B200 addition in the reference's tail padding
};

// One decoder layer: weights (row-major [out][in]), shared activation scratch,
// this layer's KV-cache slices ([cache_capacity][kKvSize], token-major).
struct alignas(16) Context {
  float *hidden;
  const float *attention_norm_weight;
  const float *q_weight;
  const float *k_weight;
  const float *v_weight;
  const float *q_bias;
  const float *k_bias;
  const float *v_bias;
  const float *out_weight;
  const float *mlp_norm_weight;
  const float *gate_weight;
  const float *up_weight;
  const float *down_weight;
  float *attention_normalized;
  float *query;
  float *key;
  float *value;
  const float *rope_cos;
  const float *rope_sin;
  float *key_cache;
  float *value_cache;
  float *mlp_normalized;
  float *activated;
  float *projected;
  TailContext *tail;
  uint32_t hidden_size;
  uint32_t query_size;
  uint32_t kv_size;
  uint32_t intermediate_size;
  uint32_t cache_capacity;
  uint32_t layer_count; // the opaque context is an array of this many
};

static_assert(std::is_standard_layout_v<Context>);
static_assert(std::is_standard_layout_v<TailContext>);
static_assert(std::is_standard_layout_v<StageProfile>);
static_assert(std::is_standard_layout_v<StageProfileEntry>);
static_assert(std::is_standard_layout_v<DecodeState>);
static_assert(std::is_standard_layout_v<Workspace>);
static_assert(sizeof(Context) == 224);
static_assert(sizeof(TailContext) == 96);
static_assert(offsetof(TailContext, stage_profile) == 80);
static_assert(offsetof(TailContext, workspace) == 88);
static_assert(sizeof(StageProfile) == 240);
static_assert(sizeof(StageProfileEntry) == 16);
static_assert(sizeof(DecodeState) == 32);
static_assert(sizeof(Workspace) == 80);
static_assert(kAttentionTaskCount <= lrrt::persistent_graph::kMaximumTasks);
static_assert(kFfnTaskCount <= lrrt::persistent_graph::kMaximumTasks);
static_assert(kMaximumTailTaskCount <= lrrt::persistent_graph::kMaximumTasks);

} // namespace lrrt::qwen::stateful_graph

#endif // LRRT_QWEN_STATEFUL_GRAPH_CONTEXT_HPP_
