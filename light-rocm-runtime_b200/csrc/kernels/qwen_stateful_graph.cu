// Qwen2 FP32 decode megakernel for sm_100a, driven by the Persistent Graph
// schedulers. Exports the seven kernels of the reference's
// benchmarks/qwen_stateful_graph_kernel.cpp:921-1083 under the same names and
// parameter blocks (ResidentArgs / HostStepArgs), so a caller of that module
// loads this cubin with lr_module_load_hsaco and runs it unchanged.
//
// Two execution paths share the task semantics of the reference workload
// (valid_qwen_task :47-77, valid_qwen_contexts :79-120, execute_task :661-761):
//
// * Generic path (any valid task table; the dynamic scheduler, the host-step
//   and matched-step kernels, and any non-canonical Program table): each task
//   runs as in the reference, one warp per output row, reading operands from
//   global memory.
//
// * Fused path (compiled kernel, canonical Qwen table, workspace bound): the
//   decode step is a weight stream plus a chain of small exchanges.
//   - Each block owns a balanced share of every weight matrix (QKV, o_proj,
//     gate/up, down, LM head) and keeps a ring of 7 x 28 KB shared-memory
//     slots filled by TMA (1-D bulk copies for weights, 2-D tensor copies for
//     its KV group's cached rows; each copy has one destination). A consumer refills the slot
//     it releases, so the stream runs ahead across stages and layers.
//   - Values one block produces for the others inside a layer (q/k/v, the
//     o_proj rows, silu(gate) * up, the down rows) travel as 64-bit exchange
//     words carrying the step as a tag; consumers poll the words they need,
//     so the wait and the data read are one round trip, and Programs 0 and 1
//     run without grid barriers. Every block keeps the residual stream in
//     shared memory and adds the exchanged o_proj and down rows itself.
//   - RMSNorm is recomputed by every block; RoPE and the KV-cache append run
//     in the QKV epilogue. Each block computes the attention of one KV group
//     (seven query heads) over the cached rows in its ring, and o_proj is
//     split along its input over the two groups. Contexts longer than the
//     ring holds use split-position attention between two grid barriers.
//   - The tail (LM-head top-1 partitions, reduce, embedding feedback) keeps
//     its grid barriers.
#include "lrrt/persistent_graph/compiled_scheduler.cuh"
#include "lrrt/persistent_graph/device_scheduler.cuh"
#include "lrrt/qwen/resident_layout.hpp"
#include "lrrt/qwen/resident_schedule.hpp"
#include "lrrt/qwen/stateful_graph_context.hpp"

#include <cstdint>

namespace sg = lrrt::persistent_graph;
namespace dev = lrrt::persistent_graph::device;
namespace qd = lrrt::qwen::stateful_graph;

namespace {

constexpr uint32_t kThreads = sg::kWorkerThreads;
constexpr uint32_t kWarps = kThreads / 32u;
constexpr uint32_t kFullMask = 0xffffffffu;

// ---------------------------------------------------------------- helpers --

__device__ __forceinline__ float warp_sum(float value) {
  for (uint32_t offset = 16; offset != 0; offset >>= 1u) {
    value += __shfl_down_sync(kFullMask, value, offset);
  }
  return value; // valid in lane 0
}

__device__ __forceinline__ float warp_all_sum(float value) {
  for (uint32_t offset = 16; offset != 0; offset >>= 1u) {
    value += __shfl_xor_sync(kFullMask, value, offset);
  }
  return value;
}

__device__ __forceinline__ float warp_all_max(float value) {
  for (uint32_t offset = 16; offset != 0; offset >>= 1u) {
    value = fmaxf(value, __shfl_xor_sync(kFullMask, value, offset));
  }
  return value;
}

// Reference better_top1 (:225-229): larger value, ties to the lower index.
__device__ __forceinline__ bool better_top1(float value, uint32_t index,
                                            float best_value, uint32_t best_index) {
  return value > best_value || (value == best_value && index < best_index);
}

__device__ __forceinline__ float silu_times(float gate, float up) {
  return (gate / (1.0f + expf(-gate))) * up;
}

__device__ __forceinline__ qd::Context *layer_context(void *opaque, const sg::State *state) {
  auto *contexts = static_cast<qd::Context *>(opaque);
  const uint32_t step = dev::load_relaxed(&state->step);
  return &contexts[step % contexts[0].layer_count];
}

__device__ __forceinline__ uint32_t decode_field(const uint32_t *field) {
  return dev::load_cg(field);
}

__device__ __forceinline__ qd::Opcode opcode_of(const sg::Task &task) {
  return static_cast<qd::Opcode>(task.opcode);
}

// ------------------------------------------------------------ validation --

// Reference valid_qwen_task (:47-77).
__device__ bool valid_qwen_task(const sg::Task &task, const qd::Context *context) {
  switch (opcode_of(task)) {
  case qd::Opcode::attention_rmsnorm_f32:
  case qd::Opcode::mlp_rmsnorm_f32:
  case qd::Opcode::final_rmsnorm_f32:
  case qd::Opcode::down_matvec_f32:
    return task.begin < task.end && task.end <= context->hidden_size;
  case qd::Opcode::qkv_projection_f32:
    return task.begin < task.end && task.end <= qd::kPackedQkvSize;
  case qd::Opcode::rope_kv_cache_f32:
    return task.begin == 0 && task.end == qd::kRotaryHeads;
  case qd::Opcode::grouped_query_attention_f32:
    return task.begin < task.end && task.end <= qd::kAttentionHeads;
  case qd::Opcode::attention_output_residual_f32:
    return task.begin < task.end && task.end <= context->hidden_size;
  case qd::Opcode::residual_advance:
    return task.begin < task.end && task.end <= context->hidden_size &&
           task.argument0 != 0;
  case qd::Opcode::gate_up_silu_f32:
    return task.begin < task.end && task.end <= context->intermediate_size;
  case qd::Opcode::lm_head_top1_partition_f32:
    return task.begin < task.end && task.end <= context->tail->vocab_size &&
           task.argument0 < context->tail->partition_count;
  case qd::Opcode::top1_reduce:
    return task.begin == 0 && task.end == context->tail->partition_count;
  case qd::Opcode::embedding_feedback_f32:
    return task.begin == 0 && task.end == context->hidden_size;
  }
  return false;
}

// Reference valid_qwen_contexts (:79-120), plus one stricter bound: every
// position the run can write (token_position .. token_position +
// maximum_tokens - 1) must lie inside the KV cache and RoPE tables. The
// reference only checks maximum_tokens <= capacity and token_position <
// capacity, which lets a prefilled cache run past its end.
__device__ bool valid_qwen_contexts(const qd::Context *contexts) {
  const qd::Context *c = contexts;
  if (contexts == nullptr || c->layer_count == 0 || c->hidden_size != qd::kHiddenSize ||
      c->query_size != qd::kQuerySize || c->kv_size != qd::kKvSize ||
      c->intermediate_size != qd::kIntermediateSize || c->tail == nullptr) {
    return false;
  }
  const qd::TailContext *tail = c->tail;
  if (tail->final_norm_weight == nullptr || tail->lm_head_weight == nullptr ||
      tail->token_embeddings == nullptr || tail->final_normalized == nullptr ||
      tail->partial_max_values == nullptr || tail->partial_max_indices == nullptr ||
      tail->decode_state == nullptr || tail->output_tokens == nullptr ||
      tail->vocab_size == 0 || tail->partition_count == 0 ||
      tail->partition_count > qd::kMaximumLmHeadPartitions ||
      tail->embedding_count != tail->vocab_size) {
    return false;
  }
  const qd::DecodeState *decode = tail->decode_state;
  const uint64_t last_position =
      uint64_t{decode->token_position} + decode->maximum_tokens;
  if (decode->maximum_tokens == 0 || decode->maximum_tokens > c->cache_capacity ||
      decode->token_position != decode->kv_length ||
      decode->token_position >= c->cache_capacity ||
      last_position > c->cache_capacity) {
    return false;
  }
  for (uint32_t layer = 1; layer < c->layer_count; ++layer) {
    const qd::Context &other = contexts[layer];
    if (other.hidden_size != c->hidden_size || other.query_size != c->query_size ||
        other.kv_size != c->kv_size ||
        other.intermediate_size != c->intermediate_size ||
        other.cache_capacity != c->cache_capacity ||
        other.layer_count != c->layer_count || other.tail != c->tail) {
      return false;
    }
  }
  return true;
}

// =========================================================== generic path ==
// One task at a time with the reference's task semantics. Operands written by
// other blocks during the launch are read through L2 (ld.cg); weights, biases,
// norms and tables never change during a launch.

// Lane-strided dot product over n columns, summed into lane 0.
__device__ __forceinline__ float dot_rows(const float *activations, const float *weights,
                                          uint32_t n, uint32_t lane) {
  float sum = 0.0f;
  for (uint32_t column = lane; column < n; column += 32u) {
    sum = fmaf(dev::load_cg(activations + column), __ldg(weights + column), sum);
  }
  return warp_sum(sum);
}

// Block-wide RMSNorm of hidden[begin,end) (reference :665-701).
__device__ void generic_rmsnorm(const sg::Task &task, qd::Context *c) {
  __shared__ float partial[kThreads];
  float sum = 0.0f;
  for (uint32_t i = task.begin + threadIdx.x; i < task.end; i += kThreads) {
    const float value = dev::load_cg(c->hidden + i);
    sum = fmaf(value, value, sum);
  }
  partial[threadIdx.x] = sum;
  __syncthreads();
  for (uint32_t stride = kThreads / 2u; stride != 0; stride >>= 1u) {
    if (threadIdx.x < stride) {
      partial[threadIdx.x] += partial[threadIdx.x + stride];
    }
    __syncthreads();
  }
  const float epsilon = __uint_as_float(task.argument0);
  const float inverse_rms =
      1.0f / sqrtf(partial[0] / static_cast<float>(task.end - task.begin) + epsilon);
  const float *weight = c->tail->final_norm_weight;
  float *out = c->tail->final_normalized;
  if (opcode_of(task) == qd::Opcode::attention_rmsnorm_f32) {
    weight = c->attention_norm_weight;
    out = c->attention_normalized;
  } else if (opcode_of(task) == qd::Opcode::mlp_rmsnorm_f32) {
    weight = c->mlp_norm_weight;
    out = c->mlp_normalized;
  }
  for (uint32_t i = task.begin + threadIdx.x; i < task.end; i += kThreads) {
    out[i] = dev::load_cg(c->hidden + i) * inverse_rms * weight[i];
  }
  __syncthreads();
}

// Packed QKV row (reference :392-427 / :436-452).
__device__ void generic_qkv_row(const qd::Context *c, uint32_t packed_row, uint32_t lane) {
  const float *weight = c->q_weight;
  const float *bias = c->q_bias;
  float *out = c->query;
  uint32_t row = packed_row;
  if (packed_row >= c->query_size + c->kv_size) {
    weight = c->v_weight;
    bias = c->v_bias;
    out = c->value;
    row -= c->query_size + c->kv_size;
  } else if (packed_row >= c->query_size) {
    weight = c->k_weight;
    bias = c->k_bias;
    out = c->key;
    row -= c->query_size;
  }
  const float sum = dot_rows(c->attention_normalized,
                             weight + size_t{row} * c->hidden_size, c->hidden_size, lane);
  if (lane == 0) {
    out[row] = sum + bias[row];
  }
}

// Reference rope_kv_cache (:517-552).
__device__ void generic_rope_kv(qd::Context *c) {
  const uint32_t position = decode_field(&c->tail->decode_state->token_position);
  const size_t rope = size_t{position} * qd::kRotarySize;
  const size_t cache_row = size_t{position} * c->kv_size;
  for (uint32_t pair = threadIdx.x; pair < qd::kRotaryHeads * qd::kRotarySize;
       pair += kThreads) {
    const uint32_t head = pair / qd::kRotarySize;
    const uint32_t f = pair % qd::kRotarySize;
    const bool is_query = head < qd::kAttentionHeads;
    const uint32_t local = is_query ? head : head - qd::kAttentionHeads;
    float *vector = is_query ? c->query : c->key;
    const uint32_t first = local * qd::kHeadSize + f;
    const uint32_t second = first + qd::kRotarySize;
    const float x0 = dev::load_cg(vector + first);
    const float x1 = dev::load_cg(vector + second);
    const float cosine = c->rope_cos[rope + f];
    const float sine = c->rope_sin[rope + f];
    const float r0 = x0 * cosine - x1 * sine;
    const float r1 = x1 * cosine + x0 * sine;
    vector[first] = r0;
    vector[second] = r1;
    if (!is_query) {
      c->key_cache[cache_row + first] = r0;
      c->key_cache[cache_row + second] = r1;
    }
  }
  for (uint32_t i = threadIdx.x; i < c->kv_size; i += kThreads) {
    c->value_cache[cache_row + i] = dev::load_cg(c->value + i);
  }
  __syncthreads();
}

// Reference grouped_query_attention (:554-600): one warp per query head,
// online softmax over positions 0..kv_length inclusive, in-place output.
__device__ void generic_gqa(const sg::Task &task, qd::Context *c) {
  const uint32_t lane = threadIdx.x & 31u;
  const uint32_t warp = threadIdx.x >> 5u;
  const uint32_t kv_length = decode_field(&c->tail->decode_state->kv_length);
  for (uint32_t head = task.begin + warp; head < task.end; head += kWarps) {
    const uint32_t kv_offset = (head / qd::kQueriesPerKvHead) * qd::kHeadSize;
    const uint32_t first = head * qd::kHeadSize + lane;
    const float q0 = dev::load_cg(c->query + first);
    const float q1 = dev::load_cg(c->query + first + 32u);
    float acc0 = 0.0f, acc1 = 0.0f, maximum = -INFINITY, denominator = 0.0f;
    for (uint32_t position = 0; position <= kv_length; ++position) {
      const size_t row = size_t{position} * c->kv_size + kv_offset;
      const float dot = warp_all_sum(q0 * dev::load_cg(c->key_cache + row + lane) +
                                     q1 * dev::load_cg(c->key_cache + row + lane + 32u));
      const float score = dot * 0.125f; // 1/sqrt(head_dim = 64)
      const float next_maximum = fmaxf(maximum, score);
      const float previous_scale = expf(maximum - next_maximum);
      const float score_scale = expf(score - next_maximum);
      denominator = denominator * previous_scale + score_scale;
      acc0 = acc0 * previous_scale +
             score_scale * dev::load_cg(c->value_cache + row + lane);
      acc1 = acc1 * previous_scale +
             score_scale * dev::load_cg(c->value_cache + row + lane + 32u);
      maximum = next_maximum;
    }
    __syncwarp();
    c->query[first] = acc0 / denominator;
    c->query[first + 32u] = acc1 / denominator;
  }
  __syncthreads();
}

// LM-head partition with per-warp then per-block top-1 (reference :231-272).
__device__ void generic_lm_head(const sg::Task &task, qd::Context *c) {
  __shared__ float values[kWarps];
  __shared__ uint32_t indices[kWarps];
  const uint32_t lane = threadIdx.x & 31u;
  const uint32_t warp = threadIdx.x >> 5u;
  float best_value = -INFINITY;
  uint32_t best_index = UINT32_MAX;
  for (uint32_t row = task.begin + warp; row < task.end; row += kWarps) {
    const float sum = dot_rows(c->tail->final_normalized,
                               c->tail->lm_head_weight + size_t{row} * c->hidden_size,
                               c->hidden_size, lane);
    if (lane == 0 && better_top1(sum, row, best_value, best_index)) {
      best_value = sum;
      best_index = row;
    }
  }
  if (lane == 0) {
    values[warp] = best_value;
    indices[warp] = best_index;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    best_value = values[0];
    best_index = indices[0];
    for (uint32_t w = 1; w < kWarps; ++w) {
      if (better_top1(values[w], indices[w], best_value, best_index)) {
        best_value = values[w];
        best_index = indices[w];
      }
    }
    c->tail->partial_max_values[task.argument0] = best_value;
    c->tail->partial_max_indices[task.argument0] = best_index;
  }
  __syncthreads();
}

// Reference reduce_top1 (:339-356).
__device__ void generic_reduce_top1(qd::Context *c) {
  if (threadIdx.x == 0) {
    qd::TailContext *tail = c->tail;
    float best_value = dev::load_cg(tail->partial_max_values);
    uint32_t best_index = dev::load_cg(tail->partial_max_indices);
    for (uint32_t p = 1; p < tail->partition_count; ++p) {
      const float value = dev::load_cg(tail->partial_max_values + p);
      const uint32_t index = dev::load_cg(tail->partial_max_indices + p);
      if (better_top1(value, index, best_value, best_index)) {
        best_value = value;
        best_index = index;
      }
    }
    tail->decode_state->sampled_logit = best_value;
    tail->decode_state->sampled_token = best_index;
  }
  __syncthreads();
}

// Reference embedding_feedback (:358-390).
__device__ void embedding_feedback(qd::Context *c, sg::State *state) {
  __shared__ uint32_t continue_with;
  qd::DecodeState *decode = c->tail->decode_state;
  if (threadIdx.x == 0) {
    // Every field is read before any is written, so the loads are in flight
    // together (one round trip instead of one per field).
    const uint32_t index = decode_field(&decode->generated_tokens);
    const uint32_t token = decode_field(&decode->sampled_token);
    const uint32_t eos_token = decode_field(&decode->eos_token);
    const uint32_t maximum = decode_field(&decode->maximum_tokens);
    const uint32_t position = decode_field(&decode->token_position);
    const uint32_t kv_length = decode_field(&decode->kv_length);
    uint32_t predicate = state->predicate_value;
    c->tail->output_tokens[index] = token;
    const uint32_t generated = index + 1u;
    decode->generated_tokens = generated;
    const bool eos = token == eos_token;
    const bool limit = generated >= maximum;
    if (eos || limit) {
      decode->stop_reason = static_cast<uint32_t>(
          eos ? qd::StopReason::eos_token : qd::StopReason::maximum_tokens);
      state->predicate_value = 1;
      predicate = 1;
    } else {
      decode->token_position = position + 1u;
      decode->kv_length = kv_length + 1u;
    }
    continue_with = predicate == 0 ? token : UINT32_MAX;
  }
  __syncthreads();
  if (continue_with != UINT32_MAX) {
    const float *row = c->tail->token_embeddings + size_t{continue_with} * c->hidden_size;
    for (uint32_t i = threadIdx.x; i < c->hidden_size; i += kThreads) {
      c->hidden[i] = row[i];
    }
  }
  __syncthreads();
}

// Reference residual_advance default branch (:749-760).
__device__ void residual_advance(const sg::Task &task, sg::State *state, qd::Context *c,
                                 bool add_projected, uint32_t step) {
  if (add_projected) {
    for (uint32_t i = task.begin + threadIdx.x; i < task.end; i += kThreads) {
      c->hidden[i] = dev::load_cg(c->hidden + i) + dev::load_cg(c->projected + i);
    }
  }
  if (threadIdx.x == 0) {
    const bool boundary = task.argument1 == 0 || (step + 1u) % c->layer_count == 0;
    if (boundary && task.argument1 == 0) {
      state->predicate_value += task.argument0;
    }
    state->branch_value = boundary ? 1u : 0u;
  }
  __syncthreads();
}

// Row-wise GEMV opcodes over [first_row, end_row), spread over `warp_count`
// warps starting at `warp_index` (a task's block, or a whole stage's grid).
__device__ void generic_rows(qd::Opcode opcode, qd::Context *c, uint32_t first_row,
                             uint32_t end_row, uint32_t warp_index, uint32_t warp_count) {
  const uint32_t lane = threadIdx.x & 31u;
  for (uint32_t row = first_row + warp_index; row < end_row; row += warp_count) {
    switch (opcode) {
    case qd::Opcode::qkv_projection_f32:
      generic_qkv_row(c, row, lane);
      break;
    case qd::Opcode::attention_output_residual_f32: {
      const float sum = dot_rows(c->query, c->out_weight + size_t{row} * c->query_size,
                                 c->query_size, lane);
      if (lane == 0) {
        c->hidden[row] = dev::load_cg(c->hidden + row) + sum;
      }
      break;
    }
    case qd::Opcode::gate_up_silu_f32: {
      const size_t offset = size_t{row} * c->hidden_size;
      const float gate = dot_rows(c->mlp_normalized, c->gate_weight + offset,
                                  c->hidden_size, lane);
      const float up = dot_rows(c->mlp_normalized, c->up_weight + offset,
                                c->hidden_size, lane);
      if (lane == 0) {
        c->activated[row] = silu_times(gate, up);
      }
      break;
    }
    case qd::Opcode::down_matvec_f32: {
      const float sum =
          dot_rows(c->activated, c->down_weight + size_t{row} * c->intermediate_size,
                   c->intermediate_size, lane);
      if (lane == 0) {
        c->projected[row] = sum;
      }
      break;
    }
    default:
      break;
    }
  }
}

__device__ bool is_row_gemv(qd::Opcode opcode) {
  return opcode == qd::Opcode::qkv_projection_f32 ||
         opcode == qd::Opcode::attention_output_residual_f32 ||
         opcode == qd::Opcode::gate_up_silu_f32 || opcode == qd::Opcode::down_matvec_f32;
}

// Reference execute_task (:661-761), whole block on one task.
__device__ void generic_execute(const sg::Task &task, sg::State *state, qd::Context *c) {
  const qd::Opcode opcode = opcode_of(task);
  switch (opcode) {
  case qd::Opcode::attention_rmsnorm_f32:
  case qd::Opcode::mlp_rmsnorm_f32:
  case qd::Opcode::final_rmsnorm_f32:
    generic_rmsnorm(task, c);
    return;
  case qd::Opcode::rope_kv_cache_f32:
    generic_rope_kv(c);
    return;
  case qd::Opcode::grouped_query_attention_f32:
    generic_gqa(task, c);
    return;
  case qd::Opcode::lm_head_top1_partition_f32:
    generic_lm_head(task, c);
    return;
  case qd::Opcode::top1_reduce:
    generic_reduce_top1(c);
    return;
  case qd::Opcode::embedding_feedback_f32:
    embedding_feedback(c, state);
    return;
  case qd::Opcode::residual_advance:
    residual_advance(task, state, c, true, dev::load_relaxed(&state->step));
    return;
  default:
    generic_rows(opcode, c, task.begin, task.end, threadIdx.x >> 5u, kWarps);
    __syncthreads();
    return;
  }
}

// Compiled-stage execution on the generic path: row GEMV stages are spread
// over every warp of the grid (as the reference does for QKV, o_proj and down,
// :183-223, :454-492, :622-659); other tasks go round-robin over blocks.
__device__ void generic_execute_stage(const sg::Stage &stage, const sg::Task *tasks,
                                      sg::State *state, void *opaque, uint32_t worker,
                                      uint32_t workers) {
  qd::Context *c = layer_context(opaque, state);
  const sg::Task &first = tasks[stage.task_offset];
  const qd::Opcode opcode = opcode_of(first);
  if (is_row_gemv(opcode)) {
    // Tasks of one row-GEMV stage form a contiguous row range in the
    // reference tables; handle each task's range so gaps stay untouched.
    const uint32_t warp_index = worker * kWarps + (threadIdx.x >> 5u);
    for (uint32_t t = 0; t < stage.task_count; ++t) {
      const sg::Task &task = tasks[stage.task_offset + t];
      generic_rows(opcode_of(task), c, task.begin, task.end, warp_index,
                   workers * kWarps);
    }
    __syncthreads();
    return;
  }
  for (uint32_t t = worker; t < stage.task_count; t += workers) {
    generic_execute(tasks[stage.task_offset + t], state, c);
  }
}

// ============================================================= fused path ==

using namespace qd::resident;
constexpr uint32_t kMaxAttentionChunks = 128;
constexpr uint32_t kKvTile = 32;                       // positions per attention tile
constexpr uint32_t kKeyStride = qd::kHeadSize + 1u;    // padded K rows (bank-conflict free)
// Up to kLocalAttentionLimit KV positions every block computes the attention
// output of its KV group's seven query heads itself from shared memory, inside
// the o_proj stage, so the attention stage needs no grid barrier; longer
// contexts use the split path.
enum Matrix : uint32_t { kMq, kMk, kMv, kMo, kMgate, kMup, kMdown };

// Block-uniform launch facts, written once by thread 0 in `begin` and kept in
// shared memory: the fused path reads them on every stream unit, and a
// per-thread copy would live in local memory, whose L1-missing loads wait
// behind the weight stream for microseconds.
struct QwenConfig {
  bool stream_empty;
  FusedShared *shared;
  const qd::Context *contexts;
  qd::Workspace *workspace;
  uint64_t *exchange;       // workspace exchange words
  const unsigned char *kv_maps; // [layer][K cache, V cache, o_proj] tensor maps
  float *logits;            // optional: every LM-head row of the step (test capture)
  const float *lm_head;
  uint32_t worker, workers, layers, vocab, lm_units;
  uint32_t limit_ms;
  uint32_t group;           // KV group whose attention this block computes
  uint32_t group_rank;      // index of this block within its group
  uint32_t group_size;      // blocks of its group
  bool group_writer;        // first block of its group: publishes the attention output
  uint64_t *attention_words; // spread-attention partial states [2][workers][kSpreadWords]
  UnitRanges ranges;
  StreamMap map;
  uint64_t policy;
  sg::Stage lm_stage;
  qd::StageProfile *unit_trace; // stage-profile runs: block 0 unit timeline
  qd::StageProfileEntry *event_trace; // stage-profile runs: every block's exchange waits
  uint32_t event_capacity;            // entries of event_trace this trace may use
  // Token position / KV length at the launch's first decode step and the
  // token index (step / layers, adjusted) they belong to: the fused path
  // derives each step's values instead of reading DecodeState, which only
  // embedding_feedback advances, by one per generated token.
  uint32_t base_position, base_kv_length;
  int32_t base_token;
  float epsilon[3];               // attention, MLP and final RMSNorm tasks
  uint32_t residual_argument[2];  // residual_advance task arguments
};
__shared__ QwenConfig block_config;

// The cache rows [first, first + rows) this block attends, and whether it
// also takes the current position, for a step with `positions` KV positions:
// all cached rows of its group when local, its group slice when spread,
// none when split (the split path reads the cache without the ring).
__device__ __forceinline__ SpreadSlice attention_slice(uint32_t positions) {
  switch (attention_mode(positions, block_config.workers)) {
  case AttentionMode::local:
    return {0u, positions - 1u, true};
  case AttentionMode::spread:
    return spread_slice(positions, block_config.group_rank, block_config.group_size);
  default:
    return {0u, 0u, false};
  }
}

// Shared-memory copies of layer Contexts, double-buffered by step parity:
// layer_cache[s & 1] holds contexts[s % layers] while step s runs. Program 1
// of step s fetches step s + 1's Context (the next Program always runs at
// that step), so no stage chases a Context pointer through global memory.
__shared__ __align__(16) qd::Context layer_cache[2];

__device__ __forceinline__ void fetch_layer_context(uint32_t step) {
  constexpr uint32_t kWords = sizeof(qd::Context) / sizeof(uint4);
  static_assert(sizeof(qd::Context) % sizeof(uint4) == 0);
  if (threadIdx.x < kWords) {
    const uint4 *source =
        reinterpret_cast<const uint4 *>(block_config.contexts + step % block_config.layers);
    reinterpret_cast<uint4 *>(&layer_cache[step & 1u])[threadIdx.x] = __ldg(source + threadIdx.x);
  }
}

// The same copy without stalling the issuing threads (cp.async), issued by
// the last warp, which is otherwise idle while the MLP norm waits for the
// o_proj exchange; those threads complete it (cp.async.wait_all) before that
// norm's block sync, which precedes the first read.
constexpr uint32_t kContextCopyThread = kThreads - 32u;
__device__ __forceinline__ void prefetch_layer_context(uint32_t step) {
  constexpr uint32_t kWords = sizeof(qd::Context) / sizeof(uint4);
  static_assert(kWords <= 32u);
  const uint32_t word = threadIdx.x - kContextCopyThread;
  if (threadIdx.x >= kContextCopyThread && word < kWords) {
    const uint4 *source =
        reinterpret_cast<const uint4 *>(block_config.contexts + step % block_config.layers);
    const uint32_t destination =
        dev::shared_address(reinterpret_cast<uint4 *>(&layer_cache[step & 1u]) + word);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n"
                 "cp.async.commit_group;" ::"r"(destination),
                 "l"(source + word)
                 : "memory");
  }
}

__device__ __forceinline__ void wait_prefetched_context() {
  asm volatile("cp.async.wait_all;" ::: "memory");
}

// Per-thread scheduler state of the Qwen workload (identical in every thread
// of a block).
struct QwenBlock {
  bool fused;
  bool split_attention;     // this step's attention runs split over blocks
  bool spread_attention;    // this step's attention is spread over its group's blocks
  bool hidden_exchanged;    // the residual's last update is the down exchange
  bool failed;              // a wait of this block gave up (block-uniform)
  uint32_t consumed;        // stream sequence number of the next unit to consume
  uint32_t traced_barriers; // stage-profile barrier trace position (thread 0)
  uint32_t program;         // current Program and stage within it
  uint32_t stage;
  uint32_t step;            // graph step of the current Program (local transitions)
  uint32_t position;        // token position and KV length of that step
  uint32_t kv_length;
};

// Stage opcodes of the canonical decode table the fused path requires
// (checked by canonical_table).
__device__ __forceinline__ qd::Opcode fused_opcode(uint32_t program, uint32_t stage) {
  using O = qd::Opcode;
  switch (program * 8u + stage) {
  case 0: return O::attention_rmsnorm_f32;
  case 1: return O::qkv_projection_f32;
  case 2: return O::rope_kv_cache_f32;
  case 3: return O::grouped_query_attention_f32;
  case 4: return O::attention_output_residual_f32;
  case 8: return O::mlp_rmsnorm_f32;
  case 9: return O::gate_up_silu_f32;
  case 10: return O::down_matvec_f32;
  case 11: return O::residual_advance;
  case 16: return O::final_rmsnorm_f32;
  case 17: return O::lm_head_top1_partition_f32;
  case 18: return O::top1_reduce;
  default: return O::embedding_feedback_f32;
  }
}

// residual_advance's branch rule (reference :749-760) for the fused path.
__device__ __forceinline__ bool fused_layer_boundary(uint32_t step) {
  return block_config.residual_argument[1] == 0 ||
         (step + 1u) % block_config.layers == 0;
}

// Stage-profile runs record, for block 0, each warp's wait and compute times
// per stream unit in the second half of StageProfile.entries.
__shared__ uint32_t unit_trace_position;
__device__ __forceinline__ void trace_unit(const QwenBlock &b, uint32_t n, uint64_t before,
                                           uint64_t ready, uint64_t done) {
  qd::StageProfile *p = block_config.unit_trace;
  if (p == nullptr || p->entries == nullptr) {
    return;
  }
  const uint32_t slot = atomicAdd(&unit_trace_position, 2u); // shared: no global round trip
  const uint32_t base = p->entry_count / 2u;
  if (base + slot + 1u < p->entry_count) {
    p->entries[base + slot] = {before, ready};
    p->entries[base + slot + 1u] = {done, (uint64_t{n} << 8) | (threadIdx.x >> 5u)};
  }
}

// Global source ranges of one stream unit (second part empty for
// single-range units). An o_proj unit is `rows` half-row copies of
// first_bytes each, `stride` floats apart.
struct UnitSource {
  const float *first;
  const float *second;
  uint32_t first_bytes;
  uint32_t second_bytes;
  uint32_t rows;
  uint32_t stride;
};

__device__ UnitSource unit_source(const QwenBlock &b, const StreamCursor &c) {
  const float *const *w = block_config.shared->layer_weights[c.layer];
  const uint32_t u = c.unit;
  switch (c.kind) {
  case kQkv: {
    // Rows f..f+3 of a head and their rotary partners f+32..f+35.
    const float *weight = w[kMq];
    uint32_t local = u;
    if (u >= kQUnits + kKUnits) {
      weight = w[kMv];
      local = u - kQUnits - kKUnits;
    } else if (u >= kQUnits) {
      weight = w[kMk];
      local = u - kQUnits;
    }
    const float *first =
        weight + size_t{(local / 8u) * qd::kHeadSize + (local % 8u) * 4u} * qd::kHiddenSize;
    return {first, first + size_t{qd::kRotarySize} * qd::kHiddenSize, 4u * kRowBytes,
            4u * kRowBytes, 1, 0};
  }
  case kOut: // filled by tensor copies in issue_unit
  case kKv:
    return {nullptr, nullptr, 0, 0, 1, 0};
  case kGateUp:
    return {w[kMgate] + size_t{u} * kGuRowsPerUnit * qd::kHiddenSize,
            w[kMup] + size_t{u} * kGuRowsPerUnit * qd::kHiddenSize,
            kGuRowsPerUnit * kRowBytes, kGuRowsPerUnit * kRowBytes, 1, 0};
  case kDown:
    return {w[kMdown] + size_t{u} * qd::kIntermediateSize, nullptr, kDownRowBytes, 0, 1, 0};
  default: { // kLmHead
    const uint32_t row = u * kSlotRows;
    return {block_config.lm_head + size_t{row} * qd::kHiddenSize, nullptr,
            min(kSlotRows, block_config.vocab - row) * kRowBytes, 0, 1, 0};
  }
  }
}

// Per-slot stream positions: slot_position[s] is where the next unit slot s
// receives sits in the block's stream. A slot receives units s, s + kSlots,
// ...; its position is touched only by the lane refilling it, which is a
// consumer of the slot's previous unit.
__shared__ StreamPosition slot_position[kSlots];

// Postponed refills: deferred_unit[s] is the sequence number slot s is still
// to receive (UINT32_MAX: none).
//  - Gate/up units the down stage would refill are first needed in the next
//    gate/up stage; issued at the end of the down stage, their bytes would
//    sit in front of the next layer's first exchanges in the memory queues,
//    so they are issued in the attention stage instead
//    (issue_deferred_refills).
//  - o_proj units' refills (not needed by a later unit of the same stage)
//    are issued by the MLP norm's last warp, which has no hidden values to
//    wait for: a copy issue holds its lane for up to a microsecond, and the
//    o_proj warps go on to the stage's final block sync.
__shared__ uint32_t deferred_unit[kSlots];

// Issues the copies of stream unit `n` into its ring slot (one lane). The
// slot's previous unit (n - kSlots) has been released by its consumers.
__device__ __noinline__ void issue_unit(const QwenBlock &b, uint32_t n) {
  FusedShared *s = block_config.shared;
  const uint32_t slot = n % kSlots;
  const StreamPosition position = slot_position[slot];
  const StreamCursor c = position_cursor(block_config.map, position);
  const UnitSource src = unit_source(b, c);
  unsigned char *destination = s->ring + size_t{slot} * kSlotBytes;
  // The slot's next position and this unit's tag are written before the unit
  // is published: the lane that refills the slot next is a consumer of this
  // unit and may run before this lane gets past the copies below. Both reach
  // other warps through the slot's mbarrier (this lane's arrive releases
  // them, the consumers' wait acquires them); the sequence number only tells
  // a consumer that the fill it waits for is the current one.
  StreamPosition next = position;
  advance_position(block_config.map, next, kSlots);
  slot_position[slot] = next;
  s->unit_tag[slot] = make_tag(c.kind, c.layer, c.unit);
  *reinterpret_cast<volatile uint32_t *>(&s->sequence[slot]) = n;
  if (c.kind == kOut) {
    // o_proj rows 16v..16v+15 (v = unit % 56), input columns of KV group
    // unit / 56: two 224-column boxes of the layer's o_proj tensor map,
    // landing as [box][16 rows][224 floats].
    dev::mbarrier_arrive_expect_tx(&s->full[slot], kOUnitBytes);
    const unsigned char *map = block_config.kv_maps +
                               (size_t{c.layer} * qd::kWorkspaceMapsPerLayer + 2u) *
                                   qd::kTensorMapBytes;
    const uint32_t x = (c.unit / kOGroupUnits) * kGroupColumns;
    const uint32_t y = (c.unit % kOGroupUnits) * kORows;
    dev::tensor_load_2d(destination, map, x, y, &s->full[slot]);
    dev::tensor_load_2d(destination + kOUnitBytes / 2u, map, x + kOBoxColumns, y, &s->full[slot]);
    return;
  }
  if (c.kind == kKv) {
    // Cached rows first + 56j .. first + 56j + 55 of this block's KV group
    // and attention slice, for the token this layer's unit belongs to (one
    // per stream cycle): K then V, each as two 32-column boxes. Units past
    // the slice's cached rows, and every unit of a step whose attention runs
    // split, carry no bytes.
    const uint32_t cached = block_config.base_position + position.cycle;
    const SpreadSlice slice = attention_slice(cached + 1u);
    const bool load = c.unit * kKvUnitPositions < slice.rows;
    dev::mbarrier_arrive_expect_tx(&s->full[slot], load ? kSlotBytes : 0u);
    if (load) {
      const unsigned char *maps =
          block_config.kv_maps + size_t{c.layer} * qd::kWorkspaceMapsPerLayer * qd::kTensorMapBytes;
      const uint32_t x = block_config.group * qd::kHeadSize;
      const uint32_t y = slice.first + c.unit * kKvUnitPositions;
      constexpr uint32_t kBox = kSlotBytes / 4u; // 32 columns x 56 rows
#pragma unroll
      for (uint32_t box = 0; box < 4; ++box) {
        dev::tensor_load_2d(destination + box * kBox, maps + (box >> 1) * qd::kTensorMapBytes,
                            x + 32u * (box & 1u), y, &s->full[slot]);
      }
    }
    return;
  }
  dev::mbarrier_arrive_expect_tx(&s->full[slot],
                                 src.rows * src.first_bytes + src.second_bytes);
  dev::bulk_copy_to_shared(destination, src.first, src.first_bytes, &s->full[slot],
                           block_config.policy);
  for (uint32_t r = 1; r < src.rows; ++r) {
    dev::bulk_copy_to_shared(destination + r * src.first_bytes, src.first + r * src.stride,
                             src.first_bytes, &s->full[slot], block_config.policy);
  }
  if (src.second_bytes != 0) {
    dev::bulk_copy_to_shared(destination + src.first_bytes, src.second, src.second_bytes,
                             &s->full[slot], block_config.policy);
  }
}

// Lane 0 of warp s issues slot s's postponed refill, if any.
__device__ __forceinline__ void issue_deferred_refills(const QwenBlock &b) {
  const uint32_t lane = threadIdx.x & 31u;
  const uint32_t warp = threadIdx.x >> 5u;
  if (lane == 0 && warp < kSlots && deferred_unit[warp] != UINT32_MAX) {
    issue_unit(b, deferred_unit[warp]);
    deferred_unit[warp] = UINT32_MAX;
  }
}

// Lane 0's verdict, shared by the warp.
__device__ __forceinline__ bool warp_uniform(bool lane0_value) {
  return __shfl_sync(kFullMask, lane0_value ? 1u : 0u, 0) != 0u;
}

// Whole warp: waits until stream unit `n` is in its slot and its bytes have
// landed, checks that it is the unit the caller expects, returns the slot.
// nullptr (warp-uniform) after a timeout, a stream mismatch, or when another
// block already failed the run.
__device__ const float *wait_unit(const QwenBlock &b, sg::State *state, uint32_t n,
                                  uint32_t tag) {
  FusedShared *s = block_config.shared;
  const uint32_t slot = n % kSlots;
  const uint32_t parity = (n / kSlots) & 1u;
  const volatile uint32_t *sequence = &s->sequence[slot];
  uint32_t spins = 0;
  uint64_t deadline_ns = 0; // taken at the first check: ready units skip the timer
  auto give_up = [&]() {
    if ((++spins & 63u) != 0u) {
      return false;
    }
    bool stop = false;
    if ((threadIdx.x & 31u) == 0u) {
      const uint64_t now = dev::global_timer_ns();
      if (deadline_ns == 0) {
        deadline_ns = now + uint64_t{block_config.limit_ms} * 1000000ull;
      }
      if (dev::detail::load_status(state) != static_cast<uint32_t>(sg::Status::running)) {
        stop = true;
      } else if (now > deadline_ns) {
        dev::detail::fail(state, sg::kErrorWaitTimeout);
        stop = true;
      }
    }
    return warp_uniform(stop);
  };
  while (__any_sync(kFullMask, *sequence != n)) { // issued (not a lap behind)
    if (give_up()) {
      return nullptr;
    }
  }
  while (__any_sync(kFullMask, !dev::mbarrier_try_wait(&s->full[slot], parity))) {
    if (give_up()) {
      return nullptr;
    }
  }
  if (!warp_uniform(s->unit_tag[slot] == tag)) {
    if ((threadIdx.x & 31u) == 0u) {
      dev::detail::fail(state, sg::kErrorStreamMismatch);
    }
    return nullptr;
  }
  return reinterpret_cast<const float *>(s->ring + size_t{slot} * kSlotBytes);
}

// A lane of the warp that consumed unit `n` last (each unit's consumers are
// done reading the slot: the warp's shuffles of the unit's sums, or a block
// sync, completed every read) refills the slot with unit n + kSlots. No
// fence is needed before the copy overwrites the slot (a CTA fence here
// waits for the lane's earlier global stores, about a microsecond while the
// weight stream runs).
__device__ __forceinline__ void release_unit(const QwenBlock &b, uint32_t n) {
  if (!block_config.stream_empty) {
    issue_unit(b, n + kSlots);
  }
}

// ------------------------------------------------------------ exchanges --

__device__ __forceinline__ uint64_t *exchange_words(uint32_t offset, uint32_t words,
                                                    uint32_t step) {
  return block_config.exchange + offset + (step & 1u) * words;
}

// One thread: waits until every word of the pairs selected by `mask` (pair i
// is the two words at address(i), 16-byte aligned) carries `tag`, and returns
// pair i's values in out[2i], out[2i + 1]. All pending pairs are loaded before
// any is checked, so one round trip serves them all. False when the run
// failed elsewhere or the wait limit passed (the run is then failed).
template <uint32_t kPairs, typename Address>
__device__ bool exchange_wait(sg::State *state, uint32_t tag, uint32_t mask, Address address,
                              float (&out)[2 * kPairs]) {
  uint32_t pending = mask;
  uint32_t polls = 0;
  uint64_t deadline_ns = 0;
  while (pending != 0) {
    uint64_t words[2 * kPairs];
#pragma unroll
    for (uint32_t i = 0; i < kPairs; ++i) {
      words[2 * i] = words[2 * i + 1] = 0;
      if ((pending >> i) & 1u) {
        dev::exchange_load2(address(i), words[2 * i], words[2 * i + 1]);
      }
    }
#pragma unroll
    for (uint32_t i = 0; i < kPairs; ++i) {
      if (((pending >> i) & 1u) && dev::exchange_tag(words[2 * i]) == tag &&
          dev::exchange_tag(words[2 * i + 1]) == tag) {
        out[2 * i] = dev::exchange_value(words[2 * i]);
        out[2 * i + 1] = dev::exchange_value(words[2 * i + 1]);
        pending &= ~(1u << i);
      }
    }
    if (pending != 0 && (++polls & 15u) == 0u) {
      const uint64_t now = dev::global_timer_ns();
      if (deadline_ns == 0) {
        deadline_ns = now + uint64_t{block_config.limit_ms} * 1000000ull;
      } else if (now > deadline_ns) {
        dev::detail::fail(state, sg::kErrorWaitTimeout);
        return false;
      }
      if (dev::detail::load_status(state) != static_cast<uint32_t>(sg::Status::running)) {
        return false;
      }
    }
  }
  return true;
}

// Stage-profile runs: thread 0 records (start, now) of an exchange wait of
// this block at entries[event * workers + worker].
__device__ __forceinline__ void trace_event(QwenBlock &b, uint64_t start_ns) {
  qd::StageProfileEntry *entries = block_config.event_trace;
  if (entries == nullptr) {
    return;
  }
  if (threadIdx.x == 0) {
    const uint64_t now = dev::global_timer_ns();
    const uint64_t index = uint64_t{b.traced_barriers} * block_config.workers + block_config.worker;
    if (index < block_config.event_capacity) {
      entries[index] = {start_ns, now};
    }
  }
  ++b.traced_barriers;
}

// Stage-profile runs: a point in this block's timeline, (marker id, now).
// Ids: 20 + opcode at a stage's entry; at a stage's end 1 attention norm,
// 2 QKV, 3 local attention, 4 o_proj, 5 MLP norm, 6 gate/up, 7 down,
// 8 final norm, 9 LM head, 10 embedding feedback, 11 spread combine. Exchange waits record
// (start, end) in the same sequence.
__device__ __forceinline__ void trace_mark(QwenBlock &b, uint32_t id) {
  if (block_config.event_trace == nullptr) {
    return;
  }
  __syncthreads();
  trace_event(b, id);
}

__device__ __forceinline__ uint64_t trace_start() {
  return block_config.event_trace != nullptr ? dev::global_timer_ns() : 0;
}

// Where a Program's first stage takes the residual from.
enum class HiddenSource : uint32_t {
  global,   // launch start, or after the tail (the next token's embedding row)
  down,     // after Program 1: hidden += down projection of step - 1
  attention // Program 1: hidden += o_proj of this step, both KV groups
};

// Brings this block's copy of the residual stream up to date and RMS-
// normalises it into shared input (every block computes the same values in
// the same order). Thread t < 224 owns hidden[4t, 4t + 4).
__device__ void fused_norm(QwenBlock &b, sg::State *state, const qd::Context *c,
                           HiddenSource source, const float *weight, float epsilon,
                           float *global_copy) {
  FusedShared *s = block_config.shared;
  constexpr uint32_t kVectors = qd::kHiddenSize / 4u; // 224
  const uint32_t t = threadIdx.x;
  float4 h = make_float4(0.f, 0.f, 0.f, 0.f);
  float4 w = make_float4(0.f, 0.f, 0.f, 0.f);
  bool ok = true;
  const uint64_t started = trace_start();
  if (t < kVectors) {
    w = __ldg(reinterpret_cast<const float4 *>(weight) + t); // in flight with the wait
    if (source == HiddenSource::global) {
      h = dev::load_cg4(c->hidden + 4u * t);
    } else if (source == HiddenSource::down) {
      h = reinterpret_cast<const float4 *>(s->hidden)[t];
      const uint32_t step = b.step - 1u;
      const uint64_t *words =
          exchange_words(qd::kExchangeDown, qd::kHiddenSize, step) + 4u * t;
      float v[4];
      ok = exchange_wait<2>(state, step + 1u, 3u, [&](uint32_t i) { return words + 2u * i; },
                            v);
      h = make_float4(h.x + v[0], h.y + v[1], h.z + v[2], h.w + v[3]);
    } else {
      h = reinterpret_cast<const float4 *>(s->hidden)[t];
      const uint64_t *words =
          exchange_words(qd::kExchangeOut, qd::kKvHeads * qd::kHiddenSize, b.step) + 4u * t;
      float v[8];
      ok = exchange_wait<4>(state, b.step + 1u, 15u,
                            [&](uint32_t i) {
                              return words + (i >> 1) * qd::kHiddenSize + 2u * (i & 1u);
                            },
                            v);
      h = make_float4((h.x + v[0]) + v[4], (h.y + v[1]) + v[5], (h.z + v[2]) + v[6],
                      (h.w + v[3]) + v[7]);
    }
    reinterpret_cast<float4 *>(s->hidden)[t] = h;
  }
  if (source == HiddenSource::attention && threadIdx.x == kContextCopyThread) {
    for (uint32_t slot = 0; slot < kSlots; ++slot) {
      if (deferred_unit[slot] != UINT32_MAX) {
        issue_unit(b, deferred_unit[slot]);
        deferred_unit[slot] = UINT32_MAX;
      }
    }
  }
  if (source == HiddenSource::attention && threadIdx.x >= kContextCopyThread) {
    wait_prefetched_context(); // the next step's Context (Program 1's begin)
  }
  float sum = fmaf(h.x, h.x, fmaf(h.y, h.y, fmaf(h.z, h.z, h.w * h.w)));
  sum = warp_sum(sum);
  if ((threadIdx.x & 31u) == 0) {
    s->reduce[threadIdx.x >> 5u] = sum;
  }
  if (__syncthreads_or(ok ? 0 : 1) != 0) {
    b.failed = true;
    return;
  }
  if (source != HiddenSource::global) {
    trace_event(b, started);
  }
  float total = 0.0f;
#pragma unroll
  for (uint32_t w8 = 0; w8 < kWarps; ++w8) {
    total += s->reduce[w8];
  }
  const float inverse_rms =
      1.0f / sqrtf(total / static_cast<float>(qd::kHiddenSize) + epsilon);
  if (t < kVectors) {
    const float4 x = make_float4(h.x * inverse_rms * w.x, h.y * inverse_rms * w.y,
                                 h.z * inverse_rms * w.z, h.w * inverse_rms * w.w);
    reinterpret_cast<float4 *>(s->input)[t] = x;
    if (global_copy != nullptr && block_config.worker == 0) {
      reinterpret_cast<float4 *>(global_copy)[t] = x;
    }
  }
  __syncthreads();
}

// Sums eight per-lane partials across the warp with a transposed butterfly
// (4 + 2 + 1 + 1 + 1 shuffles): afterwards lanes 4r..4r+3 hold row r's total,
// r = (lane >> 2) & 7.
__device__ __forceinline__ float reduce_rows8(const float (&a)[8], uint32_t lane) {
  const bool high16 = (lane & 16u) != 0;
  float q[4];
#pragma unroll
  for (uint32_t i = 0; i < 4; ++i) {
    const float send = high16 ? a[i] : a[i + 4];
    const float keep = high16 ? a[i + 4] : a[i];
    q[i] = keep + __shfl_xor_sync(kFullMask, send, 16);
  }
  const bool high8 = (lane & 8u) != 0;
  float p[2];
#pragma unroll
  for (uint32_t i = 0; i < 2; ++i) {
    const float send = high8 ? q[i] : q[i + 2];
    const float keep = high8 ? q[i + 2] : q[i];
    p[i] = keep + __shfl_xor_sync(kFullMask, send, 8);
  }
  const bool high4 = (lane & 4u) != 0;
  float v = (high4 ? p[1] : p[0]) + __shfl_xor_sync(kFullMask, high4 ? p[0] : p[1], 4);
  v += __shfl_xor_sync(kFullMask, v, 2);
  v += __shfl_xor_sync(kFullMask, v, 1);
  return v;
}

// Dot product of a 896-float shared-memory row with the register-held input;
// every lane receives the total.
__device__ __forceinline__ float row_dot(const float *row, const float4 (&x)[7],
                                         uint32_t lane) {
  const float4 *r = reinterpret_cast<const float4 *>(row);
  float a = 0.0f;
#pragma unroll
  for (uint32_t j = 0; j < 7; ++j) {
    const float4 w = r[lane + 32u * j];
    a = fmaf(w.x, x[j].x, a);
    a = fmaf(w.y, x[j].y, a);
    a = fmaf(w.z, x[j].z, a);
    a = fmaf(w.w, x[j].w, a);
  }
  return warp_all_sum(a);
}

// Consumes this block's units of an 8-row kind. Row r of a unit ends up in
// lanes 4r..4r+3 of the warp that computed it, and every lane of that warp
// runs `epilogue(unit, r, value, valid, extra)` with r = (lane >> 2) & 7;
// `valid` says the lane holds row r's dot product (the LM head's last unit
// is short, and a split unit gives each warp two rows), and lanes with
// (lane & 3) == 0 own the row's outputs. `operands(unit, r)` is loaded before
// the wait so its latency overlaps it.
//  - Many units: one whole unit per warp (warp w takes units w, w + kWarps,
//    ...); each lane accumulates its float4 columns of all eight rows
//    (eight independent FMA chains) and reduce_rows8 sums them.
//  - At most kWarps / 4 units (QKV, o_proj): four warps share a unit, warp g
//    computing the row pair (g, g + 4), so a lone unit takes a quarter of
//    the time.
struct NoOperands {
  __device__ float4 operator()(uint32_t, uint32_t) const { return make_float4(0.f, 0.f, 0.f, 0.f); }
};

constexpr uint32_t kPairWarps = 4; // warps sharing a split unit

template <typename Epilogue, typename Operands = NoOperands>
__device__ bool consume_units(QwenBlock &b, sg::State *state, uint32_t kind,
                              uint32_t layer, Epilogue epilogue,
                              Operands operands = NoOperands{}) {
  const uint32_t lane = threadIdx.x & 31u;
  const uint32_t warp = threadIdx.x >> 5u;
  const uint32_t row = (lane >> 2u) & 7u;
  float4 x[7];
  const float4 *input = reinterpret_cast<const float4 *>(block_config.shared->input);
#pragma unroll
  for (uint32_t j = 0; j < 7; ++j) {
    x[j] = input[lane + 32u * j];
  }
  const UnitRange range = block_config.ranges.of[kind];
  const uint32_t units = range.end - range.begin;
  // Units whose slots must be reused within this stage (a stage of more
  // units than ring slots) go first, four warps to a unit, so their refills
  // are issued as early as possible; so do all units of stages with at most
  // kWarps / kPairWarps units. The rest take one warp each.
  const uint32_t early = units * kPairWarps <= kWarps                ? units
                         : units > kSlots && units <= 2u * kSlots ? units - kSlots
                                                                    : 0u;
  auto process = [&](uint32_t i, bool split) -> bool {
    const uint32_t n = b.consumed + i;
    const uint32_t u = range.begin + i;
    const float4 extra = (lane & 3u) == 0u ? operands(u, row) : make_float4(0.f, 0.f, 0.f, 0.f);
    const uint64_t t_before = block_config.unit_trace != nullptr ? dev::global_timer_ns() : 0;
    const float *slot = wait_unit(b, state, n, make_tag(kind, layer, u));
    const uint64_t t_ready = block_config.unit_trace != nullptr ? dev::global_timer_ns() : 0;
    if (slot == nullptr) {
      return false;
    }
    const uint32_t rows =
        kind == kLmHead ? min(kSlotRows, block_config.vocab - u * kSlotRows) : kSlotRows;
    float value;
    bool valid;
    if (split) {
      // Rows past `rows` are never split (only full 8-row kinds get here).
      const uint32_t pair = warp % kPairWarps;
      const float a = row_dot(slot + pair * qd::kHiddenSize, x, lane);
      const float c = row_dot(slot + (pair + 4u) * qd::kHiddenSize, x, lane);
      valid = row == pair || row == pair + 4u;
      value = row == pair ? a : c;
    } else {
      // Rows past `rows` (the LM head's last unit) hold stale bytes; their
      // sums stay in their own lanes and are flagged invalid.
      const float4 *w = reinterpret_cast<const float4 *>(slot);
      float a[8];
#pragma unroll
      for (uint32_t r = 0; r < 8; ++r) {
        a[r] = 0.0f;
      }
#pragma unroll
      for (uint32_t j = 0; j < 7; ++j) {
#pragma unroll
        for (uint32_t r = 0; r < 8; ++r) {
          const float4 v = w[r * (qd::kHiddenSize / 4u) + lane + 32u * j];
          a[r] = fmaf(v.x, x[j].x, a[r]);
          a[r] = fmaf(v.y, x[j].y, a[r]);
          a[r] = fmaf(v.z, x[j].z, a[r]);
          a[r] = fmaf(v.w, x[j].w, a[r]);
        }
      }
      // The shuffles complete every lane's shared-memory reads of the slot.
      value = reduce_rows8(a, lane);
      valid = row < rows;
    }
    // The epilogue's exchange stores go first: the refill's copy issue can
    // hold its lane for several hundred nanoseconds.
    epilogue(u, row, value, valid, extra);
    if (lane == 0 && (!split || (atomicAdd(&block_config.shared->pair_done[n % kSlots], 1u) &
                                 (kPairWarps - 1u)) == kPairWarps - 1u)) {
      release_unit(b, n); // (split: the unit's last warp) refills the slot
    }
    if (lane == 0 && block_config.unit_trace != nullptr) {
      trace_unit(b, n, t_before, t_ready, dev::global_timer_ns());
    }
    __syncwarp();
    return true;
  };
  bool ok = true;
  for (uint32_t i = warp / kPairWarps; ok && i < early; i += kWarps / kPairWarps) {
    ok = process(i, true);
  }
  for (uint32_t i = early + warp; ok && i < units; i += kWarps) {
    ok = process(i, false);
  }
  b.consumed += units;
  return ok;
}

// QKV unit geometry: which projection, and the first / rotary-partner rows.
struct QkvRows {
  uint32_t which; // 0 q, 1 k, 2 v
  uint32_t first, second, frequency;
};

__device__ __forceinline__ QkvRows qkv_rows(uint32_t u, uint32_t gw) {
  uint32_t which = 0, local = u;
  if (u >= kQUnits + kKUnits) {
    which = 2;
    local = u - kQUnits - kKUnits;
  } else if (u >= kQUnits) {
    which = 1;
    local = u - kQUnits;
  }
  const uint32_t f = (local % 8u) * 4u + gw;
  const uint32_t first = (local / 8u) * qd::kHeadSize + f;
  return {which, first, first + qd::kRotarySize, f};
}

__device__ void fused_qkv(QwenBlock &b, sg::State *state, qd::Context *c, uint32_t layer) {
  const uint32_t position = b.position;
  const size_t rope = size_t{position} * qd::kRotarySize;
  const size_t cache_row = size_t{position} * qd::kKvSize;
  uint64_t *words = exchange_words(qd::kExchangeQkv, qd::kPackedQkvSize, b.step);
  const uint32_t tag = b.step + 1u;
  const bool split = b.split_attention;
  consume_units(
      b, state, kQkv, layer,
      [&](uint32_t u, uint32_t row, float value, bool valid, float4 operand) {
        // Rows 0-3 of a unit are f..f+3 of one head, rows 4-7 their rotary
        // partners f+32..f+35: lane 4r (r < 4) rotates the pair (r, r + 4)
        // (a warp holding row r also holds its partner).
        const float partner = __shfl_xor_sync(kFullMask, value, 16);
        if (row >= 4u || !valid || (threadIdx.x & 3u) != 0u) {
          return;
        }
        const QkvRows r = qkv_rows(u, row);
        const float x0 = value + operand.x;
        const float x1 = partner + operand.y;
        float r0 = x0, r1 = x1;
        if (r.which != 2) {
          r0 = x0 * operand.z - x1 * operand.w;
          r1 = x1 * operand.z + x0 * operand.w;
        }
        // The exchange words first (the other blocks wait for them), then
        // the global copies: K/V rows, the cache rows of this position, and
        // the query when the attention runs split (it reads it from there).
        uint64_t *packed = words + (r.which == 0 ? 0u
                                    : r.which == 1 ? qd::kQuerySize
                                                   : qd::kQuerySize + qd::kKvSize);
        dev::exchange_store(packed + r.first, r0, tag);
        dev::exchange_store(packed + r.second, r1, tag);
        if (r.which != 0) {
          float *out = r.which == 1 ? c->key : c->value;
          out[r.first] = r0;
          out[r.second] = r1;
          float *cache = (r.which == 1 ? c->key_cache : c->value_cache) + cache_row;
          cache[r.first] = r0;
          cache[r.second] = r1;
        } else if (split) {
          c->query[r.first] = r0;
          c->query[r.second] = r1;
        }
      },
      [&](uint32_t u, uint32_t row) {
        if (row >= 4u) {
          return make_float4(0.f, 0.f, 0.f, 0.f);
        }
        const QkvRows r = qkv_rows(u, row);
        const float *bias = r.which == 0 ? c->q_bias : (r.which == 1 ? c->k_bias : c->v_bias);
        return make_float4(bias[r.first], bias[r.second], c->rope_cos[rope + r.frequency],
                           c->rope_sin[rope + r.frequency]);
      });
}

__device__ void group_attention(QwenBlock &b, sg::State *state, const qd::Context *c,
                                uint32_t layer);

// o_proj split along its input over the two KV groups: this block's units
// are rows 8v..8v+7 restricted to its group's 448 columns, each row computed
// by one warp against the group's attention output in shared input[0, 448).
// The two groups' partial rows go to the out exchange; every block adds both
// to its residual at the start of Program 1.
__device__ void fused_out(QwenBlock &b, sg::State *state, qd::Context *c, uint32_t layer) {
  FusedShared *s = block_config.shared;
  const uint32_t lane = threadIdx.x & 31u;
  const uint32_t warp = threadIdx.x >> 5u;
  const uint32_t group = block_config.group;
  if (b.spread_attention) {
    // The group's attention output from the attention exchange (thread t <
    // 112 takes dims 4t..4t+3).
    bool ok = true;
    if (threadIdx.x < kGroupColumns / 4u) {
      const uint64_t *words = exchange_words(qd::kExchangeAttention, qd::kQuerySize, b.step) +
                              group * kGroupColumns + 4u * threadIdx.x;
      float v[4];
      ok = exchange_wait<2>(state, b.step + 1u, 3u, [&](uint32_t i) { return words + 2u * i; },
                            v);
      reinterpret_cast<float4 *>(s->input)[threadIdx.x] = make_float4(v[0], v[1], v[2], v[3]);
    }
    if (__syncthreads_or(ok ? 0 : 1) != 0) {
      b.failed = true;
      return;
    }
  } else if (!b.split_attention) {
    group_attention(b, state, c, layer);
    if (b.failed) {
      return;
    }
    trace_mark(b, 3);
  } else {
    // The split attention wrote the output over the query (grid barrier since).
    const float *source = c->query + group * kGroupColumns;
    for (uint32_t i = threadIdx.x; i < kGroupColumns / 4u; i += kThreads) {
      reinterpret_cast<float4 *>(s->input)[i] = dev::load_cg4(source + 4u * i);
    }
    __syncthreads();
  }
  constexpr uint32_t kVectors = kGroupColumns / 4u;   // 112 float4 per half row
  constexpr uint32_t kBoxVectors = kOBoxColumns / 4u; // 56 per tensor box row
  float4 x[4];
  uint32_t offset[4]; // float4 offset of input vector v = lane + 32j in a unit's row 0
#pragma unroll
  for (uint32_t j = 0; j < 4; ++j) {
    const uint32_t v = lane + 32u * j;
    x[j] = v < kVectors ? reinterpret_cast<const float4 *>(s->input)[v]
                        : make_float4(0.f, 0.f, 0.f, 0.f);
    offset[j] = v < kBoxVectors ? v : kORows * kBoxVectors + (v - kBoxVectors);
    static_assert(kORows % kWarps == 0, "every warp takes the same o_proj rows");
  }
  const UnitRange range = block_config.ranges.of[kOut];
  const uint32_t tag = b.step + 1u;
  uint64_t *words = exchange_words(qd::kExchangeOut, qd::kKvHeads * qd::kHiddenSize, b.step);
  bool ok = true;
  for (uint32_t i = 0; ok && i < range.end - range.begin; ++i) {
    const uint32_t n = b.consumed + i;
    const uint32_t u = range.begin + i;
    const float *slot = wait_unit(b, state, n, make_tag(kOut, layer, u));
    if (slot == nullptr) {
      ok = false;
      break;
    }
    // Warp w computes rows w, w + 8, ... of the unit ([box][kORows][56 float4]).
    constexpr uint32_t kRowsPerWarp = kORows / kWarps;
    float a[kRowsPerWarp];
#pragma unroll
    for (uint32_t r = 0; r < kRowsPerWarp; ++r) {
      a[r] = 0.0f;
    }
#pragma unroll
    for (uint32_t j = 0; j < 4; ++j) {
      if (lane + 32u * j < kVectors) {
#pragma unroll
        for (uint32_t r = 0; r < kRowsPerWarp; ++r) {
          const float4 w = reinterpret_cast<const float4 *>(slot)[(warp + kWarps * r) * kBoxVectors + offset[j]];
          a[r] = fmaf(w.x, x[j].x, a[r]);
          a[r] = fmaf(w.y, x[j].y, a[r]);
          a[r] = fmaf(w.z, x[j].z, a[r]);
          a[r] = fmaf(w.w, x[j].w, a[r]);
        }
      }
    }
#pragma unroll
    for (uint32_t r = 0; r < kRowsPerWarp; ++r) {
      a[r] = warp_all_sum(a[r]); // the shuffles complete the warp's reads of the slot
    }
    if (lane == 0) {
      uint64_t *group_words = words + (u / kOGroupUnits) * qd::kHiddenSize;
#pragma unroll
      for (uint32_t r = 0; r < kRowsPerWarp; ++r) {
        dev::exchange_store(group_words + (u % kOGroupUnits) * kORows + warp + kWarps * r, a[r],
                            tag);
      }
      // The unit's eighth warp hands the slot's refill to the MLP norm's
      // last warp, which waits for the o_proj exchange meanwhile.
      if ((atomicAdd(&s->rows_done[n % kSlots], 1u) & (kWarps - 1u)) == kWarps - 1u) {
        if (n + kSlots < b.consumed + (range.end - range.begin)) {
          release_unit(b, n); // a later unit of this stage takes the slot
        } else {
          deferred_unit[n % kSlots] = n + kSlots;
        }
      }
    }
  }
  b.consumed += range.end - range.begin;
  if (__syncthreads_or(ok ? 0 : 1) != 0) {
    b.failed = true;
  }
}

__device__ void fused_gate_up(QwenBlock &b, sg::State *state, qd::Context *c,
                              uint32_t layer) {
  // Rows 0-3 of a unit are gate rows 4u..4u+3, rows 4-7 the matching up rows.
  uint64_t *words = exchange_words(qd::kExchangeAct, qd::kIntermediateSize, b.step);
  const uint32_t tag = b.step + 1u;
  consume_units(b, state, kGateUp, layer,
                [&](uint32_t u, uint32_t row, float value, bool valid, float4) {
                  const float up = __shfl_xor_sync(kFullMask, value, 16);
                  if (row < 4u && valid && (threadIdx.x & 3u) == 0u) {
                    const float act = silu_times(value, up);
                    dev::exchange_store(words + u * kGuRowsPerUnit + row, act, tag);
                    c->activated[u * kGuRowsPerUnit + row] = act;
                  }
                });
}

// Down projection: one 4864-float row per unit, every row computed by all
// warps together. Warp w owns the float4 columns lane + 32k for k = w, w + 8,
// ... (five or four per lane) and takes that slice of the activated vector
// straight from the act exchange into registers. For a batch of up to kSlots rows, warp r waits for
// row r (the waits overlap), a block sync publishes the landed rows, every
// warp accumulates its columns of all rows, reduce_rows8 sums lanes, and
// lane 0 of warp r adds the eight warps' partials of row r in warp order,
// writes the row and refills its slot (one refill per warp, so they run in
// parallel instead of as divergent lanes of one warp).
__device__ void fused_down(QwenBlock &b, sg::State *state, qd::Context *c, uint32_t layer) {
  constexpr uint32_t kChunks = qd::kIntermediateSize / 4u / 32u; // 38 float4 per lane
  constexpr uint32_t kMine = (kChunks + kWarps - 1u) / kWarps;    // 5
  static_assert(kSlots < 8 && kSlots <= kWarps, "a batch of rows must fit reduce_rows8");
  const uint32_t lane = threadIdx.x & 31u;
  const uint32_t warp = threadIdx.x >> 5u;
  const uint32_t row = (lane >> 2u) & 7u;
  FusedShared *shared = block_config.shared;
  float4 x[kMine];
  {
    const uint64_t started = trace_start();
    const uint64_t *act = exchange_words(qd::kExchangeAct, qd::kIntermediateSize, b.step);
    uint32_t mask = 0;
#pragma unroll
    for (uint32_t m = 0; m < kMine; ++m) {
      mask |= warp + kWarps * m < kChunks ? 3u << (2u * m) : 0u;
    }
    float v[4 * kMine];
    const bool ok = exchange_wait<2 * kMine>(
        state, b.step + 1u, mask,
        [&](uint32_t i) { return act + 4u * (lane + 32u * (warp + kWarps * (i >> 1))) + 2u * (i & 1u); },
        v);
#pragma unroll
    for (uint32_t m = 0; m < kMine; ++m) {
      x[m] = warp + kWarps * m < kChunks
                 ? make_float4(v[4 * m], v[4 * m + 1], v[4 * m + 2], v[4 * m + 3])
                 : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    if (__syncthreads_or(ok ? 0 : 1) != 0) {
      b.failed = true;
      b.consumed += block_config.ranges.of[kDown].end - block_config.ranges.of[kDown].begin;
      return;
    }
    trace_event(b, started);
  }
  float *partial = shared->reduce; // [kWarps][kSlots]
  const UnitRange range = block_config.ranges.of[kDown];
  const uint32_t units = range.end - range.begin;
  uint64_t *words = exchange_words(qd::kExchangeDown, qd::kHiddenSize, b.step);
  for (uint32_t batch = 0; batch < units; batch += kSlots) {
    const uint32_t count = min(kSlots, units - batch);
    const bool finisher = lane == 0 && warp < count; // finishes row `warp` of the batch
    const uint32_t mine = batch + warp;
    const float residual = finisher ? shared->hidden[range.begin + mine] : 0.0f;
    bool ok = true;
    if (warp < count) {
      const uint32_t n = b.consumed + batch + warp;
      const uint64_t t_before = block_config.unit_trace != nullptr ? dev::global_timer_ns() : 0;
      ok = wait_unit(b, state, n, make_tag(kDown, layer, range.begin + batch + warp)) != nullptr;
      if (lane == 0 && block_config.unit_trace != nullptr) {
        trace_unit(b, n, t_before, dev::global_timer_ns(), dev::global_timer_ns());
      }
    }
    // Every row of the batch has landed (its waiting warp checked the tag);
    // a failed wait in any warp (the run already carries the error) ends the
    // stage for the whole block.
    if (__syncthreads_or(ok ? 0 : 1) != 0) {
      break;
    }
    float a[8];
#pragma unroll
    for (uint32_t r = 0; r < 8; ++r) {
      a[r] = 0.0f;
    }
    const dev::Deadline deadline(block_config.limit_ms);
#pragma unroll
    for (uint32_t r = 0; r < kSlots; ++r) {
      if (r < count) {
        const uint32_t n = b.consumed + batch + r;
        const uint32_t slot = n % kSlots;
        // Acquire the slot's completed fill in this warp too: another warp saw
        // it complete, so this returns at once (the deadline only bounds it).
        dev::mbarrier_wait(&shared->full[slot], (n / kSlots) & 1u, deadline);
        const float4 *w = reinterpret_cast<const float4 *>(shared->ring + size_t{slot} * kSlotBytes);
#pragma unroll
        for (uint32_t m = 0; m < kMine; ++m) {
          const uint32_t k = warp + kWarps * m;
          if (k < kChunks) {
            const float4 v = w[lane + 32u * k];
            a[r] = fmaf(v.x, x[m].x, a[r]);
            a[r] = fmaf(v.y, x[m].y, a[r]);
            a[r] = fmaf(v.z, x[m].z, a[r]);
            a[r] = fmaf(v.w, x[m].w, a[r]);
          }
        }
      }
    }
    const float value = reduce_rows8(a, lane);
    if ((lane & 3u) == 0u && row < count) {
      partial[warp * kSlots + row] = value;
    }
    __syncthreads(); // partials written; every warp is done with the batch's slots
    if (finisher) {
      float sum = 0.0f;
#pragma unroll
      for (uint32_t w = 0; w < kWarps; ++w) {
        sum += partial[w * kSlots + warp];
      }
      const uint32_t u = range.begin + mine;
      dev::exchange_store(words + u, sum, b.step + 1u);
      c->projected[u] = sum;
      c->hidden[u] = residual + sum; // the residual for a launch that resumes here
      const uint32_t n = b.consumed + mine;
      if (!block_config.stream_empty &&
          position_cursor(block_config.map, slot_position[n % kSlots]).kind == kGateUp) {
        deferred_unit[n % kSlots] = n + kSlots; // see issue_deferred_refills
      } else {
        release_unit(b, n);
      }
    }
    __syncthreads(); // partials are rewritten by the next batch
  }
  b.consumed += units;
}

// Split-position decode attention for one (kv head, chunk) item: K/V tiles
// staged in shared memory, running softmax state per query head, partial
// (acc, max, sum) written to the workspace; the last item of the kv head to
// finish combines all chunks into the attention output (written over query).
__device__ void attention_item(QwenBlock &b, qd::Context *c, uint32_t group,
                               uint32_t chunk, uint32_t chunks, uint32_t positions,
                               uint32_t item, float *scratch) {
  FusedShared *s = block_config.shared;
  const uint32_t lane = threadIdx.x & 31u;
  const uint32_t warp = threadIdx.x >> 5u;
  const uint32_t per_chunk = (positions + chunks - 1u) / chunks;
  const uint32_t begin = min(positions, chunk * per_chunk);
  const uint32_t end = min(positions, begin + per_chunk);
  constexpr uint32_t kHeads = qd::kQueriesPerKvHead;
  constexpr uint32_t kOutputs = kHeads * qd::kHeadSize; // 448
  float *keys = scratch;                                 // [32][65]
  float *values = keys + kKvTile * kKeyStride;           // [32][64]
  float *scores = values + kKvTile * qd::kHeadSize;      // [7][32]
  float *query = scores + kHeads * kKvTile;              // [7][64]
  float *run_max = s->reduce;                            // [7]
  float *run_sum = s->reduce + 8;                        // [7]
  float *scale = s->reduce + 16;                         // [7]
  const uint32_t kv_offset = group * qd::kHeadSize;
  const uint32_t head0 = group * kHeads;
  for (uint32_t o = threadIdx.x; o < kOutputs; o += kThreads) {
    query[o] = dev::load_cg(c->query + head0 * qd::kHeadSize + o);
  }
  if (threadIdx.x < kHeads) {
    run_max[threadIdx.x] = -INFINITY;
    run_sum[threadIdx.x] = 0.0f;
  }
  float acc[2] = {0.0f, 0.0f};
  __syncthreads();
  for (uint32_t tile = begin; tile < end; tile += kKvTile) {
    const uint32_t count = min(kKvTile, end - tile);
    // Stage K (padded rows) and V: 32 positions x 16 float4 each; every
    // load of the thread is issued before its shared stores.
    constexpr uint32_t kStageLoads = kKvTile * 16u / kThreads;
    float4 k4[kStageLoads], v4[kStageLoads];
#pragma unroll
    for (uint32_t i = 0; i < kStageLoads; ++i) {
      const uint32_t v = threadIdx.x + i * kThreads, p = v / 16u, q4 = v % 16u;
      k4[i] = v4[i] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (p < count) {
        const size_t row = size_t{tile + p} * qd::kKvSize + kv_offset + 4u * q4;
        k4[i] = dev::load_cg4(c->key_cache + row);
        v4[i] = dev::load_cg4(c->value_cache + row);
      }
    }
#pragma unroll
    for (uint32_t i = 0; i < kStageLoads; ++i) {
      const uint32_t v = threadIdx.x + i * kThreads, p = v / 16u, q4 = v % 16u;
      float *k = keys + p * kKeyStride + 4u * q4;
      k[0] = k4[i].x;
      k[1] = k4[i].y;
      k[2] = k4[i].z;
      k[3] = k4[i].w;
      reinterpret_cast<float4 *>(values + p * qd::kHeadSize)[q4] = v4[i];
    }
    __syncthreads();
    if (threadIdx.x < kHeads * kKvTile) {
      const uint32_t h = threadIdx.x / kKvTile, p = threadIdx.x % kKvTile;
      float dot = -INFINITY;
      if (p < count) {
        const float *q = query + h * qd::kHeadSize;
        const float *k = keys + p * kKeyStride;
        float d0 = 0.0f, d1 = 0.0f;
#pragma unroll 16
        for (uint32_t d = 0; d < qd::kHeadSize; d += 2u) {
          d0 = fmaf(q[d], k[d], d0);
          d1 = fmaf(q[d + 1u], k[d + 1u], d1);
        }
        dot = (d0 + d1) * 0.125f; // 1/sqrt(head_dim)
      }
      scores[h * kKvTile + p] = dot;
    }
    __syncthreads();
    if (warp < kHeads) {
      const uint32_t h = warp;
      const float score = scores[h * kKvTile + lane];
      const float previous = run_max[h];
      const float next = fmaxf(previous, warp_all_max(score));
      const float e = lane < count ? expf(score - next) : 0.0f;
      scores[h * kKvTile + lane] = e;
      const float total = warp_all_sum(e);
      if (lane == 0) {
        const float alpha = expf(previous - next);
        scale[h] = alpha;
        run_sum[h] = run_sum[h] * alpha + total;
        run_max[h] = next;
      }
    }
    __syncthreads();
#pragma unroll
    for (uint32_t k = 0; k < 2; ++k) {
      const uint32_t o = threadIdx.x + k * kThreads;
      if (o < kOutputs) {
        const uint32_t h = o / qd::kHeadSize, d = o % qd::kHeadSize;
        const float *e = scores + h * kKvTile;
        float value = acc[k] * scale[h];
        for (uint32_t p = 0; p < count; ++p) {
          value = fmaf(e[p], values[p * qd::kHeadSize + d], value);
        }
        acc[k] = value;
      }
    }
    __syncthreads();
  }
  float *partial = block_config.workspace->attention_partials +
                   size_t{item} * kHeads * qd::kAttentionPartialStride;
#pragma unroll
  for (uint32_t k = 0; k < 2; ++k) {
    const uint32_t o = threadIdx.x + k * kThreads;
    if (o < kOutputs) {
      partial[(o / qd::kHeadSize) * qd::kAttentionPartialStride + o % qd::kHeadSize] = acc[k];
    }
  }
  if (threadIdx.x < kHeads) {
    partial[threadIdx.x * qd::kAttentionPartialStride + qd::kHeadSize] = run_max[threadIdx.x];
    partial[threadIdx.x * qd::kAttentionPartialStride + qd::kHeadSize + 1u] =
        run_sum[threadIdx.x];
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint32_t arrived =
        dev::fetch_add_acq_rel(&block_config.workspace->attention_arrivals[group], 1u) + 1u;
    s->broadcast = arrived == chunks ? 1u : 0u;
  }
  __syncthreads();
  if (s->broadcast == 0) {
    return;
  }
  // Last arrival: weights w_j = exp(m_j - M) / sum_j l_j exp(m_j - M) per head.
  const float *group_partials = block_config.workspace->attention_partials +
                                size_t{group * chunks} * kHeads * qd::kAttentionPartialStride;
  float *maxima = scratch;                                   // [chunks][7]
  float *sums = maxima + kMaxAttentionChunks * kHeads;       // [chunks][7]
  float *weights = sums + kMaxAttentionChunks * kHeads;      // [7][chunks]
  {
    // chunks * kHeads <= 128 * 7 = 896 entries: at most four per thread,
    // all loaded before any store.
    constexpr uint32_t kPerThread = (kMaxAttentionChunks * kHeads + kThreads - 1u) / kThreads;
    float m[kPerThread], l[kPerThread];
#pragma unroll
    for (uint32_t i = 0; i < kPerThread; ++i) {
      const uint32_t t = threadIdx.x + i * kThreads;
      const float *entry = group_partials + size_t{t} * qd::kAttentionPartialStride;
      m[i] = t < chunks * kHeads ? dev::load_cg(entry + qd::kHeadSize) : 0.0f;
      l[i] = t < chunks * kHeads ? dev::load_cg(entry + qd::kHeadSize + 1u) : 0.0f;
    }
#pragma unroll
    for (uint32_t i = 0; i < kPerThread; ++i) {
      const uint32_t t = threadIdx.x + i * kThreads;
      if (t < chunks * kHeads) {
        maxima[t] = m[i];
        sums[t] = l[i];
      }
    }
  }
  __syncthreads();
  if (warp < kHeads) {
    const uint32_t h = warp;
    float maximum = -INFINITY;
    for (uint32_t j = lane; j < chunks; j += 32u) {
      maximum = fmaxf(maximum, maxima[j * kHeads + h]);
    }
    maximum = warp_all_max(maximum);
    float denominator = 0.0f;
    for (uint32_t j = lane; j < chunks; j += 32u) {
      const float e = expf(maxima[j * kHeads + h] - maximum);
      weights[h * kMaxAttentionChunks + j] = e;
      denominator += e * sums[j * kHeads + h];
    }
    denominator = warp_all_sum(denominator);
    __syncwarp();
    for (uint32_t j = lane; j < chunks; j += 32u) {
      weights[h * kMaxAttentionChunks + j] /= denominator;
    }
  }
  __syncthreads();
  // Both outputs of the thread, six chunks at a time: all 12 loads of a
  // round are issued before the multiply-adds (which stay in chunk order).
  {
    const size_t stride = size_t{kHeads} * qd::kAttentionPartialStride;
    const float *entry[2];
    const float *w[2];
    bool valid[2];
    float value[2] = {0.0f, 0.0f};
#pragma unroll
    for (uint32_t k = 0; k < 2; ++k) {
      const uint32_t o = threadIdx.x + k * kThreads;
      valid[k] = o < kOutputs;
      const uint32_t h = valid[k] ? o / qd::kHeadSize : 0u, d = o % qd::kHeadSize;
      w[k] = weights + h * kMaxAttentionChunks;
      entry[k] = group_partials + h * qd::kAttentionPartialStride + d;
    }
    constexpr uint32_t kRound = 6;
    for (uint32_t j0 = 0; j0 < chunks; j0 += kRound) {
      float x[2][kRound];
#pragma unroll
      for (uint32_t k = 0; k < 2; ++k) {
#pragma unroll
        for (uint32_t j = 0; j < kRound; ++j) {
          x[k][j] = valid[k] && j0 + j < chunks ? dev::load_cg(entry[k] + (j0 + j) * stride)
                                                : 0.0f;
        }
      }
#pragma unroll
      for (uint32_t k = 0; k < 2; ++k) {
#pragma unroll
        for (uint32_t j = 0; j < kRound; ++j) {
          if (j0 + j < chunks) {
            value[k] = fmaf(w[k][j0 + j], x[k][j], value[k]);
          }
        }
      }
    }
#pragma unroll
    for (uint32_t k = 0; k < 2; ++k) {
      const uint32_t o = threadIdx.x + k * kThreads;
      if (valid[k]) {
        c->query[(head0 + o / qd::kHeadSize) * qd::kHeadSize + o % qd::kHeadSize] = value[k];
      }
    }
  }
  if (threadIdx.x == 0) {
    block_config.workspace->attention_arrivals[group] = 0; // next use follows a grid barrier
  }
  __syncthreads();
}

// Attention of this block's KV group over its slice of the positions
// (attention_slice), from shared memory: the slice's cached K/V rows arrive
// as the layer's three KV ring units (56 positions each: K then V, each as
// two 32-column boxes of 56 rows, 128-byte rows swizzled by XOR of the
// 16-byte chunk index with row % 8); the current position's K/V and the
// group's queries come from the qkv exchange. A local step's slice is every
// position, and the output, [head][dim] of the group, goes to input[0, 448).
// A spread step publishes the slice's partial state per query head instead:
// the unnormalised value sums, the score maximum and the sum of
// exp(score - maximum) (maximum -inf and zero sums for an empty slice).
__device__ __forceinline__ const float4 *kv_chunk(const unsigned char *unit, uint32_t row,
                                                   uint32_t chunk, uint32_t part) {
  // part 0: K, 1: V; chunk = float4 index 0..15 of the 64-float row.
  constexpr uint32_t kBox = kSlotBytes / 4u;
  return reinterpret_cast<const float4 *>(unit + (2u * part + (chunk >> 3)) * kBox + row * 128u +
                                          (((chunk & 7u) ^ (row & 7u)) << 4));
}

__device__ void group_attention(QwenBlock &b, sg::State *state, const qd::Context *c,
                                uint32_t layer) {
  FusedShared *s = block_config.shared;
  float *work = s->work;
  const uint32_t lane = threadIdx.x & 31u;
  const uint32_t warp = threadIdx.x >> 5u;
  const uint32_t group = block_config.group;
  const SpreadSlice slice = attention_slice(b.kv_length + 1u);
  // Score slot p < rows is cached row slice.first + p (unit p / 56, row
  // p % 56); slot `rows` is the current position when the slice has it.
  const uint32_t rows = slice.rows;
  const uint32_t positions = rows + (slice.current ? 1u : 0u);
  const bool spread = b.spread_attention;
  uint64_t *partial = block_config.attention_words +
                      (size_t{b.step & 1u} * block_config.workers + block_config.worker) *
                          qd::kSpreadWords;
  const uint32_t tag = b.step + 1u;
  constexpr uint32_t kHeads = qd::kQueriesPerKvHead;
  // Group entries of the qkv exchange: q [448], k [64], v [64]; thread t < 144
  // takes entries 4t..4t+3 (one region each).
  bool ok = true;
  const uint64_t started = trace_start();
  if (threadIdx.x < (kGroupColumns + 2u * qd::kHeadSize) / 4u) {
    const uint32_t e = 4u * threadIdx.x;
    uint32_t index;
    if (e < kGroupColumns) {
      index = group * kGroupColumns + e;
    } else if (e < kGroupColumns + qd::kHeadSize) {
      index = qd::kQuerySize + group * qd::kHeadSize + (e - kGroupColumns);
    } else {
      index = qd::kQuerySize + qd::kKvSize + group * qd::kHeadSize +
              (e - kGroupColumns - qd::kHeadSize);
    }
    // q lands at work[0, 448), current K at work[kLocalCurrent], V after it.
    float *destination = work + (e < kGroupColumns ? kLocalQuery + e
                                                   : kLocalCurrent + (e - kGroupColumns));
    const uint64_t *words =
        exchange_words(qd::kExchangeQkv, qd::kPackedQkvSize, b.step) + index;
    float v[4];
    ok = exchange_wait<2>(state, b.step + 1u, 3u, [&](uint32_t i) { return words + 2u * i; },
                          v);
    reinterpret_cast<float4 *>(destination)[0] = make_float4(v[0], v[1], v[2], v[3]);
  }
  // The three KV units (every warp waits; an empty unit completes at once).
  const unsigned char *units[kKvUnits];
#pragma unroll
  for (uint32_t j = 0; j < kKvUnits; ++j) {
    const float *slot = wait_unit(b, state, b.consumed + j, make_tag(kKv, layer, j));
    ok = ok && slot != nullptr;
    units[j] = reinterpret_cast<const unsigned char *>(slot);
  }
  if (__syncthreads_or(ok ? 0 : 1) != 0) {
    b.failed = true;
    return;
  }
  trace_event(b, started);
  // Scores: thread p computes position p for all seven heads (each K chunk
  // read once; the query chunks are warp-wide broadcasts).
  if (threadIdx.x < positions) {
    const uint32_t p = threadIdx.x;
    const uint32_t u = p / kKvUnitPositions, row = p - u * kKvUnitPositions;
    const unsigned char *unit = units[u < kKvUnits ? u : 0u];
    float acc[kHeads];
#pragma unroll
    for (uint32_t h = 0; h < kHeads; ++h) {
      acc[h] = 0.0f;
    }
#pragma unroll 4
    for (uint32_t j = 0; j < qd::kHeadSize / 4u; ++j) {
      const float4 k = p == rows
                           ? reinterpret_cast<const float4 *>(work + kLocalCurrent)[j]
                           : *kv_chunk(unit, row, j, 0);
#pragma unroll
      for (uint32_t h = 0; h < kHeads; ++h) {
        const float4 q =
            reinterpret_cast<const float4 *>(work + kLocalQuery + h * qd::kHeadSize)[j];
        acc[h] = fmaf(q.x, k.x, fmaf(q.y, k.y, fmaf(q.z, k.z, fmaf(q.w, k.w, acc[h]))));
      }
    }
#pragma unroll
    for (uint32_t h = 0; h < kHeads; ++h) {
      work[kLocalScores + h * kLocalAttentionLimit + p] = acc[h] * 0.125f; // 1/sqrt(64)
    }
  }
  static_assert(kLocalAttentionLimit <= kThreads, "one score row per thread");
  __syncthreads();
  // Softmax of head h in warp h: exp(score - max), and 1 / sum (local) or
  // (max, sum) published (spread).
  if (warp < kHeads) {
    float *scores = work + kLocalScores + warp * kLocalAttentionLimit;
    float maximum = -INFINITY;
    for (uint32_t p = lane; p < positions; p += 32u) {
      maximum = fmaxf(maximum, scores[p]);
    }
    maximum = warp_all_max(maximum);
    float sum = 0.0f;
    for (uint32_t p = lane; p < positions; p += 32u) {
      const float e = expf(scores[p] - maximum);
      scores[p] = e;
      sum += e;
    }
    sum = warp_all_sum(sum);
    if (lane == 0) {
      if (spread) {
        dev::exchange_store2(partial + warp * qd::kAttentionPartialStride + qd::kHeadSize,
                             maximum, sum, tag);
      } else {
        s->reduce[warp] = 1.0f / sum;
      }
    }
  }
  __syncthreads();
  // Weighted values: (head, 4 dims) item t % 112 over the even (t < 112) or
  // odd (112 <= t < 224) rows of each KV unit, then the current position;
  // the odd half is added through smem.
  constexpr uint32_t kItems = kGroupColumns / 4u; // 112
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  const uint32_t item = threadIdx.x % kItems, half = threadIdx.x / kItems;
  const uint32_t h = item / (qd::kHeadSize / 4u), chunk = item % (qd::kHeadSize / 4u);
  if (half < 2u) {
    const float *e = work + kLocalScores + h * kLocalAttentionLimit;
    // V chunk `chunk` of row r: box 2 + chunk / 8, 16-byte column
    // (chunk % 8) ^ (r % 8) of the 128-byte row.
    constexpr uint32_t kBox = kSlotBytes / 4u;
    const uint32_t box = (2u + (chunk >> 3)) * kBox;
    for (uint32_t u = 0; u * kKvUnitPositions < rows; ++u) {
      const unsigned char *base = units[u] + box;
      const uint32_t unit_rows = min(kKvUnitPositions, rows - u * kKvUnitPositions);
      const float *weights = e + u * kKvUnitPositions;
#pragma unroll 2
      for (uint32_t row = half; row < unit_rows; row += 2u) {
        const float weight = weights[row];
        const float4 x = *reinterpret_cast<const float4 *>(base + row * 128u +
                                                           (((chunk & 7u) ^ (row & 7u)) << 4));
        acc.x = fmaf(weight, x.x, acc.x);
        acc.y = fmaf(weight, x.y, acc.y);
        acc.z = fmaf(weight, x.z, acc.z);
        acc.w = fmaf(weight, x.w, acc.w);
      }
    }
    if (slice.current && half == (rows & 1u)) { // the current position, in its parity's half
      const float weight = e[rows];
      const float4 x = reinterpret_cast<const float4 *>(work + kLocalCurrent + qd::kHeadSize)[chunk];
      acc.x = fmaf(weight, x.x, acc.x);
      acc.y = fmaf(weight, x.y, acc.y);
      acc.z = fmaf(weight, x.z, acc.z);
      acc.w = fmaf(weight, x.w, acc.w);
    }
    if (half == 1u) {
      reinterpret_cast<float4 *>(work + kLocalPartial)[item] = acc;
    }
  }
  __syncthreads(); // also: every thread is done with the KV units
  if (lane == 0 && warp < kKvUnits) {
    release_unit(b, b.consumed + warp);
  }
  b.consumed += kKvUnits;
  if (half == 0u && spread) {
    const float4 other = reinterpret_cast<const float4 *>(work + kLocalPartial)[item];
    uint64_t *words = partial + h * qd::kAttentionPartialStride + 4u * chunk;
    dev::exchange_store2(words, acc.x + other.x, acc.y + other.y, tag);
    dev::exchange_store2(words + 2, acc.z + other.z, acc.w + other.w, tag);
  } else if (half == 0u) {
    const float4 other = reinterpret_cast<const float4 *>(work + kLocalPartial)[item];
    const float inverse = s->reduce[h];
    const float4 out = make_float4((acc.x + other.x) * inverse, (acc.y + other.y) * inverse,
                                   (acc.z + other.z) * inverse, (acc.w + other.w) * inverse);
    reinterpret_cast<float4 *>(s->input)[item] = out;
    if (block_config.group_writer) {
      // The reference leaves the attention output in the query buffer.
      reinterpret_cast<float4 *>(c->query + group * kGroupColumns)[item] = out;
    }
  }
  __syncthreads();
}

// Merges the softmax partial state (m2, l2, x2, y2) into (m, l, x, y): both
// sums rescaled to the larger maximum; an empty state (maximum -inf) adds
// nothing.
__device__ __forceinline__ void merge_partial(float &m, float &l, float &x, float &y, float m2,
                                              float l2, float x2, float y2) {
  const float top = fmaxf(m, m2);
  const float s1 = m == -INFINITY ? 0.0f : expf(m - top);
  const float s2 = m2 == -INFINITY ? 0.0f : expf(m2 - top);
  l = l * s1 + l2 * s2;
  x = x * s1 + x2 * s2;
  y = y * s1 + y2 * s2;
  m = top;
}

// Spread attention, second half: the group's blocks' partial states merged
// into the attention output. Item i < 224 of a group is dims 2(i % 32),
// 2(i % 32) + 1 of head i / 32 and belongs to warp i % 8 of the group's
// block size - 1 - i / 8 (the group's last 28 blocks, or several items per
// warp in smaller groups). Lane l merges the partial states of the group's
// blocks l, l + 32, ... in order, the lanes then merge pairwise (xor
// butterfly), and lane 0 publishes value sum / exp sum to the attention
// exchange and, where the reference leaves the attention output, to the
// query buffer.
__device__ void spread_combine(QwenBlock &b, sg::State *state, qd::Context *c) {
  const uint32_t lane = threadIdx.x & 31u;
  const uint32_t warp = threadIdx.x >> 5u;
  const uint32_t size = block_config.group_size;
  const uint32_t group = block_config.group;
  const uint32_t workers = block_config.workers;
  const uint64_t *partials =
      block_config.attention_words +
      (size_t{b.step & 1u} * workers + (group == 0u ? 0u : attention_split(workers))) *
          qd::kSpreadWords;
  uint64_t *outputs =
      exchange_words(qd::kExchangeAttention, qd::kQuerySize, b.step) + group * kGroupColumns;
  const uint32_t tag = b.step + 1u;
  constexpr uint32_t kItems = kGroupColumns / 2u;
  constexpr uint32_t kPerLane = 3; // partial states per lane and poll round
  bool ok = true;
  for (uint32_t item = (size - 1u - block_config.group_rank) * kWarps + warp; item < kItems;
       item += kWarps * size) {
    const uint32_t head = item / 32u, dim = 2u * (item % 32u);
    const uint64_t *entry = partials + head * qd::kAttentionPartialStride;
    float m = -INFINITY, l = 0.0f, x = 0.0f, y = 0.0f;
    for (uint32_t round = 0; round < size; round += 32u * kPerLane) {
      uint32_t mask = 0;
      float v[4 * kPerLane];
#pragma unroll
      for (uint32_t k = 0; k < kPerLane; ++k) {
        mask |= round + lane + 32u * k < size ? 3u << (2u * k) : 0u;
        v[4 * k] = -INFINITY;
        v[4 * k + 1] = v[4 * k + 2] = v[4 * k + 3] = 0.0f;
      }
      // Pair 2k: (maximum, exp sum) of block round + lane + 32k; pair
      // 2k + 1: its value sums at dims (dim, dim + 1).
      ok = exchange_wait<2 * kPerLane>(
               state, tag, mask,
               [&](uint32_t i) {
                 return entry + size_t{round + lane + 32u * (i >> 1)} * qd::kSpreadWords +
                        ((i & 1u) != 0u ? dim : qd::kHeadSize);
               },
               v) &&
           ok;
      if (!__all_sync(kFullMask, ok)) {
        break;
      }
#pragma unroll
      for (uint32_t k = 0; k < kPerLane; ++k) {
        merge_partial(m, l, x, y, v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]);
      }
    }
    if (!__all_sync(kFullMask, ok)) {
      ok = false;
      break;
    }
#pragma unroll
    for (uint32_t offset = 16; offset != 0; offset >>= 1) {
      merge_partial(m, l, x, y, __shfl_xor_sync(kFullMask, m, offset),
                    __shfl_xor_sync(kFullMask, l, offset), __shfl_xor_sync(kFullMask, x, offset),
                    __shfl_xor_sync(kFullMask, y, offset));
    }
    if (lane == 0) {
      const float first = x / l, second = y / l;
      dev::exchange_store2(outputs + head * qd::kHeadSize + dim, first, second, tag);
      *reinterpret_cast<float2 *>(c->query + group * kGroupColumns + head * qd::kHeadSize +
                                  dim) = make_float2(first, second);
    }
  }
  if (__syncthreads_or(ok ? 0 : 1) != 0) {
    b.failed = true;
  }
}

__device__ void fused_attention(QwenBlock &b, sg::State *state, qd::Context *c,
                                uint32_t layer) {
  issue_deferred_refills(b); // gate/up units the last down stage postponed
  const uint32_t positions = b.kv_length + 1u;
  if (b.spread_attention) {
    group_attention(b, state, c, layer);
    if (b.failed) {
      return;
    }
    trace_mark(b, 3);
    spread_combine(b, state, c);
    trace_mark(b, 11);
    return;
  }
  if (!b.split_attention) {
    return; // computed per block inside the o_proj stage
  }
  // The layer's KV units carry no bytes for a split step; the first one's
  // slot serves as staging and combine scratch until they are released.
  bool ok = true;
  float *scratch = nullptr;
#pragma unroll
  for (uint32_t j = 0; j < kKvUnits; ++j) {
    const float *slot = wait_unit(b, state, b.consumed + j, make_tag(kKv, layer, j));
    ok = ok && slot != nullptr;
    scratch = j == 0 ? const_cast<float *>(slot) : scratch;
  }
  if (__syncthreads_or(ok ? 0 : 1) != 0) {
    b.failed = true;
    return;
  }
  uint32_t chunks = (positions + 15u) / 16u;
  chunks = min(chunks, max(1u, min(block_config.workers / 2u, kMaxAttentionChunks)));
  const uint32_t items = qd::kKvHeads * chunks;
  for (uint32_t item = block_config.worker; item < items; item += block_config.workers) {
    attention_item(b, c, item / chunks, item % chunks, chunks, positions, item, scratch);
  }
  __syncthreads();
  if ((threadIdx.x & 31u) == 0 && (threadIdx.x >> 5u) < kKvUnits) {
    release_unit(b, b.consumed + (threadIdx.x >> 5u));
  }
  b.consumed += kKvUnits;
}

// LM head: lane 0 of each warp keeps its own best (value, index) per Program
// task in shared memory; the block merges them per task and publishes
// candidate slot (worker + task) in the workspace.
__device__ void fused_lm_head(QwenBlock &b, sg::State *state, const sg::Stage &stage,
                              const sg::Task *tasks) {
  FusedShared *s = block_config.shared;
  const uint32_t warp = threadIdx.x >> 5u;
  const uint32_t task_count = stage.task_count;
  float *best_values = s->work;                                   // [8][32]
  uint32_t *best_indices =
      reinterpret_cast<uint32_t *>(best_values + kWarps * qd::kMaximumLmHeadPartitions);
  uint32_t *task_ends = best_indices + kWarps * qd::kMaximumLmHeadPartitions; // [32]
  for (uint32_t t = threadIdx.x; t < kWarps * qd::kMaximumLmHeadPartitions; t += kThreads) {
    best_values[t] = -INFINITY;
    best_indices[t] = UINT32_MAX;
  }
  if (threadIdx.x < task_count) {
    task_ends[threadIdx.x] = tasks[stage.task_offset + threadIdx.x].end;
  }
  __syncthreads();
  const UnitRange range = block_config.ranges.of[kLmHead];
  uint32_t task = 0; // lane 0's cursor: rows of a warp only increase
  const uint32_t first_row = range.begin * kSlotRows;
  while (task + 1u < task_count && task_ends[task] <= first_row) {
    ++task;
  }
  float *mine = best_values + warp * qd::kMaximumLmHeadPartitions;
  uint32_t *mine_index = best_indices + warp * qd::kMaximumLmHeadPartitions;
  auto offer = [&](uint32_t row, float value) {
    while (row >= task_ends[task]) {
      ++task;
    }
    if (better_top1(value, row, mine[task], mine_index[task])) {
      mine[task] = value;
      mine_index[task] = row;
    }
  };
  consume_units(
      b, state, kLmHead, 0,
      [&](uint32_t u, uint32_t row, float value, bool valid, float4) {
        const uint32_t lane = threadIdx.x & 31u;
        const uint32_t first = u * kSlotRows;
        const uint32_t rows = min(kSlotRows, block_config.vocab - first);
        if (block_config.logits != nullptr && valid && (lane & 3u) == 0u) {
          block_config.logits[first + row] = value; // opt-in capture for tests
        }
        uint32_t task_end = 0;
        if (lane == 0) {
          while (first >= task_ends[task]) {
            ++task;
          }
          task_end = task_ends[task];
        }
        task_end = __shfl_sync(kFullMask, task_end, 0);
        if (first + rows <= task_end) {
          // The whole unit lies in one task: warp top-1 (ties to the lower
          // row), then one offer.
          float best = valid ? value : -INFINITY;
          uint32_t index = valid ? first + row : UINT32_MAX;
#pragma unroll
          for (uint32_t offset = 4; offset < 32; offset *= 2) {
            const float other = __shfl_xor_sync(kFullMask, best, offset);
            const uint32_t other_index = __shfl_xor_sync(kFullMask, index, offset);
            if (better_top1(other, other_index, best, index)) {
              best = other;
              index = other_index;
            }
          }
          if (lane == 0) {
            offer(index, best);
          }
        } else {
          // A task boundary inside the unit: offer row by row.
#pragma unroll
          for (uint32_t r = 0; r < kSlotRows; ++r) {
            const float v = __shfl_sync(kFullMask, value, 4u * r);
            if (lane == 0 && r < rows) {
              offer(first + r, v);
            }
          }
        }
      });
  __syncthreads();
  if (threadIdx.x < task_count && range.begin < range.end) {
    const uint32_t t = threadIdx.x;
    const uint32_t task_begin = tasks[stage.task_offset + t].begin;
    const uint32_t rows_end = min(range.end * kSlotRows, block_config.vocab);
    if (task_begin < rows_end && task_ends[t] > first_row) {
      float value = -INFINITY;
      uint32_t index = UINT32_MAX;
      for (uint32_t w = 0; w < kWarps; ++w) {
        const uint32_t slot = w * qd::kMaximumLmHeadPartitions + t;
        if (better_top1(best_values[slot], best_indices[slot], value, index)) {
          value = best_values[slot];
          index = best_indices[slot];
        }
      }
      block_config.workspace->top1_values[block_config.worker + t] = value;
      block_config.workspace->top1_indices[block_config.worker + t] = index;
    }
  }
}

// Per-task top-1 over the candidate slots (loaded in one parallel pass), then
// the reference reduce_top1 over the per-task partials.
__device__ void fused_reduce_top1(QwenBlock &b, const sg::Stage &stage,
                                  const sg::Task *tasks, qd::Context *c) {
  FusedShared *s = block_config.shared;
  const sg::Task *lm_tasks = tasks + stage.task_offset;
  qd::TailContext *tail = c->tail;
  const uint32_t slots = block_config.workers + stage.task_count;
  float *values = s->work;
  uint32_t *indices = reinterpret_cast<uint32_t *>(s->work + 512);
  float *partial_values = s->work + 1024;
  uint32_t *partial_indices = reinterpret_cast<uint32_t *>(s->work + 1024 + 64);
  for (uint32_t t = threadIdx.x; t < slots; t += kThreads) {
    values[t] = dev::load_cg(block_config.workspace->top1_values + t);
    indices[t] = dev::load_cg(block_config.workspace->top1_indices + t);
  }
  __syncthreads();
  if (threadIdx.x < stage.task_count) {
    const sg::Task &task = lm_tasks[threadIdx.x];
    const uint32_t first = even_owner(task.begin / kSlotRows, block_config.lm_units, block_config.workers);
    const uint32_t last = even_owner((task.end - 1u) / kSlotRows, block_config.lm_units, block_config.workers);
    float best_value = -INFINITY;
    uint32_t best_index = UINT32_MAX;
    for (uint32_t w = first; w <= last; ++w) {
      if (better_top1(values[w + threadIdx.x], indices[w + threadIdx.x], best_value,
                      best_index)) {
        best_value = values[w + threadIdx.x];
        best_index = indices[w + threadIdx.x];
      }
    }
    tail->partial_max_values[task.argument0] = best_value;
    tail->partial_max_indices[task.argument0] = best_index;
    partial_values[task.argument0] = best_value;
    partial_indices[task.argument0] = best_index;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    // Reference reduce_top1 (:339-356) over the partials.
    float best_value = partial_values[0];
    uint32_t best_index = partial_indices[0];
    for (uint32_t p = 1; p < tail->partition_count; ++p) {
      if (better_top1(partial_values[p], partial_indices[p], best_value, best_index)) {
        best_value = partial_values[p];
        best_index = partial_indices[p];
      }
    }
    tail->decode_state->sampled_logit = best_value;
    tail->decode_state->sampled_token = best_index;
  }
  __syncthreads();
}

// Is the graph exactly the reference Qwen table (qwen_stateful_graph.cpp
// :368-485, any partition counts) compiled into its natural stages?
__device__ bool canonical_table(const sg::ResidentArgs &args, uint32_t vocab) {
  if (args.program_count != 3) {
    return false;
  }
  const sg::Program *programs = args.programs;
  if (programs[0].flags != 0 || programs[0].next_program != 1 ||
      programs[1].flags != (sg::kProgramAdvancesStep | sg::kProgramBranchesOnState) ||
      programs[1].next_program != 0 || programs[1].branch_program != 2 ||
      programs[2].flags != sg::kProgramEvaluatesPredicate ||
      programs[2].next_program != 0) {
    return false;
  }
  struct Expected {
    qd::Opcode opcode;
    uint32_t end; // union of task ranges is [0, end)
  };
  const Expected expected[3][5] = {
      {{qd::Opcode::attention_rmsnorm_f32, qd::kHiddenSize},
       {qd::Opcode::qkv_projection_f32, qd::kPackedQkvSize},
       {qd::Opcode::rope_kv_cache_f32, qd::kRotaryHeads},
       {qd::Opcode::grouped_query_attention_f32, qd::kAttentionHeads},
       {qd::Opcode::attention_output_residual_f32, qd::kHiddenSize}},
      {{qd::Opcode::mlp_rmsnorm_f32, qd::kHiddenSize},
       {qd::Opcode::gate_up_silu_f32, qd::kIntermediateSize},
       {qd::Opcode::down_matvec_f32, qd::kHiddenSize},
       {qd::Opcode::residual_advance, qd::kHiddenSize},
       {qd::Opcode::residual_advance, 0}},
      {{qd::Opcode::final_rmsnorm_f32, qd::kHiddenSize},
       {qd::Opcode::lm_head_top1_partition_f32, vocab},
       {qd::Opcode::top1_reduce, 0},
       {qd::Opcode::embedding_feedback_f32, qd::kHiddenSize},
       {qd::Opcode::residual_advance, 0}}};
  const uint32_t stage_counts[3] = {5, 4, 4};
  for (uint32_t p = 0; p < 3; ++p) {
    const sg::CompiledProgram compiled = args.compiled_programs[p];
    if (compiled.stage_count != stage_counts[p]) {
      return false;
    }
    for (uint32_t s = 0; s < compiled.stage_count; ++s) {
      const sg::Stage stage = args.stages[compiled.stage_offset + s];
      const Expected want = expected[p][s];
      uint32_t next = 0;
      for (uint32_t t = 0; t < stage.task_count; ++t) {
        const sg::Task &task = args.tasks[stage.task_offset + t];
        if (opcode_of(task) != want.opcode) {
          return false;
        }
        if (want.opcode == qd::Opcode::top1_reduce ||
            want.opcode == qd::Opcode::rope_kv_cache_f32) {
          continue;
        }
        if (task.begin != next) {
          return false;
        }
        if (want.opcode == qd::Opcode::lm_head_top1_partition_f32 && task.argument0 != t) {
          return false;
        }
        next = task.end;
      }
      if (want.opcode != qd::Opcode::top1_reduce &&
          want.opcode != qd::Opcode::rope_kv_cache_f32 && next != want.end) {
        return false;
      }
      const bool single = want.opcode == qd::Opcode::attention_rmsnorm_f32 ||
                          want.opcode == qd::Opcode::mlp_rmsnorm_f32 ||
                          want.opcode == qd::Opcode::final_rmsnorm_f32 ||
                          want.opcode == qd::Opcode::rope_kv_cache_f32 ||
                          want.opcode == qd::Opcode::residual_advance ||
                          want.opcode == qd::Opcode::top1_reduce ||
                          want.opcode == qd::Opcode::embedding_feedback_f32;
      if (single && stage.task_count != 1) {
        return false;
      }
    }
  }
  return true;
}

__device__ __forceinline__ bool aligned16(const void *pointer) {
  return (reinterpret_cast<uintptr_t>(pointer) & 15u) == 0;
}

// Fused-path preconditions; every block evaluates the same data.
__device__ bool fused_possible(const sg::ResidentArgs &args, uint32_t workers) {
  const auto *contexts = static_cast<const qd::Context *>(args.context);
  const qd::TailContext *tail = contexts[0].tail;
  const qd::Workspace *workspace = tail->workspace;
  // Every block owns at least one down row (so every block publishes to the
  // exchange that gates the next layer) and each KV group has a block; a
  // launch never starts between Programs 0 and 1 (runs only stop after
  // Program 1 or 2), so the residual it starts from is in global memory.
  if (workspace == nullptr || workspace->magic != qd::kWorkspaceMagic ||
      workspace->worker_capacity < max(workers, 2u) || workspace->exchange == nullptr ||
      workspace->attention_words == nullptr || !aligned16(workspace->attention_words) ||
      workspace->kv_maps == nullptr ||
      (reinterpret_cast<uintptr_t>(workspace->kv_maps) & 63u) != 0 ||
      !aligned16(workspace->exchange) || workers < 2u || workers > kDownUnits ||
      sg::phase_program(dev::load_relaxed(&args.state->phase)) == 1u ||
      dev::dynamic_shared_bytes() < kFusedSharedBytes || gridDim.x != workers ||
      contexts[0].layer_count > kMaxFusedLayers || tail->vocab_size >= (1u << 23) ||
      !aligned16(tail->lm_head_weight) || !aligned16(tail->final_norm_weight) ||
      !aligned16(tail->final_normalized)) {
    return false;
  }
  for (uint32_t l = 0; l < contexts[0].layer_count; ++l) {
    const qd::Context &c = contexts[l];
    if (!aligned16(c.q_weight) || !aligned16(c.k_weight) || !aligned16(c.v_weight) ||
        !aligned16(c.out_weight) || !aligned16(c.gate_weight) ||
        !aligned16(c.up_weight) || !aligned16(c.down_weight) || !aligned16(c.hidden) ||
        !aligned16(c.query) || !aligned16(c.activated) ||
        !aligned16(c.attention_norm_weight) || !aligned16(c.mlp_norm_weight) ||
        !aligned16(c.attention_normalized) || !aligned16(c.mlp_normalized)) {
      return false;
    }
  }
  return canonical_table(args, tail->vocab_size);
}

// Zeroes the exchange words this block publishes (both parities) before the
// launch returns, so a later launch, whose steps count from zero again,
// never mistakes them for its own.
__device__ void clear_exchange() {
  uint64_t *x = block_config.exchange;
  const UnitRanges &r = block_config.ranges;
  const uint32_t qkv = r.of[kQkv].end - r.of[kQkv].begin;   // 8 rows each
  const uint32_t out = r.of[kOut].end - r.of[kOut].begin;   // kORows rows each
  const uint32_t gu = r.of[kGateUp].end - r.of[kGateUp].begin; // 4 rows each
  const uint32_t down = r.of[kDown].end - r.of[kDown].begin;
  const uint32_t words = 8u * qkv + kORows * out + 4u * gu + down;
  for (uint32_t i = threadIdx.x; i < 2u * words; i += kThreads) {
    const uint32_t parity = i / words;
    uint32_t k = i % words;
    uint32_t index;
    if (k < 8u * qkv) {
      const uint32_t u = r.of[kQkv].begin + k / 8u, row = k % 8u;
      const QkvRows rows = qkv_rows(u, row % 4u);
      const uint32_t base = rows.which == 0 ? 0u
                            : rows.which == 1 ? qd::kQuerySize
                                              : qd::kQuerySize + qd::kKvSize;
      index = qd::kExchangeQkv + parity * qd::kPackedQkvSize + base +
              (row < 4u ? rows.first : rows.second);
    } else if ((k -= 8u * qkv) < kORows * out) {
      const uint32_t u = r.of[kOut].begin + k / kORows;
      index = qd::kExchangeOut + parity * qd::kKvHeads * qd::kHiddenSize +
              (u / kOGroupUnits) * qd::kHiddenSize + (u % kOGroupUnits) * kORows + k % kORows;
    } else if ((k -= kORows * out) < 4u * gu) {
      index = qd::kExchangeAct + parity * qd::kIntermediateSize +
              (r.of[kGateUp].begin + k / 4u) * kGuRowsPerUnit + k % 4u;
    } else {
      k -= 4u * gu;
      index = qd::kExchangeDown + parity * qd::kHiddenSize + r.of[kDown].begin + k;
    }
    x[index] = 0;
  }
  // Spread attention: this block's partial states and the outputs of its
  // combine items (see spread_combine), both parities.
  uint64_t *partial = block_config.attention_words + size_t{block_config.worker} * qd::kSpreadWords;
  for (uint32_t i = threadIdx.x; i < qd::kSpreadWords; i += kThreads) {
    partial[i] = 0;
    partial[size_t{block_config.workers} * qd::kSpreadWords + i] = 0;
  }
  const uint32_t size = block_config.group_size;
  const uint32_t lane = threadIdx.x & 31u;
  for (uint32_t item = (size - 1u - block_config.group_rank) * kWarps + (threadIdx.x >> 5u);
       lane < 4u && item < kGroupColumns / 2u; item += kWarps * size) {
    // lane: parity * 2 + which of the item's two dims
    x[qd::kExchangeAttention + (lane >> 1) * qd::kQuerySize + block_config.group * kGroupColumns +
      (item / 32u) * qd::kHeadSize + 2u * (item % 32u) + (lane & 1u)] = 0;
  }
}

// =============================================================== workloads ==

template <bool kStageProfile> struct QwenWorkloadT {
  using Block = QwenBlock;
  static constexpr bool kTraceBarriers = kStageProfile;

  // Stage-profile runs: every block records when it arrived at and left each
  // grid barrier into StageProfile.entries[barrier * workers + worker] when
  // the host bound an entry array.
  __device__ static void trace_barrier(QwenBlock &b, void *opaque, const sg::Stage &,
                                       const sg::Task *, uint64_t arrive_ns,
                                       uint64_t leave_ns) {
    if (b.fused) { // the entries pointer is cached in shared memory
      if (block_config.event_trace != nullptr) {
        const uint64_t index =
            uint64_t{b.traced_barriers} * block_config.workers + block_config.worker;
        if (index < block_config.event_capacity) {
          block_config.event_trace[index] = {arrive_ns, leave_ns};
        }
      }
      ++b.traced_barriers;
      return;
    }
    auto *contexts = static_cast<qd::Context *>(opaque);
    qd::StageProfile *profile = contexts[0].tail->stage_profile;
    if (profile != nullptr && profile->entries != nullptr) {
      const uint64_t index = uint64_t{b.traced_barriers} * block_config.workers + block_config.worker;
      if (index < profile->entry_count) {
        profile->entries[index] = {arrive_ns, leave_ns};
      }
    }
    ++b.traced_barriers;
  }

  __device__ static bool valid_context(const sg::State *, void *opaque) {
    return valid_qwen_contexts(static_cast<qd::Context *>(opaque));
  }
  __device__ static bool valid_task(const sg::Task &task, void *opaque) {
    return valid_qwen_task(task, static_cast<qd::Context *>(opaque));
  }
  __device__ static void execute(const sg::Task &task, sg::State *state, void *opaque) {
    generic_execute(task, state, layer_context(opaque, state));
  }

  __device__ static void begin(QwenBlock &b, const sg::ResidentArgs &args) {
    b = QwenBlock{};
    QwenConfig &k = block_config;
    extern __shared__ __align__(128) unsigned char dynamic_shared[];
    // The ring's KV units need 1024-byte aligned slots (128-byte swizzle).
    FusedShared *s = reinterpret_cast<FusedShared *>(
        (reinterpret_cast<uintptr_t>(dynamic_shared) + kFusedSharedAlign - 1u) &
        ~uintptr_t{kFusedSharedAlign - 1u});
    if (threadIdx.x == 0) {
      k = QwenConfig{};
      k.worker = blockIdx.x;
      k.workers = dev::load_relaxed(&args.state->worker_count);
      k.limit_ms = dev::detail::wait_limit_ms(args.reserved);
      const bool fused = fused_possible(args, k.workers);
      k.contexts = static_cast<const qd::Context *>(args.context);
      k.workspace = k.contexts[0].tail->workspace;
      k.group = attention_group(k.worker, k.workers);
      k.group_rank = group_rank(k.worker, k.workers);
      k.group_size = group_size(k.group, k.workers);
      k.group_writer = k.worker == 0 || k.worker == attention_split(k.workers);
      if (blockIdx.x == 0 && k.workspace != nullptr) {
        k.workspace->reserved[0] = fused ? 1u : 2u; // which path ran
      }
      if (fused) { // k.shared stays null on the generic path
        k.shared = s;
        k.lm_head = k.contexts[0].tail->lm_head_weight;
        k.exchange = k.workspace->exchange;
        k.attention_words = k.workspace->attention_words;
        k.kv_maps = static_cast<const unsigned char *>(k.workspace->kv_maps);
        k.logits = k.workspace->logits;
        k.layers = k.contexts[0].layer_count;
        k.vocab = k.contexts[0].tail->vocab_size;
        k.lm_units = lm_units_for(k.vocab);
        k.lm_stage = args.stages[args.compiled_programs[2].stage_offset + 1u];
        k.ranges = unit_ranges(k.worker, k.workers, k.vocab);
        k.policy = dev::l2_evict_first_policy();
        // The stream starts where the initial Program starts (see make_stream_map).
        k.unit_trace = kStageProfile && k.worker == 0 ? k.contexts[0].tail->stage_profile
                                                     : nullptr;
        if (kStageProfile && k.contexts[0].tail->stage_profile != nullptr) {
          k.event_trace = k.contexts[0].tail->stage_profile->entries;
          k.event_capacity = k.contexts[0].tail->stage_profile->entry_count / 2u;
        }
        unit_trace_position = 0;
        const uint32_t program = sg::phase_program(dev::load_relaxed(&args.state->phase));
        const uint32_t step = dev::load_relaxed(&args.state->step);
        k.map = make_stream_map(k.ranges, k.layers, program, step % k.layers);
        // Program 2 of token t runs at step (t + 1) * layers, before the
        // feedback that advances the decode state: a launch starting there is
        // one token behind its step.
        const qd::DecodeState *decode = k.contexts[0].tail->decode_state;
        k.base_position = decode_field(&decode->token_position);
        k.base_kv_length = decode_field(&decode->kv_length);
        k.base_token = static_cast<int32_t>(step / k.layers) - (program == 2 ? 1 : 0);
        const sg::Stage *stages = args.stages;
        const sg::CompiledProgram *compiled = args.compiled_programs;
        k.epsilon[0] = __uint_as_float(args.tasks[stages[compiled[0].stage_offset].task_offset].argument0);
        k.epsilon[1] = __uint_as_float(args.tasks[stages[compiled[1].stage_offset].task_offset].argument0);
        k.epsilon[2] = __uint_as_float(args.tasks[stages[compiled[2].stage_offset].task_offset].argument0);
        const sg::Task &advance = args.tasks[stages[compiled[1].stage_offset + 3u].task_offset];
        k.residual_argument[0] = advance.argument0;
        k.residual_argument[1] = advance.argument1;
        k.stream_empty = units_per_cycle(k.ranges, k.layers) == 0;
      }
    }
    __syncthreads();
    b.fused = k.shared != nullptr;
    if (!b.fused) {
      return;
    }
    for (uint32_t i = threadIdx.x; i < block_config.layers * kLayerMatrices; i += kThreads) {
      const qd::Context &layer = block_config.contexts[i / kLayerMatrices];
      const float *pointers[kLayerMatrices] = {layer.q_weight,    layer.k_weight,
                                               layer.v_weight,    layer.out_weight,
                                               layer.gate_weight, layer.up_weight,
                                               layer.down_weight};
      s->layer_weights[i / kLayerMatrices][i % kLayerMatrices] = pointers[i % kLayerMatrices];
    }
    fetch_layer_context(dev::load_relaxed(&args.state->step));
    if (threadIdx.x < kSlots) {
      deferred_unit[threadIdx.x] = UINT32_MAX;
      s->pair_done[threadIdx.x] = 0;
      s->rows_done[threadIdx.x] = 0;
      s->sequence[threadIdx.x] = UINT32_MAX;
      s->unit_tag[threadIdx.x] = 0;
    }
    if (threadIdx.x == 0) {
      for (uint32_t slot = 0; slot < kSlots; ++slot) {
        dev::mbarrier_init(&s->full[slot], 1);
      }
      dev::mbarrier_init_fence();

      if (block_config.worker == 0) {
        // A launch that stopped early may have left arrivals behind. No block
        // reaches attention before passing the first barrier, which block 0
        // joins only after this reset.
        for (uint32_t g = 0; g < qd::kKvHeads; ++g) {
          block_config.workspace->attention_arrivals[g] = 0;
        }
      }
    }
    __syncthreads();
    if (threadIdx.x == 0 && !block_config.stream_empty) {
      for (uint32_t n = 0; n < kSlots; ++n) {
        slot_position[n] = stream_position(block_config.map, n);
      }
      for (uint32_t n = 0; n < kSlots; ++n) {
        issue_unit(b, n);
      }
    }
  }

  __device__ static void end(QwenBlock &b) {
    if (!b.fused) {
      return;
    }
    // Wait for copies still in flight into this block's ring before exit.
    wait_prefetched_context();
    __syncthreads();
    if (threadIdx.x == 0) {
      const dev::Deadline deadline(block_config.limit_ms);
      for (uint32_t slot = 0; slot < kSlots; ++slot) {
        const uint32_t n = block_config.shared->sequence[slot];
        if (n != UINT32_MAX && n >= b.consumed &&
            !dev::mbarrier_wait(&block_config.shared->full[slot], (n / kSlots) & 1u, deadline)) {
          break;
        }
      }
    }
    clear_exchange();
    __syncthreads();
  }

  __device__ static bool local_transitions(const QwenBlock &b) { return b.fused; }
  __device__ static void barrier_poll(QwenBlock &) {}
  // Programs 0 and 1 hand their results on through the exchange words; only
  // the tail (LM-head candidates, the sampled token's embedding, the stop
  // predicate) ends with a grid barrier.
  __device__ static bool barrier_at_end(const QwenBlock &b) {
    return !b.fused || b.program == 2u;
  }
  __device__ static void program_begin(QwenBlock &b, uint32_t program, uint32_t step) {
    b.program = program;
    b.step = step;
    if (b.fused) {
      const int32_t tokens = static_cast<int32_t>(step / block_config.layers) -
                             block_config.base_token;
      b.position = block_config.base_position + static_cast<uint32_t>(tokens);
      b.kv_length = block_config.base_kv_length + static_cast<uint32_t>(tokens);
      const AttentionMode mode = attention_mode(b.kv_length + 1u, block_config.workers);
      b.split_attention = mode == AttentionMode::split;
      b.spread_attention = mode == AttentionMode::spread;
      if (program == 1) {
        // Completed in this Program's residual_advance stage, read after the
        // block syncs of its final barrier.
        prefetch_layer_context(step + 1u);
      }
    }
  }
  __device__ static void stage_begin(QwenBlock &b, uint32_t stage) { b.stage = stage; }
  __device__ static uint32_t branch_value(QwenBlock &b, const sg::State *state) {
    if (b.fused) {
      return fused_layer_boundary(b.step) ? 1u : 0u; // what residual_advance writes
    }
    return dev::load_relaxed(&state->branch_value);
  }

  __device__ static bool barrier_after(QwenBlock &b, const sg::Stage &stage,
                                       const sg::Stage &next, const sg::Task *tasks) {
    if (!b.fused) {
      return true;
    }
    const qd::Opcode op = fused_opcode(b.program, b.stage);
    const qd::Opcode following = fused_opcode(b.program, b.stage + 1u);
    switch (op) {
    case qd::Opcode::attention_rmsnorm_f32: // norm recomputed per block
    case qd::Opcode::mlp_rmsnorm_f32:
    case qd::Opcode::final_rmsnorm_f32:
    case qd::Opcode::qkv_projection_f32: // RoPE + KV append in its epilogue
    case qd::Opcode::gate_up_silu_f32:   // act exchange
    case qd::Opcode::down_matvec_f32:    // down exchange
    case qd::Opcode::top1_reduce:        // feedback runs in the same block
      return false;
    case qd::Opcode::rope_kv_cache_f32:
      // Split attention reads the query and this position's K/V from global
      // memory; local attention takes them from the qkv exchange.
      return following != qd::Opcode::rope_kv_cache_f32 && b.split_attention;
    case qd::Opcode::grouped_query_attention_f32:
      return b.split_attention;
    default:
      return true;
    }
  }

  __device__ static void execute_stage(QwenBlock &b, const sg::Stage &stage,
                                       const sg::Task *tasks, sg::State *state,
                                       void *opaque, uint32_t worker, uint32_t workers) {
    if (!b.fused) {
      generic_execute_stage(stage, tasks, state, opaque, worker, workers);
      return;
    }
    if (b.failed) {
      return; // a wait gave up; the run ends at the next Program boundary
    }
    trace_mark(b, 20u + static_cast<uint32_t>(fused_opcode(b.program, b.stage)));
    const uint32_t layer = b.step % block_config.layers;
    qd::Context *c = &layer_cache[b.step & 1u];
    switch (fused_opcode(b.program, b.stage)) {
    case qd::Opcode::attention_rmsnorm_f32:
      fused_norm(b, state, c, b.hidden_exchanged ? HiddenSource::down : HiddenSource::global,
                 c->attention_norm_weight, block_config.epsilon[0], c->attention_normalized);
      trace_mark(b, 1);
      return;
    case qd::Opcode::qkv_projection_f32:
      fused_qkv(b, state, c, layer);
      trace_mark(b, 2);
      return;
    case qd::Opcode::rope_kv_cache_f32:
      return;
    case qd::Opcode::grouped_query_attention_f32:
      fused_attention(b, state, c, layer);
      return;
    case qd::Opcode::attention_output_residual_f32:
      fused_out(b, state, c, layer);
      trace_mark(b, 4);
      return;
    case qd::Opcode::mlp_rmsnorm_f32:
      fused_norm(b, state, c, HiddenSource::attention, c->mlp_norm_weight,
                 block_config.epsilon[1], c->mlp_normalized);
      trace_mark(b, 5);
      return;
    case qd::Opcode::gate_up_silu_f32:
      fused_gate_up(b, state, c, layer);
      trace_mark(b, 6);
      return;
    case qd::Opcode::down_matvec_f32:
      fused_down(b, state, c, layer);
      trace_mark(b, 7);
      return;
    case qd::Opcode::residual_advance:
      b.hidden_exchanged = true; // the next Program adds this step's down exchange
      // The residual was added in the down epilogue; what remains is the
      // branch / predicate bookkeeping, which State carries for the host.
      if (worker == 0 && threadIdx.x == 0) {
        const bool boundary = fused_layer_boundary(b.step);
        if (boundary && block_config.residual_argument[1] == 0) {
          state->predicate_value += block_config.residual_argument[0];
        }
        state->branch_value = boundary ? 1u : 0u;
      }
      return;
    case qd::Opcode::final_rmsnorm_f32:
      fused_norm(b, state, c, b.hidden_exchanged ? HiddenSource::down : HiddenSource::global,
                 c->tail->final_norm_weight, block_config.epsilon[2],
                 c->tail->final_normalized);
      trace_mark(b, 8);
      return;
    case qd::Opcode::lm_head_top1_partition_f32:
      fused_lm_head(b, state, stage, tasks);
      trace_mark(b, 9);
      return;
    case qd::Opcode::top1_reduce:
      if (worker == 0) {
        fused_reduce_top1(b, block_config.lm_stage, tasks, c);
      }
      return;
    case qd::Opcode::embedding_feedback_f32:
      // The next Program 0 reads the residual (the new token's embedding row)
      // from global memory after the tail's final barrier.
      b.hidden_exchanged = false;
      if (worker == 0) {
        embedding_feedback(c, state);
      }
      trace_mark(b, 10);
      return;
    }
  }

  __device__ static void initialize_profile(void *opaque) {
    if constexpr (kStageProfile) {
      auto *contexts = static_cast<qd::Context *>(opaque);
      qd::StageProfile *profile = contexts[0].tail->stage_profile;
      if (profile != nullptr) {
        profile->previous_tick = dev::global_timer_ns();
      }
    }
  }

  __device__ static void complete_profile_stage(QwenBlock &, const sg::Stage &stage,
                                                const sg::Task *tasks, void *opaque) {
    if constexpr (kStageProfile) {
      auto *contexts = static_cast<qd::Context *>(opaque);
      qd::StageProfile *profile = contexts[0].tail->stage_profile;
      if (profile == nullptr) {
        return;
      }
      const uint64_t now = dev::global_timer_ns();
      const uint32_t index = profile_stage_index(opcode_of(tasks[stage.task_offset]));
      if (index < qd::kProfileStageCount) {
        profile->stage_ticks[index] += now - profile->previous_tick;
        ++profile->stage_counts[index];
      }
      profile->previous_tick = now;
    }
  }

  __device__ static uint32_t profile_stage_index(qd::Opcode opcode) {
    switch (opcode) {
    case qd::Opcode::attention_rmsnorm_f32:
      return static_cast<uint32_t>(qd::ProfileStage::attention_norm);
    case qd::Opcode::qkv_projection_f32:
      return static_cast<uint32_t>(qd::ProfileStage::qkv_projection);
    case qd::Opcode::rope_kv_cache_f32:
      return static_cast<uint32_t>(qd::ProfileStage::rope_kv_cache);
    case qd::Opcode::grouped_query_attention_f32:
      return static_cast<uint32_t>(qd::ProfileStage::attention);
    case qd::Opcode::attention_output_residual_f32:
      return static_cast<uint32_t>(qd::ProfileStage::attention_output);
    case qd::Opcode::mlp_rmsnorm_f32:
      return static_cast<uint32_t>(qd::ProfileStage::mlp_norm);
    case qd::Opcode::gate_up_silu_f32:
      return static_cast<uint32_t>(qd::ProfileStage::gate_up_silu);
    case qd::Opcode::down_matvec_f32:
      return static_cast<uint32_t>(qd::ProfileStage::down_projection);
    case qd::Opcode::residual_advance:
      return static_cast<uint32_t>(qd::ProfileStage::residual_advance);
    case qd::Opcode::final_rmsnorm_f32:
      return static_cast<uint32_t>(qd::ProfileStage::final_norm);
    case qd::Opcode::lm_head_top1_partition_f32:
      return static_cast<uint32_t>(qd::ProfileStage::lm_head_top1);
    case qd::Opcode::top1_reduce:
      return static_cast<uint32_t>(qd::ProfileStage::top1_reduce);
    case qd::Opcode::embedding_feedback_f32:
      return static_cast<uint32_t>(qd::ProfileStage::embedding_feedback);
    }
    return qd::kProfileStageCount;
  }
};

using QwenWorkload = QwenWorkloadT<false>;
using QwenStageProfileWorkload = QwenWorkloadT<true>;

// Control-only workload (reference :871-917): keeps the Programs, stages and
// barriers, and runs only the state-changing tasks (residual_advance's branch
// decision and embedding_feedback), to measure the scheduler floor.
struct QwenSchedulerProfileWorkload : dev::CompiledWorkloadDefaults {
  __device__ static bool valid_context(const sg::State *, void *opaque) {
    return valid_qwen_contexts(static_cast<qd::Context *>(opaque));
  }
  __device__ static bool valid_task(const sg::Task &task, void *opaque) {
    return valid_qwen_task(task, static_cast<qd::Context *>(opaque));
  }
  __device__ static void execute(const sg::Task &task, sg::State *state, void *opaque) {
    qd::Context *c = layer_context(opaque, state);
    if (opcode_of(task) == qd::Opcode::residual_advance) {
      residual_advance(task, state, c, true, dev::load_relaxed(&state->step));
    } else if (opcode_of(task) == qd::Opcode::embedding_feedback_f32) {
      embedding_feedback(c, state);
    }
  }
  __device__ static void execute_stage(Block &, const sg::Stage &stage,
                                       const sg::Task *tasks, sg::State *state,
                                       void *opaque, uint32_t worker, uint32_t workers) {
    for (uint32_t t = worker; t < stage.task_count; t += workers) {
      execute(tasks[stage.task_offset + t], state, opaque);
    }
  }
};

// Host-step profiling entry (reference :995-1026 / :1048-1083).
__device__ qd::StageProfileEntry *profile_entry(void *opaque, uint32_t index) {
  auto *contexts = static_cast<qd::Context *>(opaque);
  qd::StageProfile *profile = contexts[0].tail->stage_profile;
  return profile != nullptr && index < profile->entry_count ? &profile->entries[index]
                                                            : nullptr;
}

} // namespace

extern "C" __global__ void __launch_bounds__(sg::kWorkerThreads, 1)
    qwen_stateful_graph_resident_kernel(
        sg::State *state, const sg::Task *tasks, const sg::Program *programs,
        sg::MaskState *phase_states, uint32_t program_count, uint32_t total_task_count,
        uint32_t phase_state_count, void *opaque_context, const sg::Stage *,
        const sg::CompiledProgram *, uint32_t, uint32_t reserved,
        sg::ValidationState *validation_state) {
  dev::run_resident<QwenWorkload>(state, tasks, programs, phase_states, program_count,
                                  total_task_count, phase_state_count, opaque_context,
                                  validation_state, reserved);
}

#define LRRT_RESIDENT_ARGS                                                             \
  sg::State *state, const sg::Task *tasks, const sg::Program *programs,                \
      sg::MaskState *phase_states, uint32_t program_count, uint32_t total_task_count,  \
      uint32_t phase_state_count, void *opaque_context, const sg::Stage *stages,       \
      const sg::CompiledProgram *compiled_programs, uint32_t stage_count,              \
      uint32_t reserved, sg::ValidationState *validation_state
#define LRRT_PACK_RESIDENT_ARGS                                                        \
  sg::ResidentArgs {                                                                   \
    state, tasks, programs, phase_states, program_count, total_task_count,             \
        phase_state_count, opaque_context, stages, compiled_programs, stage_count,     \
        reserved, validation_state                                                     \
  }

extern "C" __global__ void __launch_bounds__(sg::kWorkerThreads, 1)
    qwen_stateful_graph_compiled_kernel(LRRT_RESIDENT_ARGS) {
  dev::run_compiled_resident<QwenWorkload>(LRRT_PACK_RESIDENT_ARGS);
}

extern "C" __global__ void __launch_bounds__(sg::kWorkerThreads, 1)
    qwen_stateful_graph_scheduler_profile_kernel(LRRT_RESIDENT_ARGS) {
  dev::run_compiled_resident<QwenSchedulerProfileWorkload>(LRRT_PACK_RESIDENT_ARGS);
}

extern "C" __global__ void __launch_bounds__(sg::kWorkerThreads, 1)
    qwen_stateful_graph_stage_profile_kernel(LRRT_RESIDENT_ARGS) {
  dev::run_compiled_resident<QwenStageProfileWorkload>(LRRT_PACK_RESIDENT_ARGS);
}

// One compiled stage per launch over gridDim.x blocks (CUDA Graph comparator
// node body, reference :979-993).
extern "C" __global__ void __launch_bounds__(sg::kWorkerThreads)
    qwen_stateful_graph_matched_step_kernel(sg::State *state, const sg::Task *tasks,
                                            uint32_t task_count, uint32_t,
                                            void *opaque_context) {
  const sg::Stage stage{0, task_count};
  generic_execute_stage(stage, tasks, state, opaque_context, blockIdx.x, gridDim.x);
  __syncthreads();
  if (blockIdx.x == 0 && threadIdx.x == 0 &&
      opcode_of(tasks[0]) == qd::Opcode::residual_advance) {
    ++state->step;
  }
}

extern "C" __global__ void __launch_bounds__(sg::kWorkerThreads)
    qwen_stateful_graph_matched_profile_step_kernel(sg::State *state,
                                                    const sg::Task *tasks,
                                                    uint32_t task_count,
                                                    uint32_t profile_index,
                                                    void *opaque_context) {
  qd::StageProfileEntry *entry = profile_entry(opaque_context, profile_index);
  if (threadIdx.x == 0 && entry != nullptr) {
    atomicMin(reinterpret_cast<unsigned long long *>(&entry->begin_tick),
              static_cast<unsigned long long>(dev::global_timer_ns()));
  }
  const sg::Stage stage{0, task_count};
  generic_execute_stage(stage, tasks, state, opaque_context, blockIdx.x, gridDim.x);
  __syncthreads();
  if (threadIdx.x == 0) {
    if (blockIdx.x == 0 && opcode_of(tasks[0]) == qd::Opcode::residual_advance) {
      ++state->step;
    }
    if (entry != nullptr) {
      atomicMax(reinterpret_cast<unsigned long long *>(&entry->end_tick),
                static_cast<unsigned long long>(dev::global_timer_ns()));
    }
  }
}

// One task per block, host-driven (reference :1028-1046).
extern "C" __global__ void __launch_bounds__(sg::kWorkerThreads)
    qwen_stateful_graph_host_step_kernel(sg::State *state, const sg::Task *tasks,
                                         uint32_t task_count, uint32_t,
                                         void *opaque_context) {
  if (blockIdx.x >= task_count) {
    return;
  }
  generic_execute(tasks[blockIdx.x], state, layer_context(opaque_context, state));
  if (threadIdx.x == 0 && opcode_of(tasks[blockIdx.x]) == qd::Opcode::residual_advance) {
    ++state->step;
  }
}

extern "C" __global__ void __launch_bounds__(sg::kWorkerThreads)
    qwen_stateful_graph_host_profile_step_kernel(sg::State *state, const sg::Task *tasks,
                                                 uint32_t task_count,
                                                 uint32_t profile_index,
                                                 void *opaque_context) {
  if (blockIdx.x >= task_count) {
    return;
  }
  qd::StageProfileEntry *entry = profile_entry(opaque_context, profile_index);
  if (threadIdx.x == 0 && entry != nullptr) {
    atomicMin(reinterpret_cast<unsigned long long *>(&entry->begin_tick),
              static_cast<unsigned long long>(dev::global_timer_ns()));
  }
  generic_execute(tasks[blockIdx.x], state, layer_context(opaque_context, state));
  if (threadIdx.x == 0) {
    if (opcode_of(tasks[blockIdx.x]) == qd::Opcode::residual_advance) {
      ++state->step;
    }
    if (entry != nullptr) {
      atomicMax(reinterpret_cast<unsigned long long *>(&entry->end_tick),
                static_cast<unsigned long long>(dev::global_timer_ns()));
    }
  }
}
