// Qwen2 FP32 resident decode driver: the host side of the decode path (C ABI
// in include/lrrt_qwen.h). It builds the reference task/Program table, owns
// the device weights, activations, KV caches, RoPE tables and per-layer
// Context array, and runs the sm_100a kernels through ResidentExecutor and the
// lr_* runtime, following light-rocm-runtime benchmarks/qwen_stateful_graph.cpp.
#include "lrrt_qwen.h"

#include "lm_head_top1_static.hpp"
#include "batch.hpp"
#include "prefill.hpp"
#include "prefill_common.hpp"

#include <cuda_runtime_api.h>
#include "lrrt/qwen/weight_bundle.hpp"

#include "lrrt/lrrt.hpp"
#include "lrrt/persistent_graph.hpp"
#include "lrrt/qwen/resident_layout.hpp"
#include "lrrt/qwen/resident_schedule.hpp"
#include "lrrt/qwen/stateful_graph_context.hpp"

#include <algorithm>
#include <array>
#include <cmath>
#include <cstring>
#include <limits>
#include <memory>
#include <mutex>
#include <optional>
#include <stdexcept>
#include <string>
#include <vector>

namespace {

namespace sg = lrrt::persistent_graph;
namespace qd = lrrt::qwen::stateful_graph;

std::mutex g_error_mutex;
std::string g_last_error;

void set_error(const std::string &text) {
  std::lock_guard<std::mutex> lock(g_error_mutex);
  g_last_error = text;
}

template <typename Body> lr_status_t guarded(const char *what, Body body) {
  try {
    body();
    return LR_SUCCESS;
  } catch (const lrrt::Error &error) {
    char detail[512] = {};
    lr_last_error_detail(detail, sizeof(detail));
    set_error(std::string(what) + ": " + error.what() +
              (detail[0] != '\0' ? std::string(" [") + detail + "]" : std::string()));
    return error.status();
  } catch (const std::invalid_argument &error) {
    set_error(std::string(what) + ": " + error.what());
    return LR_ERROR_INVALID_ARGUMENT;
  } catch (const std::logic_error &error) {
    set_error(std::string(what) + ": " + error.what());
    return LR_ERROR_INVALID_ARGUMENT;
  } catch (const std::exception &error) {
    set_error(std::string(what) + ": " + error.what());
    return LR_ERROR_RUNTIME;
  }
}

uint32_t float_bits(float value) {
  uint32_t bits;
  std::memcpy(&bits, &value, sizeof(bits));
  return bits;
}

sg::Task make_task(qd::Opcode opcode, uint64_t dependencies, uint32_t begin,
                   uint32_t end, uint32_t argument0 = 0, uint32_t argument1 = 0) {
  return {static_cast<uint32_t>(opcode),
          static_cast<uint32_t>(dependencies),
          begin,
          end,
          argument0,
          argument1,
          static_cast<uint32_t>(dependencies >> 32u),
          0};
}

sg::Program make_program(uint32_t offset, uint32_t count, uint32_t next,
                         uint32_t flags = 0, uint32_t branch = 0) {
  return {offset, count, next, flags, branch, {0, 0, 0}};
}

struct ProgramTable {
  std::vector<sg::Task> tasks;
  std::vector<sg::Program> programs;
};

// The decode graph of the reference (qwen_stateful_graph.cpp:368-485), with
// the same partitioning and dependency masks:
//   Program 0 (attention, 25 tasks): RMSNorm -> 8 QKV -> RoPE+KV -> 7 GQA
//     -> 8 o_proj+residual; next = 1.
//   Program 1 (FFN, 54 tasks): RMSNorm -> 20 gate/up/SiLU -> 32 down
//     -> residual_advance; advances the step, branches to 2 after the last
//     layer, else back to 0.
//   Program 2 (tail, P+3 tasks): final RMSNorm -> P LM-head top-1 partitions
//     -> top1_reduce -> embedding_feedback; evaluates the stop predicate.
ProgramTable make_qwen_decoder_programs(uint32_t vocab, uint32_t partitions) {
  if (vocab == 0 || partitions == 0 || partitions > qd::kMaximumLmHeadPartitions ||
      partitions > vocab) {
    throw std::invalid_argument("invalid LM head partitioning");
  }
  const uint32_t epsilon = float_bits(1.0e-6f);
  ProgramTable table;
  auto &tasks = table.tasks;
  tasks.push_back(make_task(qd::Opcode::attention_rmsnorm_f32, 0, 0, qd::kHiddenSize,
                            epsilon));
  uint64_t qkv = 0;
  for (uint32_t p = 0; p < qd::kAttentionProjectionPartitions; ++p) {
    qkv |= uint64_t{1} << tasks.size();
    tasks.push_back(make_task(
        qd::Opcode::qkv_projection_f32, 1u,
        qd::kPackedQkvSize * p / qd::kAttentionProjectionPartitions,
        qd::kPackedQkvSize * (p + 1u) / qd::kAttentionProjectionPartitions));
  }
  const uint64_t rope = uint64_t{1} << tasks.size();
  tasks.push_back(make_task(qd::Opcode::rope_kv_cache_f32, qkv, 0, qd::kRotaryHeads));
  uint64_t attention = 0;
  for (uint32_t p = 0; p < qd::kAttentionTaskPartitions; ++p) {
    attention |= uint64_t{1} << tasks.size();
    tasks.push_back(make_task(
        qd::Opcode::grouped_query_attention_f32, rope,
        qd::kAttentionHeads * p / qd::kAttentionTaskPartitions,
        qd::kAttentionHeads * (p + 1u) / qd::kAttentionTaskPartitions));
  }
  for (uint32_t p = 0; p < qd::kAttentionOutputPartitions; ++p) {
    tasks.push_back(make_task(qd::Opcode::attention_output_residual_f32, attention,
                              qd::kHiddenSize * p / qd::kAttentionOutputPartitions,
                              qd::kHiddenSize * (p + 1u) / qd::kAttentionOutputPartitions));
  }
  if (tasks.size() != qd::kAttentionTaskCount) {
    throw std::runtime_error("Qwen attention program layout mismatch");
  }
  table.programs.push_back(make_program(0, qd::kAttentionTaskCount, 1));

  const uint32_t ffn = static_cast<uint32_t>(tasks.size());
  tasks.push_back(make_task(qd::Opcode::mlp_rmsnorm_f32, 0, 0, qd::kHiddenSize, epsilon));
  uint64_t activated = 0;
  for (uint32_t p = 0; p < qd::kFfnProjectionPartitions; ++p) {
    activated |= uint64_t{1} << (tasks.size() - ffn);
    tasks.push_back(make_task(qd::Opcode::gate_up_silu_f32, 1u,
                              qd::kIntermediateSize * p / qd::kFfnProjectionPartitions,
                              qd::kIntermediateSize * (p + 1u) /
                                  qd::kFfnProjectionPartitions));
  }
  uint64_t down = 0;
  for (uint32_t p = 0; p < qd::kDownProjectionPartitions; ++p) {
    down |= uint64_t{1} << (tasks.size() - ffn);
    tasks.push_back(make_task(qd::Opcode::down_matvec_f32, activated,
                              qd::kHiddenSize * p / qd::kDownProjectionPartitions,
                              qd::kHiddenSize * (p + 1u) / qd::kDownProjectionPartitions));
  }
  tasks.push_back(make_task(qd::Opcode::residual_advance, down, 0, qd::kHiddenSize, 1, 1));
  if (tasks.size() != qd::kDecoderTaskCount) {
    throw std::runtime_error("Qwen decoder task layout mismatch");
  }
  table.programs.push_back(make_program(ffn, qd::kFfnTaskCount, 0,
                                        sg::kProgramAdvancesStep |
                                            sg::kProgramBranchesOnState,
                                        2));

  const uint32_t tail = static_cast<uint32_t>(tasks.size());
  tasks.push_back(make_task(qd::Opcode::final_rmsnorm_f32, 0, 0, qd::kHiddenSize, epsilon));
  uint64_t candidates = 0;
  for (uint32_t p = 0; p < partitions; ++p) {
    candidates |= uint64_t{1} << (tasks.size() - tail);
    tasks.push_back(make_task(
        qd::Opcode::lm_head_top1_partition_f32, 1u,
        static_cast<uint32_t>(uint64_t{vocab} * p / partitions),
        static_cast<uint32_t>(uint64_t{vocab} * (p + 1u) / partitions), p));
  }
  const uint64_t reduce = uint64_t{1} << (tasks.size() - tail);
  tasks.push_back(make_task(qd::Opcode::top1_reduce, candidates, 0, partitions));
  tasks.push_back(make_task(qd::Opcode::embedding_feedback_f32, reduce, 0, qd::kHiddenSize));
  table.programs.push_back(
      make_program(tail, partitions + 3u, 0, sg::kProgramEvaluatesPredicate));
  return table;
}

// Host launches of the reference's host-driven path (kHostStages :504-516):
// one launch per decoder stage (9 per layer) and 4 per tail, one block per task.
struct HostStage {
  uint32_t first_task;
  uint32_t task_count;
};

std::vector<HostStage> decoder_host_stages() {
  const uint32_t a = qd::kAttentionProjectionPartitions;
  const uint32_t g = qd::kAttentionTaskPartitions;
  return {{0, 1},
          {1, a},
          {1 + a, 1},
          {2 + a, g},
          {2 + a + g, qd::kAttentionOutputPartitions},
          {qd::kAttentionTaskCount, 1},
          {qd::kAttentionTaskCount + 1, qd::kFfnProjectionPartitions},
          {qd::kAttentionTaskCount + 1 + qd::kFfnProjectionPartitions,
           qd::kDownProjectionPartitions},
          {qd::kDecoderTaskCount - 1, 1}};
}

constexpr size_t kAlignFloats = 64; // 256-byte alignment of every array

size_t align_floats(size_t count) {
  return (count + kAlignFloats - 1) / kAlignFloats * kAlignFloats;
}

// Float offsets of one layer's arrays inside the weight allocation.
struct LayerLayout {
  size_t attention_norm, q, k, v, q_bias, k_bias, v_bias, o, mlp_norm, gate, up, down;
  size_t floats;
};

LayerLayout layer_layout() {
  LayerLayout l{};
  size_t at = 0;
  auto take = [&](size_t count) {
    const size_t offset = at;
    at += align_floats(count);
    return offset;
  };
  const size_t h = qd::kHiddenSize, kv = qd::kKvSize, i = qd::kIntermediateSize;
  l.attention_norm = take(h);
  l.q = take(h * h);
  l.k = take(kv * h);
  l.v = take(kv * h);
  l.q_bias = take(h);
  l.k_bias = take(kv);
  l.v_bias = take(kv);
  l.o = take(h * h);
  l.mlp_norm = take(h);
  l.gate = take(i * h);
  l.up = take(i * h);
  l.down = take(h * i);
  l.floats = at;
  return l;
}

uint64_t algorithmic_weight_bytes(uint32_t layers, uint32_t vocab) {
  const uint64_t h = qd::kHiddenSize, kv = qd::kKvSize, i = qd::kIntermediateSize;
  const uint64_t per_layer = (h * h + 2 * kv * h + qd::kPackedQkvSize + h * h +
                              3 * i * h + 2 * h) *
                             sizeof(float);
  return per_layer * layers + uint64_t{vocab} * h * sizeof(float) +
         2 * h * sizeof(float); // final norm + embedding row
}

uint32_t phase_states_for(uint32_t tokens, uint32_t layers) {
  const uint64_t count = uint64_t{tokens} * 2u * (2u * uint64_t{layers} + 1u) + 1u;
  if (count > uint64_t{sg::phase_generation(UINT32_MAX)} + 1u) {
    throw std::invalid_argument("program phase count is too large");
  }
  return static_cast<uint32_t>(count);
}

} // namespace

struct lrq_model_t {
  lrq_model_t(lrrt::Device device_, const void *image, size_t image_size,
              const lrq_model_config_t &config_)
      : device(device_), module(device_, image, image_size),
        compiled(module.kernel("qwen_stateful_graph_compiled_kernel")),
        dynamic(module.kernel("qwen_stateful_graph_resident_kernel")),
        scheduler_profile(module.kernel("qwen_stateful_graph_scheduler_profile_kernel")),
        stage_profile(module.kernel("qwen_stateful_graph_stage_profile_kernel")),
        host_step(module.kernel("qwen_stateful_graph_host_step_kernel")),
        matched_step(module.kernel("qwen_stateful_graph_matched_step_kernel")),
        config(config_), layout(layer_layout()) {}

  lrrt::Device device;
  lrrt::Module module;
  lrrt::Kernel compiled, dynamic, scheduler_profile, stage_profile, host_step, matched_step;
  lrq_model_config_t config;
  LayerLayout layout;
  uint32_t workers = 0;
  uint32_t partitions = 0;
  uint32_t phase_state_count = 0;
  uint32_t shared_bytes = 0;
  ProgramTable table;
  sg::CompiledPlan plan;

  std::optional<lrrt::DeviceBuffer> weights, embeddings, lm_head, final_norm;
  std::optional<lrrt::DeviceBuffer> key_cache, value_cache, rope_cos, rope_sin;
  std::optional<lrrt::DeviceBuffer> hidden, hidden_init, attention_normalized, query,
      key, value, mlp_normalized, activated, projected, final_normalized,
      partial_values, partial_indices, decode_state, decode_init, output_tokens,
      workspace, tail_context, contexts, profile, host_state, host_tasks;
  std::optional<sg::ResidentExecutor> compiled_executor, dynamic_executor,
      scheduler_profile_executor, stage_profile_executor;

  std::optional<lrrt::DeviceBuffer> trace; // StageProfileEntry array, optional
  std::optional<lrrt::DeviceBuffer> logits; // [vocab] logit capture, optional
  // CUDA-graph comparator: one token of matched-step launches, captured once
  // and replayed per token (LRQ_PATH_GRAPH).
  cudaGraphExec_t token_graph = nullptr;
  uint32_t token_graph_nodes = 0;
  uint32_t trace_capacity = 0;
  std::optional<std::array<uint32_t, 3>> staged_decode; // position, max, eos
  uint32_t last_path = 0;
  uint64_t device_bytes = 0;
  // Prompt prefill (optional module); weights_generation counts layer-weight
  // uploads so the prefill's TF32 weight copies know when to refresh.
  std::unique_ptr<lrrt::qwen::prefill::Prefill> prefill;
  uint64_t weights_generation = 0;
  std::vector<lrq_batch_t *> batches; // live batched decoders (they use `prefill`)

  float *layer_weight(uint32_t layer, size_t offset) const {
    return static_cast<float *>(weights->data()) + size_t{layer} * layout.floats + offset;
  }
  size_t cache_floats() const { return size_t{config.cache_capacity} * qd::kKvSize; }
};

namespace {

lrrt::DeviceBuffer allocate(lrq_model_t &m, size_t bytes) {
  m.device_bytes += bytes;
  return lrrt::DeviceBuffer(m.device, std::max<size_t>(bytes, 16));
}

void zero_fill(lrrt::DeviceBuffer &buffer) {
  const std::vector<unsigned char> zeros(buffer.size(), 0);
  lrrt::copy_to_device(buffer, zeros);
}

// One layer's KV caches and o_proj weight as the fused path's tensor maps
// see them.
struct KvCacheView {
  const float *keys;
  const float *values;
  uint32_t capacity;       // rows of [capacity][128] floats
  const float *out_weight; // [896][896]
};

// Zero-fills a workspace allocation of `bytes` (>= workspace_bytes(capacity))
// and writes its header, array pointers and each layer's 2-D tensor maps: the
// KV caches (boxes of 32 columns x 56 rows, 128-byte swizzle: the fused
// path's KV ring units) and the o_proj weight (boxes of 224 columns x 16
// rows: an OUT unit is two of them).
void init_workspace(lr_device_t device, void *workspace, uint64_t bytes, uint32_t capacity,
                    const std::vector<KvCacheView> &caches) {
  if (workspace == nullptr || capacity < 2u || bytes < qd::workspace_bytes(capacity) ||
      caches.size() > qd::kWorkspaceMapLayers ||
      (reinterpret_cast<uintptr_t>(workspace) & 255u) != 0) {
    throw std::invalid_argument(
        "invalid workspace: null, misaligned, too small for the worker count, or too many "
        "layers");
  }
  const std::vector<unsigned char> zeros(bytes, 0);
  lrrt::check(lr_memcpy(device, workspace, zeros.data(), bytes, LR_MEMCPY_HOST_TO_DEVICE),
              "lr_memcpy workspace");
  auto *base = static_cast<unsigned char *>(workspace);
  qd::Workspace header{};
  size_t at = 256;
  header.magic = qd::kWorkspaceMagic;
  header.worker_capacity = capacity;
  header.attention_partials = reinterpret_cast<float *>(base + at);
  at += size_t{capacity} * qd::kQueriesPerKvHead * qd::kAttentionPartialStride * sizeof(float);
  at = (at + 255) / 256 * 256;
  header.attention_arrivals = reinterpret_cast<uint32_t *>(base + at);
  at += 256;
  header.top1_values = reinterpret_cast<float *>(base + at);
  at += (size_t{capacity} + qd::kMaximumLmHeadPartitions) * sizeof(float);
  header.top1_indices = reinterpret_cast<uint32_t *>(base + at);
  at += (size_t{capacity} + qd::kMaximumLmHeadPartitions) * sizeof(uint32_t);
  at = (at + 255) / 256 * 256;
  header.exchange = reinterpret_cast<uint64_t *>(base + at); // zero-filled above
  at += size_t{qd::kExchangeWords} * sizeof(uint64_t);
  at = (at + 255) / 256 * 256;
  header.attention_words = reinterpret_cast<uint64_t *>(base + at);
  at += 2u * size_t{capacity} * qd::kSpreadWords * sizeof(uint64_t);
  at = (at + 255) / 256 * 256;
  std::vector<unsigned char> maps(
      size_t{qd::kWorkspaceMapLayers} * qd::kWorkspaceMapsPerLayer * qd::kTensorMapBytes, 0);
  for (size_t layer = 0; layer < caches.size(); ++layer) {
    for (uint32_t which = 0; which < 2; ++which) {
      const float *cache = which == 0 ? caches[layer].keys : caches[layer].values;
      if (cache == nullptr || (reinterpret_cast<uintptr_t>(cache) & 15u) != 0 ||
          caches[layer].capacity == 0) {
        throw std::invalid_argument("KV cache of layer " + std::to_string(layer) +
                                    " is null, misaligned or empty");
      }
      CUtensorMap map{};
      const cuuint64_t dims[2] = {qd::kKvSize, caches[layer].capacity};
      const cuuint64_t strides[1] = {qd::kKvSize * sizeof(float)};
      const cuuint32_t box[2] = {32, qd::resident::kKvUnitPositions};
      const cuuint32_t element_strides[2] = {1, 1};
      const CUresult status = lrrt::qwen::prefill::detail::encode_tiled()(
          &map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float *>(cache), dims, strides,
          box, element_strides, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
      if (status != CUDA_SUCCESS) {
        throw std::runtime_error("cuTensorMapEncodeTiled failed for a KV cache map (" +
                                 std::to_string(status) + ")");
      }
      std::memcpy(maps.data() + (layer * qd::kWorkspaceMapsPerLayer + which) * qd::kTensorMapBytes,
                  &map, sizeof(map));
    }
    const float *out = caches[layer].out_weight;
    if (out == nullptr || (reinterpret_cast<uintptr_t>(out) & 15u) != 0) {
      throw std::invalid_argument("o_proj weight of layer " + std::to_string(layer) +
                                  " is null or misaligned");
    }
    CUtensorMap map{};
    const cuuint64_t dims[2] = {qd::kHiddenSize, qd::kHiddenSize};
    const cuuint64_t strides[1] = {qd::kHiddenSize * sizeof(float)};
    const cuuint32_t box[2] = {qd::resident::kOBoxColumns, qd::resident::kORows};
    const cuuint32_t element_strides[2] = {1, 1};
    const CUresult status = lrrt::qwen::prefill::detail::encode_tiled()(
        &map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float *>(out), dims, strides, box,
        element_strides, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (status != CUDA_SUCCESS) {
      throw std::runtime_error("cuTensorMapEncodeTiled failed for an o_proj map (" +
                               std::to_string(status) + ")");
    }
    std::memcpy(maps.data() + (layer * qd::kWorkspaceMapsPerLayer + 2u) * qd::kTensorMapBytes,
                &map, sizeof(map));
  }
  header.kv_maps = base + at;
  lrrt::check(lr_memcpy(device, base + at, maps.data(), maps.size(), LR_MEMCPY_HOST_TO_DEVICE),
              "lr_memcpy KV cache maps");
  lrrt::check(lr_memcpy(device, base, &header, sizeof(header), LR_MEMCPY_HOST_TO_DEVICE),
              "lr_memcpy workspace header");
}

void build_model(lrq_model_t &m) {
  const lrq_model_config_t &c = m.config;
  if (c.layer_count == 0 || c.vocab_size == 0 || c.cache_capacity == 0 ||
      c.max_tokens_per_run == 0 || c.max_tokens_per_run > c.cache_capacity ||
      c.lm_head_partitions > qd::kMaximumLmHeadPartitions) {
    throw std::invalid_argument("invalid Qwen model configuration");
  }
  // Admission: one 256-thread block per SM with the fused path's shared memory.
  m.shared_bytes = qd::resident::kFusedSharedBytes;
  const uint32_t requested = c.worker_count == 0 ? sg::kMaximumResidentWorkers : c.worker_count;
  const sg::ResidentAdmission admission =
      sg::admit_resident_workers(m.device, m.compiled, requested, sg::kWorkerThreads,
                                 m.shared_bytes);
  m.workers = admission.worker_count;
  m.partitions = c.lm_head_partitions != 0
                     ? c.lm_head_partitions
                     : std::min({c.vocab_size, qd::kMaximumLmHeadPartitions, m.workers});
  m.partitions = std::min(m.partitions, c.vocab_size);
  m.table = make_qwen_decoder_programs(c.vocab_size, m.partitions);
  m.phase_state_count = phase_states_for(c.max_tokens_per_run, c.layer_count);

  const size_t h = qd::kHiddenSize;
  m.weights.emplace(allocate(m, sizeof(float) * m.layout.floats * c.layer_count));
  m.embeddings.emplace(allocate(m, sizeof(float) * size_t{c.vocab_size} * h));
  if (c.tied_embeddings == 0) {
    m.lm_head.emplace(allocate(m, sizeof(float) * size_t{c.vocab_size} * h));
  }
  m.final_norm.emplace(allocate(m, sizeof(float) * h));
  m.key_cache.emplace(allocate(m, sizeof(float) * m.cache_floats() * c.layer_count));
  m.value_cache.emplace(allocate(m, sizeof(float) * m.cache_floats() * c.layer_count));
  zero_fill(*m.key_cache);
  zero_fill(*m.value_cache);
  const size_t rope_floats = size_t{c.cache_capacity} * qd::kRotarySize;
  m.rope_cos.emplace(allocate(m, sizeof(float) * rope_floats));
  m.rope_sin.emplace(allocate(m, sizeof(float) * rope_floats));
  {
    std::vector<float> cos_table(rope_floats), sin_table(rope_floats);
    lrq_rope_tables(c.cache_capacity, c.rope_theta, cos_table.data(), sin_table.data());
    lrrt::copy_to_device(*m.rope_cos, cos_table);
    lrrt::copy_to_device(*m.rope_sin, sin_table);
  }
  auto vector = [&](size_t floats) { return allocate(m, sizeof(float) * floats); };
  m.hidden.emplace(vector(h));
  m.hidden_init.emplace(vector(h));
  m.attention_normalized.emplace(vector(h));
  m.query.emplace(vector(qd::kQuerySize));
  m.key.emplace(vector(qd::kKvSize));
  m.value.emplace(vector(qd::kKvSize));
  m.mlp_normalized.emplace(vector(h));
  m.activated.emplace(vector(qd::kIntermediateSize));
  m.projected.emplace(vector(h));
  m.final_normalized.emplace(vector(h));
  m.partial_values.emplace(vector(qd::kMaximumLmHeadPartitions));
  m.partial_indices.emplace(vector(qd::kMaximumLmHeadPartitions));
  m.decode_state.emplace(allocate(m, sizeof(qd::DecodeState)));
  m.decode_init.emplace(allocate(m, sizeof(qd::DecodeState)));
  m.output_tokens.emplace(allocate(m, sizeof(uint32_t) * c.max_tokens_per_run));
  m.profile.emplace(allocate(m, sizeof(qd::StageProfile)));
  m.host_state.emplace(allocate(m, sizeof(sg::State)));
  for (lrrt::DeviceBuffer *buffer :
       {&*m.hidden, &*m.hidden_init, &*m.attention_normalized, &*m.query, &*m.key,
        &*m.value, &*m.mlp_normalized, &*m.activated, &*m.projected,
        &*m.final_normalized, &*m.partial_values, &*m.partial_indices,
        &*m.decode_state, &*m.decode_init, &*m.output_tokens, &*m.profile,
        &*m.host_state}) {
    zero_fill(*buffer);
  }

  // Workspace for the fused path: header followed by its arrays.
  const uint32_t capacity = std::max(m.workers, 2u);
  m.workspace.emplace(allocate(m, qd::workspace_bytes(capacity)));
  {
    std::vector<KvCacheView> caches(c.layer_count);
    for (uint32_t layer = 0; layer < c.layer_count; ++layer) {
      caches[layer] = {static_cast<const float *>(m.key_cache->data()) + layer * m.cache_floats(),
                       static_cast<const float *>(m.value_cache->data()) + layer * m.cache_floats(),
                       c.cache_capacity, m.layer_weight(layer, m.layout.o)};
    }
    init_workspace(m.device.get(), m.workspace->data(), m.workspace->size(), capacity, caches);
  }

  qd::TailContext tail{};
  tail.final_norm_weight = static_cast<const float *>(m.final_norm->data());
  tail.lm_head_weight = static_cast<const float *>(
      c.tied_embeddings != 0 ? m.embeddings->data() : m.lm_head->data());
  tail.token_embeddings = static_cast<const float *>(m.embeddings->data());
  tail.final_normalized = static_cast<float *>(m.final_normalized->data());
  tail.partial_max_values = static_cast<float *>(m.partial_values->data());
  tail.partial_max_indices = static_cast<uint32_t *>(m.partial_indices->data());
  tail.decode_state = static_cast<qd::DecodeState *>(m.decode_state->data());
  tail.output_tokens = static_cast<uint32_t *>(m.output_tokens->data());
  tail.vocab_size = c.vocab_size;
  tail.partition_count = m.partitions;
  tail.embedding_count = c.vocab_size;
  tail.stage_profile = static_cast<qd::StageProfile *>(m.profile->data());
  tail.workspace = c.disable_fused_path != 0
                       ? nullptr
                       : static_cast<qd::Workspace *>(m.workspace->data());
  m.tail_context.emplace(allocate(m, sizeof(qd::TailContext)));
  lrrt::copy_to_device(*m.tail_context, &tail, sizeof(tail));

  std::vector<qd::Context> contexts(c.layer_count);
  for (uint32_t layer = 0; layer < c.layer_count; ++layer) {
    const LayerLayout &l = m.layout;
    qd::Context &x = contexts[layer];
    x.hidden = static_cast<float *>(m.hidden->data());
    x.attention_norm_weight = m.layer_weight(layer, l.attention_norm);
    x.q_weight = m.layer_weight(layer, l.q);
    x.k_weight = m.layer_weight(layer, l.k);
    x.v_weight = m.layer_weight(layer, l.v);
    x.q_bias = m.layer_weight(layer, l.q_bias);
    x.k_bias = m.layer_weight(layer, l.k_bias);
    x.v_bias = m.layer_weight(layer, l.v_bias);
    x.out_weight = m.layer_weight(layer, l.o);
    x.mlp_norm_weight = m.layer_weight(layer, l.mlp_norm);
    x.gate_weight = m.layer_weight(layer, l.gate);
    x.up_weight = m.layer_weight(layer, l.up);
    x.down_weight = m.layer_weight(layer, l.down);
    x.attention_normalized = static_cast<float *>(m.attention_normalized->data());
    x.query = static_cast<float *>(m.query->data());
    x.key = static_cast<float *>(m.key->data());
    x.value = static_cast<float *>(m.value->data());
    x.rope_cos = static_cast<const float *>(m.rope_cos->data());
    x.rope_sin = static_cast<const float *>(m.rope_sin->data());
    x.key_cache = static_cast<float *>(m.key_cache->data()) + layer * m.cache_floats();
    x.value_cache = static_cast<float *>(m.value_cache->data()) + layer * m.cache_floats();
    x.mlp_normalized = static_cast<float *>(m.mlp_normalized->data());
    x.activated = static_cast<float *>(m.activated->data());
    x.projected = static_cast<float *>(m.projected->data());
    x.tail = static_cast<qd::TailContext *>(m.tail_context->data());
    x.hidden_size = qd::kHiddenSize;
    x.query_size = qd::kQuerySize;
    x.kv_size = qd::kKvSize;
    x.intermediate_size = qd::kIntermediateSize;
    x.cache_capacity = c.cache_capacity;
    x.layer_count = c.layer_count;
  }
  m.contexts.emplace(allocate(m, sizeof(qd::Context) * contexts.size()));
  lrrt::copy_to_device(*m.contexts, contexts);

  const sg::ResidentConfig compiled_config{m.phase_state_count, m.workers, m.shared_bytes,
                                           0};
  const sg::ResidentConfig plain_config{m.phase_state_count, m.workers, 0, 0};
  m.plan = sg::compile_resident_plan(m.table.tasks, m.table.programs, compiled_config);
  m.compiled_executor.emplace(m.device, m.compiled, m.table.tasks, m.table.programs,
                              compiled_config, m.plan);
  m.stage_profile_executor.emplace(m.device, m.stage_profile, m.table.tasks,
                                   m.table.programs, compiled_config, m.plan);
  m.scheduler_profile_executor.emplace(m.device, m.scheduler_profile, m.table.tasks,
                                       m.table.programs, plain_config, m.plan);
  m.dynamic_executor.emplace(m.device, m.dynamic, m.table.tasks, m.table.programs,
                             plain_config);
  for (sg::ResidentExecutor *executor :
       {&*m.compiled_executor, &*m.stage_profile_executor, &*m.scheduler_profile_executor,
        &*m.dynamic_executor}) {
    executor->bind_context(m.contexts->data());
  }
  m.host_tasks.emplace(allocate(m, sizeof(sg::Task) * m.table.tasks.size()));
  lrrt::copy_to_device(*m.host_tasks, m.table.tasks);
}

sg::ResidentExecutor &executor_for(lrq_model_t &m, uint32_t path) {
  switch (path) {
  case LRQ_PATH_COMPILED:
    return *m.compiled_executor;
  case LRQ_PATH_DYNAMIC:
    return *m.dynamic_executor;
  case LRQ_PATH_SCHEDULER_PROFILE:
    return *m.scheduler_profile_executor;
  case LRQ_PATH_STAGE_PROFILE:
    return *m.stage_profile_executor;
  default:
    throw std::invalid_argument("path has no resident executor");
  }
}

lr_kernel_t *kernel_for(lrq_model_t &m, uint32_t path) {
  switch (path) {
  case LRQ_PATH_COMPILED:
    return m.compiled.get();
  case LRQ_PATH_DYNAMIC:
    return m.dynamic.get();
  case LRQ_PATH_SCHEDULER_PROFILE:
    return m.scheduler_profile.get();
  case LRQ_PATH_STAGE_PROFILE:
    return m.stage_profile.get();
  default:
    throw std::invalid_argument("path has no resident kernel");
  }
}

// Stages the DecodeState image of a request (synchronous copy only when the
// request differs from the staged one).
void stage_decode_state(lrq_model_t &m, uint32_t position, uint32_t maximum, uint32_t eos) {
  const std::array<uint32_t, 3> key = {position, maximum, eos};
  if (m.staged_decode && *m.staged_decode == key) {
    return;
  }
  const qd::DecodeState init{position, position, 0, eos, 0, maximum,
                             static_cast<uint32_t>(qd::StopReason::none), 0.0f};
  lrrt::copy_to_device(*m.decode_init, &init, sizeof(init));
  m.staged_decode = key;
}

void async_device_copy(lrq_model_t &m, lrrt::DeviceBuffer &dst, const lrrt::DeviceBuffer &src,
                       size_t bytes) {
  lrrt::check(lr_memcpy_async(m.device.get(), dst.data(), src.data(), bytes,
                              LR_MEMCPY_DEVICE_TO_DEVICE, nullptr),
              "lr_memcpy_async");
}

void reset_host_state(lrq_model_t &m, const lrq_decode_request_t &r) {
  sg::State state{};
  state.abi_version = sg::kAbiVersion;
  state.status = static_cast<uint32_t>(sg::Status::ready);
  state.phase = sg::make_phase(0, 0);
  state.max_steps = r.max_steps;
  state.stop_value = r.stop_value;
  state.worker_count = m.workers;
  lrrt::check(lr_memcpy(m.device.get(), m.host_state->data(), &state, sizeof(state),
                        LR_MEMCPY_HOST_TO_DEVICE),
              "lr_memcpy host state");
}

void launch_host_steps(lrq_model_t &m, const lrq_decode_request_t &r) {
  reset_host_state(m, r);
  const auto *tasks = static_cast<const sg::Task *>(m.host_tasks->data());
  auto launch = [&](uint32_t first, uint32_t count) {
    const sg::HostStepArgs args{static_cast<sg::State *>(m.host_state->data()),
                                tasks + first, count, 0, m.contexts->data()};
    const lr_launch_config_t config{{count * sg::kWorkerThreads, 1, 1},
                                    {sg::kWorkerThreads, 1, 1},
                                    0};
    lrrt::launch(m.host_step, config, args);
  };
  const std::vector<HostStage> stages = decoder_host_stages();
  for (uint32_t token = 0; token < r.maximum_tokens; ++token) {
    for (uint32_t layer = 0; layer < m.config.layer_count; ++layer) {
      for (const HostStage &stage : stages) {
        launch(stage.first_task, stage.task_count);
      }
    }
    launch(qd::kDecoderTaskCount, 1);
    launch(qd::kDecoderTaskCount + 1u, m.partitions);
    launch(qd::kDecoderTaskCount + 1u + m.partitions, 1);
    launch(qd::kDecoderTaskCount + 2u + m.partitions, 1);
  }
}

void check_cuda(cudaError_t status, const char *what) {
  if (status != cudaSuccess) {
    throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(status));
  }
}

void *default_stream(lrq_model_t &m) {
  void *stream = nullptr;
  lrrt::check(lr_queue_native_handle(m.device.get(), nullptr, &stream),
              "lr_queue_native_handle");
  return stream;
}

// Captures one token of the CUDA-graph comparator (reference
// benchmarks/qwen_hip_graph.hpp: one matched-step node per compiled stage over
// every worker block, in Program order: layers x (Program 0, Program 1), then
// Program 2), via stream capture of the same lr_* launches on the device's
// default queue.
void build_token_graph(lrq_model_t &m) {
  if (m.token_graph != nullptr) {
    return;
  }
  check_cuda(cudaSetDevice(static_cast<int>(m.device.index())), "cudaSetDevice");
  cudaStream_t stream = static_cast<cudaStream_t>(default_stream(m));
  m.device.synchronize();
  const auto *tasks = static_cast<const sg::Task *>(m.host_tasks->data());
  const lr_launch_config_t config{{m.workers * sg::kWorkerThreads, 1, 1},
                                  {sg::kWorkerThreads, 1, 1},
                                  0};
  uint32_t nodes = 0;
  auto stage = [&](const sg::Stage &st) {
    const sg::HostStepArgs args{static_cast<sg::State *>(m.host_state->data()),
                                tasks + st.task_offset, st.task_count, 0, m.contexts->data()};
    lrrt::launch(m.matched_step, config, args);
    ++nodes;
  };
  check_cuda(cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal),
             "cudaStreamBeginCapture");
  cudaGraph_t graph = nullptr;
  try {
    for (uint32_t layer = 0; layer < m.config.layer_count; ++layer) {
      for (uint32_t program = 0; program < 2; ++program) {
        const sg::CompiledProgram &c = m.plan.programs[program];
        for (uint32_t i = 0; i < c.stage_count; ++i) {
          stage(m.plan.stages[c.stage_offset + i]);
        }
      }
    }
    const sg::CompiledProgram &tail = m.plan.programs[2];
    for (uint32_t i = 0; i < tail.stage_count; ++i) {
      stage(m.plan.stages[tail.stage_offset + i]);
    }
  } catch (...) {
    cudaStreamEndCapture(stream, &graph);
    if (graph != nullptr) {
      cudaGraphDestroy(graph);
    }
    throw;
  }
  check_cuda(cudaStreamEndCapture(stream, &graph), "cudaStreamEndCapture");
  const cudaError_t instantiated = cudaGraphInstantiate(&m.token_graph, graph, 0);
  cudaGraphDestroy(graph);
  check_cuda(instantiated, "cudaGraphInstantiate");
  m.token_graph_nodes = nodes;
}

void launch_graph_steps(lrq_model_t &m, const lrq_decode_request_t &r) {
  build_token_graph(m);
  reset_host_state(m, r);
  cudaStream_t stream = static_cast<cudaStream_t>(default_stream(m));
  for (uint32_t token = 0; token < r.maximum_tokens; ++token) {
    check_cuda(cudaGraphLaunch(m.token_graph, stream), "cudaGraphLaunch");
  }
}

void decode_launch(lrq_model_t &m, lrq_decode_request_t r) {
  if (r.maximum_tokens == 0 || r.maximum_tokens > m.config.max_tokens_per_run ||
      uint64_t{r.token_position} + r.maximum_tokens > m.config.cache_capacity) {
    throw std::invalid_argument("decode request exceeds the model's capacity");
  }
  if (r.max_steps == 0) {
    r.max_steps = 2u * r.maximum_tokens * m.config.layer_count;
  }
  if (r.stop_value == 0) {
    r.stop_value = 1;
  }
  if ((r.path == LRQ_PATH_HOST_STEP || r.path == LRQ_PATH_GRAPH) &&
      r.eos_token != UINT32_MAX) {
    throw std::invalid_argument("the host-step and graph paths run a fixed token count (no EOS)");
  }
  stage_decode_state(m, r.token_position, r.maximum_tokens, r.eos_token);
  async_device_copy(m, *m.decode_state, *m.decode_init, sizeof(qd::DecodeState));
  async_device_copy(m, *m.hidden, *m.hidden_init, qd::kHiddenSize * sizeof(float));
  m.last_path = r.path;
  if (r.path == LRQ_PATH_HOST_STEP) {
    launch_host_steps(m, r);
    return;
  }
  if (r.path == LRQ_PATH_GRAPH) {
    launch_graph_steps(m, r);
    return;
  }
  sg::ResidentExecutor &executor = executor_for(m, r.path);
  if (r.path == LRQ_PATH_STAGE_PROFILE) {
    qd::StageProfile header{};
    if (m.trace) {
      zero_fill(*m.trace);
      header.entries = static_cast<qd::StageProfileEntry *>(m.trace->data());
      header.entry_count = m.trace_capacity;
    }
    lrrt::copy_to_device(*m.profile, &header, sizeof(header));
  }
  executor.initialize_on_device(0, r.max_steps, r.stop_value);
  sg::ResidentArgs args = executor.arguments();
  args.reserved = r.wait_limit_ms;
  lr_launch_config_t config = executor.launch_config();
  if (r.launch_workers != 0) {
    config.grid.x = r.launch_workers * sg::kWorkerThreads;
  }
  lrrt::launch(kernel_for(m, r.path), config, args);
}

void read_state(lrq_model_t &m, lrq_run_state_t *out) {
  m.device.synchronize();
  sg::State state{};
  if (m.last_path == LRQ_PATH_HOST_STEP || m.last_path == LRQ_PATH_GRAPH) {
    lrrt::copy_to_host(&state, *m.host_state, sizeof(state));
  } else {
    state = executor_for(m, m.last_path).read_state();
  }
  qd::DecodeState decode{};
  lrrt::copy_to_host(&decode, *m.decode_state, sizeof(decode));
  qd::Workspace header{};
  lrrt::copy_to_host(&header, *m.workspace, sizeof(header));
  *out = lrq_run_state_t{};
  out->status = state.status;
  out->phase = state.phase;
  out->step = state.step;
  out->max_steps = state.max_steps;
  out->stop_value = state.stop_value;
  out->error_code = state.error_code;
  out->worker_count = state.worker_count;
  out->predicate_value = state.predicate_value;
  out->branch_value = state.branch_value;
  out->executed_tasks = state.executed_tasks;
  out->token_position = decode.token_position;
  out->kv_length = decode.kv_length;
  out->sampled_token = decode.sampled_token;
  out->eos_token = decode.eos_token;
  out->generated_tokens = decode.generated_tokens;
  out->maximum_tokens = decode.maximum_tokens;
  out->stop_reason = decode.stop_reason;
  out->sampled_logit = decode.sampled_logit;
  const bool compiled_family = m.last_path == LRQ_PATH_COMPILED ||
                               m.last_path == LRQ_PATH_STAGE_PROFILE;
  out->fused_path = !compiled_family ? 0u
                    : m.config.disable_fused_path != 0 ? 2u
                                                       : header.reserved[0];
}

lrrt::DeviceBuffer &buffer_for(lrq_model_t &m, uint32_t which, uint32_t layer,
                               size_t &offset, size_t &limit) {
  offset = 0;
  auto whole = [&](lrrt::DeviceBuffer &b) -> lrrt::DeviceBuffer & {
    limit = b.size();
    return b;
  };
  switch (which) {
  case LRQ_BUFFER_HIDDEN: return whole(*m.hidden);
  case LRQ_BUFFER_ATTENTION_NORMALIZED: return whole(*m.attention_normalized);
  case LRQ_BUFFER_QUERY: return whole(*m.query);
  case LRQ_BUFFER_KEY: return whole(*m.key);
  case LRQ_BUFFER_VALUE: return whole(*m.value);
  case LRQ_BUFFER_MLP_NORMALIZED: return whole(*m.mlp_normalized);
  case LRQ_BUFFER_ACTIVATED: return whole(*m.activated);
  case LRQ_BUFFER_PROJECTED: return whole(*m.projected);
  case LRQ_BUFFER_FINAL_NORMALIZED: return whole(*m.final_normalized);
  case LRQ_BUFFER_PARTIAL_VALUES: return whole(*m.partial_values);
  case LRQ_BUFFER_PARTIAL_INDICES: return whole(*m.partial_indices);
  case LRQ_BUFFER_OUTPUT_TOKENS: return whole(*m.output_tokens);
  case LRQ_BUFFER_ROPE_COS: return whole(*m.rope_cos);
  case LRQ_BUFFER_ROPE_SIN: return whole(*m.rope_sin);
  case LRQ_BUFFER_LOGITS:
    if (!m.logits) {
      throw std::invalid_argument("logit capture is not enabled");
    }
    return whole(*m.logits);
  case LRQ_BUFFER_KEY_CACHE:
  case LRQ_BUFFER_VALUE_CACHE:
    if (layer >= m.config.layer_count) {
      throw std::invalid_argument("layer out of range");
    }
    offset = sizeof(float) * m.cache_floats() * layer;
    limit = sizeof(float) * m.cache_floats();
    return which == LRQ_BUFFER_KEY_CACHE ? *m.key_cache : *m.value_cache;
  default:
    throw std::invalid_argument("unknown buffer");
  }
}

} // namespace

extern "C" {

LRRT_API lr_status_t lrq_build_program_table(uint32_t vocab_size,
                                             uint32_t lm_head_partitions,
                                             lrq_task_t *tasks, uint32_t task_capacity,
                                             uint32_t *task_count,
                                             lrq_program_t *programs,
                                             uint32_t program_capacity,
                                             uint32_t *program_count) {
  return guarded("lrq_build_program_table", [&] {
    if (task_count == nullptr || program_count == nullptr) {
      throw std::invalid_argument("null count");
    }
    const ProgramTable table = make_qwen_decoder_programs(vocab_size, lm_head_partitions);
    *task_count = static_cast<uint32_t>(table.tasks.size());
    *program_count = static_cast<uint32_t>(table.programs.size());
    if (tasks == nullptr || programs == nullptr || task_capacity < table.tasks.size() ||
        program_capacity < table.programs.size()) {
      throw std::invalid_argument("program table capacity too small");
    }
    static_assert(sizeof(lrq_task_t) == sizeof(sg::Task));
    static_assert(sizeof(lrq_program_t) == sizeof(sg::Program));
    std::memcpy(tasks, table.tasks.data(), table.tasks.size() * sizeof(sg::Task));
    std::memcpy(programs, table.programs.data(),
                table.programs.size() * sizeof(sg::Program));
  });
}

// Reference RoPE tables (qwen_stateful_graph.cpp:912-929): float exponent
// -2f/64, angle = position * theta^exponent in float, then cos / sin.
LRRT_API lr_status_t lrq_rope_tables(uint32_t positions, float theta, float *cos_table,
                                     float *sin_table) {
  return guarded("lrq_rope_tables", [&] {
    if (cos_table == nullptr || sin_table == nullptr) {
      throw std::invalid_argument("null table");
    }
    for (uint32_t p = 0; p < positions; ++p) {
      for (uint32_t f = 0; f < qd::kRotarySize; ++f) {
        const float exponent =
            -2.0f * static_cast<float>(f) / static_cast<float>(qd::kHeadSize);
        const float angle = static_cast<float>(p) * std::pow(theta, exponent);
        cos_table[size_t{p} * qd::kRotarySize + f] = std::cos(angle);
        sin_table[size_t{p} * qd::kRotarySize + f] = std::sin(angle);
      }
    }
  });
}

LRRT_API lr_status_t lrq_model_device_bytes(const lrq_model_config_t *config,
                                            uint32_t worker_count, uint64_t *bytes) {
  return guarded("lrq_model_device_bytes", [&] {
    if (config == nullptr || bytes == nullptr) {
      throw std::invalid_argument("null argument");
    }
    const uint64_t h = qd::kHiddenSize;
    uint64_t total = sizeof(float) * layer_layout().floats * config->layer_count;
    total += sizeof(float) * uint64_t{config->vocab_size} * h *
             (config->tied_embeddings != 0 ? 1u : 2u);
    total += 2u * sizeof(float) * uint64_t{config->cache_capacity} * qd::kKvSize *
             config->layer_count;
    total += 2u * sizeof(float) * uint64_t{config->cache_capacity} * qd::kRotarySize;
    total += qd::workspace_bytes(std::max(worker_count, 2u)) + (1u << 20);
    *bytes = total;
  });
}

LRRT_API lr_status_t lrq_model_create(lr_device_t device, const void *module_image,
                                      size_t module_image_size,
                                      const lrq_model_config_t *config,
                                      lrq_model_t **model) {
  return guarded("lrq_model_create", [&] {
    if (module_image == nullptr || module_image_size == 0 || config == nullptr ||
        model == nullptr) {
      throw std::invalid_argument("null argument");
    }
    auto created = std::make_unique<lrq_model_t>(lrrt::Device(device), module_image,
                                                 module_image_size, *config);
    build_model(*created);
    *model = created.release();
  });
}

struct lrq_batch_t {
  lrq_model_t *model;
  std::unique_ptr<lrrt::qwen::prefill::BatchDecoder> decoder;
};

LRRT_API lr_status_t lrq_model_destroy(lrq_model_t *model) {
  return guarded("lrq_model_destroy", [&] {
    if (model == nullptr) {
      throw std::invalid_argument("null model");
    }
    for (lrq_batch_t *batch : model->batches) {
      delete batch;
    }
    model->batches.clear();
    if (model->token_graph != nullptr) {
      model->device.synchronize();
      cudaGraphExecDestroy(model->token_graph);
    }
    delete model;
  });
}

LRRT_API lr_status_t lrq_model_set_layer(lrq_model_t *model, uint32_t layer,
                                         const lrq_layer_weights_t *w) {
  return guarded("lrq_model_set_layer", [&] {
    if (model == nullptr || w == nullptr || layer >= model->config.layer_count) {
      throw std::invalid_argument("invalid layer upload");
    }
    const LayerLayout &l = model->layout;
    const size_t h = qd::kHiddenSize, kv = qd::kKvSize, i = qd::kIntermediateSize;
    const struct {
      const float *source;
      size_t offset, count;
    } parts[] = {{w->attention_norm, l.attention_norm, h},
                 {w->q, l.q, h * h},
                 {w->k, l.k, kv * h},
                 {w->v, l.v, kv * h},
                 {w->q_bias, l.q_bias, h},
                 {w->k_bias, l.k_bias, kv},
                 {w->v_bias, l.v_bias, kv},
                 {w->o, l.o, h * h},
                 {w->mlp_norm, l.mlp_norm, h},
                 {w->gate, l.gate, i * h},
                 {w->up, l.up, i * h},
                 {w->down, l.down, h * i}};
    ++model->weights_generation;
    for (const auto &part : parts) {
      if (part.source == nullptr) {
        throw std::invalid_argument("missing layer weight");
      }
      lrrt::check(lr_memcpy(model->device.get(), model->layer_weight(layer, part.offset),
                            part.source, part.count * sizeof(float),
                            LR_MEMCPY_HOST_TO_DEVICE),
                  "lr_memcpy layer weight");
    }
  });
}

LRRT_API lr_status_t lrq_model_replicate_layer(lrq_model_t *model, uint32_t source_layer) {
  return guarded("lrq_model_replicate_layer", [&] {
    if (model == nullptr || source_layer >= model->config.layer_count) {
      throw std::invalid_argument("invalid layer");
    }
    const size_t bytes = model->layout.floats * sizeof(float);
    ++model->weights_generation;
    for (uint32_t layer = 0; layer < model->config.layer_count; ++layer) {
      if (layer != source_layer) {
        lrrt::check(lr_memcpy(model->device.get(), model->layer_weight(layer, 0),
                              model->layer_weight(source_layer, 0), bytes,
                              LR_MEMCPY_DEVICE_TO_DEVICE),
                    "lr_memcpy layer replicate");
      }
    }
  });
}

LRRT_API lr_status_t lrq_model_set_tail(lrq_model_t *model, const float *final_norm,
                                        const float *lm_head, const float *embeddings) {
  return guarded("lrq_model_set_tail", [&] {
    if (model == nullptr || final_norm == nullptr || lm_head == nullptr) {
      throw std::invalid_argument("missing tail weight");
    }
    const size_t table = size_t{model->config.vocab_size} * qd::kHiddenSize * sizeof(float);
    ++model->weights_generation;
    lrrt::copy_to_device(*model->final_norm, final_norm, qd::kHiddenSize * sizeof(float));
    if (model->config.tied_embeddings != 0) {
      lrrt::copy_to_device(*model->embeddings, lm_head, table);
    } else {
      if (embeddings == nullptr) {
        throw std::invalid_argument("untied model needs an embedding table");
      }
      lrrt::copy_to_device(*model->lm_head, lm_head, table);
      lrrt::copy_to_device(*model->embeddings, embeddings, table);
    }
  });
}

LRRT_API lr_status_t lrq_model_load_layer_bundle(lrq_model_t *model, uint32_t layer,
                                                 const char *manifest_path) {
  return guarded("lrq_model_load_layer_bundle", [&] {
    if (model == nullptr || layer >= model->config.layer_count) {
      throw std::invalid_argument("invalid layer");
    }
    namespace wb = lrrt::executor::qwen;
    const wb::DecoderLayerWeights w = wb::load_decoder_layer_weights(manifest_path);
    if (w.shape.hidden != qd::kHiddenSize || w.shape.heads != qd::kAttentionHeads ||
        w.shape.kv_heads != qd::kKvHeads || w.shape.head_dim != qd::kHeadSize ||
        w.shape.intermediate != qd::kIntermediateSize) {
      throw std::invalid_argument(
          "weight bundle shape does not match the model (hidden 896, 14/2 heads of 64, "
          "intermediate 4864)");
    }
    if (w.rope_theta != model->config.rope_theta) {
      throw std::invalid_argument("weight bundle rope_theta differs from the model's");
    }
    const lrq_layer_weights_t upload{
        w.attention_norm_weight.data(), w.q_weight.data(), w.k_weight.data(),
        w.v_weight.data(), w.q_bias.data(), w.k_bias.data(), w.v_bias.data(),
        w.out_weight.data(), w.mlp_norm_weight.data(), w.gate_weight.data(),
        w.up_weight.data(), w.down_weight.data()};
    const lr_status_t status = lrq_model_set_layer(model, layer, &upload);
    if (status != LR_SUCCESS) {
      throw lrrt::Error(status, "lrq_model_set_layer");
    }
  });
}

LRRT_API lr_status_t lrq_model_load_tail_bundle(lrq_model_t *model, const char *manifest_path) {
  return guarded("lrq_model_load_tail_bundle", [&] {
    if (model == nullptr) {
      throw std::invalid_argument("null model");
    }
    namespace wb = lrrt::executor::qwen;
    const wb::ModelTailWeights w = wb::load_model_tail_weights(manifest_path);
    if (w.hidden != qd::kHiddenSize || w.vocab != model->config.vocab_size) {
      throw std::invalid_argument("tail bundle hidden size or vocabulary does not match the model");
    }
    // An untied model needs an embedding row for every token the decode can
    // produce: the bundle's token_ids must then be 0..vocab-1 in order.
    const float *embeddings = nullptr;
    if (model->config.tied_embeddings == 0) {
      bool complete = w.token_ids.size() == w.vocab;
      for (uint32_t i = 0; complete && i < w.vocab; ++i) {
        complete = w.token_ids[i] == i;
      }
      if (!complete) {
        throw std::invalid_argument(
            "untied model: the tail bundle must hold embeddings of token ids 0..vocab-1");
      }
      embeddings = w.token_embeddings.data();
    }
    const lr_status_t status = lrq_model_set_tail(model, w.final_norm_weight.data(),
                                                  w.lm_head_weight.data(), embeddings);
    if (status != LR_SUCCESS) {
      throw lrrt::Error(status, "lrq_model_set_tail");
    }
  });
}

LRRT_API lr_status_t lrq_model_set_kv(lrq_model_t *model, uint32_t layer,
                                      uint32_t first_position, uint32_t positions,
                                      const float *keys, const float *values) {
  return guarded("lrq_model_set_kv", [&] {
    if (model == nullptr || keys == nullptr || values == nullptr ||
        layer >= model->config.layer_count ||
        uint64_t{first_position} + positions > model->config.cache_capacity) {
      throw std::invalid_argument("invalid KV upload");
    }
    const size_t offset =
        (layer * model->cache_floats() + size_t{first_position} * qd::kKvSize) *
        sizeof(float);
    const size_t bytes = size_t{positions} * qd::kKvSize * sizeof(float);
    auto *k = static_cast<unsigned char *>(model->key_cache->data()) + offset;
    auto *v = static_cast<unsigned char *>(model->value_cache->data()) + offset;
    lrrt::check(lr_memcpy(model->device.get(), k, keys, bytes, LR_MEMCPY_HOST_TO_DEVICE),
                "lr_memcpy key cache");
    lrrt::check(lr_memcpy(model->device.get(), v, values, bytes, LR_MEMCPY_HOST_TO_DEVICE),
                "lr_memcpy value cache");
  });
}

LRRT_API lr_status_t lrq_model_set_hidden(lrq_model_t *model, const float *hidden) {
  return guarded("lrq_model_set_hidden", [&] {
    if (model == nullptr || hidden == nullptr) {
      throw std::invalid_argument("null argument");
    }
    lrrt::copy_to_device(*model->hidden_init, hidden, qd::kHiddenSize * sizeof(float));
  });
}

LRRT_API lr_status_t lrq_model_set_hidden_from_token(lrq_model_t *model, uint32_t token) {
  return guarded("lrq_model_set_hidden_from_token", [&] {
    if (model == nullptr || token >= model->config.vocab_size) {
      throw std::invalid_argument("token out of range");
    }
    const size_t row = size_t{token} * qd::kHiddenSize * sizeof(float);
    lrrt::check(lr_memcpy(model->device.get(), model->hidden_init->data(),
                          static_cast<unsigned char *>(model->embeddings->data()) + row,
                          qd::kHiddenSize * sizeof(float), LR_MEMCPY_DEVICE_TO_DEVICE),
                "lr_memcpy embedding row");
  });
}

LRRT_API lr_status_t lrq_decode_launch(lrq_model_t *model,
                                       const lrq_decode_request_t *request) {
  return guarded("lrq_decode_launch", [&] {
    if (model == nullptr || request == nullptr) {
      throw std::invalid_argument("null argument");
    }
    decode_launch(*model, *request);
  });
}

LRRT_API lr_status_t lrq_model_read_state(lrq_model_t *model, lrq_run_state_t *state) {
  return guarded("lrq_model_read_state", [&] {
    if (model == nullptr || state == nullptr) {
      throw std::invalid_argument("null argument");
    }
    read_state(*model, state);
  });
}

LRRT_API lr_status_t lrq_decode(lrq_model_t *model, const lrq_decode_request_t *request,
                                lrq_run_state_t *state, uint32_t *tokens,
                                uint32_t token_capacity) {
  return guarded("lrq_decode", [&] {
    if (model == nullptr || request == nullptr) {
      throw std::invalid_argument("null argument");
    }
    decode_launch(*model, *request);
    lrq_run_state_t local{};
    read_state(*model, state != nullptr ? state : &local);
    if (tokens != nullptr) {
      const uint32_t count = std::min(token_capacity, model->config.max_tokens_per_run);
      lrrt::copy_to_host(tokens, *model->output_tokens, count * sizeof(uint32_t));
    }
  });
}

LRRT_API lr_status_t lrq_model_ingest_prompt(lrq_model_t *model, const uint32_t *prompt,
                                             uint32_t count) {
  return guarded("lrq_model_ingest_prompt", [&] {
    if (model == nullptr || prompt == nullptr || count == 0 ||
        count > model->config.cache_capacity) {
      throw std::invalid_argument("invalid prompt");
    }
    for (uint32_t i = 0; i + 1u < count; ++i) {
      if (prompt[i] >= model->config.vocab_size) {
        throw std::invalid_argument("prompt token out of range");
      }
      lrq_model_set_hidden_from_token(model, prompt[i]);
      const lrq_decode_request_t request{i, 1, UINT32_MAX, LRQ_PATH_COMPILED, 0, 0, 0, 0};
      decode_launch(*model, request);
    }
    if (prompt[count - 1u] >= model->config.vocab_size) {
      throw std::invalid_argument("prompt token out of range");
    }
    model->device.synchronize();
    lrrt::check(static_cast<lr_status_t>(
                    lrq_model_set_hidden_from_token(model, prompt[count - 1u])),
                "stage last prompt token");
  });
}

namespace {

lrrt::qwen::prefill::ModelView prefill_view(lrq_model_t &m) {
  lrrt::qwen::prefill::ModelView view{};
  view.vocab = m.config.vocab_size;
  view.capacity = m.config.cache_capacity;
  view.epsilon = m.config.rms_epsilon;
  view.embeddings = static_cast<const float *>(m.embeddings->data());
  view.lm_head = static_cast<const float *>(m.config.tied_embeddings != 0 ? m.embeddings->data()
                                                                           : m.lm_head->data());
  view.final_norm = static_cast<const float *>(m.final_norm->data());
  view.rope_cos = static_cast<const float *>(m.rope_cos->data());
  view.rope_sin = static_cast<const float *>(m.rope_sin->data());
  const LayerLayout &l = m.layout;
  for (uint32_t layer = 0; layer < m.config.layer_count; ++layer) {
    view.layers.push_back({m.layer_weight(layer, l.attention_norm), m.layer_weight(layer, l.q),
                           m.layer_weight(layer, l.q_bias), m.layer_weight(layer, l.o),
                           m.layer_weight(layer, l.mlp_norm), m.layer_weight(layer, l.gate),
                           m.layer_weight(layer, l.down),
                           static_cast<float *>(m.key_cache->data()) + layer * m.cache_floats(),
                           static_cast<float *>(m.value_cache->data()) + layer * m.cache_floats()});
  }
  return view;
}

void prefill_tokens(lrq_model_t &m, const uint32_t *tokens, uint32_t count,
                    uint32_t first_position, uint32_t path) {
  if (!m.prefill) {
    throw std::logic_error("prefill is not enabled on this model");
  }
  if (path != LRQ_PREFILL_SIMT && path != LRQ_PREFILL_TF32X3) {
    throw std::invalid_argument("unknown prefill path");
  }
  m.prefill->run(prefill_view(m), tokens, count, first_position,
                 static_cast<lrrt::qwen::prefill::Path>(path), m.weights_generation);
}

} // namespace

LRRT_API lr_status_t lrq_model_enable_prefill(lrq_model_t *model, const void *module_image,
                                              size_t module_image_size,
                                              uint32_t max_chunk_tokens) {
  return guarded("lrq_model_enable_prefill", [&] {
    if (model == nullptr || module_image == nullptr || module_image_size == 0) {
      throw std::invalid_argument("null argument");
    }
    // q, k, v (and their biases) and gate, up must be contiguous: the prefill
    // multiplies them as single [1152][896] and [9728][896] matrices.
    const LayerLayout &l = model->layout;
    const size_t h = qd::kHiddenSize, kv = qd::kKvSize, i = qd::kIntermediateSize;
    if (l.k != l.q + h * h || l.v != l.k + kv * h || l.k_bias != l.q_bias + h ||
        l.v_bias != l.k_bias + kv || l.up != l.gate + i * h) {
      throw std::logic_error("layer layout does not keep QKV and gate/up contiguous");
    }
    if (!model->batches.empty()) {
      throw std::logic_error("destroy the model's batches before reloading the prefill module");
    }
    model->prefill.reset();
    model->prefill = std::make_unique<lrrt::qwen::prefill::Prefill>(
        model->device, module_image, module_image_size,
        max_chunk_tokens == 0 ? 512u : max_chunk_tokens);
  });
}

LRRT_API lr_status_t lrq_model_prefill_at(lrq_model_t *model, const uint32_t *tokens,
                                          uint32_t count, uint32_t first_position,
                                          uint32_t path) {
  return guarded("lrq_model_prefill_at", [&] {
    if (model == nullptr || (tokens == nullptr && count != 0)) {
      throw std::invalid_argument("null argument");
    }
    prefill_tokens(*model, tokens, count, first_position, path);
  });
}

LRRT_API lr_status_t lrq_prefill_gemm_check(lrq_model_t *model, uint32_t tile_columns,
                                            uint32_t mode, uint32_t m, uint32_t n, uint32_t k,
                                            const float *a, const float *b, const float *bias,
                                            float *c) {
  return guarded("lrq_prefill_gemm_check", [&] {
    if (model == nullptr || a == nullptr || b == nullptr || c == nullptr || mode > 2) {
      throw std::invalid_argument("invalid GEMM check");
    }
    if (!model->prefill) {
      throw std::logic_error("prefill is not enabled on this model");
    }
    model->prefill->gemm_check(tile_columns, static_cast<lrrt::qwen::prefill::GemmEpilogue>(mode),
                               m, n, k, a, b, bias, c);
  });
}

LRRT_API lr_status_t lrq_model_prefill(lrq_model_t *model, const uint32_t *prompt,
                                       uint32_t count, uint32_t path) {
  return guarded("lrq_model_prefill", [&] {
    if (model == nullptr || prompt == nullptr || count == 0 ||
        count > model->config.cache_capacity) {
      throw std::invalid_argument("invalid prompt");
    }
    if (prompt[count - 1u] >= model->config.vocab_size) {
      throw std::invalid_argument("prompt token out of range");
    }
    prefill_tokens(*model, prompt, count - 1u, 0, path);
    lrrt::check(static_cast<lr_status_t>(
                    lrq_model_set_hidden_from_token(model, prompt[count - 1u])),
                "stage last prompt token");
  });
}

LRRT_API lr_status_t lrq_batch_create(lrq_model_t *model, uint32_t streams, uint32_t capacity,
                                      uint32_t max_tokens, lrq_batch_t **batch) {
  return guarded("lrq_batch_create", [&] {
    if (model == nullptr || batch == nullptr) {
      throw std::invalid_argument("null argument");
    }
    if (!model->prefill) {
      throw std::logic_error("prefill is not enabled on this model");
    }
    auto created = std::make_unique<lrq_batch_t>();
    created->model = model;
    created->decoder = std::make_unique<lrrt::qwen::prefill::BatchDecoder>(
        *model->prefill, prefill_view(*model), streams, capacity, max_tokens);
    model->batches.push_back(created.get());
    *batch = created.release();
  });
}

LRRT_API lr_status_t lrq_batch_destroy(lrq_batch_t *batch) {
  return guarded("lrq_batch_destroy", [&] {
    if (batch == nullptr) {
      throw std::invalid_argument("null batch");
    }
    auto &list = batch->model->batches;
    list.erase(std::remove(list.begin(), list.end(), batch), list.end());
    delete batch;
  });
}

LRRT_API lr_status_t lrq_batch_prefill(lrq_batch_t *batch, uint32_t stream,
                                       const uint32_t *prompt, uint32_t count, uint32_t path) {
  return guarded("lrq_batch_prefill", [&] {
    if (batch == nullptr || prompt == nullptr) {
      throw std::invalid_argument("null argument");
    }
    if (path != LRQ_PREFILL_SIMT && path != LRQ_PREFILL_TF32X3) {
      throw std::invalid_argument("unknown prefill path");
    }
    lrq_model_t &m = *batch->model;
    batch->decoder->prefill_stream(prefill_view(m), stream, prompt, count,
                                   static_cast<lrrt::qwen::prefill::Path>(path),
                                   m.weights_generation);
  });
}

LRRT_API lr_status_t lrq_batch_decode(lrq_batch_t *batch, uint32_t steps, uint32_t *tokens,
                                      float *last_logits) {
  return guarded("lrq_batch_decode", [&] {
    if (batch == nullptr) {
      throw std::invalid_argument("null batch");
    }
    lrq_model_t &m = *batch->model;
    batch->decoder->decode(prefill_view(m), steps, m.weights_generation, tokens, last_logits);
  });
}

LRRT_API lr_status_t lrq_batch_read_cache(lrq_batch_t *batch, uint32_t stream, uint32_t layer,
                                          uint32_t positions, float *keys, float *values) {
  return guarded("lrq_batch_read_cache", [&] {
    if (batch == nullptr) {
      throw std::invalid_argument("null batch");
    }
    batch->decoder->read_cache(stream, layer, positions, keys, values);
  });
}

LRRT_API lr_status_t lrq_batch_write_cache(lrq_batch_t *batch, uint32_t stream, uint32_t layer,
                                           uint32_t first_position, uint32_t positions,
                                           const float *keys, const float *values) {
  return guarded("lrq_batch_write_cache", [&] {
    if (batch == nullptr) {
      throw std::invalid_argument("null batch");
    }
    batch->decoder->write_cache(stream, layer, first_position, positions, keys, values);
  });
}

LRRT_API lr_status_t lrq_batch_set_next(lrq_batch_t *batch, uint32_t stream, uint32_t position,
                                        uint32_t token) {
  return guarded("lrq_batch_set_next", [&] {
    if (batch == nullptr) {
      throw std::invalid_argument("null batch");
    }
    batch->decoder->set_next(stream, position, token, batch->model->config.vocab_size);
  });
}

LRRT_API lr_status_t lrq_batch_position(lrq_batch_t *batch, uint32_t stream, uint32_t *position) {
  return guarded("lrq_batch_position", [&] {
    if (batch == nullptr || position == nullptr || stream >= batch->decoder->streams()) {
      throw std::invalid_argument("invalid batch position query");
    }
    *position = batch->decoder->position(stream);
  });
}

LRRT_API lr_status_t lrq_generate(lrq_model_t *model, const float *hidden,
                                  uint32_t start_token, uint32_t token_position,
                                  uint32_t maximum_tokens, uint32_t eos_token,
                                  uint32_t *tokens, lrq_run_state_t *state) {
  return guarded("lrq_generate", [&] {
    if (model == nullptr || tokens == nullptr) {
      throw std::invalid_argument("null argument");
    }
    if (hidden != nullptr) {
      lrrt::check(lr_memcpy_async(model->device.get(), model->hidden_init->data(), hidden,
                                  qd::kHiddenSize * sizeof(float),
                                  LR_MEMCPY_HOST_TO_DEVICE, nullptr),
                  "lr_memcpy_async hidden");
    } else {
      if (start_token >= model->config.vocab_size) {
        throw std::invalid_argument("token out of range");
      }
      lrrt::check(lr_memcpy_async(model->device.get(), model->hidden_init->data(),
                                  static_cast<unsigned char *>(model->embeddings->data()) +
                                      size_t{start_token} * qd::kHiddenSize * sizeof(float),
                                  qd::kHiddenSize * sizeof(float),
                                  LR_MEMCPY_DEVICE_TO_DEVICE, nullptr),
                  "lr_memcpy_async embedding row");
    }
    const lrq_decode_request_t request{token_position, maximum_tokens, eos_token,
                                       LRQ_PATH_COMPILED, 0, 0, 0, 0};
    decode_launch(*model, request);
    lrrt::check(lr_memcpy_async(model->device.get(), tokens, model->output_tokens->data(),
                                size_t{maximum_tokens} * sizeof(uint32_t),
                                LR_MEMCPY_DEVICE_TO_HOST, nullptr),
                "lr_memcpy_async tokens");
    model->device.synchronize();
    if (state != nullptr) {
      read_state(*model, state);
    }
  });
}

LRRT_API lr_status_t lrq_model_read(lrq_model_t *model, uint32_t buffer, uint32_t layer,
                                    void *destination, size_t bytes) {
  return guarded("lrq_model_read", [&] {
    if (model == nullptr || destination == nullptr) {
      throw std::invalid_argument("null argument");
    }
    size_t offset = 0, limit = 0;
    lrrt::DeviceBuffer &source = buffer_for(*model, buffer, layer, offset, limit);
    if (bytes > limit) {
      throw std::invalid_argument("read exceeds buffer");
    }
    lrrt::check(lr_memcpy(model->device.get(), destination,
                          static_cast<unsigned char *>(source.data()) + offset, bytes,
                          LR_MEMCPY_DEVICE_TO_HOST),
                "lr_memcpy read");
  });
}

LRRT_API lr_status_t lrq_model_info(lrq_model_t *model, lrq_model_info_t *info) {
  return guarded("lrq_model_info", [&] {
    if (model == nullptr || info == nullptr) {
      throw std::invalid_argument("null argument");
    }
    info->worker_count = model->workers;
    info->lm_head_partitions = model->partitions;
    info->layer_count = model->config.layer_count;
    info->vocab_size = model->config.vocab_size;
    info->cache_capacity = model->config.cache_capacity;
    info->dynamic_shared_bytes = model->shared_bytes;
    info->phase_state_count = model->phase_state_count;
    info->task_count = static_cast<uint32_t>(model->table.tasks.size());
    info->device_bytes = model->device_bytes;
    info->weight_bytes_per_token =
        algorithmic_weight_bytes(model->config.layer_count, model->config.vocab_size);
  });
}

LRRT_API lr_status_t lrq_model_stage_profile(lrq_model_t *model, uint64_t *ticks,
                                             uint64_t *counts) {
  return guarded("lrq_model_stage_profile", [&] {
    if (model == nullptr || ticks == nullptr || counts == nullptr) {
      throw std::invalid_argument("null argument");
    }
    qd::StageProfile profile{};
    lrrt::copy_to_host(&profile, *model->profile, sizeof(profile));
    std::memcpy(ticks, profile.stage_ticks, sizeof(profile.stage_ticks));
    std::memcpy(counts, profile.stage_counts, sizeof(profile.stage_counts));
  });
}

LRRT_API lr_status_t lrq_model_run_graph(lrq_model_t *model, const lrq_task_t *tasks,
                                         uint32_t task_count, const lrq_program_t *programs,
                                         uint32_t program_count, uint32_t path,
                                         uint32_t program_index, uint32_t max_steps,
                                         uint32_t stop_value, uint32_t token_position,
                                         uint32_t maximum_tokens, lrq_run_state_t *state) {
  return guarded("lrq_model_run_graph", [&] {
    if (model == nullptr || tasks == nullptr || programs == nullptr || state == nullptr ||
        (path != LRQ_PATH_COMPILED && path != LRQ_PATH_DYNAMIC)) {
      throw std::invalid_argument("invalid custom graph run");
    }
    lrq_model_t &m = *model;
    const std::vector<sg::Task> custom_tasks(
        reinterpret_cast<const sg::Task *>(tasks),
        reinterpret_cast<const sg::Task *>(tasks) + task_count);
    const std::vector<sg::Program> custom_programs(
        reinterpret_cast<const sg::Program *>(programs),
        reinterpret_cast<const sg::Program *>(programs) + program_count);
    sg::ResidentExecutor &executor = executor_for(m, path);
    // Restore the decode graph whatever happens to the custom one.
    struct Restore {
      lrq_model_t &m;
      sg::ResidentExecutor &executor;
      uint32_t path;
      ~Restore() {
        try {
          if (path == LRQ_PATH_COMPILED) {
            executor.upload_graph(m.table.tasks, m.table.programs, m.plan);
          } else {
            executor.upload_graph(m.table.tasks, m.table.programs);
          }
        } catch (...) {
        }
      }
    } restore{m, executor, path};
    if (path == LRQ_PATH_COMPILED) {
      const sg::ResidentConfig config{m.phase_state_count, m.workers, m.shared_bytes, 0};
      const sg::CompiledPlan plan =
          sg::compile_resident_plan(custom_tasks, custom_programs, config);
      executor.upload_graph(custom_tasks, custom_programs, plan);
    } else {
      executor.upload_graph(custom_tasks, custom_programs);
    }
    stage_decode_state(m, token_position, maximum_tokens, UINT32_MAX);
    async_device_copy(m, *m.decode_state, *m.decode_init, sizeof(qd::DecodeState));
    async_device_copy(m, *m.hidden, *m.hidden_init, qd::kHiddenSize * sizeof(float));
    executor.initialize(program_index, max_steps, stop_value);
    executor.launch();
    m.last_path = path;
    read_state(m, state);
  });
}

LRRT_API lr_status_t lrq_model_set_trace(lrq_model_t *model, uint32_t entries) {
  return guarded("lrq_model_set_trace", [&] {
    if (model == nullptr) {
      throw std::invalid_argument("null model");
    }
    model->trace.reset();
    model->trace_capacity = 0;
    if (entries != 0) {
      model->trace.emplace(model->device, size_t{entries} * sizeof(qd::StageProfileEntry));
      model->trace_capacity = entries;
    }
  });
}

LRRT_API lr_status_t lrq_workspace_bytes(uint32_t worker_count, uint64_t *bytes) {
  return guarded("lrq_workspace_bytes", [&] {
    if (bytes == nullptr || worker_count == 0 || worker_count > sg::kMaximumResidentWorkers) {
      throw std::invalid_argument("null output or worker count out of range");
    }
    *bytes = qd::workspace_bytes(std::max(worker_count, 2u));
  });
}

LRRT_API lr_status_t lrq_workspace_init(lr_device_t device, void *workspace, uint64_t bytes,
                                        uint32_t worker_count, const void *contexts,
                                        uint32_t layer_count) {
  return guarded("lrq_workspace_init", [&] {
    if (contexts == nullptr || layer_count == 0 || worker_count == 0 ||
        worker_count > sg::kMaximumResidentWorkers) {
      throw std::invalid_argument("null Context array, no layers or worker count out of range");
    }
    const auto *layers = static_cast<const qd::Context *>(contexts);
    std::vector<KvCacheView> caches(layer_count);
    for (uint32_t layer = 0; layer < layer_count; ++layer) {
      caches[layer] = {layers[layer].key_cache, layers[layer].value_cache,
                       layers[layer].cache_capacity, layers[layer].out_weight};
    }
    init_workspace(device, workspace, bytes, std::max(worker_count, 2u), caches);
  });
}

LRRT_API lr_status_t lrq_workspace_path(lr_device_t device, const void *workspace,
                                        uint32_t *path) {
  return guarded("lrq_workspace_path", [&] {
    if (workspace == nullptr || path == nullptr) {
      throw std::invalid_argument("null argument");
    }
    qd::Workspace header{};
    lrrt::check(lr_memcpy(device, &header, workspace, sizeof(header), LR_MEMCPY_DEVICE_TO_HOST),
                "lr_memcpy workspace header");
    *path = header.reserved[0];
  });
}

LRRT_API lr_status_t lrq_model_set_logit_capture(lrq_model_t *model, uint32_t enable) {
  return guarded("lrq_model_set_logit_capture", [&] {
    if (model == nullptr) {
      throw std::invalid_argument("null model");
    }
    lrrt::check(lr_synchronize(model->device.get()), "lr_synchronize");
    if (enable != 0 && !model->logits) {
      model->logits.emplace(model->device, sizeof(float) * size_t{model->config.vocab_size});
      zero_fill(*model->logits);
    }
    float *pointer = enable != 0 ? static_cast<float *>(model->logits->data()) : nullptr;
    auto *field = static_cast<unsigned char *>(model->workspace->data()) +
                  offsetof(qd::Workspace, logits);
    lrrt::check(lr_memcpy(model->device.get(), field, &pointer, sizeof(pointer),
                          LR_MEMCPY_HOST_TO_DEVICE),
                "lr_memcpy logit capture");
  });
}

LRRT_API lr_status_t lrq_model_read_trace(lrq_model_t *model, uint64_t *entries,
                                          uint32_t capacity) {
  return guarded("lrq_model_read_trace", [&] {
    if (model == nullptr || entries == nullptr || !model->trace ||
        capacity > model->trace_capacity) {
      throw std::invalid_argument("invalid trace read");
    }
    lrrt::copy_to_host(entries, *model->trace, size_t{capacity} * sizeof(qd::StageProfileEntry));
  });
}

LRRT_API lr_status_t lrq_lm_head_top1_static(lr_device_t device, lr_queue_t *queue,
                                             const float *lm_head, const float *hidden,
                                             uint32_t rows, uint32_t columns,
                                             uint32_t blocks, uint32_t *token,
                                             float *logit) {
  void *stream = nullptr;
  lr_status_t status = lr_queue_native_handle(device, queue, &stream);
  if (status != LR_SUCCESS) {
    set_error("lrq_lm_head_top1_static: lr_queue_native_handle failed");
    return status;
  }
  std::string error;
  status = lrq_static::lm_head_top1(device.index, stream, lm_head, hidden, rows, columns,
                                    blocks, token, logit, error);
  if (status != LR_SUCCESS) {
    set_error("lrq_lm_head_top1_static: " + error);
  }
  return status;
}

LRRT_API const char *lrq_last_error(void) {
  std::lock_guard<std::mutex> lock(g_error_mutex);
  static thread_local std::string copy;
  copy = g_last_error;
  return copy.c_str();
}

} // extern "C"
