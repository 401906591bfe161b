// A caller that drives the sm_100a decode kernel the way the reference's
// driver does (benchmarks/qwen_stateful_graph.cpp:730-1118, 1256-1340): it
// allocates every buffer itself, builds the Context / TailContext arrays on
// the host, uploads them, and launches through ResidentExecutor. The only
// B200 additions are the two a reference caller needs for the fast path: a
// workspace initialised with lrq_workspace_init (its pointer in
// TailContext::workspace) and the fused path's dynamic shared memory in
// ResidentConfig. The pytest wrapper writes the weights and checks the
// tokens against the CPU oracle.
//
// Usage: reference_caller_test <qwen_stateful_graph.cubin> <io directory>
// The directory holds raw little-endian files: meta (u32 layers, vocab,
// position, tokens), per layer l<i>_<name> float32 arrays (attention_norm,
// q, k, v, q_bias, k_bias, v_bias, o, mlp_norm, gate, up, down), lm_head
// [vocab][896], final_norm [896], hidden [896]. It writes tokens (u32 x
// tokens) and result (u32 status, error_code, fused path, sampled_token).
#include "lrrt/lrrt.hpp"
#include "lrrt/persistent_graph.hpp"
#include "lrrt/qwen/resident_layout.hpp"
#include "lrrt/qwen/stateful_graph_context.hpp"
#include "lrrt_qwen.h"

#include <cstdio>
#include <cstring>
#include <fstream>
#include <iterator>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

namespace sg = lrrt::persistent_graph;
namespace qd = lrrt::qwen::stateful_graph;

namespace {

std::vector<unsigned char> read_file(const std::string &path) {
  std::ifstream in(path, std::ios::binary);
  if (!in) {
    throw std::runtime_error("cannot open " + path);
  }
  return std::vector<unsigned char>(std::istreambuf_iterator<char>(in), {});
}

template <typename T> std::vector<T> read_array(const std::string &path, size_t count) {
  const std::vector<unsigned char> bytes = read_file(path);
  if (bytes.size() != count * sizeof(T)) {
    throw std::runtime_error(path + ": expected " + std::to_string(count * sizeof(T)) +
                             " bytes, found " + std::to_string(bytes.size()));
  }
  std::vector<T> values(count);
  std::memcpy(values.data(), bytes.data(), bytes.size());
  return values;
}

void write_array(const std::string &path, const void *data, size_t bytes) {
  std::ofstream out(path, std::ios::binary);
  out.write(static_cast<const char *>(data), static_cast<std::streamsize>(bytes));
  if (!out) {
    throw std::runtime_error("cannot write " + path);
  }
}

void check_lrq(lr_status_t status, const char *what) {
  if (status != LR_SUCCESS) {
    throw std::runtime_error(std::string(what) + ": " + lrq_last_error());
  }
}

// Device copy of a host array, owned by `keep`.
template <typename T>
T *upload(lrrt::Device device, const std::vector<T> &host,
          std::vector<std::unique_ptr<lrrt::DeviceBuffer>> &keep) {
  keep.push_back(std::make_unique<lrrt::DeviceBuffer>(device, sizeof(T) * host.size()));
  lrrt::copy_to_device(*keep.back(), host);
  return static_cast<T *>(keep.back()->data());
}

template <typename T>
T *zeros(lrrt::Device device, size_t count,
         std::vector<std::unique_ptr<lrrt::DeviceBuffer>> &keep) {
  return upload(device, std::vector<T>(count, T{}), keep);
}

} // namespace

int main(int argc, char **argv) {
  if (argc != 3) {
    std::fprintf(stderr, "usage: %s <qwen_stateful_graph.cubin> <io directory>\n", argv[0]);
    return 2;
  }
  const std::string io = std::string(argv[2]) + "/";
  try {
    const std::vector<uint32_t> meta = read_array<uint32_t>(io + "meta", 4);
    const uint32_t layers = meta[0], vocab = meta[1], position = meta[2], tokens = meta[3];
    const uint32_t capacity = position + tokens + 8;
    constexpr uint32_t h = qd::kHiddenSize, q = qd::kQuerySize, kv = qd::kKvSize,
                       inter = qd::kIntermediateSize;

    lrrt::Runtime runtime;
    lrrt::Device device = runtime.open_device(0);
    const std::vector<unsigned char> image = read_file(argv[1]);
    lrrt::Module module(device, image.data(), image.size());
    lrrt::Kernel kernel = module.kernel("qwen_stateful_graph_compiled_kernel");
    const uint32_t shared = qd::resident::kFusedSharedBytes;
    const sg::ResidentAdmission admitted =
        sg::admit_resident_workers(device, kernel, sg::kMaximumResidentWorkers,
                                   sg::kWorkerThreads, shared);
    const uint32_t workers = admitted.worker_count;
    const uint32_t partitions = std::min({vocab, qd::kMaximumLmHeadPartitions, workers});

    // Task / Program table (make_qwen_decoder_programs) and RoPE tables.
    std::vector<lrq_task_t> table_tasks(256);
    std::vector<lrq_program_t> table_programs(4);
    uint32_t task_count = 0, program_count = 0;
    check_lrq(lrq_build_program_table(vocab, partitions, table_tasks.data(), 256, &task_count,
                                      table_programs.data(), 4, &program_count),
              "lrq_build_program_table");
    std::vector<sg::Task> tasks(task_count);
    std::vector<sg::Program> programs(program_count);
    std::memcpy(tasks.data(), table_tasks.data(), sizeof(sg::Task) * task_count);
    std::memcpy(programs.data(), table_programs.data(), sizeof(sg::Program) * program_count);
    std::vector<float> rope_cos(size_t{capacity} * qd::kRotarySize),
        rope_sin(size_t{capacity} * qd::kRotarySize);
    check_lrq(lrq_rope_tables(capacity, 1.0e6f, rope_cos.data(), rope_sin.data()),
              "lrq_rope_tables");

    // Every buffer the caller owns.
    std::vector<std::unique_ptr<lrrt::DeviceBuffer>> keep;
    float *hidden = upload(device, read_array<float>(io + "hidden", h), keep);
    float *attention_normalized = zeros<float>(device, h, keep);
    float *query = zeros<float>(device, q, keep);
    float *key = zeros<float>(device, kv, keep);
    float *value = zeros<float>(device, kv, keep);
    float *mlp_normalized = zeros<float>(device, h, keep);
    float *activated = zeros<float>(device, inter, keep);
    float *projected = zeros<float>(device, h, keep);
    const float *cos_table = upload(device, rope_cos, keep);
    const float *sin_table = upload(device, rope_sin, keep);

    qd::TailContext tail{};
    tail.final_norm_weight = upload(device, read_array<float>(io + "final_norm", h), keep);
    tail.lm_head_weight =
        upload(device, read_array<float>(io + "lm_head", size_t{vocab} * h), keep);
    tail.token_embeddings = tail.lm_head_weight; // tied
    tail.final_normalized = zeros<float>(device, h, keep);
    tail.partial_max_values = zeros<float>(device, qd::kMaximumLmHeadPartitions, keep);
    tail.partial_max_indices = zeros<uint32_t>(device, qd::kMaximumLmHeadPartitions, keep);
    qd::DecodeState decode{};
    decode.token_position = position;
    decode.kv_length = position;
    decode.eos_token = UINT32_MAX;
    decode.maximum_tokens = tokens;
    keep.push_back(std::make_unique<lrrt::DeviceBuffer>(device, sizeof(decode)));
    lrrt::copy_to_device(*keep.back(), &decode, sizeof(decode));
    tail.decode_state = static_cast<qd::DecodeState *>(keep.back()->data());
    tail.output_tokens = zeros<uint32_t>(device, tokens, keep);
    tail.vocab_size = vocab;
    tail.partition_count = partitions;
    tail.embedding_count = vocab;

    std::vector<qd::Context> contexts(layers);
    auto layer_array = [&](uint32_t layer, const char *name, size_t count) {
      return upload(device, read_array<float>(io + "l" + std::to_string(layer) + "_" + name,
                                              count),
                    keep);
    };
    for (uint32_t l = 0; l < layers; ++l) {
      qd::Context &x = contexts[l];
      x.hidden = hidden;
      x.attention_norm_weight = layer_array(l, "attention_norm", h);
      x.q_weight = layer_array(l, "q", size_t{q} * h);
      x.k_weight = layer_array(l, "k", size_t{kv} * h);
      x.v_weight = layer_array(l, "v", size_t{kv} * h);
      x.q_bias = layer_array(l, "q_bias", q);
      x.k_bias = layer_array(l, "k_bias", kv);
      x.v_bias = layer_array(l, "v_bias", kv);
      x.out_weight = layer_array(l, "o", size_t{h} * q);
      x.mlp_norm_weight = layer_array(l, "mlp_norm", h);
      x.gate_weight = layer_array(l, "gate", size_t{inter} * h);
      x.up_weight = layer_array(l, "up", size_t{inter} * h);
      x.down_weight = layer_array(l, "down", size_t{h} * inter);
      x.attention_normalized = attention_normalized;
      x.query = query;
      x.key = key;
      x.value = value;
      x.rope_cos = cos_table;
      x.rope_sin = sin_table;
      x.key_cache = zeros<float>(device, size_t{capacity} * kv, keep);
      x.value_cache = zeros<float>(device, size_t{capacity} * kv, keep);
      x.mlp_normalized = mlp_normalized;
      x.activated = activated;
      x.projected = projected;
      x.hidden_size = h;
      x.query_size = q;
      x.kv_size = kv;
      x.intermediate_size = inter;
      x.cache_capacity = capacity;
      x.layer_count = layers;
    }

    // The fast path's workspace, in the TailContext's tail padding.
    uint64_t workspace_bytes = 0;
    check_lrq(lrq_workspace_bytes(workers, &workspace_bytes), "lrq_workspace_bytes");
    lrrt::DeviceBuffer workspace(device, workspace_bytes);
    check_lrq(lrq_workspace_init(device.get(), workspace.data(), workspace_bytes, workers,
                                 contexts.data(), layers),
              "lrq_workspace_init");
    tail.workspace = static_cast<qd::Workspace *>(workspace.data());
    keep.push_back(std::make_unique<lrrt::DeviceBuffer>(device, sizeof(tail)));
    lrrt::copy_to_device(*keep.back(), &tail, sizeof(tail));
    auto *tail_device = static_cast<qd::TailContext *>(keep.back()->data());
    for (qd::Context &x : contexts) {
      x.tail = tail_device;
    }
    keep.push_back(std::make_unique<lrrt::DeviceBuffer>(device, sizeof(qd::Context) * layers));
    lrrt::copy_to_device(*keep.back(), contexts.data(), sizeof(qd::Context) * layers);
    void *context_device = keep.back()->data();

    // Resident run: the reference's phase-slot sizing, initialise, launch.
    const uint32_t phase_states = tokens * 2u * (2u * layers + 1u) + 1u;
    const sg::ResidentConfig config{phase_states, workers, shared, 0};
    const sg::CompiledPlan plan = sg::compile_resident_plan(tasks, programs, config);
    sg::ResidentExecutor executor(device, kernel, tasks, programs, config, plan);
    executor.bind_context(context_device);
    executor.initialize(0, 2u * tokens * layers, 1);
    executor.launch();
    device.synchronize();
    const sg::State state = executor.read_state();

    std::vector<uint32_t> out(tokens);
    lrrt::check(lr_memcpy(device.get(), out.data(), tail.output_tokens,
                          sizeof(uint32_t) * tokens, LR_MEMCPY_DEVICE_TO_HOST),
                "lr_memcpy tokens");
    qd::DecodeState final_decode{};
    lrrt::check(lr_memcpy(device.get(), &final_decode, tail.decode_state, sizeof(final_decode),
                          LR_MEMCPY_DEVICE_TO_HOST),
                "lr_memcpy decode state");
    uint32_t path = 0;
    check_lrq(lrq_workspace_path(device.get(), workspace.data(), &path), "lrq_workspace_path");
    write_array(io + "tokens", out.data(), sizeof(uint32_t) * tokens);
    const uint32_t result[4] = {state.status, state.error_code, path, final_decode.sampled_token};
    write_array(io + "result", result, sizeof(result));
    std::printf("reference-style run: status %u, error %u, path %u, %u workers\n", state.status,
                state.error_code, path, workers);
  } catch (const std::exception &error) {
    std::fprintf(stderr, "error: %s\n", error.what());
    return 1;
  }
  return 0;
}
