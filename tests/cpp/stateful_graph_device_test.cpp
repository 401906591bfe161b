// Scheduler fixture on the GPU through the lrrt C++ API and ResidentExecutor
// (light-rocm-runtime tests/stateful_graph_device.cpp:139-239, same graph,
// same three runs per path). Prints the observed state and arrays as JSON for
// the pytest driver, which compares them with tests/golden/scheduler_fixture.json.
// Usage: stateful_graph_device_test <stateful_graph_fixture.cubin>
#include "lrrt/lrrt.hpp"
#include "lrrt/persistent_graph.hpp"

#include <array>
#include <cstdio>
#include <fstream>
#include <iterator>
#include <stdexcept>
#include <string>
#include <vector>

namespace sg = lrrt::persistent_graph;

namespace {

struct FixtureContext {
  uint32_t magic;
  uint32_t value_count;
  uint32_t *values;
  uint32_t *step_checksums;
  uint32_t *branch_steps;
  uint32_t *task_executions;
  uint32_t *validation_calls;
};

template <size_t N> std::string json_array(const std::array<uint32_t, N> &values) {
  std::string text = "[";
  for (size_t i = 0; i < N; ++i) {
    text += (i ? "," : "") + std::to_string(values[i]);
  }
  return text + "]";
}

struct Buffers {
  explicit Buffers(lrrt::Device device)
      : values(device, 8 * 4), checksums(device, 8 * 4), branch_steps(device, 8 * 4),
        executions(device, 5 * 4), validation_calls(device, 4),
        context(device, sizeof(FixtureContext)) {}

  void reset(bool validation) {
    const std::array<uint32_t, 8> zero8{};
    const std::array<uint32_t, 5> zero5{};
    lrrt::copy_to_device(values, zero8.data(), sizeof(zero8));
    lrrt::copy_to_device(checksums, zero8.data(), sizeof(zero8));
    lrrt::copy_to_device(branch_steps, zero8.data(), sizeof(zero8));
    lrrt::copy_to_device(executions, zero5.data(), sizeof(zero5));
    if (validation) {
      const uint32_t zero = 0;
      lrrt::copy_to_device(validation_calls, &zero, sizeof(zero));
    }
    const FixtureContext host{0x53504754u,
                              8,
                              static_cast<uint32_t *>(values.data()),
                              static_cast<uint32_t *>(checksums.data()),
                              static_cast<uint32_t *>(branch_steps.data()),
                              static_cast<uint32_t *>(executions.data()),
                              static_cast<uint32_t *>(validation_calls.data())};
    lrrt::copy_to_device(context, &host, sizeof(host));
  }

  lrrt::DeviceBuffer values, checksums, branch_steps, executions, validation_calls, context;
};

std::string run_path(lrrt::Device device, const lrrt::Kernel &kernel,
                     const std::vector<sg::Task> &tasks,
                     const std::vector<sg::Program> &programs,
                     const sg::ResidentConfig &config, const sg::CompiledPlan *plan,
                     Buffers &buffers) {
  buffers.reset(true);
  sg::ResidentExecutor executor =
      plan == nullptr ? sg::ResidentExecutor(device, kernel, tasks, programs, config)
                      : sg::ResidentExecutor(device, kernel, tasks, programs, config, *plan);
  executor.bind_context(buffers.context.data());
  std::string runs = "[";
  for (uint32_t run = 0; run < 3; ++run) {
    if (run != 0) {
      buffers.reset(false);
    }
    if (run == 2) {
      executor.bind_context(buffers.context.data()); // re-binding invalidates the cache
    }
    executor.initialize(0, 8, 2);
    executor.launch();
    device.synchronize();
    const sg::State s = executor.read_state();
    std::array<uint32_t, 8> values{}, checksums{}, branch_steps{};
    std::array<uint32_t, 5> executions{};
    uint32_t calls = 0;
    lrrt::copy_to_host(values.data(), buffers.values, sizeof(values));
    lrrt::copy_to_host(checksums.data(), buffers.checksums, sizeof(checksums));
    lrrt::copy_to_host(branch_steps.data(), buffers.branch_steps, sizeof(branch_steps));
    lrrt::copy_to_host(executions.data(), buffers.executions, sizeof(executions));
    lrrt::copy_to_host(&calls, buffers.validation_calls, sizeof(calls));
    char state[512];
    std::snprintf(state, sizeof(state),
                  "{\"status\":%u,\"step\":%u,\"predicate_value\":%u,\"branch_value\":%u,"
                  "\"executed_tasks\":%llu,\"error_code\":%u,\"phase\":%u,",
                  s.status, s.step, s.predicate_value, s.branch_value,
                  static_cast<unsigned long long>(s.executed_tasks), s.error_code, s.phase);
    runs += std::string(run ? "," : "") + state + "\"values\":" + json_array(values) +
            ",\"checksums\":" + json_array(checksums) +
            ",\"branch_steps\":" + json_array(branch_steps) +
            ",\"task_executions\":" + json_array(executions) +
            ",\"validation_calls\":" + std::to_string(calls) + "}";
  }
  return runs + "]";
}

} // namespace

int main(int argc, char **argv) {
  try {
    if (argc < 2) {
      throw std::invalid_argument("usage: stateful_graph_device_test <cubin>");
    }
    lrrt::Runtime runtime;
    if (runtime.device_count() == 0) {
      std::printf("{\"skipped\": \"no GPU devices\"}\n");
      return 0;
    }
    const lrrt::Device device = runtime.open_device(0);
    std::ifstream file(argv[1], std::ios::binary);
    const std::vector<unsigned char> image((std::istreambuf_iterator<char>(file)),
                                           std::istreambuf_iterator<char>());
    const lrrt::Module module(device, image);
    const lrrt::Kernel dynamic = module.kernel("stateful_graph_dynamic_test_kernel");
    const lrrt::Kernel compiled = module.kernel("stateful_graph_compiled_test_kernel");
    const std::vector<sg::Task> tasks = {{0, 0, 0, 4, 1, 0, 0, 0},
                                         {0, 0, 4, 8, 2, 1, 0, 0},
                                         {1, 3, 0, 8, 0, 2, 0, 0},
                                         {2, 0, 0, 1, 2, 3, 0, 0},
                                         {3, 0, 0, 1, 1, 4, 0, 0}};
    const std::vector<sg::Program> programs = {
        {0, 3, 1, 0, 0, {0, 0, 0}},
        {3, 1, 0, sg::kProgramAdvancesStep | sg::kProgramBranchesOnState, 2, {0, 0, 0}},
        {4, 1, 0, sg::kProgramEvaluatesPredicate, 0, {0, 0, 0}}};
    const sg::ResidentAdmission admission = sg::admit_resident_workers(device, compiled, 4);
    const sg::ResidentConfig config{16, admission.worker_count};
    const sg::CompiledPlan plan = sg::compile_resident_plan(tasks, programs, config);
    Buffers buffers(device);
    const std::string dynamic_runs =
        run_path(device, dynamic, tasks, programs, config, nullptr, buffers);
    const std::string compiled_runs =
        run_path(device, compiled, tasks, programs, config, &plan, buffers);
    std::printf("{\"workers\":%u,\"dynamic\":%s,\"compiled\":%s}\n", admission.worker_count,
                dynamic_runs.c_str(), compiled_runs.c_str());
    return 0;
  } catch (const std::exception &error) {
    std::fprintf(stderr, "stateful graph device test: %s\n", error.what());
    return 1;
  }
}
