// Host-only checks of worker admission, graph validation and the stage
// compiler. Cases and expected values follow light-rocm-runtime
// tests/stateful_graph_resident_executor.cpp:38-112; the worker cap case uses
// this ABI's kMaximumResidentWorkers (256).
#include "lrrt/persistent_graph.hpp"

#include <cstdio>
#include <functional>
#include <stdexcept>
#include <vector>

namespace sg = lrrt::persistent_graph;

static int failures = 0;

static void expect(bool condition, const char *what) {
  if (!condition) {
    std::fprintf(stderr, "FAILED: %s\n", what);
    ++failures;
  }
}

static void expect_throws(const std::function<void()> &body, const char *what) {
  try {
    body();
  } catch (const std::invalid_argument &) {
    return;
  }
  std::fprintf(stderr, "FAILED (no invalid_argument): %s\n", what);
  ++failures;
}

int main() {
  // A 60-CU, 3-engine device admits 20 workers; smaller requests are kept.
  const lrrt::DeviceProperties rdna3{60, 32, 32, 1024, 64u * 1024u, 3};
  const lrrt::KernelProperties kernel{128, 1060, 0};
  const sg::ResidentAdmission admitted = sg::admit_resident_workers(rdna3, kernel, 128);
  expect(admitted.requested_worker_count == 128 && admitted.safe_worker_limit == 20 &&
             admitted.worker_count == 20,
         "admission caps at one engine");
  const sg::ResidentAdmission small = sg::admit_resident_workers(rdna3, kernel, 8);
  expect(small.safe_worker_limit == 20 && small.worker_count == 8,
         "admission keeps a safe request");
  // B200 as reported by lr_device_get_properties: one engine of 148 SMs.
  const lrrt::DeviceProperties b200{148, 32, 64, 1024, 232448u, 1};
  expect(sg::admit_resident_workers(b200, kernel, 1000).worker_count == 148,
         "B200 admits one worker per SM");
  expect_throws([&] { sg::resident_worker_limit({60, 32, 32, 1024, 65536u, 0}, kernel); },
                "missing engine topology");
  expect_throws([&] { sg::resident_worker_limit({61, 32, 32, 1024, 65536u, 3}, kernel); },
                "uneven engine topology");
  expect_throws([&] { sg::resident_worker_limit(rdna3, {128, 64u * 1024u + 1u, 0}); },
                "oversized shared memory");
  expect_throws([&] { sg::admit_resident_workers(rdna3, kernel, 0); }, "zero request");

  const std::vector<sg::Task> tasks = {{0, 0, 0, 1, 0, 0, 0, 0}, {1, 1, 0, 1, 0, 0, 0, 0}};
  const std::vector<sg::Program> programs = {{0, 2, 0, sg::kProgramAdvancesStep, 0, {0, 0, 0}}};
  const sg::ResidentConfig config{8, 4};
  sg::validate_resident_graph(tasks, programs, config);
  const sg::CompiledPlan plan = sg::compile_resident_plan(tasks, programs, config);
  expect(plan.programs.size() == 1 && plan.stages.size() == 2 &&
             plan.programs[0].stage_offset == 0 && plan.programs[0].stage_count == 2 &&
             plan.stages[0].task_offset == 0 && plan.stages[0].task_count == 1 &&
             plan.stages[1].task_offset == 1 && plan.stages[1].task_count == 1,
         "two-task chain compiles into two stages");

  std::vector<sg::Program> too_long = programs;
  too_long[0].task_count = sg::kMaximumTasks + 1;
  std::vector<sg::Task> bad_mask = tasks;
  bad_mask[1].dependency_mask = 4;
  std::vector<sg::Task> self_dependency = tasks;
  self_dependency[1].dependency_mask = 2;
  std::vector<sg::Task> cyclic = tasks;
  cyclic[0].dependency_mask = 2;
  std::vector<sg::Program> bad_successor = programs;
  bad_successor[0].next_program = 1;
  std::vector<sg::Program> bad_flags = programs;
  bad_flags[0].flags = 8;
  expect_throws([&] { sg::validate_resident_graph({}, programs, config); }, "empty tasks");
  expect_throws([&] { sg::validate_resident_graph(tasks, programs, {8, 0}); }, "zero workers");
  expect_throws(
      [&] {
        sg::validate_resident_graph(tasks, programs, {8, sg::kMaximumResidentWorkers + 1});
      },
      "too many workers");
  expect_throws([&] { sg::validate_resident_graph(tasks, programs, {0, 4}); },
                "zero phase states");
  expect_throws([&] { sg::validate_resident_graph(tasks, too_long, config); }, "task range");
  expect_throws([&] { sg::validate_resident_graph(bad_mask, programs, config); },
                "dependency mask out of program");
  expect_throws([&] { sg::validate_resident_graph(self_dependency, programs, config); },
                "self dependency");
  expect_throws([&] { sg::validate_resident_graph(tasks, bad_successor, config); },
                "successor out of range");
  expect_throws([&] { sg::validate_resident_graph(tasks, bad_flags, config); },
                "unknown program flags");
  expect_throws([&] { sg::compile_resident_plan(cyclic, programs, config); },
                "cyclic graph");

  // A hand-made plan that puts dependent tasks in one stage is rejected.
  sg::CompiledPlan merged{{{0, 2}}, {{0, 1}}};
  expect_throws([&] { sg::detail::validate_compiled_plan(tasks, programs, merged); },
                "dependent tasks in one stage");

  // 64-task chain uses both mask words and compiles into 64 stages.
  std::vector<sg::Task> chain;
  for (uint32_t i = 0; i < sg::kMaximumTasks; ++i) {
    const uint64_t dependency = i == 0 ? 0 : uint64_t{1} << (i - 1u);
    chain.push_back({9, static_cast<uint32_t>(dependency), 0, 1, 1, 0,
                     static_cast<uint32_t>(dependency >> 32u), 0});
  }
  const std::vector<sg::Program> chain_program = {
      {0, sg::kMaximumTasks, 0, sg::kProgramAdvancesStep | sg::kProgramEvaluatesPredicate,
       0, {0, 0, 0}}};
  const sg::CompiledPlan chain_plan = sg::compile_resident_plan(chain, chain_program, config);
  expect(chain_plan.stages.size() == sg::kMaximumTasks, "64-task chain stages");

  if (failures == 0) {
    std::printf("resident executor host checks: ok\n");
  }
  return failures == 0 ? 0 : 1;
}
