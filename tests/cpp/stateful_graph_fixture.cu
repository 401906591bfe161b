// Synthetic scheduler fixture (reference tests/stateful_graph_device_kernel.cpp
// :46-132 and tests/stateful_graph_device_context.hpp): four opcodes over an
// 8-value context exercise claims, dependency masks, step advance, branching
// and the predicate exit of both resident schedulers. The expected final
// state and arrays are the reference test's goldens
// (tests/stateful_graph_device.cpp:103-136).
#include "lrrt/persistent_graph/compiled_scheduler.cuh"
#include "lrrt/persistent_graph/device_scheduler.cuh"

#include <cstdint>

namespace sg = lrrt::persistent_graph;
namespace dev = lrrt::persistent_graph::device;

namespace {

constexpr uint32_t kContextMagic = 0x53504754u;
constexpr uint32_t kValueCount = 8;
constexpr uint32_t kMaximumSteps = 8;
constexpr uint32_t kTaskCount = 5;

enum class Opcode : uint32_t {
  add_range = 0,
  checksum = 1,
  select_branch = 2,
  advance_predicate = 3,
};

struct FixtureContext {
  uint32_t magic;
  uint32_t value_count;
  uint32_t *values;
  uint32_t *step_checksums;
  uint32_t *branch_steps;
  uint32_t *task_executions;
  uint32_t *validation_calls;
};

struct SyntheticWorkload : dev::CompiledWorkloadDefaults {
  __device__ static bool valid_context(const sg::State *, void *opaque) {
    const auto *c = static_cast<const FixtureContext *>(opaque);
    if (c != nullptr && c->validation_calls != nullptr) {
      atomicAdd(c->validation_calls, 1u);
    }
    return c != nullptr && c->magic == kContextMagic && c->value_count == kValueCount &&
           c->values != nullptr && c->step_checksums != nullptr &&
           c->branch_steps != nullptr && c->task_executions != nullptr &&
           c->validation_calls != nullptr;
  }

  __device__ static bool valid_task(const sg::Task &task, void *) {
    if (task.argument1 >= kTaskCount) {
      return false;
    }
    switch (static_cast<Opcode>(task.opcode)) {
    case Opcode::add_range:
      return task.begin < task.end && task.end <= kValueCount && task.argument0 != 0;
    case Opcode::checksum:
      return task.begin == 0 && task.end == kValueCount;
    case Opcode::select_branch:
    case Opcode::advance_predicate:
      return task.begin == 0 && task.end == 1 && task.argument0 != 0;
    }
    return false;
  }

  __device__ static void execute(const sg::Task &task, sg::State *state, void *opaque) {
    auto *c = static_cast<FixtureContext *>(opaque);
    const uint32_t step = dev::load_relaxed(&state->step);
    if (threadIdx.x == 0) {
      atomicAdd(&c->task_executions[task.argument1], 1u);
    }
    switch (static_cast<Opcode>(task.opcode)) {
    case Opcode::add_range:
      for (uint32_t i = task.begin + threadIdx.x; i < task.end; i += sg::kWorkerThreads) {
        c->values[i] = dev::load_cg(c->values + i) + task.argument0 + step;
      }
      break;
    case Opcode::checksum:
      if (threadIdx.x == 0) {
        uint32_t checksum = 0;
        for (uint32_t i = task.begin; i < task.end; ++i) {
          checksum += dev::load_cg(c->values + i);
        }
        if (step < kMaximumSteps) {
          c->step_checksums[step] = checksum;
        }
      }
      break;
    case Opcode::select_branch:
      if (threadIdx.x == 0) {
        state->branch_value = ((step + 1u) % task.argument0 == 0) ? 1u : 0u;
      }
      break;
    case Opcode::advance_predicate:
      if (threadIdx.x == 0) {
        const uint32_t predicate = state->predicate_value;
        if (predicate < kMaximumSteps) {
          c->branch_steps[predicate] = step;
        }
        state->predicate_value = predicate + task.argument0;
      }
      break;
    }
    __syncthreads();
  }

  __device__ static void execute_stage(Block &, const sg::Stage &stage,
                                       const sg::Task *tasks, sg::State *state,
                                       void *opaque, uint32_t worker, uint32_t workers) {
    for (uint32_t t = worker; t < stage.task_count; t += workers) {
      execute(tasks[stage.task_offset + t], state, opaque);
    }
  }
};

} // namespace

extern "C" __global__ void __launch_bounds__(sg::kWorkerThreads)
    stateful_graph_dynamic_test_kernel(
        sg::State *state, const sg::Task *tasks, const sg::Program *programs,
        sg::MaskState *phase_states, uint32_t program_count, uint32_t total_task_count,
        uint32_t phase_state_count, void *opaque_context, const sg::Stage *,
        const sg::CompiledProgram *, uint32_t, uint32_t reserved,
        sg::ValidationState *validation_state) {
  dev::run_resident<SyntheticWorkload>(state, tasks, programs, phase_states,
                                       program_count, total_task_count,
                                       phase_state_count, opaque_context,
                                       validation_state, reserved);
}

extern "C" __global__ void __launch_bounds__(sg::kWorkerThreads)
    stateful_graph_compiled_test_kernel(
        sg::State *state, const sg::Task *tasks, const sg::Program *programs,
        sg::MaskState *phase_states, uint32_t program_count, uint32_t total_task_count,
        uint32_t phase_state_count, void *opaque_context, const sg::Stage *stages,
        const sg::CompiledProgram *compiled_programs, uint32_t stage_count,
        uint32_t reserved, sg::ValidationState *validation_state) {
  dev::run_compiled_resident<SyntheticWorkload>(sg::ResidentArgs{
      state, tasks, programs, phase_states, program_count, total_task_count,
      phase_state_count, opaque_context, stages, compiled_programs, stage_count,
      reserved, validation_state});
}
