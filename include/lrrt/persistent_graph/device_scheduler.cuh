// Dynamic resident scheduler for sm_100a (light-rocm-runtime
// include/lrrt/persistent_graph/device_scheduler.hpp:65-305, same semantics):
// block 0 validates the graph (or reuses the cached verdict) and publishes the
// status; every block then loops claiming tasks whose dependencies completed,
// and the block completing a Program's last task performs the Program
// transition. Every spin ends at the launch's wait limit with
// status = invalid_program, error_code = kErrorWaitTimeout.
//
// Workload hooks (static): valid_context(const State*, void*),
// valid_task(const Task&, void*), execute(const Task&, State*, void*).
#ifndef LRRT_PERSISTENT_GRAPH_DEVICE_SCHEDULER_CUH_
#define LRRT_PERSISTENT_GRAPH_DEVICE_SCHEDULER_CUH_

#include "lrrt/persistent_graph/abi.hpp"
#include "lrrt/persistent_graph/device_sync.cuh"

namespace lrrt::persistent_graph::device {

namespace detail {

__device__ __forceinline__ uint32_t load_status(const State *state) {
  return load_relaxed(&state->status);
}

__device__ __forceinline__ uint64_t task_dependencies(const Task &task) {
  return uint64_t{task.dependency_mask} |
         (uint64_t{task.dependency_mask_high} << 32u);
}

__device__ __forceinline__ uint64_t all_tasks_mask(uint32_t task_count) {
  return task_count >= kMaximumTasks ? UINT64_MAX
                                     : (uint64_t{1} << task_count) - 1u;
}

__device__ __forceinline__ uint32_t wait_limit_ms(uint32_t reserved) {
  return reserved == 0 ? kDefaultWaitLimitMs : reserved;
}

// Marks the run failed; other blocks observe the status and leave.
__device__ __forceinline__ void fail(State *state, uint32_t error_code) {
  atomicCAS(&state->error_code, 0u, error_code);
  __threadfence();
  atomicExch(&state->status, static_cast<uint32_t>(Status::invalid_program));
}

template <typename Workload>
__device__ bool validate_programs(const State *state, const Task *tasks,
                                  const Program *programs,
                                  const MaskState *phase_states,
                                  uint32_t program_count,
                                  uint32_t total_task_count,
                                  uint32_t phase_state_count,
                                  void *opaque_context) {
  if (!accepted_abi_version(state->abi_version) || program_count == 0 ||
      total_task_count == 0 || program_count > kMaximumPrograms ||
      phase_program(state->phase) >= program_count ||
      phase_generation(state->phase) >= phase_state_count ||
      state->max_steps == 0 || tasks == nullptr || programs == nullptr ||
      phase_states == nullptr || phase_state_count == 0 ||
      state->worker_count == 0 || state->worker_count > kMaximumResidentWorkers ||
      !Workload::valid_context(state, opaque_context)) {
    return false;
  }
  for (uint32_t p = 0; p < program_count; ++p) {
    const Program &program = programs[p];
    if (program.task_count == 0 || program.task_count > kMaximumTasks ||
        program.task_offset > total_task_count ||
        program.task_count > total_task_count - program.task_offset ||
        program.next_program >= program_count ||
        (program.flags & ~uint32_t{kProgramAdvancesStep |
                                   kProgramEvaluatesPredicate |
                                   kProgramBranchesOnState}) != 0 ||
        ((program.flags & kProgramBranchesOnState) != 0 &&
         program.branch_program >= program_count)) {
      return false;
    }
    const Task *local = tasks + program.task_offset;
    const uint64_t valid = all_tasks_mask(program.task_count);
    for (uint32_t t = 0; t < program.task_count; ++t) {
      const uint64_t deps = task_dependencies(local[t]);
      if (!Workload::valid_task(local[t], opaque_context) || (deps & ~valid) != 0 ||
          (deps & (uint64_t{1} << t)) != 0) {
        return false;
      }
    }
    // Fixed-point walk over the dependency masks: a cycle leaves tasks that
    // never become reachable.
    uint64_t reachable = 0;
    for (uint32_t pass = 0; pass < program.task_count; ++pass) {
      for (uint32_t t = 0; t < program.task_count; ++t) {
        const uint64_t bit = uint64_t{1} << t;
        const uint64_t deps = task_dependencies(local[t]);
        if ((reachable & bit) == 0 && (deps & reachable) == deps) {
          reachable |= bit;
        }
      }
    }
    if (reachable != valid) {
      return false;
    }
  }
  return true;
}

// Program transition after its last task (shared by both schedulers). Runs on
// exactly one thread: the elected block's thread 0.
__device__ __forceinline__ void finish_program(State *state, const Program &program,
                                               uint32_t generation,
                                               uint32_t phase_state_count) {
  const uint32_t next_step =
      state->step + ((program.flags & kProgramAdvancesStep) != 0 ? 1u : 0u);
  state->step = next_step;
  state->executed_tasks += program.task_count;
  const bool predicate = (program.flags & kProgramEvaluatesPredicate) != 0 &&
                         state->predicate_value >= state->stop_value;
  __threadfence();
  if (predicate) {
    atomicExch(&state->status, static_cast<uint32_t>(Status::complete));
  } else if (next_step >= state->max_steps) {
    atomicExch(&state->status, static_cast<uint32_t>(Status::max_steps));
  } else if (generation + 1u >= phase_state_count) {
    state->error_code = kErrorPhaseSlots;
    __threadfence();
    atomicExch(&state->status, static_cast<uint32_t>(Status::invalid_program));
  } else {
    uint32_t next = program.next_program;
    if ((program.flags & kProgramBranchesOnState) != 0 && state->branch_value != 0) {
      next = program.branch_program;
    }
    atomicExch(&state->phase, make_phase(generation + 1u, next));
  }
}

// Validation prologue shared by both schedulers. Returns true when this block
// should enter the scheduling loop.
template <typename Workload, typename Validate>
__device__ bool resident_prologue(State *state, ValidationState *validation_state,
                                  uint32_t limit_ms, Validate validate) {
  __shared__ uint32_t verdict;
  if (blockIdx.x == 0) {
    if (threadIdx.x == 0) {
      const uint32_t cached =
          validation_state == nullptr
              ? static_cast<uint32_t>(ValidationStatus::unvalidated)
              : atomicAdd(&validation_state->status, 0u);
      bool valid;
      if (cached == static_cast<uint32_t>(ValidationStatus::valid)) {
        valid = true;
      } else if (cached == static_cast<uint32_t>(ValidationStatus::invalid)) {
        valid = false;
      } else {
        valid = validate();
        __threadfence();
        if (validation_state != nullptr) {
          atomicExch(&validation_state->status,
                     static_cast<uint32_t>(valid ? ValidationStatus::valid
                                                 : ValidationStatus::invalid));
        }
      }
      if (!valid) {
        state->error_code = kErrorValidation;
      }
      __threadfence();
      atomicExch(&state->status, static_cast<uint32_t>(
                                     valid ? Status::running
                                           : Status::invalid_program));
      verdict = valid ? 1u : 0u;
    }
    __syncthreads();
    return verdict != 0;
  }
  if (threadIdx.x == 0) {
    const Deadline deadline(limit_ms);
    uint32_t spins = 0;
    while (load_acquire(&state->status) == static_cast<uint32_t>(Status::ready)) {
      __nanosleep(64);
      if ((++spins & 63u) == 0u && deadline.expired()) {
        fail(state, kErrorWaitTimeout);
        break;
      }
    }
    verdict = load_acquire(&state->status) == static_cast<uint32_t>(Status::running);
  }
  __syncthreads();
  return verdict != 0;
}

} // namespace detail

template <typename Workload>
__device__ void run_resident(State *state, const Task *tasks,
                             const Program *programs, MaskState *phase_states,
                             uint32_t program_count, uint32_t total_task_count,
                             uint32_t phase_state_count, void *opaque_context,
                             ValidationState *validation_state,
                             uint32_t reserved) {
  const uint32_t limit_ms = detail::wait_limit_ms(reserved);
  const bool enter = detail::resident_prologue<Workload>(
      state, validation_state, limit_ms, [&] {
        return detail::validate_programs<Workload>(
            state, tasks, programs, phase_states, program_count, total_task_count,
            phase_state_count, opaque_context);
      });
  if (!enter) {
    return;
  }
  __shared__ uint32_t selected_task, selected_program, selected_generation, stop;
  const uint32_t worker = blockIdx.x;
  // A stall means no Program phase change for the whole wait limit.
  uint32_t last_phase = UINT32_MAX;
  Deadline progress(limit_ms);
  while (true) {
    if (threadIdx.x == 0) {
      selected_task = kNoTask;
      stop = 0;
      const uint32_t phase_before = load_acquire(&state->phase);
      if (phase_before != last_phase) {
        last_phase = phase_before;
        progress = Deadline(limit_ms);
      }
      const uint32_t generation = phase_generation(phase_before);
      const uint32_t program_index = phase_program(phase_before);
      const Program program = programs[program_index];
      const Task *local = tasks + program.task_offset;
      MaskState *mask = &phase_states[generation];
      const uint32_t claimed = load_acquire(&mask->claimed_mask);
      const uint32_t claimed_high =
          program.task_count > 32 ? load_acquire(&mask->claimed_mask_high) : 0u;
      const uint64_t completed =
          uint64_t{load_acquire(&mask->completed_mask)} |
          (program.task_count > 32
               ? uint64_t{load_acquire(&mask->completed_mask_high)} << 32u
               : 0ull);
      if (phase_before == load_acquire(&state->phase)) {
        for (uint32_t offset = 0; offset < program.task_count; ++offset) {
          const uint32_t index = (worker + offset) % program.task_count;
          const uint32_t bit = 1u << (index & 31u);
          const uint32_t word = index < 32 ? claimed : claimed_high;
          const uint64_t deps = detail::task_dependencies(local[index]);
          if ((word & bit) == 0 && (deps & completed) == deps) {
            uint32_t *target =
                index < 32 ? &mask->claimed_mask : &mask->claimed_mask_high;
            if ((atomicOr(target, bit) & bit) == 0) {
              selected_task = index;
              selected_program = program_index;
              selected_generation = generation;
              break;
            }
          }
        }
      }
      if (selected_task == kNoTask && progress.expired() &&
          detail::load_status(state) == static_cast<uint32_t>(Status::running)) {
        detail::fail(state, kErrorWaitTimeout);
      }
    }
    __syncthreads();

    if (selected_task == kNoTask) {
      if (threadIdx.x == 0) {
        __nanosleep(100);
      }
    } else {
      const Program program = programs[selected_program];
      const Task *local = tasks + program.task_offset;
      MaskState *mask = &phase_states[selected_generation];
      Workload::execute(local[selected_task], state, opaque_context);
      __syncthreads();
      if (threadIdx.x == 0) {
        __threadfence();
        const uint32_t bit = 1u << (selected_task & 31u);
        atomicOr(selected_task < 32 ? &mask->completed_mask
                                    : &mask->completed_mask_high,
                 bit);
        // One counter elects the transition owner without needing a coherent
        // snapshot of both mask words.
        const uint32_t done = fetch_add_acq_rel(&mask->completed_count, 1u) + 1u;
        if (done == program.task_count) {
          detail::finish_program(state, program, selected_generation,
                                 phase_state_count);
        }
      }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      stop = detail::load_status(state) != static_cast<uint32_t>(Status::running);
    }
    __syncthreads();
    if (stop) {
      return;
    }
  }
}

} // namespace lrrt::persistent_graph::device

#endif // LRRT_PERSISTENT_GRAPH_DEVICE_SCHEDULER_CUH_
