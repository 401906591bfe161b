// Compiled resident scheduler for sm_100a (light-rocm-runtime
// include/lrrt/persistent_graph/compiled_scheduler.hpp:15-218, same Program /
// Stage semantics): every block executes each compiled stage of the current
// Program, then meets the others at a software grid barrier counted
// cumulatively in the generation's MaskState (claimed_mask = arrivals,
// completed_mask = barriers released). The last arrival at a Program's final
// barrier performs the Program transition.
//
// B200 differences:
//  * Cooperative launch (lr_kernel_set_resident) guarantees co-residency.
//  * Every spin has a %globaltimer deadline (launch wait limit) after which the
//    run ends with invalid_program / kErrorWaitTimeout; blocks also leave a
//    barrier early once another block has failed the run.
//  * Workloads may declare that a stage boundary needs no grid barrier
//    (barrier_after), because they carry the dependency inside each block
//    (e.g. a norm recomputed per block, or a RoPE epilogue fused into the
//    projection). Barriers are then counted per executed barrier, not per
//    stage; the Program's final stage always ends with a barrier.
//  * Workloads get a per-block state object (Workload::Block) created before
//    the loop (begin) and retired after it (end), so a block can keep a TMA
//    weight-streaming ring running across stages and barriers.
//
// Workload interface (static members):
//   struct Block;                       // per-block state
//   valid_context, valid_task           // as in the dynamic scheduler
//   begin(Block&, const ResidentArgs&)  // after validation, before the loop
//   execute_stage(Block&, const Stage&, const Task*, State*, void* context,
//                 uint32_t worker, uint32_t active_workers)
//   barrier_after(Block&, const Stage&, const Stage& next, const Task*)
//   end(Block&)                         // before the block returns
//   initialize_profile(void*)
//   complete_profile_stage(Block&, const Stage&, const Task*, void*)
#ifndef LRRT_PERSISTENT_GRAPH_COMPILED_SCHEDULER_CUH_
#define LRRT_PERSISTENT_GRAPH_COMPILED_SCHEDULER_CUH_

#include "lrrt/persistent_graph/device_scheduler.cuh"

namespace lrrt::persistent_graph::device {

namespace detail {

template <typename Workload>
__device__ bool validate_plan(const State *state, const Task *tasks,
                              const Program *programs, const MaskState *phase_states,
                              const Stage *stages,
                              const CompiledProgram *compiled_programs,
                              uint32_t program_count, uint32_t total_task_count,
                              uint32_t phase_state_count, uint32_t stage_count,
                              void *opaque_context) {
  if (!validate_programs<Workload>(state, tasks, programs, phase_states,
                                   program_count, total_task_count,
                                   phase_state_count, opaque_context) ||
      stages == nullptr || compiled_programs == nullptr || stage_count == 0) {
    return false;
  }
  for (uint32_t p = 0; p < program_count; ++p) {
    const Program program = programs[p];
    const CompiledProgram compiled = compiled_programs[p];
    if (compiled.stage_count == 0 || compiled.stage_offset > stage_count ||
        compiled.stage_count > stage_count - compiled.stage_offset) {
      return false;
    }
    uint32_t next_task = program.task_offset;
    uint64_t done = 0;
    for (uint32_t s = 0; s < compiled.stage_count; ++s) {
      const Stage stage = stages[compiled.stage_offset + s];
      const uint32_t finished = next_task - program.task_offset;
      if (stage.task_count == 0 || stage.task_offset != next_task ||
          stage.task_count > program.task_count - finished) {
        return false;
      }
      for (uint32_t t = 0; t < stage.task_count; ++t) {
        const uint64_t deps = task_dependencies(tasks[stage.task_offset + t]);
        if ((deps & done) != deps) {
          return false;
        }
      }
      done |= all_tasks_mask(stage.task_count) << finished;
      next_task += stage.task_count;
    }
    if (next_task != program.task_offset + program.task_count) {
      return false;
    }
  }
  return true;
}

// Grid barrier number `index` (0-based within the generation). The last
// arrival runs `on_last` (thread 0 of that block only) before releasing the
// others. Returns false when the run failed or the wait limit passed.
template <typename OnLast>
__device__ bool grid_barrier(State *state, MaskState *barrier, uint32_t index,
                             uint32_t workers, const Deadline &deadline,
                             OnLast on_last) {
  __shared__ uint32_t barrier_ok;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const uint32_t target = (index + 1u) * workers;
    const uint32_t arrived = fetch_add_acq_rel(&barrier->claimed_mask, 1u) + 1u;
    if (arrived == target) {
      on_last();
      __threadfence();
      store_release(&barrier->completed_mask, index + 1u);
    }
    uint32_t ok = 1;
    uint32_t spins = 0;
    while (load_acquire(&barrier->completed_mask) < index + 1u) {
      if ((++spins & 127u) == 0u) {
        if (load_status(state) != static_cast<uint32_t>(Status::running)) {
          ok = 0;
          break;
        }
        if (deadline.expired()) {
          fail(state, kErrorWaitTimeout);
          ok = 0;
          break;
        }
      }
    }
    __threadfence();
    barrier_ok = ok;
  }
  __syncthreads();
  return barrier_ok != 0;
}

} // namespace detail

// Default hooks for workloads without per-block state or fusion.
struct CompiledWorkloadDefaults {
  struct Block {};
  __device__ static void begin(Block &, const ResidentArgs &) {}
  __device__ static bool barrier_after(Block &, const Stage &, const Stage &,
                                       const Task *) {
    return true;
  }
  __device__ static void end(Block &) {}
  __device__ static void initialize_profile(void *) {}
  __device__ static void complete_profile_stage(Block &, const Stage &,
                                                const Task *, void *) {}
};

template <typename Workload>
__device__ void run_compiled_resident(const ResidentArgs &args) {
  State *state = args.state;
  const uint32_t limit_ms = detail::wait_limit_ms(args.reserved);
  const bool enter = detail::resident_prologue<Workload>(
      state, args.validation_state, limit_ms, [&] {
        return detail::validate_plan<Workload>(
            state, args.tasks, args.programs, args.phase_states, args.stages,
            args.compiled_programs, args.program_count, args.task_count,
            args.phase_state_count, args.stage_count, args.context);
      });
  if (!enter) {
    return;
  }
  // Block 0 arrives at every barrier, so initialising here precedes the first
  // complete_profile_stage call of any block.
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    Workload::initialize_profile(args.context);
  }
  const uint32_t worker = blockIdx.x;
  typename Workload::Block block{};
  Workload::begin(block, args);
  __shared__ uint32_t loop_phase, loop_running;
  while (true) {
    if (threadIdx.x == 0) {
      loop_phase = load_acquire(&state->phase);
    }
    __syncthreads();
    const uint32_t phase = loop_phase;
    const uint32_t generation = phase_generation(phase);
    const Program program = args.programs[phase_program(phase)];
    const CompiledProgram compiled = args.compiled_programs[phase_program(phase)];
    MaskState *barrier = &args.phase_states[generation];
    const uint32_t workers = load_relaxed(&state->worker_count);
    const Deadline deadline(limit_ms);
    uint32_t barrier_index = 0;
    bool ok = true;
    for (uint32_t s = 0; s < compiled.stage_count && ok; ++s) {
      const Stage stage = args.stages[compiled.stage_offset + s];
      if (worker < workers) {
        Workload::execute_stage(block, stage, args.tasks, state, args.context,
                                worker, workers);
      }
      const bool last = s + 1u == compiled.stage_count;
      if (!last && !Workload::barrier_after(
                       block, stage, args.stages[compiled.stage_offset + s + 1u],
                       args.tasks)) {
        continue;
      }
      ok = detail::grid_barrier(state, barrier, barrier_index++, workers,
                                deadline, [&] {
                                  if (last) {
                                    detail::finish_program(state, program,
                                                           generation,
                                                           args.phase_state_count);
                                  }
                                  Workload::complete_profile_stage(
                                      block, stage, args.tasks, args.context);
                                });
    }
    // One thread reads the status so every thread of the block takes the same
    // branch even if another block fails the run concurrently.
    if (threadIdx.x == 0) {
      loop_running = ok && detail::load_status(state) ==
                               static_cast<uint32_t>(Status::running);
    }
    __syncthreads();
    if (!loop_running) {
      break;
    }
  }
  Workload::end(block);
}

} // namespace lrrt::persistent_graph::device

#endif // LRRT_PERSISTENT_GRAPH_COMPILED_SCHEDULER_CUH_
