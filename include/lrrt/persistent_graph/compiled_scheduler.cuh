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
//    projection) or exchange the data through self-validating words.
//    Barriers are then counted per executed barrier, not per stage. The
//    Program's final stage ends with a barrier unless the workload runs in
//    local-transition mode and barrier_at_end says otherwise.
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
//   barrier_at_end(const Block&)        // local mode: barrier after the last stage
//   barrier_poll(Block&)                // thread 0, between grid-barrier polls
//   end(Block&)                         // before the block returns
//   initialize_profile(void*)
//   complete_profile_stage(Block&, const Stage&, const Task*, void*)
//   kTraceBarriers, trace_barrier(Block&, void* context, const Stage&,
//                                 const Task*, arrive_ns, leave_ns)
//                                       // optional per-block barrier trace
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

// Grid barrier number `index` (0-based within the generation); `workers`
// blocks arrive. Arrivals accumulate in claimed_mask: a barrier inside a
// Program is complete once claimed_mask reaches (index + 1) * workers. At a
// Program's final barrier the last arrival first runs `on_last` (the Program
// transition, on thread 0 of that block only) and then publishes
// completed_mask = index + 1, which the other blocks wait for. Returns false
// when the run failed or the wait limit passed. Thread 0 calls `on_poll`
// between polls (the workload's barrier_poll hook).
//
// The block-wide __syncthreads before the arrival orders every thread's writes
// before thread 0's release; thread 0's acquire and the __syncthreads after the
// wait order every thread's later reads after the other blocks' writes.
template <typename OnLast, typename OnPoll>
__device__ bool grid_barrier(State *state, MaskState *barrier, uint32_t index,
                             uint32_t workers, bool final, const Deadline &deadline,
                             OnLast on_last, OnPoll on_poll) {
  __shared__ uint32_t barrier_ok;
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint32_t target = (index + 1u) * workers;
    const uint32_t *watched = &barrier->claimed_mask;
    uint32_t goal = target;
    if (final) {
      const uint32_t arrived = fetch_add_acq_rel(&barrier->claimed_mask, 1u) + 1u;
      if (arrived == target) {
        on_last();
        store_release(&barrier->completed_mask, index + 1u);
      }
      watched = &barrier->completed_mask;
      goal = index + 1u;
    } else {
      add_release(&barrier->claimed_mask, 1u);
    }
    uint32_t ok = 1;
    uint32_t spins = 0;
    while (load_acquire(watched) < goal) {
      on_poll();
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
    barrier_ok = ok;
  }
  __syncthreads();
  return barrier_ok != 0;
}

} // namespace detail

// Default hooks for workloads without per-block state or fusion.
struct CompiledWorkloadDefaults {
  static constexpr bool kTraceBarriers = false;
  struct Block {};
  __device__ static void trace_barrier(Block &, void *, const Stage &, const Task *,
                                       uint64_t, uint64_t) {}
  __device__ static void begin(Block &, const ResidentArgs &) {}
  __device__ static bool local_transitions(const Block &) { return false; }
  // Thread 0, between polls of a grid barrier.
  __device__ static void barrier_poll(Block &) {}
  // Local-transition mode: whether the current Program ends with a grid
  // barrier. A workload that carries every dependency across the Program
  // boundary itself (and whose transition needs no other block's writes) may
  // skip it.
  __device__ static bool barrier_at_end(const Block &) { return true; }
  __device__ static void program_begin(Block &, uint32_t /*program*/, uint32_t /*step*/) {}
  __device__ static void stage_begin(Block &, uint32_t /*stage index in program*/) {}
  // Local-transition mode: the branch_value the finished Program's tasks
  // wrote. A workload that can compute it from its own state (the same rule
  // its task applies) avoids a global read.
  __device__ static uint32_t branch_value(Block &, const State *state) {
    return load_relaxed(&state->branch_value);
  }
  __device__ static bool barrier_after(Block &, const Stage &, const Stage &,
                                       const Task *) {
    return true;
  }
  __device__ static void end(Block &) {}
  __device__ static void initialize_profile(void *) {}
  __device__ static void complete_profile_stage(Block &, const Stage &,
                                                const Task *, void *) {}
};

namespace detail {

// Program state a block tracks for itself in local-transition mode.
struct LocalControl {
  uint32_t phase;
  uint32_t step;
  uint32_t status;
  uint32_t error_code;
  uint64_t executed_tasks;
};

// The Program transition of finish_program computed from the block's own copy
// of the control state; predicate_value was written by the Program's tasks
// before its final barrier, `branch` is the branch_value they produced.
__device__ __forceinline__ void local_transition(LocalControl &c, const State *state,
                                                 const Program &program,
                                                 uint32_t generation,
                                                 uint32_t phase_state_count,
                                                 uint32_t max_steps, uint32_t stop_value,
                                                 uint32_t branch) {
  const uint32_t next_step =
      c.step + ((program.flags & kProgramAdvancesStep) != 0 ? 1u : 0u);
  c.step = next_step;
  c.executed_tasks += program.task_count;
  const bool predicate =
      (program.flags & kProgramEvaluatesPredicate) != 0 &&
      load_relaxed(&state->predicate_value) >= stop_value;
  if (predicate) {
    c.status = static_cast<uint32_t>(Status::complete);
  } else if (next_step >= max_steps) {
    c.status = static_cast<uint32_t>(Status::max_steps);
  } else if (generation + 1u >= phase_state_count) {
    c.status = static_cast<uint32_t>(Status::invalid_program);
    c.error_code = kErrorPhaseSlots;
  } else {
    uint32_t next = program.next_program;
    if ((program.flags & kProgramBranchesOnState) != 0 && branch != 0) {
      next = program.branch_program;
    }
    c.phase = make_phase(generation + 1u, next);
  }
}

// Block 0 mirrors the local control state into State for the host.
__device__ __forceinline__ void publish_control(State *state, const LocalControl &c) {
  state->step = c.step;
  state->executed_tasks = c.executed_tasks;
  state->phase = c.phase;
  if (c.status != static_cast<uint32_t>(Status::running)) {
    if (c.error_code != 0) {
      atomicCAS(&state->error_code, 0u, c.error_code);
    }
    __threadfence();
    atomicCAS(&state->status, static_cast<uint32_t>(Status::running), c.status);
  }
}

} // namespace detail

// Workloads may opt into block-local Program transitions
// (local_transitions(block) == true, the same answer in every block): each
// block then evaluates the transition of a finished Program itself, every grid
// barrier is a plain counting barrier, and block 0 mirrors the control state
// into State. The workload must then take the step from program_begin()
// instead of reading State during the run.
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
  // Small plans are copied into shared memory once: the loop reads a Program
  // per transition and a Stage per stage, and a global read costs an L2 round
  // trip behind whatever else the kernel streams.
  constexpr uint32_t kCachedPrograms = 8;
  constexpr uint32_t kCachedStages = 64;
  __shared__ Program program_cache[kCachedPrograms];
  __shared__ CompiledProgram compiled_cache[kCachedPrograms];
  __shared__ Stage stage_cache[kCachedStages];
  const bool cached =
      args.program_count <= kCachedPrograms && args.stage_count <= kCachedStages;
  if (cached) {
    for (uint32_t i = threadIdx.x; i < args.program_count; i += blockDim.x) {
      program_cache[i] = args.programs[i];
      compiled_cache[i] = args.compiled_programs[i];
    }
    for (uint32_t i = threadIdx.x; i < args.stage_count; i += blockDim.x) {
      stage_cache[i] = args.stages[i];
    }
  }
  const Program *programs = cached ? program_cache : args.programs;
  const CompiledProgram *compiled_programs =
      cached ? compiled_cache : args.compiled_programs;
  const Stage *stages = cached ? stage_cache : args.stages;
  typename Workload::Block block{};
  Workload::begin(block, args);
  const bool local = Workload::local_transitions(block);
  const uint32_t workers = load_relaxed(&state->worker_count);
  __shared__ uint32_t loop_phase, loop_running;
  __shared__ detail::LocalControl shared_control;
  detail::LocalControl control{};
  uint32_t status_seen = static_cast<uint32_t>(Status::running); // thread 0
  if (threadIdx.x == 0) {
    shared_control = {load_relaxed(&state->phase), load_relaxed(&state->step),
                      static_cast<uint32_t>(Status::running), 0,
                      static_cast<uint64_t>(atomicAdd(
                          reinterpret_cast<unsigned long long *>(&state->executed_tasks),
                          0ull))};
  }
  __syncthreads();
  control = shared_control;
  const uint32_t max_steps = load_relaxed(&state->max_steps);
  const uint32_t stop_value = load_relaxed(&state->stop_value);
  while (true) {
    if (!local) {
      if (threadIdx.x == 0) {
        loop_phase = load_acquire(&state->phase);
      }
      __syncthreads();
    }
    const uint32_t phase = local ? control.phase : loop_phase;
    const uint32_t generation = phase_generation(phase);
    const Program program = programs[phase_program(phase)];
    const CompiledProgram compiled = compiled_programs[phase_program(phase)];
    MaskState *barrier = &args.phase_states[generation];
    const Deadline deadline(limit_ms);
    if (local && threadIdx.x == 0) {
      // Read now, used at the transition: a failure elsewhere is noticed one
      // Program later (or by any wait), without a read on the critical path.
      status_seen = load_relaxed(&state->status);
    }
    Workload::program_begin(block, phase_program(phase), control.step);
    uint32_t barrier_index = 0;
    bool ok = true;
    bool ended_with_barrier = false;
    for (uint32_t s = 0; s < compiled.stage_count && ok; ++s) {
      const Stage stage = stages[compiled.stage_offset + s];
      Workload::stage_begin(block, s);
      if (worker < workers) {
        Workload::execute_stage(block, stage, args.tasks, state, args.context,
                                worker, workers);
      }
      const bool last = s + 1u == compiled.stage_count;
      const bool skip =
          last ? local && !Workload::barrier_at_end(block)
               : !Workload::barrier_after(block, stage,
                                          stages[compiled.stage_offset + s + 1u], args.tasks);
      if (skip) {
        continue;
      }
      ended_with_barrier = last;
      const uint64_t arrive_ns = Workload::kTraceBarriers ? global_timer_ns() : 0;
      ok = detail::grid_barrier(state, barrier, barrier_index++, workers, last && !local,
                                deadline, [&] {
                                  if (last) {
                                    detail::finish_program(state, program,
                                                           generation,
                                                           args.phase_state_count);
                                  }
                                  Workload::complete_profile_stage(
                                      block, stage, args.tasks, args.context);
                                },
                                [&] { Workload::barrier_poll(block); });
      if (Workload::kTraceBarriers && threadIdx.x == 0) {
        Workload::trace_barrier(block, args.context, stage, args.tasks, arrive_ns,
                                global_timer_ns());
      }
      if (local && ok && worker == 0 && threadIdx.x == 0) {
        // No block is elected as the last arrival in local mode; block 0
        // records the stage profile after each barrier instead.
        Workload::complete_profile_stage(block, stage, args.tasks, args.context);
      }
    }
    // One thread decides whether to continue so every thread of the block
    // takes the same branch even if another block fails the run concurrently.
    if (threadIdx.x == 0) {
      if (local && ok) {
        const uint32_t branch = (program.flags & kProgramBranchesOnState) != 0
                                    ? Workload::branch_value(block, state)
                                    : 0u;
        detail::local_transition(shared_control, state, program, generation,
                                 args.phase_state_count, max_steps, stop_value, branch);
        // State is mirrored only where every block is known to have read the
        // launch's initial State: after a Program-ending grid barrier, or when
        // the run stops (which needs every block's contribution).
        if (worker == 0 &&
            (ended_with_barrier ||
             shared_control.status != static_cast<uint32_t>(Status::running))) {
          detail::publish_control(state, shared_control);
        }
      }
      const uint32_t status =
          local ? status_seen : detail::load_status(state);
      loop_running = ok &&
                     (!local ||
                      shared_control.status == static_cast<uint32_t>(Status::running)) &&
                     status == static_cast<uint32_t>(Status::running);
    }
    __syncthreads();
    if (local) {
      control = shared_control;
    }
    if (!loop_running) {
      break;
    }
  }
  Workload::end(block);
}

} // namespace lrrt::persistent_graph::device

#endif // LRRT_PERSISTENT_GRAPH_COMPILED_SCHEDULER_CUH_
