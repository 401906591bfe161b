// Host side of the Persistent Graph: worker admission, graph validation, the
// greedy stage compiler, and ResidentExecutor, which owns the device control
// buffers of one resident graph and launches its kernel.
//
// Public names, argument meaning and the exceptions thrown follow
// light-rocm-runtime include/lrrt/persistent_graph/resident_executor.hpp:19-475:
//   admission ............ :30-89    validate_resident_graph ... :115-172
//   validate_compiled_plan :174-217  compile_resident_plan ..... :227-263
//   ResidentExecutor ..... :268-475
// B200 differences:
//   * ResidentConfig has two optional trailing fields (dynamic shared memory of
//     the resident kernel, device wait limit); two-field aggregate
//     initialisation as in reference callers still compiles.
//   * The constructor marks the kernel resident (lr_kernel_set_resident), so
//     launches are cooperative and over-subscription fails at launch time.
//   * initialize_on_device() re-arms the control state with device-to-device
//     copies from a pristine image, for timed loops with no host copies.
#ifndef LRRT_PERSISTENT_GRAPH_RESIDENT_EXECUTOR_HPP_
#define LRRT_PERSISTENT_GRAPH_RESIDENT_EXECUTOR_HPP_

#include "lrrt/lrrt.hpp"
#include "lrrt/persistent_graph/abi.hpp"

#include <algorithm>
#include <array>
#include <cstddef>
#include <cstdint>
#include <limits>
#include <optional>
#include <stdexcept>
#include <utility>
#include <vector>

namespace lrrt::persistent_graph {

struct ResidentConfig {
  uint32_t phase_state_count;
  uint32_t worker_count;
  uint32_t dynamic_shared_memory_bytes = 0;
  uint32_t wait_limit_ms = 0; // 0 = kDefaultWaitLimitMs
};

struct ResidentAdmission {
  uint32_t requested_worker_count;
  uint32_t safe_worker_limit;
  uint32_t worker_count;
};

// Largest resident grid the admission rule accepts: one block per compute
// unit of one shader engine, capped at kMaximumResidentWorkers, after checking
// that one block fits the device's workgroup, wave and shared-memory limits.
// On B200 lr_device_get_properties reports one engine of 148 SMs.
inline uint32_t resident_worker_limit(const DeviceProperties &device,
                                      const KernelProperties &kernel,
                                      uint32_t block_threads = kWorkerThreads,
                                      uint32_t dynamic_group_segment_size = 0) {
  if (device.compute_unit_count == 0 || device.wavefront_size == 0 ||
      device.maximum_waves_per_compute_unit == 0 ||
      device.maximum_workgroup_size == 0 || device.shader_engine_count == 0 ||
      device.shader_engine_count > device.compute_unit_count ||
      device.compute_unit_count % device.shader_engine_count != 0 ||
      block_threads == 0) {
    throw std::invalid_argument("incomplete resident resource properties");
  }
  if (block_threads > device.maximum_workgroup_size) {
    throw std::invalid_argument("resident workgroup exceeds device limit");
  }
  const uint32_t waves =
      (block_threads + device.wavefront_size - 1u) / device.wavefront_size;
  if (waves > device.maximum_waves_per_compute_unit) {
    throw std::invalid_argument("resident workgroup exceeds wave limit");
  }
  const uint64_t shared_bytes =
      uint64_t{kernel.group_segment_size} + dynamic_group_segment_size;
  if (shared_bytes > device.group_segment_size) {
    throw std::invalid_argument("resident workgroup exceeds LDS limit");
  }
  const uint32_t per_engine =
      device.compute_unit_count / device.shader_engine_count;
  return std::min(per_engine, kMaximumResidentWorkers);
}

inline ResidentAdmission
admit_resident_workers(const DeviceProperties &device,
                       const KernelProperties &kernel,
                       uint32_t requested_worker_count,
                       uint32_t block_threads = kWorkerThreads,
                       uint32_t dynamic_group_segment_size = 0) {
  if (requested_worker_count == 0) {
    throw std::invalid_argument("resident worker request must be nonzero");
  }
  const uint32_t limit = resident_worker_limit(device, kernel, block_threads,
                                               dynamic_group_segment_size);
  return {requested_worker_count, limit,
          std::min(requested_worker_count, limit)};
}

// Device overload: additionally bounds the grid by the driver's occupancy
// figure for this kernel, which the cooperative launch will enforce.
inline ResidentAdmission
admit_resident_workers(Device device, const Kernel &kernel,
                       uint32_t requested_worker_count,
                       uint32_t block_threads = kWorkerThreads,
                       uint32_t dynamic_group_segment_size = 0) {
  ResidentAdmission admission = admit_resident_workers(
      device.properties(), kernel.properties(), requested_worker_count,
      block_threads, dynamic_group_segment_size);
  uint32_t resident_blocks = 0;
  check(lr_kernel_max_resident_blocks(kernel.get(), block_threads,
                                      dynamic_group_segment_size,
                                      &resident_blocks),
        "lr_kernel_max_resident_blocks");
  if (resident_blocks == 0) {
    throw std::invalid_argument("resident kernel cannot be made resident");
  }
  admission.safe_worker_limit =
      std::min(admission.safe_worker_limit, resident_blocks);
  admission.worker_count =
      std::min(admission.requested_worker_count, admission.safe_worker_limit);
  return admission;
}

struct CompiledPlan {
  std::vector<Stage> stages;
  std::vector<CompiledProgram> programs;
};

namespace detail {

struct ValidatedGraph {
  size_t task_bytes;
  size_t program_bytes;
  size_t phase_state_bytes;
};

inline uint64_t task_dependencies(const Task &task) {
  return uint64_t{task.dependency_mask} |
         (uint64_t{task.dependency_mask_high} << 32u);
}

inline uint64_t valid_task_mask(uint32_t task_count) {
  return task_count >= kMaximumTasks ? UINT64_MAX
                                     : (uint64_t{1} << task_count) - 1u;
}

inline ValidatedGraph validate_resident_graph(const std::vector<Task> &tasks,
                                              const std::vector<Program> &programs,
                                              ResidentConfig config) {
  if (tasks.empty()) {
    throw std::invalid_argument("stateful graph must contain tasks");
  }
  if (tasks.size() > std::numeric_limits<uint32_t>::max()) {
    throw std::invalid_argument("invalid stateful graph task count");
  }
  if (programs.empty() || programs.size() > kMaximumPrograms) {
    throw std::invalid_argument("invalid stateful graph program count");
  }
  constexpr uint32_t kMaximumPhaseStates =
      phase_generation(std::numeric_limits<uint32_t>::max()) + 1u;
  if (config.phase_state_count == 0 ||
      config.phase_state_count > kMaximumPhaseStates) {
    throw std::invalid_argument("invalid stateful graph phase-state count");
  }
  if (config.worker_count == 0 || config.worker_count > kMaximumResidentWorkers) {
    throw std::invalid_argument("invalid stateful graph resident worker count");
  }
  const size_t program_count = programs.size();
  for (const Program &program : programs) {
    if (program.task_count == 0 || program.task_count > kMaximumTasks ||
        program.task_offset > tasks.size() ||
        program.task_count > tasks.size() - program.task_offset) {
      throw std::invalid_argument("invalid stateful graph task range");
    }
    const bool branches = (program.flags & kProgramBranchesOnState) != 0;
    if (program.next_program >= program_count ||
        (branches && program.branch_program >= program_count)) {
      throw std::invalid_argument("invalid stateful graph successor");
    }
    if ((program.flags & ~uint32_t{kProgramAdvancesStep |
                                   kProgramEvaluatesPredicate |
                                   kProgramBranchesOnState}) != 0) {
      throw std::invalid_argument("invalid stateful graph program flags");
    }
    const uint64_t allowed = valid_task_mask(program.task_count);
    for (uint32_t local = 0; local < program.task_count; ++local) {
      const uint64_t deps = task_dependencies(tasks[program.task_offset + local]);
      if ((deps & ~allowed) != 0 || (deps & (uint64_t{1} << local)) != 0) {
        throw std::invalid_argument("invalid stateful graph dependency mask");
      }
    }
  }
  return {tasks.size() * sizeof(Task), programs.size() * sizeof(Program),
          size_t{config.phase_state_count} * sizeof(MaskState)};
}

inline void validate_compiled_plan(const std::vector<Task> &tasks,
                                   const std::vector<Program> &programs,
                                   const CompiledPlan &plan) {
  if (plan.stages.empty() || plan.programs.size() != programs.size()) {
    throw std::invalid_argument("invalid stateful graph compiled plan size");
  }
  for (size_t index = 0; index < programs.size(); ++index) {
    const Program &program = programs[index];
    const CompiledProgram &compiled = plan.programs[index];
    if (compiled.stage_count == 0 || compiled.stage_offset > plan.stages.size() ||
        compiled.stage_count > plan.stages.size() - compiled.stage_offset) {
      throw std::invalid_argument("invalid stateful graph compiled stages");
    }
    uint32_t next_task = program.task_offset;
    uint64_t done = 0;
    for (uint32_t s = 0; s < compiled.stage_count; ++s) {
      const Stage &stage = plan.stages[compiled.stage_offset + s];
      const uint32_t finished = next_task - program.task_offset;
      if (stage.task_count == 0 || stage.task_offset != next_task ||
          stage.task_count > program.task_count - finished) {
        throw std::invalid_argument("invalid stateful graph compiled stage");
      }
      for (uint32_t t = 0; t < stage.task_count; ++t) {
        const uint64_t deps = task_dependencies(tasks[stage.task_offset + t]);
        if ((deps & done) != deps) {
          throw std::invalid_argument("compiled stage contains dependent tasks");
        }
      }
      done |= valid_task_mask(stage.task_count) << finished;
      next_task += stage.task_count;
    }
    if (next_task != program.task_offset + program.task_count) {
      throw std::invalid_argument("compiled plan does not cover program");
    }
  }
}

} // namespace detail

inline void validate_resident_graph(const std::vector<Task> &tasks,
                                    const std::vector<Program> &programs,
                                    ResidentConfig config) {
  (void)detail::validate_resident_graph(tasks, programs, config);
}

// Splits each Program, in task order, into maximal runs of tasks whose
// dependencies are all satisfied by earlier runs. A task that depends on a
// later task (or on itself through a cycle) cannot be placed and is rejected.
inline CompiledPlan compile_resident_plan(const std::vector<Task> &tasks,
                                          const std::vector<Program> &programs,
                                          ResidentConfig config) {
  validate_resident_graph(tasks, programs, config);
  CompiledPlan plan;
  plan.programs.reserve(programs.size());
  for (const Program &program : programs) {
    const uint32_t first_stage = static_cast<uint32_t>(plan.stages.size());
    uint64_t done = 0;
    uint32_t local = 0;
    while (local < program.task_count) {
      const uint32_t begin = local;
      while (local < program.task_count) {
        const uint64_t deps =
            detail::task_dependencies(tasks[program.task_offset + local]);
        if ((deps & done) != deps) {
          break;
        }
        ++local;
      }
      if (local == begin) {
        throw std::invalid_argument(
            "stateful graph tasks are not in topological stage order");
      }
      plan.stages.push_back({program.task_offset + begin, local - begin});
      done |= detail::valid_task_mask(local - begin) << begin;
    }
    plan.programs.push_back(
        {first_stage, static_cast<uint32_t>(plan.stages.size()) - first_stage});
  }
  detail::validate_compiled_plan(tasks, programs, plan);
  return plan;
}

// Owns State, task/Program tables, per-generation MaskStates, the validation
// cache and (optionally) the compiled plan of one resident graph on one device.
// Task semantics stay in the kernel's workload; the executor only binds an
// opaque device context pointer.
class ResidentExecutor {
public:
  ResidentExecutor(Device device, const Kernel &kernel,
                   const std::vector<Task> &tasks,
                   const std::vector<Program> &programs, ResidentConfig config)
      : ResidentExecutor(device, kernel, tasks, programs, config,
                         detail::validate_resident_graph(tasks, programs, config)) {}

  ResidentExecutor(Device device, const Kernel &kernel,
                   const std::vector<Task> &tasks,
                   const std::vector<Program> &programs, ResidentConfig config,
                   const CompiledPlan &plan)
      : ResidentExecutor(device, kernel, tasks, programs, config) {
    upload_compiled_plan(tasks, programs, plan);
  }

  ResidentExecutor(const ResidentExecutor &) = delete;
  ResidentExecutor &operator=(const ResidentExecutor &) = delete;
  ResidentExecutor(ResidentExecutor &&) = default;
  ResidentExecutor &operator=(ResidentExecutor &&) = default;

  void upload_graph(const std::vector<Task> &tasks,
                    const std::vector<Program> &programs) {
    const detail::ValidatedGraph graph =
        detail::validate_resident_graph(tasks, programs, config_);
    if (graph.task_bytes > task_buffer_.size() ||
        graph.program_bytes > program_buffer_.size()) {
      throw std::invalid_argument(
          "stateful graph exceeds resident executor capacity");
    }
    copy_to_device(task_buffer_, tasks);
    copy_to_device(program_buffer_, programs);
    task_count_ = static_cast<uint32_t>(tasks.size());
    program_count_ = static_cast<uint32_t>(programs.size());
    stage_count_ = 0;
    invalidate_validation();
    initialized_ = false;
  }

  void upload_graph(const std::vector<Task> &tasks,
                    const std::vector<Program> &programs,
                    const CompiledPlan &plan) {
    upload_graph(tasks, programs);
    upload_compiled_plan(tasks, programs, plan);
  }

  void bind_context(void *device_context) {
    context_ = device_context;
    invalidate_validation();
  }

  // Forget the cached device validation. Needed after changing
  // validation-relevant data behind an already bound context; uploads,
  // bind_context() and new initialize() parameters do this automatically.
  void invalidate_validation() {
    const ValidationState fresh{};
    copy_to_device(validation_buffer_, &fresh, sizeof(fresh));
    validation_key_.reset();
  }

  void initialize(uint32_t program_index, uint32_t max_steps,
                  uint32_t stop_value) {
    prepare_initial_state(program_index, max_steps, stop_value);
    copy_to_device(state_buffer_, &initial_state_, sizeof(initial_state_));
    copy_to_device(phase_state_buffer_, empty_phase_states_);
    initialized_ = true;
  }

  // Same state as initialize(), but written by asynchronous device-to-device
  // copies on the default queue from a pristine image kept on the device. The
  // image is refreshed (synchronously) only when the parameters change.
  void initialize_on_device(uint32_t program_index, uint32_t max_steps,
                            uint32_t stop_value) {
    prepare_initial_state(program_index, max_steps, stop_value);
    const std::array<uint32_t, 3> key = {program_index, max_steps, stop_value};
    if (!pristine_) {
      pristine_.emplace(state_buffer_.device(),
                        sizeof(State) + phase_state_buffer_.size());
    }
    if (!pristine_key_ || *pristine_key_ != key) {
      std::vector<unsigned char> image(pristine_->size(), 0);
      std::copy_n(reinterpret_cast<const unsigned char *>(&initial_state_),
                  sizeof(State), image.begin());
      copy_to_device(*pristine_, image);
      pristine_key_ = key;
    }
    check(lr_memcpy_async(state_buffer_.device(), state_buffer_.data(),
                          pristine_->data(), sizeof(State),
                          LR_MEMCPY_DEVICE_TO_DEVICE, nullptr),
          "lr_memcpy_async state");
    check(lr_memcpy_async(state_buffer_.device(), phase_state_buffer_.data(),
                          detail_offset(*pristine_, sizeof(State)),
                          phase_state_buffer_.size(), LR_MEMCPY_DEVICE_TO_DEVICE,
                          nullptr),
          "lr_memcpy_async phase states");
    initialized_ = true;
  }

  void launch() const {
    require_initialized();
    const ResidentArgs args = arguments();
    lrrt::launch(kernel_, launch_config_, args);
  }

  void launch(const Queue &queue,
              const std::vector<const Event *> &dependencies = {}) const {
    require_initialized();
    const ResidentArgs args = arguments();
    lrrt::launch(queue, kernel_, launch_config_, args, dependencies);
  }

  State read_state() const {
    require_initialized();
    State state{};
    copy_to_host(&state, state_buffer_, sizeof(state));
    return state;
  }

  State *device_state() const { return static_cast<State *>(state_buffer_.data()); }
  const Task *device_tasks() const {
    return static_cast<const Task *>(task_buffer_.data());
  }
  MaskState *device_phase_states() const {
    return static_cast<MaskState *>(phase_state_buffer_.data());
  }
  uint32_t task_count() const { return task_count_; }
  uint32_t program_count() const { return program_count_; }
  uint32_t phase_state_count() const { return config_.phase_state_count; }
  uint32_t worker_count() const { return config_.worker_count; }
  bool has_compiled_plan() const { return stage_count_ != 0; }
  const lr_launch_config_t &launch_config() const { return launch_config_; }
  ResidentArgs arguments() const {
    return {
        static_cast<State *>(state_buffer_.data()),
        static_cast<const Task *>(task_buffer_.data()),
        static_cast<const Program *>(program_buffer_.data()),
        static_cast<MaskState *>(phase_state_buffer_.data()),
        program_count_,
        task_count_,
        config_.phase_state_count,
        context_,
        stage_buffer_ ? static_cast<const Stage *>(stage_buffer_->data()) : nullptr,
        compiled_program_buffer_ ? static_cast<const CompiledProgram *>(
                                       compiled_program_buffer_->data())
                                 : nullptr,
        stage_count_,
        config_.wait_limit_ms,
        static_cast<ValidationState *>(validation_buffer_.data()),
    };
  }

private:
  ResidentExecutor(Device device, const Kernel &kernel,
                   const std::vector<Task> &tasks,
                   const std::vector<Program> &programs, ResidentConfig config,
                   detail::ValidatedGraph graph)
      : kernel_(kernel.get()), config_(config),
        launch_config_{{config.worker_count * kWorkerThreads, 1, 1},
                       {kWorkerThreads, 1, 1},
                       config.dynamic_shared_memory_bytes},
        state_buffer_(device, sizeof(State)),
        task_buffer_(device, graph.task_bytes),
        program_buffer_(device, graph.program_bytes),
        phase_state_buffer_(device, graph.phase_state_bytes),
        validation_buffer_(device, sizeof(ValidationState)),
        empty_phase_states_(config.phase_state_count) {
    check(lr_kernel_set_resident(kernel_, 1), "lr_kernel_set_resident");
    upload_graph(tasks, programs);
  }

  static void *detail_offset(const DeviceBuffer &buffer, size_t bytes) {
    return static_cast<unsigned char *>(buffer.data()) + bytes;
  }

  void prepare_initial_state(uint32_t program_index, uint32_t max_steps,
                             uint32_t stop_value) {
    if (program_index >= program_count_) {
      throw std::invalid_argument("invalid stateful graph initial program");
    }
    if (max_steps == 0) {
      throw std::invalid_argument("stateful graph max steps must be nonzero");
    }
    const std::array<uint32_t, 3> key = {program_index, max_steps, stop_value};
    if (!validation_key_ || *validation_key_ != key) {
      invalidate_validation();
      validation_key_ = key;
    }
    initial_state_ = State{};
    initial_state_.abi_version = kAbiVersion;
    initial_state_.status = static_cast<uint32_t>(Status::ready);
    initial_state_.phase = make_phase(0, program_index);
    initial_state_.max_steps = max_steps;
    initial_state_.stop_value = stop_value;
    initial_state_.worker_count = config_.worker_count;
  }

  void upload_compiled_plan(const std::vector<Task> &tasks,
                            const std::vector<Program> &programs,
                            const CompiledPlan &plan) {
    detail::validate_compiled_plan(tasks, programs, plan);
    const size_t stage_bytes = plan.stages.size() * sizeof(Stage);
    const size_t program_bytes = plan.programs.size() * sizeof(CompiledProgram);
    if (!stage_buffer_) {
      stage_buffer_.emplace(state_buffer_.device(), stage_bytes);
      compiled_program_buffer_.emplace(state_buffer_.device(), program_bytes);
    } else if (stage_bytes > stage_buffer_->size() ||
               program_bytes > compiled_program_buffer_->size()) {
      throw std::invalid_argument(
          "compiled plan exceeds resident executor capacity");
    }
    copy_to_device(*stage_buffer_, plan.stages);
    copy_to_device(*compiled_program_buffer_, plan.programs);
    stage_count_ = static_cast<uint32_t>(plan.stages.size());
    invalidate_validation();
    initialized_ = false;
  }

  void require_initialized() const {
    if (!initialized_) {
      throw std::logic_error("stateful graph executor is not initialized");
    }
  }

  lr_kernel_t *kernel_;
  ResidentConfig config_;
  lr_launch_config_t launch_config_;
  DeviceBuffer state_buffer_;
  DeviceBuffer task_buffer_;
  DeviceBuffer program_buffer_;
  DeviceBuffer phase_state_buffer_;
  DeviceBuffer validation_buffer_;
  std::optional<DeviceBuffer> stage_buffer_;
  std::optional<DeviceBuffer> compiled_program_buffer_;
  std::optional<DeviceBuffer> pristine_;
  std::vector<MaskState> empty_phase_states_;
  State initial_state_{};
  void *context_ = nullptr;
  uint32_t task_count_ = 0;
  uint32_t program_count_ = 0;
  uint32_t stage_count_ = 0;
  bool initialized_ = false;
  std::optional<std::array<uint32_t, 3>> validation_key_;
  std::optional<std::array<uint32_t, 3>> pristine_key_;
};

} // namespace lrrt::persistent_graph

#endif // LRRT_PERSISTENT_GRAPH_RESIDENT_EXECUTOR_HPP_
