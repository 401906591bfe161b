// Persistent Graph ABI shared by the host executor and the sm_100a resident
// kernels.
//
// Byte layouts of every struct are those of light-rocm-runtime
// include/lrrt/persistent_graph/abi.hpp:42-168 (the static_asserts below pin
// them) so task tables, Program tables and ResidentArgs blobs built for that
// ABI are accepted unchanged. Two constants differ, and kAbiVersion moves from 9
// to 10 because of them:
//   * kMaximumResidentWorkers is 256 instead of 32. The reference caps a
//     resident grid at one AMD shader engine because HSA has no cooperative
//     dispatch; a B200 resident grid is one block per SM (148) launched
//     cooperatively, so co-residency is guaranteed by the driver.
//   * ResidentArgs::reserved, zero in reference callers, now carries an
//     optional device wait limit in milliseconds (0 = default). Every spin
//     wait in the resident schedulers gives up after that limit and reports
//     Status::invalid_program with error_code kErrorWaitTimeout instead of
//     hanging the GPU.
#ifndef LRRT_PERSISTENT_GRAPH_ABI_HPP_
#define LRRT_PERSISTENT_GRAPH_ABI_HPP_

#include <cstddef>
#include <cstdint>
#include <type_traits>

#if defined(__CUDACC__)
#define LRRT_HOST_DEVICE __host__ __device__
#else
#define LRRT_HOST_DEVICE
#endif

namespace lrrt::persistent_graph {

constexpr uint32_t kAbiVersion = 10;
// State::abi_version values the resident kernels accept: this ABI and the
// reference's 9, whose struct layouts are the same (a State built by a
// reference caller carries 9).
constexpr uint32_t kReferenceAbiVersion = 9;
LRRT_HOST_DEVICE constexpr bool accepted_abi_version(uint32_t version) {
  return version == kAbiVersion || version == kReferenceAbiVersion;
}
constexpr uint32_t kWorkerThreads = 256;
constexpr uint32_t kMaximumResidentWorkers = 256;
constexpr uint32_t kMaximumTasks = 64;
constexpr uint32_t kMaximumPrograms = 256;
constexpr uint32_t kNoTask = UINT32_MAX;
constexpr uint32_t kProgramIndexBits = 8;
constexpr uint32_t kProgramIndexMask = (1u << kProgramIndexBits) - 1u;

// error_code values written into State when status becomes invalid_program.
constexpr uint32_t kErrorValidation = 1;      // graph or context rejected
constexpr uint32_t kErrorPhaseSlots = 2;      // phase_state_count exhausted
constexpr uint32_t kErrorWaitTimeout = 3;     // a device wait hit its limit
constexpr uint32_t kErrorStreamMismatch = 4;  // weight stream out of step
constexpr uint32_t kDefaultWaitLimitMs = 2000;

LRRT_HOST_DEVICE constexpr uint32_t make_phase(uint32_t generation,
                                               uint32_t program_index) {
  return (generation << kProgramIndexBits) | program_index;
}
LRRT_HOST_DEVICE constexpr uint32_t phase_generation(uint32_t phase) {
  return phase >> kProgramIndexBits;
}
LRRT_HOST_DEVICE constexpr uint32_t phase_program(uint32_t phase) {
  return phase & kProgramIndexMask;
}

enum class Status : uint32_t {
  ready = 0,
  running = 1,
  complete = 2,
  max_steps = 3,
  invalid_program = 4,
};

// Device-resident control word block. `phase` packs the generation (which
// MaskState slot the current Program uses) with the active Program index.
struct alignas(64) State {
  uint32_t abi_version;
  uint32_t status;
  uint32_t phase;
  uint32_t step;
  uint32_t max_steps;
  uint32_t stop_value;
  uint32_t error_code;
  uint32_t worker_count;
  uint64_t executed_tasks;
  uint32_t predicate_value;
  // Nonzero when a Program flagged kProgramBranchesOnState completes selects
  // its branch_program instead of next_program.
  uint32_t branch_value;
  uint32_t reserved[4];
};

// One task: an opcode with a [begin, end) range, two opcode-specific
// arguments, and a 64-bit dependency mask over the tasks of its Program.
struct alignas(32) Task {
  uint32_t opcode;
  uint32_t dependency_mask;
  uint32_t begin;
  uint32_t end;
  uint32_t argument0;
  uint32_t argument1;
  uint32_t dependency_mask_high;
  uint32_t reserved;
};

enum ProgramFlags : uint32_t {
  kProgramAdvancesStep = 1u << 0u,
  kProgramEvaluatesPredicate = 1u << 1u,
  kProgramBranchesOnState = 1u << 2u,
};

// A Program is a contiguous task range forming one DAG plus its successor(s).
struct alignas(16) Program {
  uint32_t task_offset;
  uint32_t task_count;
  uint32_t next_program;
  uint32_t flags;
  uint32_t branch_program;
  uint32_t reserved[3];
};

// Per-generation scheduling state. The dynamic scheduler uses all fields; the
// compiled scheduler counts barrier arrivals in claimed_mask and publishes the
// number of released barriers in completed_mask.
struct MaskState {
  uint32_t claimed_mask;
  uint32_t completed_mask;
  uint32_t claimed_mask_high;
  uint32_t completed_mask_high;
  uint32_t completed_count;
};

enum class ValidationStatus : uint32_t {
  unvalidated = 0,
  valid = 1,
  invalid = 2,
};

// Caches device-side validation across launches of an unchanged graph.
struct alignas(8) ValidationState {
  uint32_t status;
  uint32_t reserved;
};

// A compiled stage: consecutive tasks with no dependencies among themselves.
struct alignas(8) Stage {
  uint32_t task_offset;
  uint32_t task_count;
};

struct alignas(8) CompiledProgram {
  uint32_t stage_offset;
  uint32_t stage_count;
};

// Kernel parameter block of every resident kernel (13 scalar parameters).
struct ResidentArgs {
  State *state;
  const Task *tasks;
  const Program *programs;
  MaskState *phase_states;
  uint32_t program_count;
  uint32_t task_count;
  uint32_t phase_state_count;
  void *context;
  const Stage *stages;
  const CompiledProgram *compiled_programs;
  uint32_t stage_count;
  uint32_t reserved; // wait limit in ms, 0 = kDefaultWaitLimitMs
  ValidationState *validation_state;
};

// Kernel parameter block of the host-driven single-step kernels.
struct HostStepArgs {
  State *state;
  const Task *tasks;
  uint32_t task_count;
  uint32_t reserved;
  void *context;
};

static_assert(std::is_standard_layout_v<State>);
static_assert(std::is_standard_layout_v<Task>);
static_assert(std::is_standard_layout_v<Program>);
static_assert(std::is_standard_layout_v<MaskState>);
static_assert(std::is_standard_layout_v<ValidationState>);
static_assert(std::is_standard_layout_v<Stage>);
static_assert(std::is_standard_layout_v<CompiledProgram>);
static_assert(std::is_standard_layout_v<ResidentArgs>);
static_assert(std::is_standard_layout_v<HostStepArgs>);
static_assert(sizeof(State) == 64);
static_assert(sizeof(Task) == 32);
static_assert(sizeof(Program) == 32);
static_assert(sizeof(MaskState) == 20);
static_assert(sizeof(ValidationState) == 8);
static_assert(sizeof(Stage) == 8);
static_assert(sizeof(CompiledProgram) == 8);
static_assert(sizeof(ResidentArgs) == 88);
static_assert(sizeof(HostStepArgs) == 32);
static_assert(offsetof(ResidentArgs, reserved) == 76);

} // namespace lrrt::persistent_graph

#endif // LRRT_PERSISTENT_GRAPH_ABI_HPP_
