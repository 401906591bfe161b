// lr_* C ABI over the CUDA driver API (sm_100a, B200).
//
// Semantics follow light-rocm-runtime's runtime core (src/runtime.cpp,
// src/memory.cpp, src/launch.cpp:988-1335, src/event.cpp, src/queue.cpp):
//   * process-global init with a registry mutex; every call validates its
//     handles against live registries, so stale or foreign handles return
//     LR_ERROR_INVALID_ARGUMENT instead of being dereferenced;
//   * a device must be opened before queues, events or memory are created on it;
//   * each opened device owns a default queue (one in-order CUDA stream) that
//     lr_launch, lr_memcpy_async and lr_event_record use, which gives the
//     reference's completion ordering between launches and async copies;
//   * launch grids are counted in threads and must be >= block per dimension,
//     blocks are <= 65535 per dimension, args fit the kernel parameter block;
//   * lr_free / lr_module_destroy / lr_shutdown drain the device first.
// The HSA/AQL queue machinery of the reference has no counterpart: CUDA
// streams, events and cooperative launches replace it.
#include "driver.hpp"
#include "lrrt/lrrt.h"

#include <dlfcn.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <memory>
#include <mutex>
#include <string>
#include <unordered_map>
#include <unordered_set>
#include <vector>

struct lr_queue_t {
  uint32_t device;
  CUstream stream;
};

struct lr_event_t {
  uint32_t device;
  CUevent begin;
  CUevent end;
  bool recorded;
};

struct lr_kernel_t {
  lr_module_t *module;
  CUfunction function;
  std::string name;
  uint32_t kernarg_size;
  std::vector<size_t> parameter_offsets;
  uint32_t static_shared_bytes;
  uint32_t local_bytes;
  uint32_t dynamic_shared_limit; // last MAX_DYNAMIC_SHARED_SIZE_BYTES set
  bool resident;
  bool overlapped; // launches carry programmatic stream serialization
};

struct lr_module_t {
  uint32_t device;
  CUmodule module;
  std::vector<std::unique_ptr<lr_kernel_t>> kernels;
};

namespace lrrt_b200 {

#define LRRT_STRINGIFY_(x) #x
#define LRRT_STRINGIFY(x) LRRT_STRINGIFY_(x)

bool load_driver(Driver &driver) {
  if (driver.loaded) {
    return true;
  }
  void *library = dlopen("libcuda.so.1", RTLD_NOW | RTLD_LOCAL);
  if (library == nullptr) {
    return false;
  }
  Driver candidate;
  bool complete = true;
#define LRRT_LOAD_DRIVER_FUNCTION(fn)                                          \
  candidate.fn##_ =                                                            \
      reinterpret_cast<decltype(&fn)>(dlsym(library, LRRT_STRINGIFY(fn)));     \
  complete = complete && candidate.fn##_ != nullptr;
  LRRT_DRIVER_FUNCTIONS(LRRT_LOAD_DRIVER_FUNCTION)
#undef LRRT_LOAD_DRIVER_FUNCTION
  if (!complete) {
    dlclose(library);
    return false;
  }
  candidate.library = library;
  candidate.loaded = true;
  driver = candidate;
  return true;
}

namespace {

struct DeviceState {
  bool open = false;
  CUdevice device = 0;
  CUcontext context = nullptr;
  CUstream stream = nullptr;
  lr_memory_stats_t stats{};
  std::unordered_map<void *, size_t> allocations;
  std::unordered_map<void *, size_t> host_allocations;
  uint32_t sm_count = 0;
};

std::mutex g_mutex;
bool g_initialized = false;
Driver g_driver;
std::vector<DeviceState> g_devices;
std::unordered_set<lr_queue_t *> g_queues;
std::unordered_set<lr_event_t *> g_events;
std::unordered_set<lr_module_t *> g_modules;
std::unordered_set<lr_kernel_t *> g_kernels;
std::string g_last_error;

using Lock = std::lock_guard<std::mutex>;

void note_error(const char *what, CUresult result) {
  const char *name = nullptr;
  const char *text = nullptr;
  if (g_driver.loaded) {
    g_driver.cuGetErrorName_(result, &name);
    g_driver.cuGetErrorString_(result, &text);
  }
  char buffer[512];
  std::snprintf(buffer, sizeof(buffer), "%s: %s (%d): %s", what,
                name ? name : "CUDA error", static_cast<int>(result),
                text ? text : "");
  g_last_error = buffer;
}

lr_status_t to_status(CUresult result) {
  switch (result) {
  case CUDA_SUCCESS:
    return LR_SUCCESS;
  case CUDA_ERROR_INVALID_VALUE:
  case CUDA_ERROR_INVALID_HANDLE:
  case CUDA_ERROR_NOT_FOUND:
  case CUDA_ERROR_INVALID_IMAGE:
  case CUDA_ERROR_NO_BINARY_FOR_GPU:
  case CUDA_ERROR_INVALID_SOURCE:
  case CUDA_ERROR_COOPERATIVE_LAUNCH_TOO_LARGE:
  case CUDA_ERROR_LAUNCH_OUT_OF_RESOURCES:
  case CUDA_ERROR_OUT_OF_MEMORY:
    return LR_ERROR_INVALID_ARGUMENT;
  case CUDA_ERROR_NOT_SUPPORTED:
    return LR_ERROR_NOT_SUPPORTED;
  case CUDA_ERROR_ILLEGAL_ADDRESS:
  case CUDA_ERROR_ILLEGAL_INSTRUCTION:
  case CUDA_ERROR_MISALIGNED_ADDRESS:
  case CUDA_ERROR_INVALID_ADDRESS_SPACE:
  case CUDA_ERROR_INVALID_PC:
  case CUDA_ERROR_HARDWARE_STACK_ERROR:
  case CUDA_ERROR_ASSERT:
  case CUDA_ERROR_LAUNCH_FAILED:
  case CUDA_ERROR_LAUNCH_TIMEOUT:
  case CUDA_ERROR_ECC_UNCORRECTABLE:
    return LR_ERROR_DEVICE_FAULT;
  default:
    return LR_ERROR_RUNTIME;
  }
}

lr_status_t cu(CUresult result, const char *what) {
  if (result != CUDA_SUCCESS) {
    note_error(what, result);
  }
  return to_status(result);
}

#define LR_TRY(expression)                                                     \
  do {                                                                         \
    const lr_status_t lr_try_status_ = (expression);                           \
    if (lr_try_status_ != LR_SUCCESS) {                                        \
      return lr_try_status_;                                                   \
    }                                                                          \
  } while (0)

DeviceState *open_device_state(uint32_t index) {
  if (index >= g_devices.size() || !g_devices[index].open) {
    return nullptr;
  }
  return &g_devices[index];
}

lr_status_t make_current(const DeviceState &state) {
  return cu(g_driver.cuCtxSetCurrent_(state.context), "cuCtxSetCurrent");
}

lr_status_t drain(const DeviceState &state) {
  LR_TRY(make_current(state));
  return cu(g_driver.cuCtxSynchronize_(), "cuCtxSynchronize");
}

void count_copy(DeviceState &state, size_t size, lr_memcpy_kind_t kind) {
  switch (kind) {
  case LR_MEMCPY_HOST_TO_DEVICE:
    state.stats.h2d_copy_bytes += size;
    break;
  case LR_MEMCPY_DEVICE_TO_HOST:
    state.stats.d2h_copy_bytes += size;
    break;
  case LR_MEMCPY_DEVICE_TO_DEVICE:
    state.stats.d2d_copy_bytes += size;
    break;
  }
  ++state.stats.memcpy_count;
}

bool valid_kind(lr_memcpy_kind_t kind) {
  return kind == LR_MEMCPY_HOST_TO_DEVICE || kind == LR_MEMCPY_DEVICE_TO_HOST ||
         kind == LR_MEMCPY_DEVICE_TO_DEVICE;
}

// Waits, on `stream`, for every listed event. All must be live, recorded and
// belong to `device`.
lr_status_t wait_for_events(uint32_t device, CUstream stream,
                            lr_event_t *const *events, size_t count) {
  if (count != 0 && events == nullptr) {
    return LR_ERROR_INVALID_ARGUMENT;
  }
  for (size_t i = 0; i < count; ++i) {
    lr_event_t *event = events[i];
    if (event == nullptr || g_events.count(event) == 0 ||
        event->device != device) {
      return LR_ERROR_INVALID_ARGUMENT;
    }
  }
  for (size_t i = 0; i < count; ++i) {
    if (events[i]->recorded) {
      LR_TRY(cu(g_driver.cuStreamWaitEvent_(stream, events[i]->end, 0),
                "cuStreamWaitEvent"));
    }
  }
  return LR_SUCCESS;
}

lr_status_t record_marker(lr_event_t *event, CUstream stream) {
  if (event->recorded) {
    LR_TRY(cu(g_driver.cuEventSynchronize_(event->end), "cuEventSynchronize"));
  }
  LR_TRY(cu(g_driver.cuEventRecord_(event->begin, stream), "cuEventRecord"));
  LR_TRY(cu(g_driver.cuEventRecord_(event->end, stream), "cuEventRecord"));
  event->recorded = true;
  return LR_SUCCESS;
}

lr_status_t async_copy(uint32_t device_index, void *dst, const void *src,
                       size_t size, lr_memcpy_kind_t kind, lr_event_t *event,
                       lr_event_t *const *dependencies, size_t dependency_count,
                       bool explicit_dependencies) {
  DeviceState *state = open_device_state(device_index);
  if (state == nullptr || dst == nullptr || src == nullptr || size == 0 ||
      !valid_kind(kind)) {
    return LR_ERROR_INVALID_ARGUMENT;
  }
  if (event != nullptr &&
      (g_events.count(event) == 0 || event->device != device_index)) {
    return LR_ERROR_INVALID_ARGUMENT;
  }
  if (explicit_dependencies) {
    if (dependency_count != 0 && dependencies == nullptr) {
      return LR_ERROR_INVALID_ARGUMENT;
    }
    for (size_t i = 0; i < dependency_count; ++i) {
      if (dependencies[i] == nullptr) {
        return LR_ERROR_INVALID_ARGUMENT;
      }
    }
  }
  LR_TRY(make_current(*state));
  if (explicit_dependencies) {
    LR_TRY(wait_for_events(device_index, state->stream, dependencies,
                           dependency_count));
  }
  if (event != nullptr) {
    if (event->recorded) {
      LR_TRY(cu(g_driver.cuEventSynchronize_(event->end), "cuEventSynchronize"));
    }
    LR_TRY(cu(g_driver.cuEventRecord_(event->begin, state->stream),
              "cuEventRecord"));
  }
  LR_TRY(cu(g_driver.cuMemcpyAsync_(reinterpret_cast<CUdeviceptr>(dst),
                                    reinterpret_cast<CUdeviceptr>(src), size,
                                    state->stream),
            "cuMemcpyAsync"));
  if (event != nullptr) {
    LR_TRY(cu(g_driver.cuEventRecord_(event->end, state->stream),
              "cuEventRecord"));
    event->recorded = true;
  }
  count_copy(*state, size, kind);
  return LR_SUCCESS;
}

lr_status_t set_dynamic_shared(lr_kernel_t *kernel, uint32_t bytes) {
  if (bytes <= 48u * 1024u || bytes <= kernel->dynamic_shared_limit) {
    return LR_SUCCESS;
  }
  LR_TRY(cu(g_driver.cuFuncSetAttribute_(
                kernel->function, CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES,
                static_cast<int>(bytes)),
            "cuFuncSetAttribute(max dynamic shared)"));
  kernel->dynamic_shared_limit = bytes;
  return LR_SUCCESS;
}

lr_status_t launch_impl(lr_kernel_t *kernel, const lr_launch_config_t *config,
                        const void *args, size_t args_size, lr_queue_t *queue,
                        lr_event_t *const *dependencies,
                        size_t dependency_count) {
  if (!g_initialized) {
    return LR_ERROR_NOT_INITIALIZED;
  }
  if (kernel == nullptr || config == nullptr || args == nullptr || args_size == 0) {
    return LR_ERROR_INVALID_ARGUMENT;
  }
  const lr_dim3_t &grid = config->grid;
  const lr_dim3_t &block = config->block;
  if (grid.x == 0 || grid.y == 0 || grid.z == 0 || block.x == 0 ||
      block.y == 0 || block.z == 0) {
    return LR_ERROR_INVALID_ARGUMENT;
  }
  if (grid.x < block.x || grid.y < block.y || grid.z < block.z) {
    return LR_ERROR_INVALID_ARGUMENT;
  }
  if (block.x > UINT16_MAX || block.y > UINT16_MAX || block.z > UINT16_MAX) {
    return LR_ERROR_INVALID_ARGUMENT;
  }
  if (g_kernels.count(kernel) == 0) {
    return LR_ERROR_INVALID_ARGUMENT;
  }
  const uint32_t device_index = kernel->module->device;
  DeviceState *state = open_device_state(device_index);
  if (state == nullptr || args_size > kernel->kernarg_size) {
    return LR_ERROR_INVALID_ARGUMENT;
  }
  CUstream stream = state->stream;
  if (queue != nullptr) {
    if (g_queues.count(queue) == 0 || queue->device != device_index) {
      return LR_ERROR_INVALID_ARGUMENT;
    }
    stream = queue->stream;
  }
  LR_TRY(make_current(*state));
  LR_TRY(wait_for_events(device_index, stream, dependencies, dependency_count));
  LR_TRY(set_dynamic_shared(kernel, config->shared_memory_bytes));

  // The packed blob is laid out exactly like the kernel parameter block; each
  // parameter pointer handed to the driver points into the zero-padded copy.
  std::vector<unsigned char> block_bytes(std::max<size_t>(kernel->kernarg_size, 1), 0);
  std::memcpy(block_bytes.data(), args, args_size);
  std::vector<void *> parameters;
  parameters.reserve(kernel->parameter_offsets.size());
  for (size_t offset : kernel->parameter_offsets) {
    parameters.push_back(block_bytes.data() + offset);
  }

  CUlaunchConfig launch{};
  launch.gridDimX = (grid.x + block.x - 1u) / block.x;
  launch.gridDimY = (grid.y + block.y - 1u) / block.y;
  launch.gridDimZ = (grid.z + block.z - 1u) / block.z;
  launch.blockDimX = block.x;
  launch.blockDimY = block.y;
  launch.blockDimZ = block.z;
  launch.sharedMemBytes = config->shared_memory_bytes;
  launch.hStream = stream;
  CUlaunchAttribute attributes[2]{};
  uint32_t attribute_count = 0;
  if (kernel->resident) {
    attributes[attribute_count].id = CU_LAUNCH_ATTRIBUTE_COOPERATIVE;
    attributes[attribute_count++].value.cooperative = 1;
  }
  if (kernel->overlapped) {
    attributes[attribute_count].id = CU_LAUNCH_ATTRIBUTE_PROGRAMMATIC_STREAM_SERIALIZATION;
    attributes[attribute_count++].value.programmaticStreamSerializationAllowed = 1;
  }
  if (attribute_count != 0) {
    launch.attrs = attributes;
    launch.numAttrs = attribute_count;
  }
  return cu(g_driver.cuLaunchKernelEx_(&launch, kernel->function,
                                       parameters.empty() ? nullptr
                                                          : parameters.data(),
                                       nullptr),
            "cuLaunchKernelEx");
}

void release_device(DeviceState &state) {
  if (!state.open) {
    return;
  }
  g_driver.cuCtxSetCurrent_(state.context);
  g_driver.cuCtxSynchronize_();
  for (auto it = g_modules.begin(); it != g_modules.end();) {
    lr_module_t *module = *it;
    if (&g_devices[module->device] == &state) {
      for (auto &kernel : module->kernels) {
        g_kernels.erase(kernel.get());
      }
      g_driver.cuModuleUnload_(module->module);
      delete module;
      it = g_modules.erase(it);
    } else {
      ++it;
    }
  }
  for (auto it = g_queues.begin(); it != g_queues.end();) {
    if (&g_devices[(*it)->device] == &state) {
      g_driver.cuStreamDestroy_((*it)->stream);
      delete *it;
      it = g_queues.erase(it);
    } else {
      ++it;
    }
  }
  for (auto it = g_events.begin(); it != g_events.end();) {
    if (&g_devices[(*it)->device] == &state) {
      g_driver.cuEventDestroy_((*it)->begin);
      g_driver.cuEventDestroy_((*it)->end);
      delete *it;
      it = g_events.erase(it);
    } else {
      ++it;
    }
  }
  for (auto &entry : state.allocations) {
    g_driver.cuMemFree_(reinterpret_cast<CUdeviceptr>(entry.first));
  }
  for (auto &entry : state.host_allocations) {
    g_driver.cuMemFreeHost_(entry.first);
  }
  g_driver.cuStreamDestroy_(state.stream);
  g_driver.cuDevicePrimaryCtxRelease_(state.device);
  state = DeviceState{};
}

} // namespace
} // namespace lrrt_b200

using namespace lrrt_b200;

extern "C" {

LRRT_API const char *lr_status_string(lr_status_t status) {
  switch (status) {
  case LR_SUCCESS:
    return "LR_SUCCESS";
  case LR_ERROR_INVALID_ARGUMENT:
    return "LR_ERROR_INVALID_ARGUMENT";
  case LR_ERROR_NOT_INITIALIZED:
    return "LR_ERROR_NOT_INITIALIZED";
  case LR_ERROR_ALREADY_INITIALIZED:
    return "LR_ERROR_ALREADY_INITIALIZED";
  case LR_ERROR_NOT_SUPPORTED:
    return "LR_ERROR_NOT_SUPPORTED";
  case LR_ERROR_RUNTIME:
    return "LR_ERROR_RUNTIME";
  case LR_ERROR_DEVICE_FAULT:
    return "LR_ERROR_DEVICE_FAULT";
  }
  return "LR_ERROR_UNKNOWN";
}

LRRT_API lr_status_t lr_init(void) {
  Lock lock(g_mutex);
  if (g_initialized) {
    return LR_ERROR_ALREADY_INITIALIZED;
  }
  g_devices.clear();
  int count = 0;
  if (load_driver(g_driver)) {
    const CUresult init = g_driver.cuInit_(0);
    if (init == CUDA_SUCCESS) {
      if (g_driver.cuDeviceGetCount_(&count) != CUDA_SUCCESS) {
        count = 0;
      }
    } else if (init != CUDA_ERROR_NO_DEVICE) {
      note_error("cuInit", init);
    }
  }
  g_devices.resize(static_cast<size_t>(std::max(count, 0)));
  g_initialized = true;
  return LR_SUCCESS;
}

LRRT_API lr_status_t lr_shutdown(void) {
  Lock lock(g_mutex);
  if (!g_initialized) {
    return LR_ERROR_NOT_INITIALIZED;
  }
  for (DeviceState &state : g_devices) {
    release_device(state);
  }
  g_devices.clear();
  g_queues.clear();
  g_events.clear();
  g_modules.clear();
  g_kernels.clear();
  g_initialized = false;
  return LR_SUCCESS;
}

LRRT_API lr_status_t lr_device_count(uint32_t *count) {
  Lock lock(g_mutex);
  if (!g_initialized) {
    return LR_ERROR_NOT_INITIALIZED;
  }
  if (count == nullptr) {
    return LR_ERROR_INVALID_ARGUMENT;
  }
  *count = static_cast<uint32_t>(g_devices.size());
  return LR_SUCCESS;
}

LRRT_API lr_status_t lr_device_open(uint32_t index, lr_device_t *device) {
  Lock lock(g_mutex);
  if (!g_initialized) {
    return LR_ERROR_NOT_INITIALIZED;
  }
  if (device == nullptr || index >= g_devices.size()) {
    return LR_ERROR_INVALID_ARGUMENT;
  }
  DeviceState &state = g_devices[index];
  if (!state.open) {
    DeviceState fresh;
    LR_TRY(cu(g_driver.cuDeviceGet_(&fresh.device, static_cast<int>(index)),
              "cuDeviceGet"));
    LR_TRY(cu(g_driver.cuDevicePrimaryCtxRetain_(&fresh.context, fresh.device),
              "cuDevicePrimaryCtxRetain"));
    lr_status_t status = cu(g_driver.cuCtxSetCurrent_(fresh.context), "cuCtxSetCurrent");
    if (status == LR_SUCCESS) {
      status = cu(g_driver.cuStreamCreate_(&fresh.stream, CU_STREAM_NON_BLOCKING),
                  "cuStreamCreate");
    }
    int sms = 0;
    if (status == LR_SUCCESS) {
      status = cu(g_driver.cuDeviceGetAttribute_(
                      &sms, CU_DEVICE_ATTRIBUTE_MULTIPROCESSOR_COUNT, fresh.device),
                  "cuDeviceGetAttribute");
    }
    if (status != LR_SUCCESS) {
      g_driver.cuDevicePrimaryCtxRelease_(fresh.device);
      return status;
    }
    fresh.sm_count = static_cast<uint32_t>(sms);
    fresh.open = true;
    state = std::move(fresh);
  }
  device->index = index;
  return LR_SUCCESS;
}

LRRT_API lr_status_t lr_device_name(lr_device_t device, char *name,
                                    size_t name_size) {
  Lock lock(g_mutex);
  if (!g_initialized) {
    return LR_ERROR_NOT_INITIALIZED;
  }
  DeviceState *state = open_device_state(device.index);
  if (state == nullptr || name == nullptr || name_size == 0) {
    return LR_ERROR_INVALID_ARGUMENT;
  }
  char text[256] = {};
  LR_TRY(cu(g_driver.cuDeviceGetName_(text, sizeof(text), state->device),
            "cuDeviceGetName"));
  const size_t length = std::strlen(text);
  if (length + 1 > name_size) {
    return LR_ERROR_INVALID_ARGUMENT;
  }
  std::memcpy(name, text, length + 1);
  return LR_SUCCESS;
}

LRRT_API lr_status_t lr_device_get_properties(lr_device_t device,
                                              lr_device_properties_t *properties) {
  Lock lock(g_mutex);
  if (!g_initialized) {
    return LR_ERROR_NOT_INITIALIZED;
  }
  DeviceState *state = open_device_state(device.index);
  if (state == nullptr || properties == nullptr) {
    return LR_ERROR_INVALID_ARGUMENT;
  }
  int warp = 0, threads_per_sm = 0, threads_per_block = 0, shared_optin = 0;
  LR_TRY(cu(g_driver.cuDeviceGetAttribute_(&warp, CU_DEVICE_ATTRIBUTE_WARP_SIZE,
                                           state->device),
            "cuDeviceGetAttribute"));
  LR_TRY(cu(g_driver.cuDeviceGetAttribute_(
                &threads_per_sm, CU_DEVICE_ATTRIBUTE_MAX_THREADS_PER_MULTIPROCESSOR,
                state->device),
            "cuDeviceGetAttribute"));
  LR_TRY(cu(g_driver.cuDeviceGetAttribute_(
                &threads_per_block, CU_DEVICE_ATTRIBUTE_MAX_THREADS_PER_BLOCK,
                state->device),
            "cuDeviceGetAttribute"));
  LR_TRY(cu(g_driver.cuDeviceGetAttribute_(
                &shared_optin, CU_DEVICE_ATTRIBUTE_MAX_SHARED_MEMORY_PER_BLOCK_OPTIN,
                state->device),
            "cuDeviceGetAttribute"));
  properties->compute_unit_count = state->sm_count;
  properties->wavefront_size = static_cast<uint32_t>(warp);
  properties->maximum_waves_per_compute_unit =
      static_cast<uint32_t>(threads_per_sm / std::max(warp, 1));
  properties->maximum_workgroup_size = static_cast<uint32_t>(threads_per_block);
  properties->group_segment_size = static_cast<uint64_t>(shared_optin);
  properties->shader_engine_count = 1;
  return LR_SUCCESS;
}

LRRT_API lr_status_t lr_get_memory_stats(lr_device_t device,
                                         lr_memory_stats_t *stats) {
  Lock lock(g_mutex);
  if (!g_initialized) {
    return LR_ERROR_NOT_INITIALIZED;
  }
  DeviceState *state = open_device_state(device.index);
  if (device.index >= g_devices.size() || stats == nullptr) {
    return LR_ERROR_INVALID_ARGUMENT;
  }
  *stats = state != nullptr ? state->stats : lr_memory_stats_t{};
  return LR_SUCCESS;
}

LRRT_API lr_status_t lr_reset_memory_stats(lr_device_t device) {
  Lock lock(g_mutex);
  if (!g_initialized) {
    return LR_ERROR_NOT_INITIALIZED;
  }
  if (device.index >= g_devices.size()) {
    return LR_ERROR_INVALID_ARGUMENT;
  }
  DeviceState *state = open_device_state(device.index);
  if (state != nullptr) {
    // Live/peak figures describe current allocations and survive a reset.
    lr_memory_stats_t fresh{};
    fresh.live_bytes = state->stats.live_bytes;
    fresh.peak_live_bytes = state->stats.live_bytes;
    fresh.pinned_host_live_bytes = state->stats.pinned_host_live_bytes;
    fresh.pinned_host_peak_live_bytes = state->stats.pinned_host_live_bytes;
    state->stats = fresh;
  }
  return LR_SUCCESS;
}

LRRT_API lr_status_t lr_queue_create(lr_device_t device, lr_queue_t **queue) {
  Lock lock(g_mutex);
  if (!g_initialized) {
    return LR_ERROR_NOT_INITIALIZED;
  }
  DeviceState *state = open_device_state(device.index);
  if (state == nullptr || queue == nullptr) {
    return LR_ERROR_INVALID_ARGUMENT;
  }
  LR_TRY(make_current(*state));
  CUstream stream = nullptr;
  LR_TRY(cu(g_driver.cuStreamCreate_(&stream, CU_STREAM_NON_BLOCKING),
            "cuStreamCreate"));
  lr_queue_t *created = new lr_queue_t{device.index, stream};
  g_queues.insert(created);
  *queue = created;
  return LR_SUCCESS;
}

LRRT_API lr_status_t lr_queue_destroy(lr_queue_t *queue) {
  Lock lock(g_mutex);
  if (!g_initialized) {
    return LR_ERROR_NOT_INITIALIZED;
  }
  if (queue == nullptr || g_queues.count(queue) == 0) {
    return LR_ERROR_INVALID_ARGUMENT;
  }
  DeviceState *state = open_device_state(queue->device);
  if (state != nullptr) {
    make_current(*state);
    g_driver.cuStreamSynchronize_(queue->stream);
    g_driver.cuStreamDestroy_(queue->stream);
  }
  g_queues.erase(queue);
  delete queue;
  return LR_SUCCESS;
}

LRRT_API lr_status_t lr_queue_synchronize(lr_queue_t *queue) {
  CUstream stream = nullptr;
  {
    Lock lock(g_mutex);
    if (!g_initialized) {
      return LR_ERROR_NOT_INITIALIZED;
    }
    if (queue == nullptr || g_queues.count(queue) == 0) {
      return LR_ERROR_INVALID_ARGUMENT;
    }
    DeviceState *state = open_device_state(queue->device);
    if (state == nullptr) {
      return LR_ERROR_INVALID_ARGUMENT;
    }
    LR_TRY(make_current(*state));
    stream = queue->stream;
  }
  const CUresult result = g_driver.cuStreamSynchronize_(stream);
  Lock lock(g_mutex);
  return cu(result, "cuStreamSynchronize");
}

LRRT_API lr_status_t lr_event_create(lr_device_t device, lr_event_t **event) {
  Lock lock(g_mutex);
  if (!g_initialized) {
    return LR_ERROR_NOT_INITIALIZED;
  }
  DeviceState *state = open_device_state(device.index);
  if (state == nullptr || event == nullptr) {
    return LR_ERROR_INVALID_ARGUMENT;
  }
  LR_TRY(make_current(*state));
  CUevent begin = nullptr, end = nullptr;
  LR_TRY(cu(g_driver.cuEventCreate_(&begin, CU_EVENT_DEFAULT), "cuEventCreate"));
  const lr_status_t status =
      cu(g_driver.cuEventCreate_(&end, CU_EVENT_DEFAULT), "cuEventCreate");
  if (status != LR_SUCCESS) {
    g_driver.cuEventDestroy_(begin);
    return status;
  }
  lr_event_t *created = new lr_event_t{device.index, begin, end, false};
  g_events.insert(created);
  *event = created;
  return LR_SUCCESS;
}

LRRT_API lr_status_t lr_event_destroy(lr_event_t *event) {
  Lock lock(g_mutex);
  if (!g_initialized) {
    return LR_ERROR_NOT_INITIALIZED;
  }
  if (event == nullptr || g_events.count(event) == 0) {
    return LR_ERROR_INVALID_ARGUMENT;
  }
  DeviceState *state = open_device_state(event->device);
  if (state != nullptr) {
    make_current(*state);
    if (event->recorded) {
      g_driver.cuEventSynchronize_(event->end);
    }
    g_driver.cuEventDestroy_(event->begin);
    g_driver.cuEventDestroy_(event->end);
  }
  g_events.erase(event);
  delete event;
  return LR_SUCCESS;
}

LRRT_API lr_status_t lr_event_record(lr_event_t *event) {
  Lock lock(g_mutex);
  if (!g_initialized) {
    return LR_ERROR_NOT_INITIALIZED;
  }
  if (event == nullptr || g_events.count(event) == 0) {
    return LR_ERROR_INVALID_ARGUMENT;
  }
  DeviceState *state = open_device_state(event->device);
  if (state == nullptr) {
    return LR_ERROR_INVALID_ARGUMENT;
  }
  LR_TRY(make_current(*state));
  return record_marker(event, state->stream);
}

LRRT_API lr_status_t lr_event_record_on_queue(lr_event_t *event,
                                              lr_queue_t *queue) {
  Lock lock(g_mutex);
  if (!g_initialized) {
    return LR_ERROR_NOT_INITIALIZED;
  }
  if (event == nullptr || g_events.count(event) == 0 || queue == nullptr ||
      g_queues.count(queue) == 0 || queue->device != event->device) {
    return LR_ERROR_INVALID_ARGUMENT;
  }
  DeviceState *state = open_device_state(event->device);
  if (state == nullptr) {
    return LR_ERROR_INVALID_ARGUMENT;
  }
  LR_TRY(make_current(*state));
  return record_marker(event, queue->stream);
}

LRRT_API lr_status_t lr_event_synchronize(lr_event_t *event) {
  CUevent handle = nullptr;
  {
    Lock lock(g_mutex);
    if (!g_initialized) {
      return LR_ERROR_NOT_INITIALIZED;
    }
    if (event == nullptr || g_events.count(event) == 0) {
      return LR_ERROR_INVALID_ARGUMENT;
    }
    if (!event->recorded) {
      return LR_SUCCESS;
    }
    DeviceState *state = open_device_state(event->device);
    if (state == nullptr) {
      return LR_ERROR_INVALID_ARGUMENT;
    }
    LR_TRY(make_current(*state));
    handle = event->end;
  }
  const CUresult result = g_driver.cuEventSynchronize_(handle);
  Lock lock(g_mutex);
  return cu(result, "cuEventSynchronize");
}

namespace {
lr_status_t elapsed_between(CUevent from, CUevent to, uint64_t *elapsed_ns) {
  LR_TRY(cu(g_driver.cuEventSynchronize_(from), "cuEventSynchronize"));
  LR_TRY(cu(g_driver.cuEventSynchronize_(to), "cuEventSynchronize"));
  float milliseconds = 0.0f;
  LR_TRY(cu(g_driver.cuEventElapsedTime_(&milliseconds, from, to),
            "cuEventElapsedTime"));
  *elapsed_ns = milliseconds <= 0.0f
                    ? 0u
                    : static_cast<uint64_t>(static_cast<double>(milliseconds) * 1.0e6);
  return LR_SUCCESS;
}
} // namespace

LRRT_API lr_status_t lr_event_elapsed_time_ns(const lr_event_t *start,
                                              const lr_event_t *end,
                                              uint64_t *elapsed_ns) {
  Lock lock(g_mutex);
  if (!g_initialized) {
    return LR_ERROR_NOT_INITIALIZED;
  }
  lr_event_t *first = const_cast<lr_event_t *>(start);
  lr_event_t *last = const_cast<lr_event_t *>(end);
  if (first == nullptr || last == nullptr || elapsed_ns == nullptr ||
      g_events.count(first) == 0 || g_events.count(last) == 0 ||
      first->device != last->device || !first->recorded || !last->recorded) {
    return LR_ERROR_INVALID_ARGUMENT;
  }
  DeviceState *state = open_device_state(first->device);
  if (state == nullptr) {
    return LR_ERROR_INVALID_ARGUMENT;
  }
  LR_TRY(make_current(*state));
  return elapsed_between(first->end, last->end, elapsed_ns);
}

LRRT_API lr_status_t lr_event_duration_ns(const lr_event_t *event,
                                          uint64_t *duration_ns) {
  Lock lock(g_mutex);
  if (!g_initialized) {
    return LR_ERROR_NOT_INITIALIZED;
  }
  lr_event_t *handle = const_cast<lr_event_t *>(event);
  if (handle == nullptr || duration_ns == nullptr ||
      g_events.count(handle) == 0 || !handle->recorded) {
    return LR_ERROR_INVALID_ARGUMENT;
  }
  DeviceState *state = open_device_state(handle->device);
  if (state == nullptr) {
    return LR_ERROR_INVALID_ARGUMENT;
  }
  LR_TRY(make_current(*state));
  return elapsed_between(handle->begin, handle->end, duration_ns);
}

LRRT_API lr_status_t lr_malloc(lr_device_t device, size_t size, void **ptr) {
  Lock lock(g_mutex);
  if (!g_initialized) {
    return LR_ERROR_NOT_INITIALIZED;
  }
  DeviceState *state = open_device_state(device.index);
  if (state == nullptr || ptr == nullptr || size == 0) {
    return LR_ERROR_INVALID_ARGUMENT;
  }
  LR_TRY(make_current(*state));
  CUdeviceptr address = 0;
  LR_TRY(cu(g_driver.cuMemAlloc_(&address, size), "cuMemAlloc"));
  void *pointer = reinterpret_cast<void *>(address);
  state->allocations[pointer] = size;
  lr_memory_stats_t &stats = state->stats;
  stats.live_bytes += size;
  stats.peak_live_bytes = std::max(stats.peak_live_bytes, stats.live_bytes);
  stats.total_allocated_bytes += size;
  ++stats.allocation_count;
  *ptr = pointer;
  return LR_SUCCESS;
}

LRRT_API lr_status_t lr_free(lr_device_t device, void *ptr) {
  Lock lock(g_mutex);
  if (!g_initialized) {
    return LR_ERROR_NOT_INITIALIZED;
  }
  DeviceState *state = open_device_state(device.index);
  if (state == nullptr || ptr == nullptr) {
    return LR_ERROR_INVALID_ARGUMENT;
  }
  auto found = state->allocations.find(ptr);
  if (found == state->allocations.end()) {
    return LR_ERROR_INVALID_ARGUMENT;
  }
  LR_TRY(drain(*state));
  LR_TRY(cu(g_driver.cuMemFree_(reinterpret_cast<CUdeviceptr>(ptr)), "cuMemFree"));
  state->stats.live_bytes -= found->second;
  state->stats.total_freed_bytes += found->second;
  ++state->stats.free_count;
  state->allocations.erase(found);
  return LR_SUCCESS;
}

LRRT_API lr_status_t lr_host_malloc(lr_device_t device, size_t size, void **ptr) {
  Lock lock(g_mutex);
  if (!g_initialized) {
    return LR_ERROR_NOT_INITIALIZED;
  }
  DeviceState *state = open_device_state(device.index);
  if (state == nullptr || ptr == nullptr || size == 0) {
    return LR_ERROR_INVALID_ARGUMENT;
  }
  LR_TRY(make_current(*state));
  void *pointer = nullptr;
  LR_TRY(cu(g_driver.cuMemHostAlloc_(&pointer, size,
                                     CU_MEMHOSTALLOC_PORTABLE |
                                         CU_MEMHOSTALLOC_DEVICEMAP),
            "cuMemHostAlloc"));
  state->host_allocations[pointer] = size;
  lr_memory_stats_t &stats = state->stats;
  stats.pinned_host_live_bytes += size;
  stats.pinned_host_peak_live_bytes =
      std::max(stats.pinned_host_peak_live_bytes, stats.pinned_host_live_bytes);
  stats.pinned_host_total_allocated_bytes += size;
  ++stats.pinned_host_allocation_count;
  *ptr = pointer;
  return LR_SUCCESS;
}

LRRT_API lr_status_t lr_host_free(lr_device_t device, void *ptr) {
  Lock lock(g_mutex);
  if (!g_initialized) {
    return LR_ERROR_NOT_INITIALIZED;
  }
  DeviceState *state = open_device_state(device.index);
  if (state == nullptr || ptr == nullptr) {
    return LR_ERROR_INVALID_ARGUMENT;
  }
  auto found = state->host_allocations.find(ptr);
  if (found == state->host_allocations.end()) {
    return LR_ERROR_INVALID_ARGUMENT;
  }
  LR_TRY(drain(*state));
  LR_TRY(cu(g_driver.cuMemFreeHost_(ptr), "cuMemFreeHost"));
  state->stats.pinned_host_live_bytes -= found->second;
  state->stats.pinned_host_total_freed_bytes += found->second;
  ++state->stats.pinned_host_free_count;
  state->host_allocations.erase(found);
  return LR_SUCCESS;
}

LRRT_API lr_status_t lr_memcpy(lr_device_t device, void *dst, const void *src,
                               size_t size, lr_memcpy_kind_t kind) {
  Lock lock(g_mutex);
  if (!g_initialized) {
    return LR_ERROR_NOT_INITIALIZED;
  }
  DeviceState *state = open_device_state(device.index);
  if (state == nullptr || dst == nullptr || src == nullptr || !valid_kind(kind)) {
    return LR_ERROR_INVALID_ARGUMENT;
  }
  if (size == 0) {
    return LR_SUCCESS;
  }
  // Synchronous in the full sense: earlier work is drained, the copy runs on
  // the device's (non-blocking) queue and has landed when this returns. A
  // plain cuMemcpy would run on the legacy stream, which the queues do not
  // wait for, and may return before a pageable host-to-device DMA or a
  // device-to-device copy has completed; queue work issued next (a decode
  // that re-arms its state from a freshly written image) could then read
  // the old bytes.
  LR_TRY(drain(*state));
  LR_TRY(cu(g_driver.cuMemcpyAsync_(reinterpret_cast<CUdeviceptr>(dst),
                                    reinterpret_cast<CUdeviceptr>(src), size, state->stream),
            "cuMemcpyAsync"));
  LR_TRY(drain(*state));
  count_copy(*state, size, kind);
  return LR_SUCCESS;
}

LRRT_API lr_status_t lr_memcpy_async(lr_device_t device, void *dst,
                                     const void *src, size_t size,
                                     lr_memcpy_kind_t kind, lr_event_t *event) {
  Lock lock(g_mutex);
  if (!g_initialized) {
    return LR_ERROR_NOT_INITIALIZED;
  }
  return async_copy(device.index, dst, src, size, kind, event, nullptr, 0, false);
}

LRRT_API lr_status_t lr_memcpy_async_with_dependencies(
    lr_device_t device, void *dst, const void *src, size_t size,
    lr_memcpy_kind_t kind, lr_event_t *event, lr_event_t *const *dependencies,
    size_t dependency_count) {
  Lock lock(g_mutex);
  if (!g_initialized) {
    return LR_ERROR_NOT_INITIALIZED;
  }
  return async_copy(device.index, dst, src, size, kind, event, dependencies,
                    dependency_count, true);
}

LRRT_API lr_status_t lr_module_load_hsaco(lr_device_t device, const void *image,
                                          size_t image_size,
                                          lr_module_t **module) {
  Lock lock(g_mutex);
  if (!g_initialized) {
    return LR_ERROR_NOT_INITIALIZED;
  }
  DeviceState *state = open_device_state(device.index);
  if (state == nullptr || image == nullptr || image_size == 0 ||
      module == nullptr) {
    return LR_ERROR_INVALID_ARGUMENT;
  }
  LR_TRY(make_current(*state));
  CUmodule handle = nullptr;
  LR_TRY(cu(g_driver.cuModuleLoadData_(&handle, image), "cuModuleLoadData"));
  lr_module_t *created = new lr_module_t{device.index, handle, {}};
  g_modules.insert(created);
  *module = created;
  return LR_SUCCESS;
}

LRRT_API lr_status_t lr_module_destroy(lr_module_t *module) {
  Lock lock(g_mutex);
  if (!g_initialized) {
    return LR_ERROR_NOT_INITIALIZED;
  }
  if (module == nullptr || g_modules.count(module) == 0) {
    return LR_ERROR_INVALID_ARGUMENT;
  }
  DeviceState *state = open_device_state(module->device);
  if (state != nullptr) {
    drain(*state);
    g_driver.cuModuleUnload_(module->module);
  }
  for (auto &kernel : module->kernels) {
    g_kernels.erase(kernel.get());
  }
  g_modules.erase(module);
  delete module;
  return LR_SUCCESS;
}

LRRT_API lr_status_t lr_kernel_get(lr_module_t *module, const char *name,
                                   lr_kernel_t **kernel) {
  Lock lock(g_mutex);
  if (!g_initialized) {
    return LR_ERROR_NOT_INITIALIZED;
  }
  if (module == nullptr || g_modules.count(module) == 0 || name == nullptr ||
      kernel == nullptr) {
    return LR_ERROR_INVALID_ARGUMENT;
  }
  for (auto &existing : module->kernels) {
    if (existing->name == name) {
      *kernel = existing.get();
      return LR_SUCCESS;
    }
  }
  DeviceState *state = open_device_state(module->device);
  if (state == nullptr) {
    return LR_ERROR_INVALID_ARGUMENT;
  }
  LR_TRY(make_current(*state));
  CUfunction function = nullptr;
  LR_TRY(cu(g_driver.cuModuleGetFunction_(&function, module->module, name),
            "cuModuleGetFunction"));
  auto created = std::make_unique<lr_kernel_t>();
  created->module = module;
  created->function = function;
  created->name = name;
  size_t end = 0;
  for (size_t index = 0;; ++index) {
    size_t offset = 0, size = 0;
    if (g_driver.cuFuncGetParamInfo_(function, index, &offset, &size) !=
        CUDA_SUCCESS) {
      break;
    }
    created->parameter_offsets.push_back(offset);
    end = std::max(end, offset + size);
  }
  created->kernarg_size = static_cast<uint32_t>(end);
  int shared = 0, local = 0;
  LR_TRY(cu(g_driver.cuFuncGetAttribute_(&shared, CU_FUNC_ATTRIBUTE_SHARED_SIZE_BYTES,
                                         function),
            "cuFuncGetAttribute"));
  LR_TRY(cu(g_driver.cuFuncGetAttribute_(&local, CU_FUNC_ATTRIBUTE_LOCAL_SIZE_BYTES,
                                         function),
            "cuFuncGetAttribute"));
  created->static_shared_bytes = static_cast<uint32_t>(shared);
  created->local_bytes = static_cast<uint32_t>(local);
  created->dynamic_shared_limit = 48u * 1024u;
  created->resident = false;
  created->overlapped = false;
  lr_kernel_t *handle = created.get();
  module->kernels.push_back(std::move(created));
  g_kernels.insert(handle);
  *kernel = handle;
  return LR_SUCCESS;
}

LRRT_API lr_status_t lr_kernel_get_properties(lr_kernel_t *kernel,
                                              lr_kernel_properties_t *properties) {
  Lock lock(g_mutex);
  if (!g_initialized) {
    return LR_ERROR_NOT_INITIALIZED;
  }
  if (kernel == nullptr || properties == nullptr || g_kernels.count(kernel) == 0) {
    return LR_ERROR_INVALID_ARGUMENT;
  }
  properties->kernarg_size = kernel->kernarg_size;
  properties->group_segment_size = kernel->static_shared_bytes;
  properties->private_segment_size = kernel->local_bytes;
  return LR_SUCCESS;
}

LRRT_API lr_status_t lr_launch(lr_kernel_t *kernel,
                               const lr_launch_config_t *config,
                               const void *args, size_t args_size) {
  Lock lock(g_mutex);
  return launch_impl(kernel, config, args, args_size, nullptr, nullptr, 0);
}

LRRT_API lr_status_t lr_launch_with_dependencies(
    lr_kernel_t *kernel, const lr_launch_config_t *config, const void *args,
    size_t args_size, lr_event_t *const *dependencies, size_t dependency_count) {
  Lock lock(g_mutex);
  if (g_initialized && dependency_count != 0 && dependencies == nullptr) {
    return LR_ERROR_INVALID_ARGUMENT;
  }
  return launch_impl(kernel, config, args, args_size, nullptr, dependencies,
                     dependency_count);
}

LRRT_API lr_status_t lr_launch_on_queue(lr_queue_t *queue, lr_kernel_t *kernel,
                                        const lr_launch_config_t *config,
                                        const void *args, size_t args_size) {
  Lock lock(g_mutex);
  if (g_initialized && queue == nullptr) {
    return LR_ERROR_INVALID_ARGUMENT;
  }
  return launch_impl(kernel, config, args, args_size, queue, nullptr, 0);
}

LRRT_API lr_status_t lr_launch_on_queue_with_dependencies(
    lr_queue_t *queue, lr_kernel_t *kernel, const lr_launch_config_t *config,
    const void *args, size_t args_size, lr_event_t *const *dependencies,
    size_t dependency_count) {
  Lock lock(g_mutex);
  if (g_initialized &&
      (queue == nullptr || (dependency_count != 0 && dependencies == nullptr))) {
    return LR_ERROR_INVALID_ARGUMENT;
  }
  return launch_impl(kernel, config, args, args_size, queue, dependencies,
                     dependency_count);
}

LRRT_API lr_status_t lr_synchronize(lr_device_t device) {
  CUcontext context = nullptr;
  {
    Lock lock(g_mutex);
    if (!g_initialized) {
      return LR_ERROR_NOT_INITIALIZED;
    }
    DeviceState *state = open_device_state(device.index);
    if (state == nullptr) {
      return LR_ERROR_INVALID_ARGUMENT;
    }
    context = state->context;
  }
  // Wait without the registry lock so other host threads keep submitting.
  CUresult result = g_driver.cuCtxSetCurrent_(context);
  if (result == CUDA_SUCCESS) {
    result = g_driver.cuCtxSynchronize_();
  }
  Lock lock(g_mutex);
  return cu(result, "cuCtxSynchronize");
}

LRRT_API lr_status_t lr_kernel_set_resident(lr_kernel_t *kernel,
                                            uint32_t resident) {
  Lock lock(g_mutex);
  if (!g_initialized) {
    return LR_ERROR_NOT_INITIALIZED;
  }
  if (kernel == nullptr || g_kernels.count(kernel) == 0) {
    return LR_ERROR_INVALID_ARGUMENT;
  }
  kernel->resident = resident != 0;
  return LR_SUCCESS;
}

LRRT_API lr_status_t lr_kernel_set_overlapped(lr_kernel_t *kernel, uint32_t overlapped) {
  Lock lock(g_mutex);
  if (!g_initialized) {
    return LR_ERROR_NOT_INITIALIZED;
  }
  if (kernel == nullptr || g_kernels.count(kernel) == 0) {
    return LR_ERROR_INVALID_ARGUMENT;
  }
  kernel->overlapped = overlapped != 0;
  return LR_SUCCESS;
}

LRRT_API lr_status_t lr_kernel_max_resident_blocks(
    lr_kernel_t *kernel, uint32_t block_threads,
    uint32_t dynamic_shared_memory_bytes, uint32_t *blocks) {
  Lock lock(g_mutex);
  if (!g_initialized) {
    return LR_ERROR_NOT_INITIALIZED;
  }
  if (kernel == nullptr || g_kernels.count(kernel) == 0 || blocks == nullptr ||
      block_threads == 0) {
    return LR_ERROR_INVALID_ARGUMENT;
  }
  DeviceState *state = open_device_state(kernel->module->device);
  if (state == nullptr) {
    return LR_ERROR_INVALID_ARGUMENT;
  }
  LR_TRY(make_current(*state));
  LR_TRY(set_dynamic_shared(kernel, dynamic_shared_memory_bytes));
  int per_sm = 0;
  LR_TRY(cu(g_driver.cuOccupancyMaxActiveBlocksPerMultiprocessor_(
                &per_sm, kernel->function, static_cast<int>(block_threads),
                dynamic_shared_memory_bytes),
            "cuOccupancyMaxActiveBlocksPerMultiprocessor"));
  *blocks = static_cast<uint32_t>(std::max(per_sm, 0)) * state->sm_count;
  return LR_SUCCESS;
}

LRRT_API lr_status_t lr_queue_native_handle(lr_device_t device, lr_queue_t *queue,
                                            void **stream) {
  Lock lock(g_mutex);
  if (!g_initialized) {
    return LR_ERROR_NOT_INITIALIZED;
  }
  DeviceState *state = open_device_state(device.index);
  if (state == nullptr || stream == nullptr) {
    return LR_ERROR_INVALID_ARGUMENT;
  }
  if (queue == nullptr) {
    *stream = state->stream;
    return LR_SUCCESS;
  }
  if (g_queues.count(queue) == 0 || queue->device != device.index) {
    return LR_ERROR_INVALID_ARGUMENT;
  }
  *stream = queue->stream;
  return LR_SUCCESS;
}

LRRT_API lr_status_t lr_last_error_detail(char *text, size_t text_size) {
  Lock lock(g_mutex);
  if (text == nullptr || text_size == 0) {
    return LR_ERROR_INVALID_ARGUMENT;
  }
  const size_t length = std::min(g_last_error.size(), text_size - 1);
  std::memcpy(text, g_last_error.data(), length);
  text[length] = '\0';
  return LR_SUCCESS;
}

} // extern "C"
