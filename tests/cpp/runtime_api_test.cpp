// lr_* status contract, following light-rocm-runtime tests/runtime_api.cpp
// :15-487: every entry point reports LR_ERROR_NOT_INITIALIZED before lr_init,
// double init is LR_ERROR_ALREADY_INITIALIZED, null and stale handles are
// LR_ERROR_INVALID_ARGUMENT. With no GPU (no driver) the device checks are
// skipped after lr_device_count reports zero, as in the reference.
#include "lrrt/lrrt.h"

#include <cstdio>
#include <cstring>

static int failures = 0;

static void expect(lr_status_t actual, lr_status_t wanted, const char *what) {
  if (actual != wanted) {
    std::fprintf(stderr, "FAILED: %s returned %s, expected %s\n", what,
                 lr_status_string(actual), lr_status_string(wanted));
    ++failures;
  }
}

static void before_init() {
  uint32_t count = 0;
  lr_device_t device{0};
  lr_device_properties_t properties{};
  lr_memory_stats_t stats{};
  char name[64] = {};
  auto *queue = reinterpret_cast<lr_queue_t *>(1);
  auto *event = reinterpret_cast<lr_event_t *>(1);
  lr_event_t *dependencies[1] = {event};
  auto *module = reinterpret_cast<lr_module_t *>(1);
  auto *kernel = reinterpret_cast<lr_kernel_t *>(1);
  const lr_launch_config_t config{{1, 1, 1}, {1, 1, 1}, 0};
  int args = 0;
  void *pointer = reinterpret_cast<void *>(1);
  uint64_t value = 0;
  const lr_status_t n = LR_ERROR_NOT_INITIALIZED;
  expect(lr_device_count(&count), n, "lr_device_count");
  expect(lr_device_open(0, &device), n, "lr_device_open");
  expect(lr_device_name(device, name, sizeof(name)), n, "lr_device_name");
  expect(lr_device_get_properties(device, &properties), n, "lr_device_get_properties");
  expect(lr_get_memory_stats(device, &stats), n, "lr_get_memory_stats");
  expect(lr_reset_memory_stats(device), n, "lr_reset_memory_stats");
  expect(lr_queue_create(device, &queue), n, "lr_queue_create");
  expect(lr_queue_synchronize(queue), n, "lr_queue_synchronize");
  expect(lr_queue_destroy(queue), n, "lr_queue_destroy");
  expect(lr_event_create(device, &event), n, "lr_event_create");
  expect(lr_event_record(event), n, "lr_event_record");
  expect(lr_event_record_on_queue(event, queue), n, "lr_event_record_on_queue");
  expect(lr_event_synchronize(event), n, "lr_event_synchronize");
  expect(lr_event_elapsed_time_ns(event, event, &value), n, "lr_event_elapsed_time_ns");
  expect(lr_event_duration_ns(event, &value), n, "lr_event_duration_ns");
  expect(lr_event_destroy(event), n, "lr_event_destroy");
  expect(lr_malloc(device, sizeof(args), &pointer), n, "lr_malloc");
  expect(lr_free(device, pointer), n, "lr_free");
  expect(lr_host_malloc(device, sizeof(args), &pointer), n, "lr_host_malloc");
  expect(lr_host_free(device, pointer), n, "lr_host_free");
  expect(lr_memcpy(device, pointer, &args, sizeof(args), LR_MEMCPY_HOST_TO_DEVICE), n,
         "lr_memcpy");
  expect(lr_memcpy_async(device, pointer, &args, sizeof(args), LR_MEMCPY_HOST_TO_DEVICE,
                         event),
         n, "lr_memcpy_async");
  expect(lr_memcpy_async_with_dependencies(device, pointer, &args, sizeof(args),
                                           LR_MEMCPY_HOST_TO_DEVICE, event, dependencies, 1),
         n, "lr_memcpy_async_with_dependencies");
  expect(lr_module_load_hsaco(device, &args, sizeof(args), &module), n,
         "lr_module_load_hsaco");
  expect(lr_module_destroy(module), n, "lr_module_destroy");
  expect(lr_kernel_get(module, "kernel", &kernel), n, "lr_kernel_get");
  expect(lr_launch(kernel, &config, &args, sizeof(args)), n, "lr_launch");
  expect(lr_launch_with_dependencies(kernel, &config, &args, sizeof(args), dependencies, 1),
         n, "lr_launch_with_dependencies");
  expect(lr_launch_on_queue(queue, kernel, &config, &args, sizeof(args)), n,
         "lr_launch_on_queue");
  expect(lr_launch_on_queue_with_dependencies(queue, kernel, &config, &args, sizeof(args),
                                              dependencies, 1),
         n, "lr_launch_on_queue_with_dependencies");
  expect(lr_synchronize(device), n, "lr_synchronize");
  expect(lr_shutdown(), n, "lr_shutdown");
}

static void with_devices(uint32_t count) {
  const lr_status_t bad = LR_ERROR_INVALID_ARGUMENT;
  lr_device_t invalid{count};
  lr_memory_stats_t stats{};
  expect(lr_get_memory_stats(invalid, &stats), bad, "stats of invalid device");
  lr_device_t device{0};
  lr_queue_t *queue = nullptr;
  lr_event_t *event = nullptr;
  expect(lr_queue_create(device, &queue), bad, "queue before open");
  expect(lr_event_create(device, &event), bad, "event before open");
  expect(lr_synchronize(device), bad, "synchronize before open");
  if (queue != nullptr || event != nullptr) {
    std::fprintf(stderr, "FAILED: handle written on error\n");
    ++failures;
  }
  expect(lr_device_open(0, &device), LR_SUCCESS, "lr_device_open");
  expect(lr_device_open(count, &device), bad, "open out of range");
  char tiny[1] = {};
  expect(lr_device_name(device, tiny, sizeof(tiny)), bad, "name buffer too small");
  lr_device_properties_t p{};
  expect(lr_device_get_properties(device, &p), LR_SUCCESS, "properties");
  if (p.compute_unit_count == 0 || p.wavefront_size == 0 ||
      p.maximum_waves_per_compute_unit == 0 || p.maximum_workgroup_size == 0 ||
      p.group_segment_size == 0 || p.shader_engine_count == 0 ||
      p.shader_engine_count > p.compute_unit_count ||
      p.compute_unit_count % p.shader_engine_count != 0) {
    std::fprintf(stderr, "FAILED: incomplete device properties\n");
    ++failures;
  }
  expect(lr_device_get_properties(device, nullptr), bad, "properties null");
  expect(lr_device_get_properties(invalid, &p), bad, "properties invalid device");
  expect(lr_get_memory_stats(device, nullptr), bad, "stats null");
  expect(lr_reset_memory_stats(invalid), bad, "reset invalid device");
  expect(lr_queue_create(device, nullptr), bad, "queue null");
  expect(lr_queue_synchronize(nullptr), bad, "queue sync null");
  expect(lr_queue_destroy(nullptr), bad, "queue destroy null");
  expect(lr_queue_create(device, &queue), LR_SUCCESS, "queue create");
  expect(lr_queue_destroy(queue), LR_SUCCESS, "queue destroy");
  expect(lr_queue_synchronize(queue), bad, "stale queue sync");
  expect(lr_queue_destroy(queue), bad, "stale queue destroy");
  expect(lr_event_create(device, nullptr), bad, "event null");
  expect(lr_event_synchronize(nullptr), bad, "event sync null");
  expect(lr_event_destroy(nullptr), bad, "event destroy null");
  expect(lr_event_create(device, &event), LR_SUCCESS, "event create");
  expect(lr_event_synchronize(event), LR_SUCCESS, "unrecorded event sync");
  uint64_t value = 1;
  expect(lr_event_elapsed_time_ns(event, event, &value), bad, "unrecorded elapsed");
  expect(lr_event_duration_ns(event, &value), bad, "unrecorded duration");
  expect(lr_event_destroy(event), LR_SUCCESS, "event destroy");
  expect(lr_event_synchronize(event), bad, "stale event sync");
  expect(lr_event_record(event), bad, "stale event record");
  expect(lr_event_destroy(event), bad, "stale event destroy");
  lr_event_t *null_dependency[1] = {nullptr};
  expect(lr_memcpy_async_with_dependencies(device, &stats, &stats, sizeof(stats),
                                           LR_MEMCPY_DEVICE_TO_DEVICE, event,
                                           null_dependency, 1),
         bad, "async copy null dependency");
  expect(lr_synchronize(invalid), bad, "synchronize invalid device");
  // Round trip through device memory, then launch validation failures.
  void *buffer = nullptr;
  expect(lr_malloc(device, 64, &buffer), LR_SUCCESS, "lr_malloc");
  const char text[16] = "lrrt on sm_100a";
  char back[16] = {};
  expect(lr_memcpy(device, buffer, text, sizeof(text), LR_MEMCPY_HOST_TO_DEVICE),
         LR_SUCCESS, "h2d");
  expect(lr_memcpy(device, back, buffer, sizeof(back), LR_MEMCPY_DEVICE_TO_HOST),
         LR_SUCCESS, "d2h");
  if (std::memcmp(text, back, sizeof(text)) != 0) {
    std::fprintf(stderr, "FAILED: device round trip\n");
    ++failures;
  }
  expect(lr_free(device, buffer), LR_SUCCESS, "lr_free");
  expect(lr_free(device, buffer), bad, "double free");
}

int main() {
  before_init();
  expect(lr_init(), LR_SUCCESS, "lr_init");
  expect(lr_init(), LR_ERROR_ALREADY_INITIALIZED, "double lr_init");
  expect(lr_device_count(nullptr), LR_ERROR_INVALID_ARGUMENT, "count null");
  uint32_t count = 123;
  expect(lr_device_count(&count), LR_SUCCESS, "lr_device_count");
  expect(lr_device_open(0, nullptr), LR_ERROR_INVALID_ARGUMENT, "open null");
  if (count == 0) {
    std::printf("runtime api: no GPU devices, device checks skipped\n");
  } else {
    with_devices(count);
  }
  expect(lr_shutdown(), LR_SUCCESS, "lr_shutdown");
  expect(lr_device_count(&count), LR_ERROR_NOT_INITIALIZED, "count after shutdown");
  if (failures == 0) {
    std::printf("runtime api: ok\n");
  }
  return failures == 0 ? 0 : 1;
}
