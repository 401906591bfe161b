/*
 * lrrt C ABI, B200 (sm_100a) implementation.
 *
 * The entry points, status codes and structs below keep the names, argument
 * meaning and error behaviour of light-rocm-runtime's C ABI
 * (include/lrrt/lrrt.h:17-232 in that project) so that callers of that ABI
 * recompile against this header unchanged. The implementation lives in
 * light-rocm-runtime_b200/csrc/runtime/ and drives the CUDA driver API, which
 * it loads lazily: on a machine without an NVIDIA driver lr_init() succeeds and
 * lr_device_count() reports zero devices.
 *
 * Conventions kept from the reference ABI:
 *  - lr_launch_config_t.grid counts WORK-ITEMS (threads) per dimension, not
 *    blocks; the CUDA grid is ceil(grid / block) per dimension.
 *  - lr_module_load_hsaco() accepts the device code image; on B200 that image
 *    is a cubin or fatbin built for sm_100a (the name is kept for the ABI).
 *  - Launch arguments are a packed kernarg blob no larger than the kernel's
 *    parameter block (lr_kernel_properties_t.kernarg_size).
 *  - Launches are asynchronous; device errors surface at lr_synchronize() or
 *    at a later call that waits for pending work.
 *
 * B200 additions are grouped at the end of this header.
 */
#ifndef LRRT_LRRT_H_
#define LRRT_LRRT_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define LRRT_API __attribute__((visibility("default")))

typedef enum lr_status_t {
  LR_SUCCESS = 0,
  LR_ERROR_INVALID_ARGUMENT = 1,
  LR_ERROR_NOT_INITIALIZED = 2,
  LR_ERROR_ALREADY_INITIALIZED = 3,
  LR_ERROR_NOT_SUPPORTED = 4,
  LR_ERROR_RUNTIME = 5,
  LR_ERROR_DEVICE_FAULT = 6
} lr_status_t;

typedef enum lr_memcpy_kind_t {
  LR_MEMCPY_HOST_TO_DEVICE = 0,
  LR_MEMCPY_DEVICE_TO_HOST = 1,
  LR_MEMCPY_DEVICE_TO_DEVICE = 2
} lr_memcpy_kind_t;

typedef struct lr_device_t {
  uint32_t index;
} lr_device_t;

typedef struct lr_event_t lr_event_t;
typedef struct lr_queue_t lr_queue_t;
typedef struct lr_module_t lr_module_t;
typedef struct lr_kernel_t lr_kernel_t;

typedef struct lr_dim3_t {
  uint32_t x;
  uint32_t y;
  uint32_t z;
} lr_dim3_t;

typedef struct lr_launch_config_t {
  lr_dim3_t grid;  /* total threads per dimension */
  lr_dim3_t block; /* threads per block */
  uint32_t shared_memory_bytes; /* dynamic shared memory per block */
} lr_launch_config_t;

typedef struct lr_memory_stats_t {
  uint64_t live_bytes;
  uint64_t peak_live_bytes;
  uint64_t total_allocated_bytes;
  uint64_t total_freed_bytes;
  uint64_t allocation_count;
  uint64_t free_count;
  uint64_t h2d_copy_bytes;
  uint64_t d2h_copy_bytes;
  uint64_t d2d_copy_bytes;
  uint64_t memcpy_count;
  uint64_t pinned_host_live_bytes;
  uint64_t pinned_host_peak_live_bytes;
  uint64_t pinned_host_total_allocated_bytes;
  uint64_t pinned_host_total_freed_bytes;
  uint64_t pinned_host_allocation_count;
  uint64_t pinned_host_free_count;
} lr_memory_stats_t;

/*
 * On B200: compute_unit_count = SMs (148), wavefront_size = 32,
 * maximum_waves_per_compute_unit = resident warps per SM,
 * maximum_workgroup_size = 1024, group_segment_size = opt-in shared memory per
 * block, shader_engine_count = 1 (cooperative launch guarantees co-residency of
 * a resident grid, so the whole GPU counts as one engine for admission).
 */
typedef struct lr_device_properties_t {
  uint32_t compute_unit_count;
  uint32_t wavefront_size;
  uint32_t maximum_waves_per_compute_unit;
  uint32_t maximum_workgroup_size;
  uint64_t group_segment_size;
  uint32_t shader_engine_count;
} lr_device_properties_t;

/* kernarg_size = parameter block bytes; group_segment_size = static shared
 * memory; private_segment_size = local memory per thread. */
typedef struct lr_kernel_properties_t {
  uint32_t kernarg_size;
  uint32_t group_segment_size;
  uint32_t private_segment_size;
} lr_kernel_properties_t;

LRRT_API const char *lr_status_string(lr_status_t status);

LRRT_API lr_status_t lr_init(void);

/* Drains every opened device, then releases all runtime resources. */
LRRT_API lr_status_t lr_shutdown(void);

LRRT_API lr_status_t lr_device_count(uint32_t *count);
LRRT_API lr_status_t lr_device_open(uint32_t index, lr_device_t *device);
LRRT_API lr_status_t lr_device_name(lr_device_t device, char *name,
                                    size_t name_size);
LRRT_API lr_status_t lr_device_get_properties(
    lr_device_t device, lr_device_properties_t *properties);
LRRT_API lr_status_t lr_get_memory_stats(lr_device_t device,
                                         lr_memory_stats_t *stats);
LRRT_API lr_status_t lr_reset_memory_stats(lr_device_t device);

LRRT_API lr_status_t lr_queue_create(lr_device_t device, lr_queue_t **queue);
/* Drains the queue, then releases it. */
LRRT_API lr_status_t lr_queue_destroy(lr_queue_t *queue);
LRRT_API lr_status_t lr_queue_synchronize(lr_queue_t *queue);

LRRT_API lr_status_t lr_event_create(lr_device_t device, lr_event_t **event);
/* Waits for a pending event, then releases the handle. */
LRRT_API lr_status_t lr_event_destroy(lr_event_t *event);
/* Marker after all work previously submitted to the device's default queue. A
 * pending event is waited for before it is recorded again. */
LRRT_API lr_status_t lr_event_record(lr_event_t *event);
LRRT_API lr_status_t lr_event_record_on_queue(lr_event_t *event,
                                              lr_queue_t *queue);
/* Succeeds immediately for an event that was never recorded. */
LRRT_API lr_status_t lr_event_synchronize(lr_event_t *event);
LRRT_API lr_status_t lr_event_elapsed_time_ns(const lr_event_t *start,
                                              const lr_event_t *end,
                                              uint64_t *elapsed_ns);
/* Device duration of the operation an event completed: the copy for an
 * asynchronous copy, zero-length for a plain marker. */
LRRT_API lr_status_t lr_event_duration_ns(const lr_event_t *event,
                                          uint64_t *duration_ns);

LRRT_API lr_status_t lr_malloc(lr_device_t device, size_t size, void **ptr);
/* Drains the device before releasing ptr. */
LRRT_API lr_status_t lr_free(lr_device_t device, void *ptr);

/* Page-locked, device-mapped host memory tied to device. */
LRRT_API lr_status_t lr_host_malloc(lr_device_t device, size_t size,
                                    void **ptr);
/* Drains the device; ptr must be the base pointer from lr_host_malloc. */
LRRT_API lr_status_t lr_host_free(lr_device_t device, void *ptr);

/* Synchronous: drains the device, then copies. */
LRRT_API lr_status_t lr_memcpy(lr_device_t device, void *dst, const void *src,
                               size_t size, lr_memcpy_kind_t kind);

/* Asynchronous copy on the device's default queue, ordered after earlier
 * launches and copies there; completion is recorded in event. */
LRRT_API lr_status_t lr_memcpy_async(lr_device_t device, void *dst,
                                     const void *src, size_t size,
                                     lr_memcpy_kind_t kind, lr_event_t *event);

/* Asynchronous copy that starts after the listed events. dependencies may be
 * NULL when dependency_count is zero. */
LRRT_API lr_status_t lr_memcpy_async_with_dependencies(
    lr_device_t device, void *dst, const void *src, size_t size,
    lr_memcpy_kind_t kind, lr_event_t *event, lr_event_t *const *dependencies,
    size_t dependency_count);

/* image: a cubin or fatbin for sm_100a. */
LRRT_API lr_status_t lr_module_load_hsaco(lr_device_t device, const void *image,
                                          size_t image_size,
                                          lr_module_t **module);
/* Drains the module's device, then unloads it and its kernels. */
LRRT_API lr_status_t lr_module_destroy(lr_module_t *module);

LRRT_API lr_status_t lr_kernel_get(lr_module_t *module, const char *name,
                                   lr_kernel_t **kernel);
LRRT_API lr_status_t lr_kernel_get_properties(
    lr_kernel_t *kernel, lr_kernel_properties_t *properties);

/* Enqueues a launch on the device's default queue; returns once submitted. */
LRRT_API lr_status_t lr_launch(lr_kernel_t *kernel,
                               const lr_launch_config_t *config,
                               const void *args, size_t args_size);

/* Launch that also waits for the listed events. */
LRRT_API lr_status_t lr_launch_with_dependencies(
    lr_kernel_t *kernel, const lr_launch_config_t *config, const void *args,
    size_t args_size, lr_event_t *const *dependencies, size_t dependency_count);

LRRT_API lr_status_t lr_launch_on_queue(lr_queue_t *queue, lr_kernel_t *kernel,
                                        const lr_launch_config_t *config,
                                        const void *args, size_t args_size);

LRRT_API lr_status_t lr_launch_on_queue_with_dependencies(
    lr_queue_t *queue, lr_kernel_t *kernel, const lr_launch_config_t *config,
    const void *args, size_t args_size, lr_event_t *const *dependencies,
    size_t dependency_count);

/* Waits for all work enqueued on the device, on every queue. */
LRRT_API lr_status_t lr_synchronize(lr_device_t device);

/* ------------------------------------------------------------------------ *
 * B200 additions (no counterpart in the reference ABI).                     *
 * ------------------------------------------------------------------------ */

/*
 * Marks a kernel as a resident (persistent) kernel: its launches become
 * cooperative launches, so the driver either makes every block co-resident or
 * fails the launch with LR_ERROR_INVALID_ARGUMENT instead of letting a software
 * grid barrier wait on a block that was never scheduled. The reference runtime
 * has no cooperative dispatch and admits workers conservatively instead.
 */
LRRT_API lr_status_t lr_kernel_set_resident(lr_kernel_t *kernel,
                                            uint32_t resident);

/*
 * Marks a kernel for overlapped (programmatic dependent) launches: each launch
 * carries CUDA's programmatic stream serialization, so the kernel may begin
 * while the previous kernel on the same queue is finishing. The kernel must
 * execute `griddepcontrol.wait` before it reads anything an earlier launch
 * wrote (and may execute `griddepcontrol.launch_dependents` to let the next
 * overlapped launch begin). Unmarked kernels launch in plain stream order.
 */
LRRT_API lr_status_t lr_kernel_set_overlapped(lr_kernel_t *kernel, uint32_t overlapped);

/*
 * Maximum number of blocks of `kernel` with `block_threads` threads and
 * `dynamic_shared_memory_bytes` of dynamic shared memory that can be resident
 * on the device at once (SMs x blocks per SM).
 */
LRRT_API lr_status_t lr_kernel_max_resident_blocks(
    lr_kernel_t *kernel, uint32_t block_threads,
    uint32_t dynamic_shared_memory_bytes, uint32_t *blocks);

/* Raw CUDA stream behind a queue (NULL queue = the device's default queue),
 * for interop with other CUDA code on the same device. */
LRRT_API lr_status_t lr_queue_native_handle(lr_device_t device,
                                            lr_queue_t *queue, void **stream);

/* Copies a human-readable description of the most recent driver failure seen
 * by any lr_* call of this process (empty when there was none). */
LRRT_API lr_status_t lr_last_error_detail(char *text, size_t text_size);

#ifdef __cplusplus
}
#endif

#endif // LRRT_LRRT_H_
