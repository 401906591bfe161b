// Device and pinned-host buffers plus copy helpers over lr_memcpy*. Names and
// argument order follow light-rocm-runtime include/lrrt/memory.hpp:10-311 so
// code written against that header (ResidentExecutor, the Qwen driver, tests)
// compiles unchanged.
#ifndef LRRT_MEMORY_HPP_
#define LRRT_MEMORY_HPP_

#include "lrrt/runtime.hpp"

#include <utility>
#include <vector>

namespace lrrt {

class PinnedHostBuffer {
public:
  PinnedHostBuffer(lr_device_t device, size_t size) : device_(device), size_(size) {
    check(lr_host_malloc(device_, size_, &ptr_), "lr_host_malloc");
  }
  PinnedHostBuffer(Device device, size_t size)
      : PinnedHostBuffer(device.get(), size) {}
  ~PinnedHostBuffer() { reset(); }
  PinnedHostBuffer(PinnedHostBuffer &&other) noexcept
      : device_(other.device_), ptr_(std::exchange(other.ptr_, nullptr)),
        size_(std::exchange(other.size_, 0)) {}
  PinnedHostBuffer &operator=(PinnedHostBuffer &&other) noexcept {
    if (this != &other) {
      reset();
      device_ = other.device_;
      ptr_ = std::exchange(other.ptr_, nullptr);
      size_ = std::exchange(other.size_, 0);
    }
    return *this;
  }
  PinnedHostBuffer(const PinnedHostBuffer &) = delete;
  PinnedHostBuffer &operator=(const PinnedHostBuffer &) = delete;

  void *data() const { return ptr_; }
  size_t size() const { return size_; }
  lr_device_t device() const { return device_; }

private:
  void reset() noexcept {
    if (ptr_ != nullptr) {
      lr_host_free(device_, ptr_);
    }
    ptr_ = nullptr;
    size_ = 0;
  }
  lr_device_t device_;
  void *ptr_ = nullptr;
  size_t size_ = 0;
};

// Owning device allocation, or a non-owning view() of memory owned elsewhere.
class DeviceBuffer {
public:
  DeviceBuffer(lr_device_t device, size_t size) : device_(device), size_(size) {
    check(lr_malloc(device_, size_, &ptr_), "lr_malloc");
  }
  DeviceBuffer(Device device, size_t size) : DeviceBuffer(device.get(), size) {}

  static DeviceBuffer view(lr_device_t device, void *ptr, size_t size) {
    DeviceBuffer buffer;
    buffer.device_ = device;
    buffer.ptr_ = ptr;
    buffer.size_ = size;
    buffer.owner_ = false;
    return buffer;
  }

  ~DeviceBuffer() { reset(); }
  DeviceBuffer(DeviceBuffer &&other) noexcept
      : device_(other.device_), ptr_(std::exchange(other.ptr_, nullptr)),
        size_(std::exchange(other.size_, 0)),
        owner_(std::exchange(other.owner_, true)) {}
  DeviceBuffer &operator=(DeviceBuffer &&other) noexcept {
    if (this != &other) {
      reset();
      device_ = other.device_;
      ptr_ = std::exchange(other.ptr_, nullptr);
      size_ = std::exchange(other.size_, 0);
      owner_ = std::exchange(other.owner_, true);
    }
    return *this;
  }
  DeviceBuffer(const DeviceBuffer &) = delete;
  DeviceBuffer &operator=(const DeviceBuffer &) = delete;

  void *data() const { return ptr_; }
  size_t size() const { return size_; }
  lr_device_t device() const { return device_; }

private:
  DeviceBuffer() : device_{0} {}
  void reset() noexcept {
    if (ptr_ != nullptr && owner_) {
      lr_free(device_, ptr_);
    }
    ptr_ = nullptr;
    size_ = 0;
    owner_ = true;
  }
  lr_device_t device_;
  void *ptr_ = nullptr;
  size_t size_ = 0;
  bool owner_ = true;
};

namespace detail {
inline void require_range(const DeviceBuffer &dst, size_t dst_offset,
                          const DeviceBuffer &src, size_t src_offset,
                          size_t size) {
  if (dst_offset > dst.size() || src_offset > src.size() ||
      size > dst.size() - dst_offset || size > src.size() - src_offset) {
    throw Error(LR_ERROR_INVALID_ARGUMENT,
                "lr_memcpy device to device offset is out of range");
  }
}
inline void *offset(const DeviceBuffer &buffer, size_t bytes) {
  return static_cast<unsigned char *>(buffer.data()) + bytes;
}
} // namespace detail

// ---- host -> device ------------------------------------------------------
inline void copy_to_device(DeviceBuffer &dst, const void *src, size_t size) {
  check(lr_memcpy(dst.device(), dst.data(), src, size, LR_MEMCPY_HOST_TO_DEVICE),
        "lr_memcpy host to device");
}
inline void copy_to_device_async(DeviceBuffer &dst, const void *src, size_t size,
                                 const Event &event) {
  check(lr_memcpy_async(dst.device(), dst.data(), src, size,
                        LR_MEMCPY_HOST_TO_DEVICE, event.get()),
        "lr_memcpy_async host to device");
}
inline void copy_to_device_async(DeviceBuffer &dst, const void *src, size_t size,
                                 const Event &event,
                                 const std::vector<const Event *> &dependencies) {
  std::vector<lr_event_t *> handles = event_handles(dependencies);
  check(lr_memcpy_async_with_dependencies(dst.device(), dst.data(), src, size,
                                          LR_MEMCPY_HOST_TO_DEVICE, event.get(),
                                          handles.data(), handles.size()),
        "lr_memcpy_async_with_dependencies host to device");
}
template <typename T, size_t N>
inline void copy_to_device(DeviceBuffer &dst, const T (&src)[N]) {
  copy_to_device(dst, src, sizeof(src));
}
template <typename T, size_t N>
inline void copy_to_device_async(DeviceBuffer &dst, const T (&src)[N],
                                 const Event &event) {
  copy_to_device_async(dst, src, sizeof(src), event);
}
template <typename T>
inline void copy_to_device(DeviceBuffer &dst, const std::vector<T> &src) {
  if (!src.empty()) {
    copy_to_device(dst, src.data(), src.size() * sizeof(T));
  }
}
template <typename T>
inline void copy_to_device_async(DeviceBuffer &dst, const std::vector<T> &src,
                                 const Event &event) {
  if (!src.empty()) {
    copy_to_device_async(dst, src.data(), src.size() * sizeof(T), event);
  }
}

// ---- device -> host ------------------------------------------------------
inline void copy_to_host(void *dst, const DeviceBuffer &src, size_t size) {
  check(lr_memcpy(src.device(), dst, src.data(), size, LR_MEMCPY_DEVICE_TO_HOST),
        "lr_memcpy device to host");
}
inline void copy_to_host_async(void *dst, const DeviceBuffer &src, size_t size,
                               const Event &event) {
  check(lr_memcpy_async(src.device(), dst, src.data(), size,
                        LR_MEMCPY_DEVICE_TO_HOST, event.get()),
        "lr_memcpy_async device to host");
}
inline void copy_to_host_async(void *dst, const DeviceBuffer &src, size_t size,
                               const Event &event,
                               const std::vector<const Event *> &dependencies) {
  std::vector<lr_event_t *> handles = event_handles(dependencies);
  check(lr_memcpy_async_with_dependencies(src.device(), dst, src.data(), size,
                                          LR_MEMCPY_DEVICE_TO_HOST, event.get(),
                                          handles.data(), handles.size()),
        "lr_memcpy_async_with_dependencies device to host");
}
template <typename T, size_t N>
inline void copy_to_host(T (&dst)[N], const DeviceBuffer &src) {
  copy_to_host(dst, src, sizeof(dst));
}
template <typename T, size_t N>
inline void copy_to_host_async(T (&dst)[N], const DeviceBuffer &src,
                               const Event &event) {
  copy_to_host_async(dst, src, sizeof(dst), event);
}
template <typename T>
inline void copy_to_host(std::vector<T> &dst, const DeviceBuffer &src) {
  if (!dst.empty()) {
    copy_to_host(dst.data(), src, dst.size() * sizeof(T));
  }
}
template <typename T>
inline void copy_to_host_async(std::vector<T> &dst, const DeviceBuffer &src,
                               const Event &event) {
  if (!dst.empty()) {
    copy_to_host_async(dst.data(), src, dst.size() * sizeof(T), event);
  }
}

// ---- device -> device ----------------------------------------------------
inline void copy_device_to_device(DeviceBuffer &dst, const DeviceBuffer &src,
                                  size_t size) {
  check(lr_memcpy(dst.device(), dst.data(), src.data(), size,
                  LR_MEMCPY_DEVICE_TO_DEVICE),
        "lr_memcpy device to device");
}
inline void copy_device_to_device(DeviceBuffer &dst, size_t dst_offset,
                                  const DeviceBuffer &src, size_t src_offset,
                                  size_t size) {
  detail::require_range(dst, dst_offset, src, src_offset, size);
  check(lr_memcpy(dst.device(), detail::offset(dst, dst_offset),
                  detail::offset(src, src_offset), size,
                  LR_MEMCPY_DEVICE_TO_DEVICE),
        "lr_memcpy device to device");
}
inline void copy_device_to_device_async(DeviceBuffer &dst, const DeviceBuffer &src,
                                        size_t size, const Event &event) {
  check(lr_memcpy_async(dst.device(), dst.data(), src.data(), size,
                        LR_MEMCPY_DEVICE_TO_DEVICE, event.get()),
        "lr_memcpy_async device to device");
}
inline void copy_device_to_device_async(DeviceBuffer &dst, size_t dst_offset,
                                        const DeviceBuffer &src,
                                        size_t src_offset, size_t size,
                                        const Event &event) {
  detail::require_range(dst, dst_offset, src, src_offset, size);
  check(lr_memcpy_async(dst.device(), detail::offset(dst, dst_offset),
                        detail::offset(src, src_offset), size,
                        LR_MEMCPY_DEVICE_TO_DEVICE, event.get()),
        "lr_memcpy_async device to device");
}
inline void
copy_device_to_device_async(DeviceBuffer &dst, const DeviceBuffer &src,
                            size_t size, const Event &event,
                            const std::vector<const Event *> &dependencies) {
  std::vector<lr_event_t *> handles = event_handles(dependencies);
  check(lr_memcpy_async_with_dependencies(
            dst.device(), dst.data(), src.data(), size,
            LR_MEMCPY_DEVICE_TO_DEVICE, event.get(), handles.data(),
            handles.size()),
        "lr_memcpy_async_with_dependencies device to device");
}
inline void
copy_device_to_device_async(DeviceBuffer &dst, size_t dst_offset,
                            const DeviceBuffer &src, size_t src_offset,
                            size_t size, const Event &event,
                            const std::vector<const Event *> &dependencies) {
  detail::require_range(dst, dst_offset, src, src_offset, size);
  std::vector<lr_event_t *> handles = event_handles(dependencies);
  check(lr_memcpy_async_with_dependencies(
            dst.device(), detail::offset(dst, dst_offset),
            detail::offset(src, src_offset), size, LR_MEMCPY_DEVICE_TO_DEVICE,
            event.get(), handles.data(), handles.size()),
        "lr_memcpy_async_with_dependencies device to device");
}

} // namespace lrrt

#endif // LRRT_MEMORY_HPP_
