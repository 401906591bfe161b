// RAII C++ layer over the lr_* runtime calls: Runtime, Device, Queue, Event.
// Names and semantics follow light-rocm-runtime include/lrrt/runtime.hpp:15-185
// (move-only handles, exceptions via lrrt::check).
#ifndef LRRT_RUNTIME_HPP_
#define LRRT_RUNTIME_HPP_

#include "lrrt/error.hpp"

#include <stdint.h>
#include <string>
#include <utility>
#include <vector>

namespace lrrt {

using MemoryStats = lr_memory_stats_t;
using DeviceProperties = lr_device_properties_t;

class Device {
public:
  explicit Device(lr_device_t device) : device_(device) {}
  lr_device_t get() const { return device_; }
  uint32_t index() const { return device_.index; }
  std::string name() const {
    char text[128] = {};
    check(lr_device_name(device_, text, sizeof(text)), "lr_device_name");
    return std::string(text);
  }
  DeviceProperties properties() const {
    DeviceProperties value{};
    check(lr_device_get_properties(device_, &value), "lr_device_get_properties");
    return value;
  }
  void synchronize() const { check(lr_synchronize(device_), "lr_synchronize"); }
  MemoryStats memory_stats() const {
    MemoryStats value{};
    check(lr_get_memory_stats(device_, &value), "lr_get_memory_stats");
    return value;
  }
  void reset_memory_stats() const {
    check(lr_reset_memory_stats(device_), "lr_reset_memory_stats");
  }

private:
  lr_device_t device_;
};

inline void synchronize(Device device) {
  check(lr_synchronize(device.get()), "lr_synchronize");
}

// Move-only owner of one lr_* handle type; Destroy releases it.
template <typename Handle, lr_status_t (*Destroy)(Handle *)>
class OwnedHandle {
public:
  OwnedHandle() = default;
  explicit OwnedHandle(Handle *handle) : handle_(handle) {}
  ~OwnedHandle() { reset(); }
  OwnedHandle(OwnedHandle &&other) noexcept
      : handle_(std::exchange(other.handle_, nullptr)) {}
  OwnedHandle &operator=(OwnedHandle &&other) noexcept {
    if (this != &other) {
      reset();
      handle_ = std::exchange(other.handle_, nullptr);
    }
    return *this;
  }
  OwnedHandle(const OwnedHandle &) = delete;
  OwnedHandle &operator=(const OwnedHandle &) = delete;
  Handle *get() const { return handle_; }

protected:
  Handle **out() { return &handle_; }

private:
  void reset() noexcept {
    if (handle_ != nullptr) {
      Destroy(handle_);
      handle_ = nullptr;
    }
  }
  Handle *handle_ = nullptr;
};

class Queue : public OwnedHandle<lr_queue_t, lr_queue_destroy> {
public:
  explicit Queue(lr_device_t device) {
    check(lr_queue_create(device, out()), "lr_queue_create");
  }
  explicit Queue(Device device) : Queue(device.get()) {}
  void synchronize() const {
    check(lr_queue_synchronize(get()), "lr_queue_synchronize");
  }
};

class Event : public OwnedHandle<lr_event_t, lr_event_destroy> {
public:
  explicit Event(lr_device_t device) {
    check(lr_event_create(device, out()), "lr_event_create");
  }
  explicit Event(Device device) : Event(device.get()) {}
  void record() const { check(lr_event_record(get()), "lr_event_record"); }
  void record(const Queue &queue) const {
    check(lr_event_record_on_queue(get(), queue.get()),
          "lr_event_record_on_queue");
  }
  void synchronize() const {
    check(lr_event_synchronize(get()), "lr_event_synchronize");
  }
};

inline std::vector<lr_event_t *>
event_handles(const std::vector<const Event *> &dependencies) {
  std::vector<lr_event_t *> handles;
  handles.reserve(dependencies.size());
  for (const Event *event : dependencies) {
    handles.push_back(event != nullptr ? event->get() : nullptr);
  }
  return handles;
}

inline uint64_t elapsed_time_ns(const Event &start, const Event &end) {
  uint64_t value = 0;
  check(lr_event_elapsed_time_ns(start.get(), end.get(), &value),
        "lr_event_elapsed_time_ns");
  return value;
}

inline uint64_t duration_ns(const Event &event) {
  uint64_t value = 0;
  check(lr_event_duration_ns(event.get(), &value), "lr_event_duration_ns");
  return value;
}

class Runtime {
public:
  Runtime() { check(lr_init(), "lr_init"); }
  ~Runtime() { lr_shutdown(); }
  Runtime(const Runtime &) = delete;
  Runtime &operator=(const Runtime &) = delete;
  uint32_t device_count() const {
    uint32_t count = 0;
    check(lr_device_count(&count), "lr_device_count");
    return count;
  }
  Device open_device(uint32_t index) const {
    lr_device_t device{0};
    check(lr_device_open(index, &device), "lr_device_open");
    return Device(device);
  }
};

} // namespace lrrt

#endif // LRRT_RUNTIME_HPP_
