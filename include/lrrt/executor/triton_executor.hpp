// Generic per-operation bundle executor for sm_100a: named lrrt::Bundle
// kernels, named device buffers (optionally packed into one arena
// allocation) and a launch helper that binds kernel arguments by name.
//
// The public surface (namespace, class and function names, signatures and
// the text of every error) is that of light-rocm-runtime
// executor/triton/triton_executor.hpp:21-312, so executors written against
// that header compile and report errors unchanged; the bundles' code objects
// are sm_100a cubins and queues are CUDA streams. The implementation is this
// file's own: each set is one ordered table of named records (so listings are
// sorted without copying), a buffer record owns either its allocation or a
// view into the arena, and the arena layout is computed in one pass at
// finalize().
#ifndef LRRT_EXECUTOR_TRITON_EXECUTOR_HPP_
#define LRRT_EXECUTOR_TRITON_EXECUTOR_HPP_

#include "lrrt/bundle.hpp"
#include "lrrt/lrrt.hpp"

#include <cstddef>
#include <cstdint>
#include <cstring>
#include <initializer_list>
#include <limits>
#include <map>
#include <memory>
#include <set>
#include <stdexcept>
#include <string>
#include <vector>

namespace lrrt::executor::triton {

namespace detail {

// The keys of an ordered table as "a, b, c", or "<none>" for an empty one.
template <typename Table> std::string listing(const Table &table) {
  std::string text;
  for (const auto &[name, unused] : table) {
    (void)unused;
    text.append(text.empty() ? "" : ", ").append(name);
  }
  return text.empty() ? std::string("<none>") : text;
}

inline std::string kernel_label(const lrrt::KernelManifest &manifest) {
  return manifest.name + " (" + manifest.symbol + ")";
}

// a * b, or throws std::overflow_error(message) when it does not fit size_t.
inline size_t checked_product(size_t a, size_t b, const std::string &message) {
  if (b != 0 && a > std::numeric_limits<size_t>::max() / b) {
    throw std::overflow_error(message);
  }
  return a * b;
}

} // namespace detail

// Kernels by name; each entry is one kernel of a bundle manifest.
class BundleSet {
public:
  explicit BundleSet(lrrt::Device device) : device_(device) {}

  void add(const std::string &name, const char *manifest_path, const std::string &kernel_name) {
    std::unique_ptr<lrrt::Bundle> bundle;
    try {
      bundle = std::make_unique<lrrt::Bundle>(device_, manifest_path, kernel_name.c_str());
    } catch (const std::exception &error) {
      throw std::runtime_error("failed to load Triton executor bundle '" + name +
                               "' from manifest '" +
                               (manifest_path != nullptr ? manifest_path : "<null>") +
                               "' for kernel '" + kernel_name + "': " + error.what());
    }
    table_[name] = std::move(bundle);
  }

  lrrt::Bundle &get(const std::string &name) const {
    if (auto hit = table_.find(name); hit != table_.end()) {
      return *hit->second;
    }
    throw std::runtime_error("unknown Triton executor bundle '" + name +
                             "'; available bundles: " + detail::listing(table_));
  }

private:
  lrrt::Device device_;
  std::map<std::string, std::unique_ptr<lrrt::Bundle>> table_;
};

// Device buffers by name. Without an arena every allocate_*() call allocates
// at once and the set is usable immediately. With an arena, allocate_*()
// only records a name and a size; finalize() places the recorded buffers, in
// the order they were first recorded, at 256-byte aligned offsets of one
// allocation, so that a whole input set can be staged in a host image (pack)
// and uploaded with one copy.
class BufferSet {
public:
  explicit BufferSet(lrrt::Device device, bool arena = false)
      : device_(device), arena_(arena), open_(arena) {}

  void allocate_bytes(const std::string &name, size_t bytes) {
    if (arena_) {
      if (!open_) {
        throw std::runtime_error("Triton executor arena buffer set is finalized");
      }
      auto [entry, added] = table_.try_emplace(name);
      if (added) {
        entry->second.order = recorded_++;
      }
      entry->second.bytes = bytes;
      return;
    }
    try {
      Record &record = table_[name];
      record.bytes = bytes;
      record.storage = std::make_unique<lrrt::DeviceBuffer>(device_, bytes);
    } catch (const std::exception &error) {
      table_.erase(name);
      throw std::runtime_error("failed to allocate Triton executor buffer '" + name + "' (" +
                               std::to_string(bytes) + " bytes): " + error.what());
    }
  }

  template <typename T> void allocate(const std::string &name, size_t count) {
    allocate_bytes(name, detail::checked_product(
                             count, sizeof(T),
                             "Triton executor buffer allocation overflows size_t for buffer '" +
                                 name + "'"));
  }

  // Lays out and allocates the arena (no effect without one, or twice).
  void finalize() {
    if (!open_) {
      return;
    }
    std::vector<Record *> placement(table_.size());
    for (auto &[name, record] : table_) {
      (void)name;
      placement[record.order] = &record;
    }
    size_t cursor = 0;
    for (Record *record : placement) {
      record->offset = round_up(cursor);
      if (record->bytes > std::numeric_limits<size_t>::max() - record->offset) {
        throw std::overflow_error("Triton executor arena allocation overflows size_t");
      }
      cursor = record->offset + record->bytes;
    }
    backing_ = std::make_unique<lrrt::DeviceBuffer>(device_, cursor);
    auto *base = static_cast<unsigned char *>(backing_->data());
    for (auto &[name, record] : table_) {
      (void)name;
      record.storage = std::make_unique<lrrt::DeviceBuffer>(
          lrrt::DeviceBuffer::view(device_.get(), base + record.offset, record.bytes));
    }
    arena_bytes_ = cursor;
    open_ = false;
  }

  lrrt::DeviceBuffer &get(const std::string &name) const { return *find(name).storage; }

  template <typename T> T *ptr(const std::string &name, size_t element_offset = 0) const {
    lrrt::DeviceBuffer &buffer = get(name);
    const size_t at = detail::checked_product(
        element_offset, sizeof(T),
        "Triton executor buffer offset overflows size_t for buffer '" + name + "'");
    if (at > buffer.size()) {
      throw std::out_of_range("Triton executor buffer offset is out of range for '" + name +
                              "': element_offset=" + std::to_string(element_offset) +
                              ", element_size=" + std::to_string(sizeof(T)) +
                              ", byte_offset=" + std::to_string(at) +
                              ", buffer_size=" + std::to_string(buffer.size()));
    }
    return reinterpret_cast<T *>(static_cast<unsigned char *>(buffer.data()) + at);
  }

  template <typename T> void copy_to(const std::string &name, const std::vector<T> &src) const {
    lrrt::copy_to_device(get(name), src);
  }

  template <typename T> void copy_from(std::vector<T> &dst, const std::string &name) const {
    lrrt::copy_to_host(dst, get(name));
  }

  bool uses_arena() const { return arena_; }
  size_t arena_size() const { return arena_bytes_; }

  size_t byte_offset(const std::string &name) const {
    if (!arena_ || open_) {
      throw std::runtime_error("Triton executor buffer set does not have arena offsets");
    }
    return find(name).offset;
  }

  // Copies `src` into `dst`, a host image of the whole arena, at the offset
  // of buffer `name`.
  template <typename T>
  void pack(std::vector<unsigned char> &dst, const std::string &name,
            const std::vector<T> &src) const {
    const size_t bytes = sizeof(T) * src.size();
    if (bytes > get(name).size()) {
      throw std::runtime_error("Triton executor packed copy overflows buffer '" + name + "'");
    }
    const size_t at = byte_offset(name);
    if (at > dst.size() || dst.size() - at < bytes) {
      throw std::runtime_error("Triton executor packed copy is out of range for '" + name + "'");
    }
    if (bytes != 0) {
      std::memcpy(dst.data() + at, src.data(), bytes);
    }
  }

  void copy_arena_to_device(const std::vector<unsigned char> &src) const {
    if (backing_ == nullptr || src.size() != arena_bytes_) {
      throw std::runtime_error("Triton executor arena copy size mismatch");
    }
    lrrt::copy_to_device(*backing_, src);
  }

private:
  struct Record {
    size_t bytes = 0;
    size_t offset = 0;                            // arena sets only
    size_t order = 0;                             // arena sets: position in the layout
    std::unique_ptr<lrrt::DeviceBuffer> storage;  // allocation, or view into the arena
  };

  static constexpr size_t kAlignment = 256;

  static size_t round_up(size_t value) {
    if (value > std::numeric_limits<size_t>::max() - (kAlignment - 1)) {
      throw std::overflow_error("Triton executor arena alignment overflows size_t");
    }
    return (value + kAlignment - 1) & ~(kAlignment - 1);
  }

  const Record &find(const std::string &name) const {
    if (open_) {
      throw std::runtime_error("Triton executor buffer set is not finalized");
    }
    if (auto hit = table_.find(name); hit != table_.end()) {
      return hit->second;
    }
    throw std::runtime_error("unknown Triton executor buffer '" + name +
                             "'; available buffers: " + detail::listing(table_));
  }

  lrrt::Device device_;
  bool arena_;
  bool open_;   // arena sets: allocations still being recorded
  size_t arena_bytes_ = 0;
  size_t recorded_ = 0; // buffers recorded in an arena set
  std::unique_ptr<lrrt::DeviceBuffer> backing_;
  std::map<std::string, Record> table_;
};

// One named kernel argument as raw bytes.
struct LaunchArg {
  std::string name;
  std::vector<unsigned char> value;
};

template <typename T> LaunchArg arg(const char *name, const T &value) {
  if (name == nullptr || *name == '\0') {
    throw std::invalid_argument("Triton executor launch argument name is empty");
  }
  const auto *bytes = reinterpret_cast<const unsigned char *>(&value);
  return LaunchArg{name, std::vector<unsigned char>(bytes, bytes + sizeof(T))};
}

// Binds `args` by name (each name at most once), leaves unbound optional
// pointer arguments null and launches `bundle` for problem size n on `queue`
// after `dependencies`.
inline void launch(const lrrt::Queue &queue, lrrt::Bundle &bundle, uint32_t n,
                   std::initializer_list<LaunchArg> args,
                   const std::vector<const lrrt::Event *> &dependencies = {}) {
  const std::string label = detail::kernel_label(bundle.manifest());
  lrrt::KernargBuffer kernargs = bundle.make_args();
  std::set<std::string> bound;
  for (const LaunchArg &argument : args) {
    if (!bound.insert(argument.name).second) {
      throw std::runtime_error("duplicate Triton executor launch argument '" + argument.name +
                               "' for kernel " + label);
    }
    try {
      kernargs.set_raw(argument.name.c_str(), argument.value.data(), argument.value.size());
    } catch (const std::exception &error) {
      throw std::runtime_error("failed to bind Triton executor launch argument '" +
                               argument.name + "' for kernel " + label + ": " + error.what());
    }
  }
  try {
    kernargs.bind_optional_nulls();
    bundle.launch(queue, n, kernargs, dependencies);
  } catch (const std::exception &error) {
    throw std::runtime_error("failed to launch Triton executor kernel " + label + ": " +
                             error.what());
  }
}

} // namespace lrrt::executor::triton

#endif // LRRT_EXECUTOR_TRITON_EXECUTOR_HPP_
