// Generic per-operation bundle executor: named lrrt::Bundle kernels, named
// device buffers (optionally carved out of one arena allocation) and a
// launch helper that binds kernel arguments by name. Same classes,
// functions and error texts as light-rocm-runtime
// executor/triton/triton_executor.hpp:21-312, so executors written against
// that header (the Triton per-op examples) compile unchanged; on B200 the
// bundles' code objects are sm_100a cubins and the queue is a CUDA stream.
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
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <unordered_set>
#include <vector>

namespace lrrt::executor::triton {

namespace detail {

// "a, b, c" (sorted, so messages do not depend on hash order), or "<none>".
template <typename Map> std::string names_of(const Map &entries) {
  std::map<std::string, int> sorted;
  for (const auto &entry : entries) {
    sorted.emplace(entry.first, 0);
  }
  if (sorted.empty()) {
    return "<none>";
  }
  std::string text;
  for (const auto &entry : sorted) {
    text += (text.empty() ? "" : ", ") + entry.first;
  }
  return text;
}

inline std::string kernel_label(const lrrt::KernelManifest &manifest) {
  return manifest.name + " (" + manifest.symbol + ")";
}

inline const char *display_string(const char *value) { return value ? value : "<null>"; }

} // namespace detail

// Bundles by name; each entry is one kernel of a manifest.
class BundleSet {
public:
  explicit BundleSet(lrrt::Device device) : device_(device) {}

  void add(const std::string &name, const char *manifest_path, const std::string &kernel_name) {
    try {
      entries_[name] = std::make_unique<lrrt::Bundle>(device_, manifest_path, kernel_name.c_str());
    } catch (const std::exception &error) {
      throw std::runtime_error("failed to load Triton executor bundle '" + name +
                               "' from manifest '" + detail::display_string(manifest_path) +
                               "' for kernel '" + kernel_name + "': " + error.what());
    }
  }

  lrrt::Bundle &get(const std::string &name) const {
    const auto found = entries_.find(name);
    if (found == entries_.end()) {
      throw std::runtime_error("unknown Triton executor bundle '" + name +
                               "'; available bundles: " + detail::names_of(entries_));
    }
    return *found->second;
  }

private:
  lrrt::Device device_;
  std::unordered_map<std::string, std::unique_ptr<lrrt::Bundle>> entries_;
};

// Device buffers by name. With `arena`, allocations are recorded until
// finalize() and then placed in one device allocation at 256-byte aligned
// offsets (so a whole input set can be uploaded with one copy); without it
// each buffer is its own allocation and the set is usable at once.
class BufferSet {
public:
  explicit BufferSet(lrrt::Device device, bool arena = false)
      : device_(device), arena_enabled_(arena), finalized_(!arena) {}

  void allocate_bytes(const std::string &name, size_t bytes) {
    if (arena_enabled_) {
      if (finalized_) {
        throw std::runtime_error("Triton executor arena buffer set is finalized");
      }
      pending_.push_back({name, bytes});
      return;
    }
    try {
      buffers_[name] = std::make_unique<lrrt::DeviceBuffer>(device_, bytes);
    } catch (const std::exception &error) {
      throw std::runtime_error("failed to allocate Triton executor buffer '" + name + "' (" +
                               std::to_string(bytes) + " bytes): " + error.what());
    }
  }

  template <typename T> void allocate(const std::string &name, size_t count) {
    if (count > std::numeric_limits<size_t>::max() / sizeof(T)) {
      throw std::overflow_error(
          "Triton executor buffer allocation overflows size_t for buffer '" + name + "'");
    }
    allocate_bytes(name, count * sizeof(T));
  }

  void finalize() {
    if (finalized_) {
      return;
    }
    size_t end = 0;
    std::vector<size_t> offsets;
    offsets.reserve(pending_.size());
    for (const Pending &buffer : pending_) {
      end = align_up(end);
      if (buffer.bytes > std::numeric_limits<size_t>::max() - end) {
        throw std::overflow_error("Triton executor arena allocation overflows size_t");
      }
      offsets.push_back(end);
      end += buffer.bytes;
    }
    arena_ = std::make_unique<lrrt::DeviceBuffer>(device_, end);
    auto *base = static_cast<unsigned char *>(arena_->data());
    for (size_t i = 0; i < pending_.size(); ++i) {
      offsets_[pending_[i].name] = offsets[i];
      buffers_[pending_[i].name] = std::make_unique<lrrt::DeviceBuffer>(
          lrrt::DeviceBuffer::view(device_.get(), base + offsets[i], pending_[i].bytes));
    }
    arena_size_ = end;
    pending_.clear();
    finalized_ = true;
  }

  lrrt::DeviceBuffer &get(const std::string &name) const {
    if (!finalized_) {
      throw std::runtime_error("Triton executor buffer set is not finalized");
    }
    const auto found = buffers_.find(name);
    if (found == buffers_.end()) {
      throw std::runtime_error("unknown Triton executor buffer '" + name +
                               "'; available buffers: " + detail::names_of(buffers_));
    }
    return *found->second;
  }

  template <typename T> T *ptr(const std::string &name, size_t element_offset = 0) const {
    lrrt::DeviceBuffer &buffer = get(name);
    if (element_offset > std::numeric_limits<size_t>::max() / sizeof(T)) {
      throw std::overflow_error("Triton executor buffer offset overflows size_t for buffer '" +
                                name + "'");
    }
    const size_t byte_offset = element_offset * sizeof(T);
    if (byte_offset > buffer.size()) {
      throw std::out_of_range("Triton executor buffer offset is out of range for '" + name +
                              "': element_offset=" + std::to_string(element_offset) +
                              ", element_size=" + std::to_string(sizeof(T)) +
                              ", byte_offset=" + std::to_string(byte_offset) +
                              ", buffer_size=" + std::to_string(buffer.size()));
    }
    return reinterpret_cast<T *>(static_cast<unsigned char *>(buffer.data()) + byte_offset);
  }

  template <typename T> void copy_to(const std::string &name, const std::vector<T> &src) const {
    lrrt::copy_to_device(get(name), src);
  }

  template <typename T> void copy_from(std::vector<T> &dst, const std::string &name) const {
    lrrt::copy_to_host(dst, get(name));
  }

  bool uses_arena() const { return arena_enabled_; }
  size_t arena_size() const { return arena_size_; }

  size_t byte_offset(const std::string &name) const {
    if (!finalized_ || !arena_enabled_) {
      throw std::runtime_error("Triton executor buffer set does not have arena offsets");
    }
    const auto found = offsets_.find(name);
    if (found == offsets_.end()) {
      throw std::runtime_error("unknown Triton executor buffer '" + name +
                               "'; available buffers: " + detail::names_of(offsets_));
    }
    return found->second;
  }

  // Copies `src` into a host image of the whole arena at the buffer's offset.
  template <typename T>
  void pack(std::vector<unsigned char> &dst, const std::string &name,
            const std::vector<T> &src) const {
    const size_t bytes = src.size() * sizeof(T);
    if (bytes > get(name).size()) {
      throw std::runtime_error("Triton executor packed copy overflows buffer '" + name + "'");
    }
    const size_t offset = byte_offset(name);
    if (offset > dst.size() || bytes > dst.size() - offset) {
      throw std::runtime_error("Triton executor packed copy is out of range for '" + name + "'");
    }
    if (bytes != 0) {
      std::memcpy(dst.data() + offset, src.data(), bytes);
    }
  }

  void copy_arena_to_device(const std::vector<unsigned char> &src) const {
    if (!arena_ || src.size() != arena_size_) {
      throw std::runtime_error("Triton executor arena copy size mismatch");
    }
    lrrt::copy_to_device(*arena_, src);
  }

private:
  static constexpr size_t kArenaAlignment = 256;

  struct Pending {
    std::string name;
    size_t bytes;
  };

  static size_t align_up(size_t value) {
    const size_t padding = (kArenaAlignment - value % kArenaAlignment) % kArenaAlignment;
    if (value > std::numeric_limits<size_t>::max() - padding) {
      throw std::overflow_error("Triton executor arena alignment overflows size_t");
    }
    return value + padding;
  }

  lrrt::Device device_;
  bool arena_enabled_;
  bool finalized_;
  size_t arena_size_ = 0;
  std::vector<Pending> pending_;
  std::unique_ptr<lrrt::DeviceBuffer> arena_;
  std::unordered_map<std::string, size_t> offsets_;
  std::unordered_map<std::string, std::unique_ptr<lrrt::DeviceBuffer>> buffers_;
};

// One named kernel argument as raw bytes.
struct LaunchArg {
  std::string name;
  std::vector<unsigned char> value;
};

template <typename T> LaunchArg arg(const char *name, const T &value) {
  if (name == nullptr || name[0] == '\0') {
    throw std::invalid_argument("Triton executor launch argument name is empty");
  }
  LaunchArg bound{name, std::vector<unsigned char>(sizeof(T))};
  std::memcpy(bound.value.data(), &value, sizeof(T));
  return bound;
}

// Binds `args` by name (each at most once), sets unbound optional pointers to
// null and launches the bundle for problem size n on `queue`.
inline void launch(const lrrt::Queue &queue, lrrt::Bundle &bundle, uint32_t n,
                   std::initializer_list<LaunchArg> args,
                   const std::vector<const lrrt::Event *> &dependencies = {}) {
  lrrt::KernargBuffer kernargs = bundle.make_args();
  std::unordered_set<std::string> seen;
  for (const LaunchArg &entry : args) {
    if (!seen.insert(entry.name).second) {
      throw std::runtime_error("duplicate Triton executor launch argument '" + entry.name +
                               "' for kernel " + detail::kernel_label(bundle.manifest()));
    }
    try {
      kernargs.set_raw(entry.name.c_str(), entry.value.data(), entry.value.size());
    } catch (const std::exception &error) {
      throw std::runtime_error("failed to bind Triton executor launch argument '" + entry.name +
                               "' for kernel " + detail::kernel_label(bundle.manifest()) + ": " +
                               error.what());
    }
  }
  try {
    kernargs.bind_optional_nulls();
    bundle.launch(queue, n, kernargs, dependencies);
  } catch (const std::exception &error) {
    throw std::runtime_error("failed to launch Triton executor kernel " +
                             detail::kernel_label(bundle.manifest()) + ": " + error.what());
  }
}

} // namespace lrrt::executor::triton

#endif // LRRT_EXECUTOR_TRITON_EXECUTOR_HPP_
