// Kernel bundles: a JSON manifest describing kernels in code objects next to
// it (symbol, block size, grid rule, kernarg layout), a kernarg buffer that
// packs and checks arguments against that layout, and a Bundle that loads
// the code object and launches through the lr_* ABI.
//
// Interface, manifest format and error texts are those of light-rocm-runtime
// include/lrrt/bundle.hpp:14-134 and src/bundle.cpp (callers and their tests
// match on the messages). On B200 the code object is an sm_100a cubin and
// the manifest's "target" is informational ("sm_100a"), as the reference
// does not check it against the device either.
//
// Manifest (version 1):
//   { "manifest_version": 1, "target": "<arch>",
//     "kernels": [ { "name", "symbol", "code_object" (relative path inside
//       the bundle directory), "kernarg_size", "block": [x, y, z],
//       "grid": ["ceil_div(n, D) * M", 1, 1],
//       "args": [ {"name", "type", "offset", "size", "optional"?}, ... ],
//       "shared_memory_bytes"? (default 0), "workspace_bytes"? (default 0) } ] }
// Field order is free and unknown fields are ignored. The launch grid for a
// problem size n is ceil(n / D) * M threads in x (lr_* grids count threads).
#ifndef LRRT_BUNDLE_HPP_
#define LRRT_BUNDLE_HPP_

#include "lrrt/lrrt.hpp"

#include <cstddef>
#include <cstdint>
#include <stdexcept>
#include <string>
#include <vector>

namespace lrrt {

static constexpr uint32_t kSupportedBundleManifestVersion = 1;

struct KernelArgument {
  std::string name;
  std::string type;
  size_t offset;
  size_t size;
  bool optional;
};

struct KernelManifest {
  uint32_t manifest_version;
  std::string target;
  std::string name;
  std::string symbol;
  std::string code_object;
  uint32_t block[3];
  uint32_t grid_multiplier;
  uint32_t grid_divisor;
  size_t kernarg_size;
  uint32_t shared_memory_bytes;
  uint64_t workspace_bytes;
  std::vector<size_t> arg_offsets;
  std::vector<KernelArgument> args;
};

// First kernel of the manifest, the kernel called `kernel_name`, or all
// kernels in manifest order.
LRRT_API KernelManifest parse_bundle_manifest(const void *data, size_t size);
LRRT_API KernelManifest parse_bundle_manifest(const void *data, size_t size,
                                              const char *kernel_name);
LRRT_API std::vector<KernelManifest> parse_bundle_manifests(const void *data,
                                                            size_t size);

inline KernelManifest parse_bundle_manifest(const std::vector<unsigned char> &data) {
  return parse_bundle_manifest(data.data(), data.size());
}
inline KernelManifest parse_bundle_manifest(const std::vector<unsigned char> &data,
                                            const char *kernel_name) {
  return parse_bundle_manifest(data.data(), data.size(), kernel_name);
}
inline std::vector<KernelManifest>
parse_bundle_manifests(const std::vector<unsigned char> &data) {
  return parse_bundle_manifests(data.data(), data.size());
}

// Launch configuration for problem size n (grid = ceil(n / D) * M threads).
LRRT_API lr_launch_config_t launch_config_from_manifest(const KernelManifest &manifest,
                                                        uint32_t n);

// Throws unless the manifest's kernarg size and argument offsets are these.
LRRT_API void require_kernarg_layout(const KernelManifest &manifest, size_t kernarg_size,
                                     const std::vector<size_t> &arg_offsets);

class LRRT_API KernargBuffer {
public:
  explicit KernargBuffer(const KernelManifest &manifest);

  void set_raw(size_t index, const void *value, size_t value_size);
  void set_raw(const char *name, const void *value, size_t value_size);

  template <typename T> void set(size_t index, const T &value) {
    set_raw(index, &value, sizeof(T));
  }
  template <typename T> void set(int index, const T &value) {
    if (index < 0) {
      throw std::out_of_range("bundle kernarg index is out of range");
    }
    set_raw(static_cast<size_t>(index), &value, sizeof(T));
  }
  template <typename T> void set(const char *name, const T &value) {
    set_raw(name, &value, sizeof(T));
  }
  template <typename T> void set(const std::string &name, const T &value) {
    set_raw(name.c_str(), &value, sizeof(T));
  }

  // Every required argument bound (and, with a manifest, the same layout).
  void validate() const;
  void validate(const KernelManifest &manifest) const;
  // Binds every unbound optional pointer argument to null.
  void bind_optional_nulls();

  const void *data() const { return data_.data(); }
  void *data() { return data_.data(); }
  size_t size() const { return data_.size(); }
  const std::vector<unsigned char> &bytes() const { return data_; }

private:
  std::vector<unsigned char> data_;
  std::vector<KernelArgument> args_;
  std::vector<bool> bound_;
};

class LRRT_API Bundle {
public:
  Bundle(Device device, const char *manifest_path);
  Bundle(Device device, const char *manifest_path, const char *kernel_name);

  const KernelManifest &manifest() const { return manifest_; }
  Kernel kernel() const { return kernel_; }
  KernargBuffer make_args() const;
  lr_launch_config_t launch_config(uint32_t n) const;
  void launch(uint32_t n, const KernargBuffer &args) const;
  void launch(uint32_t n, const KernargBuffer &args,
              const std::vector<const Event *> &dependencies) const;
  void launch(const Queue &queue, uint32_t n, const KernargBuffer &args,
              const std::vector<const Event *> &dependencies = {}) const;

private:
  static KernelManifest load_manifest(const char *manifest_path, const char *kernel_name);
  static std::vector<unsigned char> read_code_object(const char *manifest_path,
                                                     const KernelManifest &manifest);

  KernelManifest manifest_;
  Module module_;
  Kernel kernel_;
};

} // namespace lrrt

#endif // LRRT_BUNDLE_HPP_
