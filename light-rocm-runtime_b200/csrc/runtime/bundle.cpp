// lrrt::bundle: manifest parsing, kernarg packing and bundle launches.
//
// The manifest is read into a small JSON document tree first (any field
// order, unknown fields ignored, standard string escapes), then each kernel
// entry is checked field by field. Validation rules and error texts follow
// light-rocm-runtime src/bundle.cpp (manifest :88-245 and :470-600, launch
// configuration :640-670, kernarg buffer :672-760, Bundle :762-810), because
// callers and their tests match on those messages.
#include "lrrt/bundle.hpp"

#include "lrrt/launch.hpp"

#include "../common/json.hpp"

#include <cstdio>
#include <cstring>
#include <limits>
#include <memory>
#include <utility>

namespace lrrt {
namespace {

using ManifestError = std::runtime_error;
using json::Json;
using json::JsonReader;

// ------------------------------------------------------ manifest fields --

const Json &require(const Json &object, const char *field) {
  const Json *value = object.find(field);
  if (value == nullptr) {
    throw ManifestError(std::string("missing manifest token \"") + field + "\"");
  }
  return *value;
}

// A non-negative integer token no larger than `maximum`.
uint64_t integer_value(const Json &value, const char *field, uint64_t maximum) {
  if (value.kind != Json::Kind::number) {
    throw ManifestError(std::string("manifest field is not integer: ") + field);
  }
  uint64_t result = 0;
  bool overflow = false;
  for (const char c : value.text) {
    if (c < '0' || c > '9') {
      throw ManifestError(std::string("invalid manifest integer: ") + field);
    }
    const uint64_t digit = static_cast<uint64_t>(c - '0');
    if (result > (std::numeric_limits<uint64_t>::max() - digit) / 10u) {
      overflow = true;
      break;
    }
    result = result * 10u + digit;
  }
  if (value.text.empty()) {
    throw ManifestError(std::string("invalid manifest integer: ") + field);
  }
  if (overflow || result > maximum) {
    throw ManifestError(std::string("manifest field is too large: ") + field);
  }
  return result;
}

uint64_t read_integer(const Json &object, const char *field, uint64_t maximum) {
  return integer_value(require(object, field), field, maximum);
}

uint64_t read_optional_integer(const Json &object, const char *field, uint64_t fallback,
                               uint64_t maximum) {
  const Json *value = object.find(field);
  return value == nullptr ? fallback : integer_value(*value, field, maximum);
}

std::string read_string(const Json &object, const char *field) {
  const Json &value = require(object, field);
  if (value.kind != Json::Kind::string) {
    throw ManifestError(std::string("manifest field is not string: ") + field);
  }
  return value.text;
}

bool read_optional_bool(const Json &object, const char *field, bool fallback) {
  const Json *value = object.find(field);
  if (value == nullptr) {
    return fallback;
  }
  if (value->kind != Json::Kind::boolean) {
    throw ManifestError(std::string("manifest field is not boolean: ") + field);
  }
  return value->flag;
}

constexpr uint64_t kU32 = std::numeric_limits<uint32_t>::max();
constexpr uint64_t kSize = std::numeric_limits<size_t>::max();

bool has_parent_component(const std::string &path) {
  size_t begin = 0;
  while (begin <= path.size()) {
    size_t end = path.find('/', begin);
    if (end == std::string::npos) {
      end = path.size();
    }
    if (path.compare(begin, end - begin, "..") == 0 && end - begin == 2) {
      return true;
    }
    begin = end + 1;
  }
  return false;
}

bool stays_in_bundle(const std::string &path) {
  return !path.empty() && path[0] != '/' && !has_parent_component(path);
}

// "ceil_div(n, D) * M" with optional spaces between tokens.
void parse_grid_expression(const std::string &expression, uint32_t *divisor,
                           uint32_t *multiplier) {
  size_t at = 0;
  auto space = [&] {
    while (at < expression.size() && expression[at] == ' ') {
      ++at;
    }
  };
  auto word = [&](const char *text) {
    space();
    const size_t length = std::strlen(text);
    if (expression.compare(at, length, text) != 0) {
      throw ManifestError("unsupported bundle grid expression");
    }
    at += length;
  };
  auto number = [&]() -> uint32_t {
    space();
    const size_t begin = at;
    uint64_t value = 0;
    while (at < expression.size() && expression[at] >= '0' && expression[at] <= '9') {
      value = value * 10u + static_cast<uint64_t>(expression[at] - '0');
      if (value > kU32) {
        throw ManifestError("bundle grid expression is too large");
      }
      ++at;
    }
    if (at == begin) {
      throw ManifestError("unsupported bundle grid expression");
    }
    return static_cast<uint32_t>(value);
  };
  word("ceil_div");
  word("(");
  word("n");
  word(",");
  *divisor = number();
  word(")");
  word("*");
  *multiplier = number();
  space();
  if (at != expression.size()) {
    throw ManifestError("unsupported bundle grid expression");
  }
}

void read_launch_shape(const Json &kernel, KernelManifest &m) {
  const Json &block = require(kernel, "block");
  if (block.kind != Json::Kind::array) {
    throw ManifestError("manifest field is not array: block");
  }
  if (block.items.size() != 3) {
    throw ManifestError("invalid manifest array: block");
  }
  for (size_t i = 0; i < 3; ++i) {
    if (block.items[i].kind != Json::Kind::number) {
      throw ManifestError("invalid manifest array: block");
    }
    m.block[i] = static_cast<uint32_t>(integer_value(block.items[i], "block", kU32));
  }
  const Json &grid = require(kernel, "grid");
  if (grid.kind != Json::Kind::array) {
    throw ManifestError("manifest grid is not array");
  }
  if (grid.items.empty() || grid.items[0].kind != Json::Kind::string) {
    throw ManifestError("manifest grid[0] is not expression string");
  }
  if (grid.items.size() != 3) {
    throw ManifestError("invalid manifest grid array");
  }
  if (integer_value(grid.items[1], "grid", kU32) != 1) {
    throw ManifestError("bundle grid y dimension must be 1");
  }
  if (integer_value(grid.items[2], "grid", kU32) != 1) {
    throw ManifestError("bundle grid z dimension must be 1");
  }
  parse_grid_expression(grid.items[0].text, &m.grid_divisor, &m.grid_multiplier);
}

std::string argument_context(size_t index, const KernelArgument &argument) {
  std::string context = "args[" + std::to_string(index) + "]";
  if (!argument.name.empty()) {
    context += " '" + argument.name + "'";
  }
  return context;
}

void read_arguments(const Json &kernel, KernelManifest &m) {
  const Json &args = require(kernel, "args");
  if (args.kind != Json::Kind::array) {
    throw ManifestError("manifest args is not array");
  }
  for (size_t i = 0; i < args.items.size(); ++i) {
    const Json &entry = args.items[i];
    if (entry.kind != Json::Kind::object) {
      throw ManifestError("invalid manifest args array");
    }
    KernelArgument argument{};
    try {
      argument.name = read_string(entry, "name");
      argument.type = read_string(entry, "type");
      argument.offset = static_cast<size_t>(read_integer(entry, "offset", kSize));
      argument.size = static_cast<size_t>(read_integer(entry, "size", kSize));
      argument.optional = read_optional_bool(entry, "optional", false);
    } catch (const std::exception &error) {
      throw ManifestError("args[" + std::to_string(i) + "]: " + error.what());
    }
    m.args.push_back(std::move(argument));
  }
  if (m.args.empty()) {
    throw ManifestError("bundle manifest has no arguments");
  }
  // Strictly increasing, in-range, uniquely named arguments.
  for (size_t i = 0; i < m.args.size(); ++i) {
    const KernelArgument &a = m.args[i];
    if (a.name.empty() || a.type.empty() || a.size == 0) {
      throw ManifestError(argument_context(i, a) + ": invalid bundle argument manifest");
    }
    if (a.offset >= m.kernarg_size || a.size > m.kernarg_size ||
        a.offset + a.size > m.kernarg_size) {
      throw ManifestError(argument_context(i, a) + ": argument range exceeds kernarg_size");
    }
    if (i > 0 && a.offset <= m.args[i - 1].offset) {
      throw ManifestError(argument_context(i, a) +
                  ": argument offsets must be strictly increasing");
    }
    for (size_t j = 0; j < i; ++j) {
      if (m.args[j].name == a.name) {
        throw ManifestError(argument_context(i, a) + ": duplicate argument name");
      }
    }
    m.arg_offsets.push_back(a.offset);
  }
}

KernelManifest read_kernel(const Json &kernel, uint32_t version, const std::string &target) {
  KernelManifest m{};
  m.manifest_version = version;
  m.target = target;
  m.name = read_string(kernel, "name");
  m.symbol = read_string(kernel, "symbol");
  m.code_object = read_string(kernel, "code_object");
  if (!stays_in_bundle(m.code_object)) {
    throw ManifestError("bundle code object path must stay in bundle");
  }
  m.kernarg_size = static_cast<size_t>(read_integer(kernel, "kernarg_size", kSize));
  const uint64_t shared = read_optional_integer(kernel, "shared_memory_bytes", 0,
                                                std::numeric_limits<uint64_t>::max());
  if (shared > kU32) {
    throw ManifestError("bundle shared memory requirement is too large");
  }
  m.shared_memory_bytes = static_cast<uint32_t>(shared);
  m.workspace_bytes = read_optional_integer(kernel, "workspace_bytes", 0,
                                            std::numeric_limits<uint64_t>::max());
  read_launch_shape(kernel, m);
  read_arguments(kernel, m);
  return m;
}

std::vector<KernelManifest> parse_document(const void *data, size_t size) {
  if (data == nullptr || size == 0) {
    throw std::invalid_argument("bundle manifest is empty");
  }
  const Json root = JsonReader(static_cast<const char *>(data), size).document();
  if (root.kind != Json::Kind::object) {
    throw ManifestError("bundle manifest root is not object");
  }
  const uint32_t version = static_cast<uint32_t>(read_integer(root, "manifest_version", kU32));
  if (version != kSupportedBundleManifestVersion) {
    throw ManifestError("unsupported bundle manifest_version: " + std::to_string(version));
  }
  const std::string target = read_string(root, "target");
  if (target.empty()) {
    throw ManifestError("bundle manifest target is empty");
  }
  const Json &kernels = require(root, "kernels");
  if (kernels.kind != Json::Kind::array) {
    throw ManifestError("manifest kernels is not array");
  }
  std::vector<KernelManifest> manifests;
  for (size_t i = 0; i < kernels.items.size(); ++i) {
    const Json &kernel = kernels.items[i];
    if (kernel.kind != Json::Kind::object) {
      throw ManifestError("invalid kernel manifest array");
    }
    KernelManifest m;
    try {
      m = read_kernel(kernel, version, target);
    } catch (const std::exception &error) {
      std::string context = "bundle manifest kernels[" + std::to_string(i) + "]";
      const Json *name = kernel.find("name");
      if (name != nullptr && name->kind == Json::Kind::string && !name->text.empty()) {
        context += " '" + name->text + "'";
      }
      throw ManifestError(context + ": " + error.what());
    }
    for (const KernelManifest &previous : manifests) {
      if (previous.name == m.name) {
        throw ManifestError("duplicate kernel name in bundle manifest: " + m.name);
      }
    }
    manifests.push_back(std::move(m));
  }
  if (manifests.empty()) {
    throw ManifestError("bundle manifest has no kernels");
  }
  return manifests;
}

std::vector<unsigned char> read_file(const char *path) {
  if (path == nullptr || path[0] == '\0') {
    throw std::invalid_argument("bundle path is empty");
  }
  std::unique_ptr<FILE, int (*)(FILE *)> file(std::fopen(path, "rb"), &std::fclose);
  if (!file) {
    throw ManifestError(std::string("failed to open ") + path);
  }
  std::vector<unsigned char> bytes;
  unsigned char chunk[65536];
  size_t got;
  while ((got = std::fread(chunk, 1, sizeof(chunk), file.get())) > 0) {
    bytes.insert(bytes.end(), chunk, chunk + got);
  }
  if (std::ferror(file.get())) {
    throw ManifestError(std::string("failed to read ") + path);
  }
  if (bytes.empty()) {
    throw ManifestError(std::string("empty file ") + path);
  }
  return bytes;
}

bool same_layout(const std::vector<KernelArgument> &a, const std::vector<KernelArgument> &b) {
  if (a.size() != b.size()) {
    return false;
  }
  for (size_t i = 0; i < a.size(); ++i) {
    if (a[i].name != b[i].name || a[i].type != b[i].type || a[i].offset != b[i].offset ||
        a[i].size != b[i].size || a[i].optional != b[i].optional) {
      return false;
    }
  }
  return true;
}

} // namespace

// ------------------------------------------------------------ public API --

std::vector<KernelManifest> parse_bundle_manifests(const void *data, size_t size) {
  return parse_document(data, size);
}

KernelManifest parse_bundle_manifest(const void *data, size_t size) {
  return parse_document(data, size).front();
}

KernelManifest parse_bundle_manifest(const void *data, size_t size, const char *kernel_name) {
  if (kernel_name == nullptr || kernel_name[0] == '\0') {
    throw std::invalid_argument("bundle kernel name is empty");
  }
  for (KernelManifest &manifest : parse_document(data, size)) {
    if (manifest.name == kernel_name) {
      return std::move(manifest);
    }
  }
  throw ManifestError(std::string("bundle kernel not found: ") + kernel_name);
}

lr_launch_config_t launch_config_from_manifest(const KernelManifest &manifest, uint32_t n) {
  const uint32_t *block = manifest.block;
  if (block[0] == 0 || block[1] == 0 || block[2] == 0) {
    throw ManifestError("bundle launch block dimensions must be non-zero");
  }
  // The reference's message names HSA dispatch packets (16-bit workgroup
  // sizes); the same bound is kept so manifests behave identically.
  if (block[0] > 0xffffu || block[1] > 0xffffu || block[2] > 0xffffu) {
    throw ManifestError("bundle launch block dimensions exceed HSA packet limits");
  }
  if (manifest.grid_divisor == 0 || manifest.grid_multiplier == 0) {
    throw ManifestError("invalid bundle launch configuration");
  }
  const uint64_t programs =
      (uint64_t{n} + manifest.grid_divisor - 1u) / manifest.grid_divisor;
  const uint64_t threads = programs * manifest.grid_multiplier;
  if (threads > kU32) {
    throw ManifestError("bundle grid size is too large");
  }
  if (threads == 0) {
    throw ManifestError("bundle launch grid dimensions must be non-zero");
  }
  if (threads < block[0]) {
    throw ManifestError("bundle launch grid dimensions must cover the workgroup");
  }
  lr_launch_config_t config{};
  config.grid = {static_cast<uint32_t>(threads), 1u, 1u};
  config.block = {block[0], block[1], block[2]};
  config.shared_memory_bytes = manifest.shared_memory_bytes;
  return config;
}

void require_kernarg_layout(const KernelManifest &manifest, size_t kernarg_size,
                            const std::vector<size_t> &arg_offsets) {
  if (manifest.kernarg_size != kernarg_size || manifest.arg_offsets != arg_offsets) {
    throw ManifestError("bundle manifest does not match kernarg layout");
  }
}

KernargBuffer::KernargBuffer(const KernelManifest &manifest)
    : data_(manifest.kernarg_size, 0), args_(manifest.args),
      bound_(manifest.args.size(), false) {
  if (data_.empty() || args_.empty()) {
    throw ManifestError("invalid bundle kernarg layout");
  }
}

void KernargBuffer::set_raw(size_t index, const void *value, size_t value_size) {
  if (value == nullptr && value_size != 0) {
    throw std::invalid_argument("bundle kernarg value is null");
  }
  if (index >= args_.size()) {
    throw std::out_of_range("bundle kernarg index is out of range");
  }
  const KernelArgument &argument = args_[index];
  if (argument.offset > data_.size() || argument.size > data_.size() - argument.offset) {
    throw ManifestError("invalid bundle kernarg offset");
  }
  if (value_size > argument.size) {
    throw ManifestError("bundle kernarg value exceeds argument slot");
  }
  unsigned char *slot = data_.data() + argument.offset;
  std::memset(slot, 0, argument.size);
  if (value_size != 0) {
    std::memcpy(slot, value, value_size);
  }
  bound_[index] = true;
}

void KernargBuffer::set_raw(const char *name, const void *value, size_t value_size) {
  if (name == nullptr || name[0] == '\0') {
    throw std::invalid_argument("bundle kernarg name is empty");
  }
  for (size_t i = 0; i < args_.size(); ++i) {
    if (args_[i].name == name) {
      set_raw(i, value, value_size);
      return;
    }
  }
  throw std::out_of_range(std::string("bundle kernarg not found: ") + name);
}

void KernargBuffer::validate() const {
  for (size_t i = 0; i < args_.size(); ++i) {
    if (!bound_[i] && !args_[i].optional) {
      throw ManifestError("missing required bundle kernarg: " + args_[i].name);
    }
  }
}

void KernargBuffer::validate(const KernelManifest &manifest) const {
  if (data_.size() != manifest.kernarg_size || !same_layout(args_, manifest.args)) {
    throw ManifestError("bundle kernarg buffer does not match kernel manifest");
  }
  validate();
}

void KernargBuffer::bind_optional_nulls() {
  const void *null_pointer = nullptr;
  for (size_t i = 0; i < args_.size(); ++i) {
    if (args_[i].optional && !bound_[i]) {
      if (args_[i].type != "ptr") {
        throw ManifestError("optional null binding requires ptr argument: " + args_[i].name);
      }
      set_raw(i, &null_pointer, sizeof(null_pointer));
    }
  }
}

Bundle::Bundle(Device device, const char *manifest_path)
    : manifest_(load_manifest(manifest_path, nullptr)),
      module_(device, read_code_object(manifest_path, manifest_)),
      kernel_(module_.kernel(manifest_.symbol.c_str())) {}

Bundle::Bundle(Device device, const char *manifest_path, const char *kernel_name)
    : manifest_(load_manifest(manifest_path, kernel_name)),
      module_(device, read_code_object(manifest_path, manifest_)),
      kernel_(module_.kernel(manifest_.symbol.c_str())) {}

KernargBuffer Bundle::make_args() const { return KernargBuffer(manifest_); }

lr_launch_config_t Bundle::launch_config(uint32_t n) const {
  return launch_config_from_manifest(manifest_, n);
}

void Bundle::launch(uint32_t n, const KernargBuffer &args) const {
  args.validate(manifest_);
  lrrt::launch(kernel_, launch_config(n), args.data(), args.size());
}

void Bundle::launch(uint32_t n, const KernargBuffer &args,
                    const std::vector<const Event *> &dependencies) const {
  args.validate(manifest_);
  lrrt::launch(kernel_, launch_config(n), args.data(), args.size(), dependencies);
}

void Bundle::launch(const Queue &queue, uint32_t n, const KernargBuffer &args,
                    const std::vector<const Event *> &dependencies) const {
  args.validate(manifest_);
  lrrt::launch(queue, kernel_, launch_config(n), args.data(), args.size(), dependencies);
}

KernelManifest Bundle::load_manifest(const char *manifest_path, const char *kernel_name) {
  const std::vector<unsigned char> data = read_file(manifest_path);
  return kernel_name != nullptr ? parse_bundle_manifest(data, kernel_name)
                                : parse_bundle_manifest(data);
}

std::vector<unsigned char> Bundle::read_code_object(const char *manifest_path,
                                                    const KernelManifest &manifest) {
  if (!stays_in_bundle(manifest.code_object)) {
    throw ManifestError("bundle code object path must stay in bundle");
  }
  const std::string manifest_file(manifest_path);
  const size_t slash = manifest_file.find_last_of('/');
  const std::string path = slash == std::string::npos
                               ? manifest.code_object
                               : manifest_file.substr(0, slash + 1) + manifest.code_object;
  return read_file(path.c_str());
}

} // namespace lrrt
