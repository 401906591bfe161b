// FP32 weight bundles (include/lrrt/qwen/weight_bundle.hpp): manifest
// parsing on the shared JSON reader, tensor extraction with the reference's
// checks and messages (light-rocm-runtime executor/qwen/weight_bundle.hpp:
// shape rules :74-90, data path :139-156, tensor lookup :332-370, loaders
// :460-602, writers :606-756), and writers producing the same format.
#include "lrrt/qwen/weight_bundle.hpp"

#include "../common/json.hpp"

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <limits>
#include <memory>
#include <stdexcept>
#include <string>

namespace lrrt::executor::qwen {
namespace {

using json::Json;

constexpr uint64_t kMaxU32 = std::numeric_limits<uint32_t>::max();

std::vector<unsigned char> read_file(const std::string &path) {
  std::unique_ptr<FILE, int (*)(FILE *)> file(std::fopen(path.c_str(), "rb"), &std::fclose);
  if (!file) {
    throw std::runtime_error("failed to open mini decoder weight file: " + path);
  }
  std::vector<unsigned char> bytes;
  unsigned char chunk[1 << 16];
  size_t got;
  while ((got = std::fread(chunk, 1, sizeof(chunk), file.get())) > 0) {
    bytes.insert(bytes.end(), chunk, chunk + got);
  }
  if (std::ferror(file.get())) {
    throw std::runtime_error("failed to read mini decoder weight file: " + path);
  }
  if (bytes.empty()) {
    throw std::runtime_error("mini decoder weight file is empty: " + path);
  }
  return bytes;
}

bool has_parent_component(const std::string &path) {
  size_t begin = 0;
  while (begin <= path.size()) {
    size_t end = path.find('/', begin);
    if (end == std::string::npos) {
      end = path.size();
    }
    if (end - begin == 2 && path.compare(begin, 2, "..") == 0) {
      return true;
    }
    begin = end + 1;
  }
  return false;
}

// `file_name` resolved next to the manifest; it must stay in that directory.
std::string relative_path(const char *manifest_path, const std::string &file_name) {
  if (file_name.empty() || file_name[0] == '/' || has_parent_component(file_name)) {
    throw std::runtime_error("invalid mini decoder weight data path: " + file_name);
  }
  const std::string manifest(manifest_path);
  const size_t slash = manifest.find_last_of('/');
  return slash == std::string::npos ? file_name : manifest.substr(0, slash + 1) + file_name;
}

Json read_manifest(const char *path) {
  const std::vector<unsigned char> text = read_file(path);
  return json::JsonReader(reinterpret_cast<const char *>(text.data()), text.size(),
                          "invalid mini decoder weight manifest")
      .document();
}

const Json &field(const Json &object, const char *name) {
  const Json *value = object.kind == Json::Kind::object ? object.find(name) : nullptr;
  if (value == nullptr) {
    throw std::runtime_error(std::string("missing mini decoder weight manifest field: ") + name);
  }
  return *value;
}

uint64_t integer_of(const Json &value, const char *name, uint64_t maximum) {
  if (value.kind != Json::Kind::number || value.text.empty()) {
    throw std::runtime_error(std::string("invalid mini decoder weight manifest field: ") + name);
  }
  uint64_t result = 0;
  for (const char c : value.text) {
    if (c < '0' || c > '9') {
      throw std::runtime_error(std::string("invalid mini decoder weight manifest field: ") +
                               name);
    }
    const uint64_t digit = static_cast<uint64_t>(c - '0');
    if (result > (std::numeric_limits<uint64_t>::max() - digit) / 10u ||
        result * 10u + digit > maximum) {
      throw std::runtime_error(std::string("mini decoder weight manifest integer is too large: ") +
                               name);
    }
    result = result * 10u + digit;
  }
  return result;
}

uint32_t u32_field(const Json &object, const char *name) {
  return static_cast<uint32_t>(integer_of(field(object, name), name, kMaxU32));
}

std::string string_field(const Json &object, const char *name) {
  const Json &value = field(object, name);
  if (value.kind != Json::Kind::string) {
    throw std::runtime_error(std::string("invalid mini decoder weight manifest field: ") + name);
  }
  return value.text;
}

float f32_field(const Json &object, const char *name) {
  const Json &value = field(object, name);
  if (value.kind != Json::Kind::number) {
    throw std::runtime_error(std::string("invalid mini decoder weight manifest field: ") + name);
  }
  char *end = nullptr;
  const double parsed = std::strtod(value.text.c_str(), &end);
  if (end == value.text.c_str() || *end != '\0') {
    throw std::runtime_error(std::string("invalid mini decoder weight manifest field: ") + name);
  }
  return static_cast<float>(parsed);
}

size_t checked_multiply(size_t left, size_t right, const char *context) {
  if (left != 0 && right > std::numeric_limits<size_t>::max() / left) {
    throw std::overflow_error(std::string(context) + " overflows size_t");
  }
  return left * right;
}

void validate_shape(const DecoderLayerShape &shape) {
  if (shape.keys == 0 || shape.hidden == 0 || shape.heads == 0 || shape.kv_heads == 0 ||
      shape.head_dim == 0 || shape.head_dim % 2 != 0 || shape.intermediate == 0) {
    throw std::runtime_error("mini decoder weight manifest has invalid shape");
  }
  if (shape.kv_heads > shape.heads || shape.heads % shape.kv_heads != 0) {
    throw std::runtime_error("mini decoder weight manifest has invalid GQA shape");
  }
  if (shape.heads > kMaxU32 / shape.head_dim) {
    throw std::overflow_error("mini decoder q dimension overflows uint32");
  }
  if (shape.kv_heads > kMaxU32 / shape.head_dim) {
    throw std::overflow_error("mini decoder kv dimension overflows uint32");
  }
}

// The entry of `tensors` named `name` (exactly one).
const Json &tensor_entry(const Json &manifest, const char *name) {
  const Json &tensors = field(manifest, "tensors");
  if (tensors.kind != Json::Kind::array) {
    throw std::runtime_error("invalid mini decoder weight manifest field: tensors");
  }
  const Json *found = nullptr;
  for (const Json &entry : tensors.items) {
    const Json *entry_name = entry.kind == Json::Kind::object ? entry.find("name") : nullptr;
    if (entry_name != nullptr && entry_name->kind == Json::Kind::string &&
        entry_name->text == name) {
      if (found != nullptr) {
        throw std::runtime_error(std::string("duplicate mini decoder weight tensor: ") + name);
      }
      found = &entry;
    }
  }
  if (found == nullptr) {
    throw std::runtime_error(std::string("missing mini decoder weight tensor: ") + name);
  }
  return *found;
}

// Copies tensor `name` (`count` floats expected) out of `data`; returns the
// byte offset just past it.
uint64_t extract(const Json &manifest, const std::vector<unsigned char> &data, const char *name,
                 size_t count, const char *kind, std::vector<float> *out) {
  const Json &entry = tensor_entry(manifest, name);
  const uint64_t offset = integer_of(field(entry, "offset"), "offset",
                                     std::numeric_limits<uint64_t>::max());
  const uint64_t listed = integer_of(field(entry, "count"), "count",
                                     std::numeric_limits<uint64_t>::max());
  if (listed != count) {
    throw std::runtime_error(std::string(kind) + " tensor '" + name + "' has unexpected count");
  }
  const uint64_t bytes = checked_multiply(count, sizeof(float), name);
  if (offset > std::numeric_limits<uint64_t>::max() - bytes) {
    throw std::runtime_error(std::string(kind) + " tensor '" + name + "' overflows offset");
  }
  if (offset + bytes > data.size()) {
    throw std::runtime_error(std::string("mini decoder weight tensor '") + name +
                             "' is out of range");
  }
  out->resize(count);
  if (bytes != 0) {
    std::memcpy(out->data(), data.data() + offset, bytes);
  }
  return offset + bytes;
}

struct OutputFile {
  std::unique_ptr<FILE, int (*)(FILE *)> file{nullptr, &std::fclose};
  OutputFile(const std::string &path, const char *what) : file(std::fopen(path.c_str(), "wb"), &std::fclose) {
    if (!file) {
      throw std::runtime_error(std::string(what) + path);
    }
  }
};

// Appends `values` to the data file and its {name, offset, count} entry to
// the manifest text.
void append_tensor(FILE *data, std::string &manifest, const char *name,
                   const std::vector<float> &values, uint64_t &offset) {
  if (offset != 0) {
    manifest += ",\n";
  }
  manifest += "    {\"name\": \"" + std::string(name) + "\", \"offset\": " +
              std::to_string(offset) + ", \"count\": " + std::to_string(values.size()) + "}";
  const size_t bytes = checked_multiply(values.size(), sizeof(float), name);
  if (bytes != 0 && std::fwrite(values.data(), 1, bytes, data) != bytes) {
    throw std::runtime_error(std::string("failed to write mini decoder weight tensor: ") + name);
  }
  if (offset > std::numeric_limits<uint64_t>::max() - bytes) {
    throw std::overflow_error("mini decoder weight data offset overflows");
  }
  offset += bytes;
}

void write_text(const char *path, const std::string &text, const char *create_error,
                const char *write_error) {
  OutputFile out(path, create_error);
  if (std::fwrite(text.data(), 1, text.size(), out.file.get()) != text.size()) {
    throw std::runtime_error(write_error);
  }
}

std::string number(float value) {
  char text[32];
  std::snprintf(text, sizeof(text), "%.9g", static_cast<double>(value));
  std::string out(text);
  if (out.find_first_of(".eEn") == std::string::npos) {
    out += ".0"; // keep JSON numbers of floats recognisable as such
  }
  return out;
}

} // namespace

DecoderLayerWeights load_decoder_layer_weights(const char *manifest_path) {
  if (manifest_path == nullptr || manifest_path[0] == '\0') {
    throw std::invalid_argument("mini decoder weight manifest path is empty");
  }
  const Json manifest = read_manifest(manifest_path);
  if (manifest.kind != Json::Kind::object) {
    throw std::runtime_error("invalid mini decoder weight manifest: root is not an object");
  }
  if (u32_field(manifest, "version") != 2) {
    throw std::runtime_error("unsupported mini decoder weight manifest version");
  }
  const std::string format = string_field(manifest, "format");
  if (format != "lrrt.mini_decoder_weights") {
    throw std::runtime_error("unsupported mini decoder weight manifest format: " + format);
  }
  const std::string dtype = string_field(manifest, "dtype");
  if (dtype != "f32") {
    throw std::runtime_error("unsupported mini decoder weight dtype: " + dtype);
  }
  DecoderLayerWeights w{};
  w.shape.keys = u32_field(manifest, "keys");
  w.shape.hidden = u32_field(manifest, "hidden");
  w.shape.heads = u32_field(manifest, "heads");
  w.shape.kv_heads = manifest.find("kv_heads") != nullptr ? u32_field(manifest, "kv_heads")
                                                          : w.shape.heads;
  w.shape.head_dim = u32_field(manifest, "head_dim");
  w.shape.intermediate = u32_field(manifest, "intermediate");
  if (manifest.find("rope_theta") != nullptr) {
    w.rope_theta = f32_field(manifest, "rope_theta");
  }
  validate_shape(w.shape);
  const std::vector<unsigned char> data =
      read_file(relative_path(manifest_path, string_field(manifest, "data")));
  const size_t hidden = w.shape.hidden, q = w.shape.q_dim(), kv = w.shape.kv_dim(),
               inter = w.shape.intermediate;
  struct Spec {
    const char *name;
    size_t count;
    std::vector<float> *out;
  };
  const Spec specs[] = {
      {"attention_norm_weight", hidden, &w.attention_norm_weight},
      {"mlp_norm_weight", hidden, &w.mlp_norm_weight},
      {"q_weight", checked_multiply(q, hidden, "q_weight"), &w.q_weight},
      {"k_weight", checked_multiply(kv, hidden, "k_weight"), &w.k_weight},
      {"v_weight", checked_multiply(kv, hidden, "v_weight"), &w.v_weight},
      {"q_bias", q, &w.q_bias},
      {"k_bias", kv, &w.k_bias},
      {"v_bias", kv, &w.v_bias},
      {"out_weight", checked_multiply(hidden, q, "out_weight"), &w.out_weight},
      {"gate_weight", checked_multiply(inter, hidden, "gate_weight"), &w.gate_weight},
      {"up_weight", checked_multiply(inter, hidden, "up_weight"), &w.up_weight},
      {"down_weight", checked_multiply(hidden, inter, "down_weight"), &w.down_weight},
  };
  uint64_t used = 0;
  for (const Spec &spec : specs) {
    used = std::max(used, extract(manifest, data, spec.name, spec.count, "mini decoder weight",
                                  spec.out));
  }
  if (used != data.size()) {
    throw std::runtime_error("mini decoder weight data size mismatch");
  }
  return w;
}

ModelTailWeights load_model_tail_weights(const char *manifest_path) {
  if (manifest_path == nullptr || manifest_path[0] == '\0') {
    throw std::invalid_argument("mini model tail manifest path is empty");
  }
  const Json manifest = read_manifest(manifest_path);
  if (manifest.kind != Json::Kind::object) {
    throw std::runtime_error("invalid mini decoder weight manifest: root is not an object");
  }
  if (u32_field(manifest, "version") != 1) {
    throw std::runtime_error("unsupported mini model tail manifest version");
  }
  const std::string format = string_field(manifest, "format");
  if (format != "lrrt.mini_model_tail_weights") {
    throw std::runtime_error("unsupported mini model tail manifest format: " + format);
  }
  const std::string dtype = string_field(manifest, "dtype");
  if (dtype != "f32") {
    throw std::runtime_error("unsupported mini model tail dtype: " + dtype);
  }
  ModelTailWeights w{};
  w.hidden = u32_field(manifest, "hidden");
  w.vocab = u32_field(manifest, "vocab");
  const Json &ids = field(manifest, "token_ids");
  if (ids.kind != Json::Kind::array) {
    throw std::runtime_error("invalid mini decoder weight manifest field: token_ids");
  }
  for (const Json &id : ids.items) {
    w.token_ids.push_back(static_cast<uint32_t>(integer_of(id, "token_ids", kMaxU32)));
  }
  if (w.hidden == 0 || w.vocab == 0 || w.token_ids.empty()) {
    throw std::runtime_error("mini model tail manifest has invalid shape");
  }
  for (const uint32_t id : w.token_ids) {
    if (id >= w.vocab) {
      throw std::runtime_error("mini model tail manifest has invalid token id");
    }
  }
  const std::vector<unsigned char> data =
      read_file(relative_path(manifest_path, string_field(manifest, "data")));
  uint64_t used = 0;
  used = std::max(used, extract(manifest, data, "token_embeddings",
                                checked_multiply(w.token_ids.size(), w.hidden, "token_embeddings"),
                                "mini model tail", &w.token_embeddings));
  used = std::max(used, extract(manifest, data, "final_norm_weight", w.hidden, "mini model tail",
                                &w.final_norm_weight));
  used = std::max(used, extract(manifest, data, "lm_head_weight",
                                checked_multiply(w.vocab, w.hidden, "lm_head_weight"),
                                "mini model tail", &w.lm_head_weight));
  if (used != data.size()) {
    throw std::runtime_error("mini model tail data size mismatch");
  }
  return w;
}

void write_decoder_layer_weights(const char *manifest_path, const char *data_file_name,
                                 const DecoderLayerWeights &w) {
  if (manifest_path == nullptr || manifest_path[0] == '\0' || data_file_name == nullptr ||
      data_file_name[0] == '\0') {
    throw std::invalid_argument("mini decoder weight output path is empty");
  }
  validate_shape(w.shape);
  const size_t hidden = w.shape.hidden, q = w.shape.q_dim(), kv = w.shape.kv_dim(),
               inter = w.shape.intermediate;
  if (!(w.rope_theta > 0.0f) || w.attention_norm_weight.size() != hidden ||
      w.mlp_norm_weight.size() != hidden || w.q_weight.size() != q * hidden ||
      w.k_weight.size() != kv * hidden || w.v_weight.size() != kv * hidden ||
      w.q_bias.size() != q || w.k_bias.size() != kv || w.v_bias.size() != kv ||
      w.out_weight.size() != hidden * q || w.gate_weight.size() != inter * hidden ||
      w.up_weight.size() != inter * hidden || w.down_weight.size() != hidden * inter) {
    throw std::runtime_error("mini decoder weights have invalid tensor sizes");
  }
  const std::string data_path = relative_path(manifest_path, data_file_name);
  OutputFile data(data_path, "failed to create mini decoder weight data file: ");
  std::string manifest = "{\n  \"format\": \"lrrt.mini_decoder_weights\",\n  \"version\": 2,\n"
                         "  \"dtype\": \"f32\",\n  \"data\": \"" + std::string(data_file_name) +
                         "\",\n  \"keys\": " + std::to_string(w.shape.keys) +
                         ",\n  \"hidden\": " + std::to_string(w.shape.hidden) +
                         ",\n  \"heads\": " + std::to_string(w.shape.heads) +
                         ",\n  \"kv_heads\": " + std::to_string(w.shape.kv_heads) +
                         ",\n  \"head_dim\": " + std::to_string(w.shape.head_dim) +
                         ",\n  \"intermediate\": " + std::to_string(w.shape.intermediate) +
                         ",\n  \"rope_theta\": " + number(w.rope_theta) + ",\n  \"tensors\": [\n";
  uint64_t offset = 0;
  append_tensor(data.file.get(), manifest, "attention_norm_weight", w.attention_norm_weight, offset);
  append_tensor(data.file.get(), manifest, "mlp_norm_weight", w.mlp_norm_weight, offset);
  append_tensor(data.file.get(), manifest, "q_weight", w.q_weight, offset);
  append_tensor(data.file.get(), manifest, "k_weight", w.k_weight, offset);
  append_tensor(data.file.get(), manifest, "v_weight", w.v_weight, offset);
  append_tensor(data.file.get(), manifest, "q_bias", w.q_bias, offset);
  append_tensor(data.file.get(), manifest, "k_bias", w.k_bias, offset);
  append_tensor(data.file.get(), manifest, "v_bias", w.v_bias, offset);
  append_tensor(data.file.get(), manifest, "out_weight", w.out_weight, offset);
  append_tensor(data.file.get(), manifest, "gate_weight", w.gate_weight, offset);
  append_tensor(data.file.get(), manifest, "up_weight", w.up_weight, offset);
  append_tensor(data.file.get(), manifest, "down_weight", w.down_weight, offset);
  manifest += "\n  ]\n}\n";
  if (std::fflush(data.file.get()) != 0) {
    throw std::runtime_error("failed to write mini decoder weight data file: " + data_path);
  }
  write_text(manifest_path, manifest, "failed to create mini decoder weight manifest: ",
             "failed to write mini decoder weight manifest");
}

void write_model_tail_weights(const char *manifest_path, const char *data_file_name,
                              const ModelTailWeights &w) {
  if (manifest_path == nullptr || manifest_path[0] == '\0' || data_file_name == nullptr ||
      data_file_name[0] == '\0') {
    throw std::invalid_argument("mini model tail output path is empty");
  }
  if (w.hidden == 0 || w.vocab == 0 || w.token_ids.empty() ||
      w.token_embeddings.size() != w.token_ids.size() * size_t{w.hidden} ||
      w.final_norm_weight.size() != w.hidden ||
      w.lm_head_weight.size() != size_t{w.vocab} * w.hidden) {
    throw std::runtime_error("mini model tail weights have invalid sizes");
  }
  for (const uint32_t id : w.token_ids) {
    if (id >= w.vocab) {
      throw std::runtime_error("mini model tail weights have invalid token id");
    }
  }
  const std::string data_path = relative_path(manifest_path, data_file_name);
  OutputFile data(data_path, "failed to create mini model tail data file: ");
  std::string manifest = "{\n  \"format\": \"lrrt.mini_model_tail_weights\",\n  \"version\": 1,\n"
                         "  \"dtype\": \"f32\",\n  \"data\": \"" + std::string(data_file_name) +
                         "\",\n  \"hidden\": " + std::to_string(w.hidden) +
                         ",\n  \"vocab\": " + std::to_string(w.vocab) + ",\n  \"token_ids\": [";
  for (size_t i = 0; i < w.token_ids.size(); ++i) {
    manifest += (i == 0 ? "" : ", ") + std::to_string(w.token_ids[i]);
  }
  manifest += "],\n  \"tensors\": [\n";
  uint64_t offset = 0;
  append_tensor(data.file.get(), manifest, "token_embeddings", w.token_embeddings, offset);
  append_tensor(data.file.get(), manifest, "final_norm_weight", w.final_norm_weight, offset);
  append_tensor(data.file.get(), manifest, "lm_head_weight", w.lm_head_weight, offset);
  manifest += "\n  ]\n}\n";
  if (std::fflush(data.file.get()) != 0) {
    throw std::runtime_error("failed to write mini model tail data file: " + data_path);
  }
  write_text(manifest_path, manifest, "failed to create mini model tail manifest: ",
             "failed to write mini model tail manifest");
}

} // namespace lrrt::executor::qwen
