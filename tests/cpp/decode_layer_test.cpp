// Device check of the generic bundle executor (lrrt/executor/triton_executor.hpp)
// and of one Qwen2 decoder layer's decode step composed from per-operation
// bundles (lrrt/executor/triton_decode_layer.hpp, kernels in
// csrc/kernels/decoder_ops.cu). BASELINE config 1's shapes: hidden 896, 14
// query heads, 2 KV heads, head_dim 64, intermediate 4864, RoPE theta 1e6,
// RMSNorm eps 1e-6, weights N(0, 0.02), norm gains 1, KV cache prefilled with
// 128 positions of N(0, 1), hidden N(0, 1). Usage:
//   decode_layer_test <decoder_ops manifest> [<io directory>]
// Without a directory the weights and inputs come from a local generator and
// the step is checked against the same layer computed in double precision
// here. With one, they are read from raw float32 files in the directory
// (attention_norm, q, k, v, q_bias, k_bias, v_bias, o, mlp_norm, gate, up,
// down, cache_keys [128][128], cache_values, hidden) and the layer output and
// appended key row are written to out.f32 and key.f32 for the caller to check
// (the pytest wrapper compares them with the CPU oracle's decode step).
#include "lrrt/executor/triton_decode_layer.hpp"

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <fstream>
#include <random>
#include <string>
#include <vector>

namespace {

namespace tr = lrrt::executor::triton;
namespace qw = lrrt::executor::qwen;

int failures = 0;

void expect(bool condition, const std::string &what) {
  if (!condition) {
    std::fprintf(stderr, "FAILED: %s\n", what.c_str());
    ++failures;
  }
}

template <typename Body> void expect_throw(Body body, const std::string &needle) {
  try {
    body();
    expect(false, "expected an error containing '" + needle + "'");
  } catch (const std::exception &error) {
    expect(std::string(error.what()).find(needle) != std::string::npos,
           "error '" + std::string(error.what()) + "' contains '" + needle + "'");
  }
}

std::vector<float> normal(std::mt19937 &rng, size_t count, float sigma) {
  std::normal_distribution<float> dist(0.0f, sigma);
  std::vector<float> values(count);
  for (float &v : values) {
    v = dist(rng);
  }
  return values;
}

using Vector = std::vector<double>;

Vector matvec(const std::vector<float> &w, const Vector &x, size_t rows) {
  Vector out(rows, 0.0);
  for (size_t r = 0; r < rows; ++r) {
    for (size_t c = 0; c < x.size(); ++c) {
      out[r] += double(w[r * x.size() + c]) * x[c];
    }
  }
  return out;
}

Vector rmsnorm(const Vector &x, const std::vector<float> &weight, double eps) {
  double sum = 0.0;
  for (double v : x) {
    sum += v * v;
  }
  const double inverse = 1.0 / std::sqrt(sum / x.size() + eps);
  Vector out(x.size());
  for (size_t i = 0; i < x.size(); ++i) {
    out[i] = x[i] * inverse * weight[i];
  }
  return out;
}

// The layer in double precision; `keys` and `values` are the cache rows
// [position][kv_dim] before this step; returns the layer output and the
// appended (rotated) key row.
Vector reference_step(const qw::DecoderLayerWeights &w, const Vector &hidden,
                      std::vector<Vector> keys, std::vector<Vector> values, uint32_t position,
                      float theta, double eps, Vector *key_row) {
  const auto &s = w.shape;
  const size_t half = s.head_dim / 2;
  const Vector norm = rmsnorm(hidden, w.attention_norm_weight, eps);
  Vector q = matvec(w.q_weight, norm, s.q_dim()), k = matvec(w.k_weight, norm, s.kv_dim()),
         v = matvec(w.v_weight, norm, s.kv_dim());
  for (size_t i = 0; i < q.size(); ++i) q[i] += w.q_bias[i];
  for (size_t i = 0; i < k.size(); ++i) k[i] += w.k_bias[i], v[i] += w.v_bias[i];
  auto rope = [&](Vector &x, uint32_t heads) {
    for (uint32_t h = 0; h < heads; ++h) {
      for (size_t f = 0; f < half; ++f) {
        // The tables are float on the device; use the same float angle.
        const float exponent = -2.0f * float(f) / float(s.head_dim);
        const float angle = float(position) * std::pow(theta, exponent);
        const double c = std::cos(angle), sn = std::sin(angle);
        const double x0 = x[h * s.head_dim + f], x1 = x[h * s.head_dim + f + half];
        x[h * s.head_dim + f] = x0 * c - x1 * sn;
        x[h * s.head_dim + f + half] = x1 * c + x0 * sn;
      }
    }
  };
  rope(q, s.heads);
  rope(k, s.kv_heads);
  *key_row = k;
  keys.push_back(k);
  values.push_back(v);
  Vector attention(s.q_dim(), 0.0);
  const uint32_t group_size = s.heads / s.kv_heads;
  for (uint32_t h = 0; h < s.heads; ++h) {
    const uint32_t g = h / group_size;
    std::vector<double> scores(keys.size());
    double maximum = -INFINITY;
    for (size_t p = 0; p < keys.size(); ++p) {
      double dot = 0.0;
      for (uint32_t d = 0; d < s.head_dim; ++d) {
        dot += q[h * s.head_dim + d] * keys[p][g * s.head_dim + d];
      }
      scores[p] = dot / std::sqrt(double(s.head_dim));
      maximum = std::max(maximum, scores[p]);
    }
    double total = 0.0;
    for (double &score : scores) {
      score = std::exp(score - maximum);
      total += score;
    }
    for (size_t p = 0; p < keys.size(); ++p) {
      for (uint32_t d = 0; d < s.head_dim; ++d) {
        attention[h * s.head_dim + d] += scores[p] / total * values[p][g * s.head_dim + d];
      }
    }
  }
  Vector residual = matvec(w.out_weight, attention, s.hidden);
  for (size_t i = 0; i < residual.size(); ++i) residual[i] += hidden[i];
  const Vector mlp = rmsnorm(residual, w.mlp_norm_weight, eps);
  const Vector gate = matvec(w.gate_weight, mlp, s.intermediate),
               up = matvec(w.up_weight, mlp, s.intermediate);
  Vector activated(s.intermediate);
  for (size_t i = 0; i < activated.size(); ++i) {
    activated[i] = gate[i] / (1.0 + std::exp(-gate[i])) * up[i];
  }
  Vector out = matvec(w.down_weight, activated, s.hidden);
  for (size_t i = 0; i < out.size(); ++i) out[i] += residual[i];
  return out;
}

std::vector<float> read_floats(const std::string &path, size_t count) {
  std::vector<float> values(count);
  std::ifstream in(path, std::ios::binary);
  in.read(reinterpret_cast<char *>(values.data()),
          static_cast<std::streamsize>(count * sizeof(float)));
  if (!in || in.gcount() != static_cast<std::streamsize>(count * sizeof(float))) {
    throw std::runtime_error("cannot read " + std::to_string(count) + " floats from " + path);
  }
  return values;
}

void write_floats(const std::string &path, const std::vector<float> &values) {
  std::ofstream out(path, std::ios::binary);
  out.write(reinterpret_cast<const char *>(values.data()),
            static_cast<std::streamsize>(values.size() * sizeof(float)));
  if (!out) {
    throw std::runtime_error("cannot write " + path);
  }
}

double relative_error(const std::vector<float> &got, const Vector &want) {
  double scale = 0.0, worst = 0.0;
  for (size_t i = 0; i < want.size(); ++i) {
    scale = std::max(scale, std::abs(want[i]));
    worst = std::max(worst, std::abs(double(got[i]) - want[i]));
  }
  return worst / std::max(scale, 1e-30);
}

} // namespace

int main(int argc, char **argv) {
  if (argc != 2 && argc != 3) {
    std::fprintf(stderr, "usage: %s <decoder_ops manifest> [<io directory>]\n", argv[0]);
    return 2;
  }
  const std::string io = argc == 3 ? std::string(argv[2]) + "/" : std::string();
  try {
    lrrt::Runtime runtime;
    if (runtime.device_count() == 0) {
      std::fprintf(stderr, "no CUDA device\n");
      return 2;
    }
    lrrt::Device device = runtime.open_device(0);

    // Executor API: names, arena layout and the reference's error texts.
    tr::BundleSet bundles(device);
    bundles.add("norm", argv[1], "rmsnorm");
    expect_throw([&] { bundles.get("missing"); },
                 "unknown Triton executor bundle 'missing'; available bundles: norm");
    expect_throw([&] { bundles.add("bad", argv[1], "no_such_kernel"); },
                 "failed to load Triton executor bundle 'bad'");
    tr::BufferSet arena(device, true);
    arena.allocate<float>("a", 3);
    arena.allocate<float>("b", 100);
    expect_throw([&] { arena.get("a"); }, "Triton executor buffer set is not finalized");
    arena.finalize();
    expect(arena.byte_offset("a") == 0 && arena.byte_offset("b") == 256, "arena offsets");
    expect(arena.arena_size() == 256 + 400, "arena size");
    expect_throw([&] { arena.allocate<float>("c", 1); },
                 "Triton executor arena buffer set is finalized");
    expect_throw([&] { arena.get("zz"); }, "unknown Triton executor buffer 'zz'");
    expect_throw([&] { tr::arg("", 1u); }, "Triton executor launch argument name is empty");
    lrrt::Queue queue(device);
    expect_throw(
        [&] {
          tr::launch(queue, bundles.get("norm"), 1, {tr::arg("n", 1u), tr::arg("n", 2u)});
        },
        "duplicate Triton executor launch argument 'n' for kernel rmsnorm (ops_rmsnorm_f32)");
    expect_throw([&] { tr::launch(queue, bundles.get("norm"), 1, {tr::arg("nope", 1u)}); },
                 "failed to bind Triton executor launch argument 'nope'");

    // One decoder layer's decode step at position 128 (config 1).
    const uint32_t capacity = 256, position = 128;
    const float theta = 1.0e6f, eps = 1.0e-6f;
    qw::DecoderLayerWeights w;
    w.shape = qw::DecoderLayerShape{capacity, 896, 14, 2, 64, 4864};
    w.rope_theta = theta;
    std::mt19937 rng(0);
    const auto &s = w.shape;
    if (!io.empty()) {
      // Weights and inputs from the caller; outputs back to it.
      const size_t h = s.hidden, q = s.q_dim(), kv = s.kv_dim(), i = s.intermediate;
      w.attention_norm_weight = read_floats(io + "attention_norm", h);
      w.mlp_norm_weight = read_floats(io + "mlp_norm", h);
      w.q_weight = read_floats(io + "q", q * h);
      w.k_weight = read_floats(io + "k", kv * h);
      w.v_weight = read_floats(io + "v", kv * h);
      w.q_bias = read_floats(io + "q_bias", q);
      w.k_bias = read_floats(io + "k_bias", kv);
      w.v_bias = read_floats(io + "v_bias", kv);
      w.out_weight = read_floats(io + "o", h * q);
      w.gate_weight = read_floats(io + "gate", i * h);
      w.up_weight = read_floats(io + "up", i * h);
      w.down_weight = read_floats(io + "down", h * i);
      const std::vector<float> keys = read_floats(io + "cache_keys", size_t{position} * kv);
      const std::vector<float> values = read_floats(io + "cache_values", size_t{position} * kv);
      const std::vector<float> input = read_floats(io + "hidden", h);
      tr::DecodeLayer layer(device, argv[1], capacity, s, theta, eps);
      layer.set_weights(w);
      layer.set_kv(0, position, keys.data(), values.data());
      std::vector<float> out;
      layer.step(input, position, out);
      std::vector<float> k_cache(size_t{capacity} * kv);
      layer.buffers().copy_from(k_cache, "k_cache");
      write_floats(io + "out.f32", out);
      write_floats(io + "key.f32",
                   std::vector<float>(k_cache.begin() + size_t{position} * kv,
                                      k_cache.begin() + size_t{position + 1} * kv));
    }
    w.attention_norm_weight.assign(s.hidden, 1.0f);
    w.mlp_norm_weight.assign(s.hidden, 1.0f);
    w.q_weight = normal(rng, s.q_dim() * s.hidden, 0.02f);
    w.k_weight = normal(rng, s.kv_dim() * s.hidden, 0.02f);
    w.v_weight = normal(rng, s.kv_dim() * s.hidden, 0.02f);
    w.q_bias = normal(rng, s.q_dim(), 0.02f);
    w.k_bias = normal(rng, s.kv_dim(), 0.02f);
    w.v_bias = normal(rng, s.kv_dim(), 0.02f);
    w.out_weight = normal(rng, s.hidden * s.q_dim(), 0.02f);
    w.gate_weight = normal(rng, size_t{s.intermediate} * s.hidden, 0.02f);
    w.up_weight = normal(rng, size_t{s.intermediate} * s.hidden, 0.02f);
    w.down_weight = normal(rng, size_t{s.hidden} * s.intermediate, 0.02f);
    const std::vector<float> cache_keys = normal(rng, size_t{position} * s.kv_dim(), 1.0f);
    const std::vector<float> cache_values = normal(rng, size_t{position} * s.kv_dim(), 1.0f);
    const std::vector<float> hidden = normal(rng, s.hidden, 1.0f);

    tr::DecodeLayer layer(device, argv[1], capacity, s, theta, eps);
    layer.set_weights(w);
    layer.set_kv(0, position, cache_keys.data(), cache_values.data());
    std::vector<float> out;
    layer.step(hidden, position, out);

    std::vector<Vector> keys(position), values(position);
    for (uint32_t p = 0; p < position; ++p) {
      keys[p].assign(cache_keys.begin() + size_t{p} * s.kv_dim(),
                     cache_keys.begin() + size_t{p + 1} * s.kv_dim());
      values[p].assign(cache_values.begin() + size_t{p} * s.kv_dim(),
                       cache_values.begin() + size_t{p + 1} * s.kv_dim());
    }
    Vector key_row;
    const Vector want = reference_step(w, Vector(hidden.begin(), hidden.end()), keys, values,
                                       position, theta, eps, &key_row);
    const double error = relative_error(out, want);
    std::vector<float> k_cache(size_t{capacity} * s.kv_dim());
    layer.buffers().copy_from(k_cache, "k_cache");
    const std::vector<float> appended(k_cache.begin() + size_t{position} * s.kv_dim(),
                                      k_cache.begin() + size_t{position + 1} * s.kv_dim());
    const double key_error = relative_error(appended, key_row);
    std::printf("decode layer: output max relative error %.3e, appended key %.3e\n", error,
                key_error);
    expect(error <= 1.0e-4, "layer output within 1e-4 of the double-precision reference");
    expect(key_error <= 1.0e-4, "appended key row within 1e-4");
  } catch (const std::exception &error) {
    std::fprintf(stderr, "error: %s\n", error.what());
    return 1;
  }
  if (failures != 0) {
    return 1;
  }
  std::printf("decode layer checks: ok\n");
  return 0;
}
