// Host checks of the FP32 weight bundles (include/lrrt/qwen/weight_bundle.hpp):
// the committed fixture written by the reference's own converter loads with
// the expected shapes and values, our writer round-trips, and malformed
// manifests fail with the reference's messages (light-rocm-runtime
// tests/qwen_weight_bundle.cpp:160-240 checks the same cases).
// Usage: weight_bundle_test <tests/golden/weight_bundles> <scratch dir>
#include "lrrt/qwen/weight_bundle.hpp"

#include <cmath>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <stdexcept>
#include <string>
#include <vector>

namespace wb = lrrt::executor::qwen;

namespace {

int failures = 0;

void expect(bool condition, const char *what) {
  if (!condition) {
    std::fprintf(stderr, "FAILED: %s\n", what);
    ++failures;
  }
}

template <typename Body> void expect_error(Body body, const char *text, const char *what) {
  try {
    body();
  } catch (const std::exception &error) {
    if (std::strstr(error.what(), text) == nullptr) {
      std::fprintf(stderr, "FAILED: %s: '%s' lacks '%s'\n", what, error.what(), text);
      ++failures;
    }
    return;
  }
  std::fprintf(stderr, "FAILED: %s: no error\n", what);
  ++failures;
}

// Element i of the k-th tensor of the fixture (make_weight_bundles.py).
bool matches(const std::vector<float> &v, int k, size_t count) {
  if (v.size() != count) {
    return false;
  }
  for (size_t i = 0; i < count; ++i) {
    const float want = static_cast<float>(k + 1 + 0.001 * static_cast<double>(i % 97));
    if (v[i] != want) {
      return false;
    }
  }
  return true;
}

void write_text(const std::string &path, const std::string &text) {
  std::ofstream(path, std::ios::binary) << text;
}

std::string read_text(const std::string &path) {
  std::ifstream in(path, std::ios::binary);
  return std::string(std::istreambuf_iterator<char>(in), std::istreambuf_iterator<char>());
}

std::string replace(std::string text, const std::string &from, const std::string &to) {
  const size_t at = text.find(from);
  if (at != std::string::npos) {
    text.replace(at, from.size(), to);
  }
  return text;
}

} // namespace

int main(int argc, char **argv) {
  if (argc != 3) {
    std::fprintf(stderr, "usage: %s <fixture dir> <scratch dir>\n", argv[0]);
    return 2;
  }
  const std::string fixture = argv[1], scratch = argv[2];
  try {
    // Reference-written layer bundle.
    const wb::DecoderLayerWeights w =
        wb::load_decoder_layer_weights((fixture + "/layer_0/weights.json").c_str());
    expect(w.shape.keys == 4 && w.shape.hidden == 8 && w.shape.heads == 2 &&
               w.shape.kv_heads == 1 && w.shape.head_dim == 4 && w.shape.intermediate == 12,
           "layer shape");
    expect(w.rope_theta == 1000000.0f, "rope_theta");
    const std::vector<float> *order[] = {&w.attention_norm_weight, &w.mlp_norm_weight,
                                         &w.q_weight,  &w.k_weight,  &w.v_weight,
                                         &w.q_bias,    &w.k_bias,    &w.v_bias,
                                         &w.out_weight, &w.gate_weight, &w.up_weight,
                                         &w.down_weight};
    const size_t counts[] = {8, 8, 64, 32, 32, 8, 4, 4, 64, 96, 96, 96};
    for (int k = 0; k < 12; ++k) {
      expect(matches(*order[k], k, counts[k]), "layer tensor values");
    }
    // Reference-written tail bundle.
    const wb::ModelTailWeights t =
        wb::load_model_tail_weights((fixture + "/model_tail/weights.json").c_str());
    expect(t.hidden == 8 && t.vocab == 10 && t.token_ids == std::vector<uint32_t>({1, 5, 7}),
           "tail shape and token ids");
    expect(matches(t.token_embeddings, 0, 24) && matches(t.final_norm_weight, 1, 8) &&
               matches(t.lm_head_weight, 2, 80),
           "tail tensor values");

    // Our writer round-trips both.
    const std::string layer_manifest = scratch + "/layer.json";
    wb::write_decoder_layer_weights(layer_manifest.c_str(), "layer.bin", w);
    const wb::DecoderLayerWeights again = wb::load_decoder_layer_weights(layer_manifest.c_str());
    expect(again.rope_theta == w.rope_theta && again.q_weight == w.q_weight &&
               again.down_weight == w.down_weight && again.v_bias == w.v_bias,
           "layer round trip");
    const std::string tail_manifest = scratch + "/tail.json";
    wb::write_model_tail_weights(tail_manifest.c_str(), "tail.bin", t);
    const wb::ModelTailWeights tail_again = wb::load_model_tail_weights(tail_manifest.c_str());
    expect(tail_again.token_ids == t.token_ids && tail_again.lm_head_weight == t.lm_head_weight,
           "tail round trip");

    // Malformed manifests (the data file stays next to them).
    const std::string text = read_text(layer_manifest);
    const std::string bad = scratch + "/bad.json";
    auto load_bad = [&] { wb::load_decoder_layer_weights(bad.c_str()); };
    write_text(bad, replace(text, "\"down_weight\"", "\"down_weights\""));
    expect_error(load_bad, "missing mini decoder weight tensor: down_weight", "missing tensor");
    write_text(bad, replace(text, "\"layer.bin\"", "\"../layer.bin\""));
    expect_error(load_bad, "invalid mini decoder weight data path", "data path outside");
    write_text(bad, replace(text, "\"f32\"", "\"bf16\""));
    expect_error(load_bad, "unsupported mini decoder weight dtype: bf16", "dtype");
    write_text(bad, replace(text, "\"version\": 2", "\"version\": 1"));
    expect_error(load_bad, "unsupported mini decoder weight manifest version", "version");
    write_text(bad, replace(text, "\"lrrt.mini_decoder_weights\"", "\"other\""));
    expect_error(load_bad, "unsupported mini decoder weight manifest format: other", "format");
    write_text(bad, replace(text, "\"kv_heads\": 1", "\"kv_heads\": 3"));
    expect_error(load_bad, "invalid GQA shape", "GQA shape");
    write_text(bad, replace(text, "\"head_dim\": 4", "\"head_dim\": 3"));
    expect_error(load_bad, "has invalid shape", "odd head_dim");
    write_text(bad, replace(text, "\"count\": 96}", "\"count\": 95}"));
    expect_error(load_bad, "has unexpected count", "count");
    write_text(bad, replace(text, "\"intermediate\": 12", "\"intermediate\": 11"));
    expect_error(load_bad, "unexpected count", "shape / data disagreement");
    const std::string tail_text = read_text(tail_manifest);
    write_text(bad, replace(tail_text, "[1, 5, 7]", "[1, 5, 10]"));
    expect_error([&] { wb::load_model_tail_weights(bad.c_str()); },
                 "mini model tail manifest has invalid token id", "tail token id");
    write_text(bad, replace(tail_text, "\"version\": 1", "\"version\": 2"));
    expect_error([&] { wb::load_model_tail_weights(bad.c_str()); },
                 "unsupported mini model tail manifest version", "tail version");
    // A data file longer than the tensors it lists.
    {
      std::ofstream(scratch + "/layer.bin", std::ios::binary | std::ios::app) << "pad!";
      expect_error([&] { wb::load_decoder_layer_weights(layer_manifest.c_str()); },
                   "mini decoder weight data size mismatch", "trailing bytes");
    }
    expect_error([] { wb::load_decoder_layer_weights(""); }, "manifest path is empty",
                 "empty path");
  } catch (const std::exception &error) {
    std::fprintf(stderr, "FAILED: %s\n", error.what());
    return 1;
  }
  if (failures == 0) {
    std::printf("weight bundle checks: ok\n");
  }
  return failures == 0 ? 0 : 1;
}
