// One Qwen2 decoder layer's decode step composed from per-operation bundles
// (the decoder_ops manifest built next to decoder_ops.cubin) through the
// generic executor (triton_executor.hpp): the B200 counterpart of
// light-rocm-runtime's Triton mini decoder layer
// (examples/triton/mini_decoder_layer.hpp:179-632), restricted to the decode
// step of one token at `position` against a token-major KV cache.
//
// Per step, in order (each a bundle launch on the layer's queue):
//   rmsnorm -> matvec q/k/v (+ bias) -> rope q, rope k -> kv_cache_update ->
//   attention_score (keys 0..position, scale 1/sqrt(head_dim)) ->
//   causal_softmax -> value_aggregation -> matvec o (+ residual) ->
//   rmsnorm -> matvec gate, up -> silu_mul -> matvec down (+ residual).
// Weights are the FP32 weight-bundle layout (lrrt/qwen/weight_bundle.hpp).
#ifndef LRRT_EXECUTOR_TRITON_DECODE_LAYER_HPP_
#define LRRT_EXECUTOR_TRITON_DECODE_LAYER_HPP_

#include "lrrt/executor/triton_executor.hpp"
#include "lrrt/qwen/weight_bundle.hpp"

#include <cmath>
#include <string>
#include <vector>

namespace lrrt::executor::triton {

inline std::shared_ptr<BundleSet> make_decode_layer_bundles(lrrt::Device device,
                                                            const std::string &manifest) {
  auto bundles = std::make_shared<BundleSet>(device);
  for (const char *kernel : {"rmsnorm", "matvec", "rope", "kv_cache_update", "attention_score",
                             "causal_softmax", "value_aggregation", "silu_mul", "vector_add"}) {
    bundles->add(kernel, manifest.c_str(), kernel);
  }
  return bundles;
}

class DecodeLayer {
public:
  DecodeLayer(lrrt::Device device, const std::string &manifest, uint32_t capacity,
              const qwen::DecoderLayerShape &shape, float rope_theta, float epsilon)
      : queue_(device), bundles_(make_decode_layer_bundles(device, manifest)),
        buffers_(device, true), capacity_(capacity), shape_(shape), epsilon_(epsilon) {
    if (shape.heads == 0 || shape.kv_heads == 0 || shape.heads % shape.kv_heads != 0 ||
        shape.head_dim == 0 || shape.head_dim % 2 != 0 || capacity == 0) {
      throw std::runtime_error("decode layer invalid shape");
    }
    const size_t h = shape.hidden, q = shape.q_dim(), kv = shape.kv_dim(),
                 i = shape.intermediate, half = shape.head_dim / 2;
    for (const auto &[name, count] : std::vector<std::pair<const char *, size_t>>{
             {"attention_norm_weight", h}, {"mlp_norm_weight", h}, {"q_weight", q * h},
             {"k_weight", kv * h}, {"v_weight", kv * h}, {"q_bias", q}, {"k_bias", kv},
             {"v_bias", kv}, {"out_weight", h * q}, {"gate_weight", i * h}, {"up_weight", i * h},
             {"down_weight", h * i}, {"k_cache", capacity * kv}, {"v_cache", capacity * kv},
             {"cos", capacity * half}, {"sin", capacity * half}, {"hidden", h},
             {"attention_norm", h}, {"q", q}, {"k", kv}, {"v", kv},
             {"scores", size_t{shape.heads} * capacity}, {"probs", size_t{shape.heads} * capacity},
             {"attention", q}, {"attention_residual", h}, {"mlp_norm", h}, {"gate", i},
             {"up", i}, {"activated", i}, {"out", h}}) {
      buffers_.allocate<float>(name, count);
    }
    buffers_.finalize();
    // RoPE tables: angle = p * theta^(-2f / head_dim) in float.
    std::vector<float> cos_table(capacity * half), sin_table(capacity * half);
    for (uint32_t p = 0; p < capacity; ++p) {
      for (uint32_t f = 0; f < half; ++f) {
        const float exponent = -2.0f * static_cast<float>(f) / static_cast<float>(shape.head_dim);
        const float angle = static_cast<float>(p) * std::pow(rope_theta, exponent);
        cos_table[size_t{p} * half + f] = std::cos(angle);
        sin_table[size_t{p} * half + f] = std::sin(angle);
      }
    }
    buffers_.copy_to("cos", cos_table);
    buffers_.copy_to("sin", sin_table);
    std::vector<float> zeros(capacity * kv, 0.0f);
    buffers_.copy_to("k_cache", zeros);
    buffers_.copy_to("v_cache", zeros);
  }

  void set_weights(const qwen::DecoderLayerWeights &w) {
    const qwen::DecoderLayerShape &s = w.shape;
    if (s.hidden != shape_.hidden || s.heads != shape_.heads || s.kv_heads != shape_.kv_heads ||
        s.head_dim != shape_.head_dim || s.intermediate != shape_.intermediate) {
      throw std::runtime_error("decode layer weights do not match the layer shape");
    }
    buffers_.copy_to("attention_norm_weight", w.attention_norm_weight);
    buffers_.copy_to("mlp_norm_weight", w.mlp_norm_weight);
    buffers_.copy_to("q_weight", w.q_weight);
    buffers_.copy_to("k_weight", w.k_weight);
    buffers_.copy_to("v_weight", w.v_weight);
    buffers_.copy_to("q_bias", w.q_bias);
    buffers_.copy_to("k_bias", w.k_bias);
    buffers_.copy_to("v_bias", w.v_bias);
    buffers_.copy_to("out_weight", w.out_weight);
    buffers_.copy_to("gate_weight", w.gate_weight);
    buffers_.copy_to("up_weight", w.up_weight);
    buffers_.copy_to("down_weight", w.down_weight);
  }

  // Cache rows [first, first + positions), host arrays [positions][kv_dim].
  void set_kv(uint32_t first, uint32_t positions, const float *keys, const float *values) {
    const size_t kv = shape_.kv_dim();
    if (uint64_t{first} + positions > capacity_) {
      throw std::out_of_range("decode layer KV rows exceed the capacity");
    }
    const size_t bytes = sizeof(float) * positions * kv;
    lrrt::check(lr_memcpy(queue_device(), buffers_.ptr<float>("k_cache", first * kv), keys, bytes,
                          LR_MEMCPY_HOST_TO_DEVICE),
                "lr_memcpy k_cache");
    lrrt::check(lr_memcpy(queue_device(), buffers_.ptr<float>("v_cache", first * kv), values,
                          bytes, LR_MEMCPY_HOST_TO_DEVICE),
                "lr_memcpy v_cache");
  }

  // hidden_out = layer(hidden_in) for the token at `position`; writes cache
  // row `position` and attends to rows 0..position. Waits for the queue.
  void step(const std::vector<float> &hidden_in, uint32_t position,
            std::vector<float> &hidden_out) {
    if (position >= capacity_ || hidden_in.size() != shape_.hidden) {
      throw std::out_of_range("decode layer step outside the cache or with a wrong hidden size");
    }
    buffers_.copy_to("hidden", hidden_in);
    const uint32_t h = shape_.hidden, q = shape_.q_dim(), kv = shape_.kv_dim(),
                   i = shape_.intermediate, heads = shape_.heads, kv_heads = shape_.kv_heads,
                   head_dim = shape_.head_dim, keys = position + 1u;
    const float scale = 1.0f / std::sqrt(static_cast<float>(head_dim));
    auto p = [&](const char *name) { return buffers_.ptr<float>(name); };
    auto bundle = [&](const char *name) -> lrrt::Bundle & { return bundles_->get(name); };
    auto rmsnorm = [&](const char *x, const char *weight, const char *out) {
      launch(queue_, bundle("rmsnorm"), h,
             {arg("x", p(x)), arg("weight", p(weight)), arg("out", p(out)), arg("n", h),
              arg("eps", epsilon_)});
    };
    auto matvec = [&](const char *w, const char *x, const char *bias, const char *residual,
                      const char *out, uint32_t rows, uint32_t columns) {
      launch(queue_, bundle("matvec"), rows,
             {arg("w", p(w)), arg("x", p(x)), arg("bias", bias ? p(bias) : nullptr),
              arg("residual", residual ? p(residual) : nullptr), arg("out", p(out)),
              arg("rows", rows), arg("columns", columns)});
    };
    rmsnorm("hidden", "attention_norm_weight", "attention_norm");
    matvec("q_weight", "attention_norm", "q_bias", nullptr, "q", q, h);
    matvec("k_weight", "attention_norm", "k_bias", nullptr, "k", kv, h);
    matvec("v_weight", "attention_norm", "v_bias", nullptr, "v", kv, h);
    for (const auto &[x, count] : {std::pair<const char *, uint32_t>{"q", heads}, {"k", kv_heads}}) {
      launch(queue_, bundle("rope"), count * (head_dim / 2u),
             {arg("x", p(x)), arg("cos", p("cos")), arg("sin", p("sin")), arg("position", position),
              arg("heads", count), arg("head_dim", head_dim)});
    }
    launch(queue_, bundle("kv_cache_update"), kv,
           {arg("k", p("k")), arg("v", p("v")), arg("k_cache", p("k_cache")),
            arg("v_cache", p("v_cache")), arg("position", position), arg("kv_dim", kv)});
    launch(queue_, bundle("attention_score"), heads * keys,
           {arg("q", p("q")), arg("k_cache", p("k_cache")), arg("scores", p("scores")),
            arg("keys", keys), arg("heads", heads), arg("kv_heads", kv_heads),
            arg("head_dim", head_dim), arg("scale", scale)});
    launch(queue_, bundle("causal_softmax"), heads,
           {arg("scores", p("scores")), arg("probs", p("probs")), arg("keys", keys),
            arg("heads", heads)});
    launch(queue_, bundle("value_aggregation"), heads * head_dim,
           {arg("probs", p("probs")), arg("v_cache", p("v_cache")), arg("out", p("attention")),
            arg("keys", keys), arg("heads", heads), arg("kv_heads", kv_heads),
            arg("head_dim", head_dim)});
    matvec("out_weight", "attention", nullptr, "hidden", "attention_residual", h, q);
    rmsnorm("attention_residual", "mlp_norm_weight", "mlp_norm");
    matvec("gate_weight", "mlp_norm", nullptr, nullptr, "gate", i, h);
    matvec("up_weight", "mlp_norm", nullptr, nullptr, "up", i, h);
    launch(queue_, bundle("silu_mul"), i,
           {arg("gate", p("gate")), arg("up", p("up")), arg("out", p("activated")), arg("n", i)});
    matvec("down_weight", "activated", nullptr, "attention_residual", "out", h, i);
    queue_.synchronize();
    hidden_out.resize(h);
    buffers_.copy_from(hidden_out, "out");
  }

  const BufferSet &buffers() const { return buffers_; }

private:
  lr_device_t queue_device() const { return buffers_.get("k_cache").device(); }

  lrrt::Queue queue_;
  std::shared_ptr<BundleSet> bundles_;
  BufferSet buffers_;
  uint32_t capacity_;
  qwen::DecoderLayerShape shape_;
  float epsilon_;
};

} // namespace lrrt::executor::triton

#endif // LRRT_EXECUTOR_TRITON_DECODE_LAYER_HPP_
