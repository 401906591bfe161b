// FP32 weight bundles of the Qwen decode path: one decoder layer
// ("lrrt.mini_decoder_weights", version 2) or the model tail
// ("lrrt.mini_model_tail_weights", version 1), each a JSON manifest next to
// one binary file of little-endian float32 tensors laid end to end.
//
// Format, names, shapes and error texts are those of light-rocm-runtime
// executor/qwen/weight_bundle.hpp:20-758 and tools/convert_qwen_layer.py
// :421-539 (the converter that writes them from Hugging Face checkpoints),
// so bundles written for the reference load unchanged. The usual layout is
// <dir>/layer_<i>/weights.json and <dir>/model_tail/weights.json.
//
// Decoder manifest fields: format, version, dtype ("f32"), data (a relative
// file name inside the manifest's directory), keys, hidden, heads,
// kv_heads (optional, default heads), head_dim, intermediate, rope_theta
// (optional, default 10000), tensors: [{name, offset (bytes), count}] for
// attention_norm_weight, mlp_norm_weight, q/k/v_weight, q/k/v_bias,
// out_weight, gate_weight, up_weight, down_weight (row-major [out][in]).
// Tail manifest fields: format, version, dtype, data, hidden, vocab,
// token_ids (the rows token_embeddings holds), tensors: token_embeddings
// [tokens][hidden], final_norm_weight [hidden], lm_head_weight [vocab][hidden].
#ifndef LRRT_QWEN_WEIGHT_BUNDLE_HPP_
#define LRRT_QWEN_WEIGHT_BUNDLE_HPP_

#include "lrrt/lrrt.h"

#include <cstdint>
#include <vector>

namespace lrrt::executor::qwen {

struct DecoderLayerShape {
  uint32_t keys;
  uint32_t hidden;
  uint32_t heads;
  uint32_t kv_heads;
  uint32_t head_dim;
  uint32_t intermediate;

  uint32_t q_dim() const { return heads * head_dim; }
  uint32_t kv_dim() const { return kv_heads * head_dim; }
  uint32_t qkv_dim() const { return q_dim(); }
};

struct DecoderLayerWeights {
  DecoderLayerShape shape;
  float rope_theta = 10000.0f;
  std::vector<float> attention_norm_weight;
  std::vector<float> mlp_norm_weight;
  std::vector<float> q_weight;
  std::vector<float> k_weight;
  std::vector<float> v_weight;
  std::vector<float> q_bias;
  std::vector<float> k_bias;
  std::vector<float> v_bias;
  std::vector<float> out_weight;
  std::vector<float> gate_weight;
  std::vector<float> up_weight;
  std::vector<float> down_weight;
};

struct ModelTailWeights {
  uint32_t hidden;
  uint32_t vocab;
  std::vector<uint32_t> token_ids;
  std::vector<float> token_embeddings;
  std::vector<float> final_norm_weight;
  std::vector<float> lm_head_weight;
};

LRRT_API DecoderLayerWeights load_decoder_layer_weights(const char *manifest_path);
LRRT_API ModelTailWeights load_model_tail_weights(const char *manifest_path);
// Writes the manifest and, next to it, `data_file_name` (a plain file name).
LRRT_API void write_decoder_layer_weights(const char *manifest_path,
                                          const char *data_file_name,
                                          const DecoderLayerWeights &weights);
LRRT_API void write_model_tail_weights(const char *manifest_path, const char *data_file_name,
                                       const ModelTailWeights &weights);

} // namespace lrrt::executor::qwen

#endif // LRRT_QWEN_WEIGHT_BUNDLE_HPP_
