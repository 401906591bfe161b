// Batched multi-stream greedy decode on one GPU: B independent streams
// (own KV caches, positions, tokens) share the model's weights, so each
// decode step streams the weights once for all B tokens. A step runs the
// prefill module's kernels over B rows, one row per stream: 3xTF32 GEMMs
// (M = B), RoPE + KV append at each stream's own position and cache, split
// decode attention over each stream's cache, the LM-head GEMM and a
// per-row greedy argmax. The step is captured once as a CUDA graph and
// replayed per token.
//
// light-rocm-runtime decodes one stream per launch (one DecodeState per
// context); this is the batched mode that its single-stream ABI leaves out.
// Per stream the arithmetic is the decode step's (RMSNorm, QKV + bias, RoPE,
// GQA with the inclusive 0..kv_length online softmax, o_proj, SwiGLU, down,
// final norm, LM head with the lower-index tie rule); sums run in GEMM
// order, so logits match single-stream decoding to FP32 rounding.
#ifndef LRRT_B200_QWEN_BATCH_HPP_
#define LRRT_B200_QWEN_BATCH_HPP_

#include "prefill.hpp"

#include <cuda_runtime_api.h>

#include <cstdint>
#include <optional>
#include <vector>

namespace lrrt::qwen::prefill {

class BatchDecoder {
public:
  // streams <= the prefill's chunk size; capacity = KV positions per stream;
  // max_tokens = tokens one decode() call may generate per stream.
  BatchDecoder(Prefill &prefill, const ModelView &model, uint32_t streams, uint32_t capacity,
               uint32_t max_tokens);
  ~BatchDecoder();
  BatchDecoder(const BatchDecoder &) = delete;
  BatchDecoder &operator=(const BatchDecoder &) = delete;

  // Prompt of one stream: positions 0..count-2 through the prefill into the
  // stream's cache, prompt[count-1] becomes its next input token.
  void prefill_stream(const ModelView &model, uint32_t stream, const uint32_t *prompt,
                      uint32_t count, Path path, uint64_t weights_generation);
  // Greedy decode of `steps` tokens for every stream, tokens[stream * steps + i];
  // last_logits (optional, [streams]) receives each stream's last chosen logit.
  void decode(const ModelView &model, uint32_t steps, uint64_t weights_generation,
              uint32_t *tokens, float *last_logits);
  // Writes cache rows [first, first + positions) of one stream and layer
  // ([positions][128] each; keys or values may be null).
  void write_cache(uint32_t stream, uint32_t layer, uint32_t first, uint32_t positions,
                   const float *keys, const float *values);
  // Sets a stream's position and the token it takes as input there (its
  // cache must hold rows 0..position-1).
  void set_next(uint32_t stream, uint32_t position, uint32_t token, uint32_t vocab);
  // Cache rows [0, positions) of one stream and layer, [positions][128] each.
  void read_cache(uint32_t stream, uint32_t layer, uint32_t positions, float *keys,
                  float *values);
  uint32_t position(uint32_t stream) const { return positions_host_.at(stream); }
  uint32_t streams() const { return streams_; }
  uint64_t device_bytes() const { return device_bytes_; }

private:
  DeviceBuffer allocate(size_t bytes);
  ModelView stream_view(const ModelView &model, uint32_t stream) const;
  void capture_step(const ModelView &model);
  void enqueue_step(const ModelView &model);

  Prefill &prefill_;
  uint32_t streams_, capacity_, max_tokens_, layers_;
  uint32_t splits_, chunk_;
  uint64_t device_bytes_ = 0;
  std::optional<DeviceBuffer> key_cache_, value_cache_, positions_, next_tokens_, generated_,
      tokens_, logits_, logit_values_, attention_partials_, candidate_values_,
      candidate_indices_, arrivals_, attention_arrivals_;
  std::vector<uint32_t> positions_host_, next_host_;
  cudaGraphExec_t graph_ = nullptr; // one step; kernels read positions from the device
};

} // namespace lrrt::qwen::prefill

#endif // LRRT_B200_QWEN_BATCH_HPP_
