// Batched multi-stream greedy decode: per-stream caches and counters, the
// step's launch sequence over B stream rows, and its CUDA graph.
#include "batch.hpp"

#include "prefill_common.hpp"

#include <algorithm>

namespace lrrt::qwen::prefill {

using namespace detail;

namespace {

void check_cuda(cudaError_t status, const char *what) {
  if (status != cudaSuccess) {
    throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(status));
  }
}

} // namespace

BatchDecoder::BatchDecoder(Prefill &prefill, const ModelView &model, uint32_t streams,
                           uint32_t capacity, uint32_t max_tokens)
    : prefill_(prefill), streams_(streams), capacity_(capacity), max_tokens_(max_tokens),
      layers_(static_cast<uint32_t>(model.layers.size())) {
  if (streams_ == 0 || streams_ > prefill_.max_chunk_tokens() || capacity_ == 0 ||
      capacity_ > model.capacity || max_tokens_ == 0 || max_tokens_ > capacity_) {
    throw std::invalid_argument(
        "batch needs 1..prefill-chunk streams, capacity <= the model's RoPE rows and "
        "1..capacity tokens per decode");
  }
  // Position splits: as many as one wave of kDecodeBlocksPerSm blocks per SM
  // holds (streams x KV heads x splits blocks), at most one per key tile and
  // at most kDecodeMaximumSplits; each block streams its tiles double
  // buffered.
  const uint32_t tiles = ceil_div(capacity_, kDecodeTileKeys);
  const uint32_t per_head = std::max(1u, kSms * kDecodeBlocksPerSm / (streams_ * qd::kKvHeads));
  splits_ = std::max(1u, std::min({per_head, tiles, kDecodeMaximumSplits}));
  chunk_ = ceil_div(tiles, splits_) * kDecodeTileKeys;
  const size_t cache = size_t{streams_} * layers_ * capacity_ * qd::kKvSize;
  key_cache_.emplace(allocate(sizeof(float) * cache));
  value_cache_.emplace(allocate(sizeof(float) * cache));
  positions_.emplace(allocate(sizeof(uint32_t) * streams_));
  next_tokens_.emplace(allocate(sizeof(uint32_t) * streams_));
  generated_.emplace(allocate(sizeof(uint32_t) * streams_));
  tokens_.emplace(allocate(sizeof(uint32_t) * streams_ * max_tokens_));
  logits_.emplace(allocate(sizeof(float) * streams_ * size_t{model.vocab}));
  logit_values_.emplace(allocate(sizeof(float) * streams_));
  attention_partials_.emplace(allocate(sizeof(float) * streams_ * qd::kKvHeads * splits_ *
                                       qd::kQueriesPerKvHead * kDecodePartialStride));
  candidate_values_.emplace(allocate(sizeof(float) * streams_ * kArgmaxPartitions));
  candidate_indices_.emplace(allocate(sizeof(uint32_t) * streams_ * kArgmaxPartitions));
  arrivals_.emplace(allocate(sizeof(uint32_t) * streams_));
  attention_arrivals_.emplace(allocate(sizeof(uint32_t) * streams_ * qd::kKvHeads));
  // Zeroed caches: rows a stream has not written are never read (each
  // stream attends to its own positions 0..position only).
  const std::vector<unsigned char> zeros(1u << 20, 0);
  for (DeviceBuffer *buffer : {&*key_cache_, &*value_cache_}) {
    for (size_t at = 0; at < buffer->size(); at += zeros.size()) {
      const size_t bytes = std::min(zeros.size(), buffer->size() - at);
      check(lr_memcpy(prefill_.device_.get(), static_cast<unsigned char *>(buffer->data()) + at,
                      zeros.data(), bytes, LR_MEMCPY_HOST_TO_DEVICE),
            "lr_memcpy zero cache");
    }
  }
  positions_host_.assign(streams_, 0);
  next_host_.assign(streams_, 0);
  copy_to_device(*arrivals_, positions_host_.data(), sizeof(uint32_t) * streams_);
  const std::vector<uint32_t> no_arrivals(size_t{streams_} * qd::kKvHeads, 0);
  copy_to_device(*attention_arrivals_, no_arrivals.data(), sizeof(uint32_t) * no_arrivals.size());
  copy_to_device(*positions_, positions_host_.data(), sizeof(uint32_t) * streams_);
  copy_to_device(*next_tokens_, next_host_.data(), sizeof(uint32_t) * streams_);
}

BatchDecoder::~BatchDecoder() {
  if (graph_ != nullptr) {
    lr_synchronize(prefill_.device_.get());
    cudaGraphExecDestroy(graph_);
  }
}

DeviceBuffer BatchDecoder::allocate(size_t bytes) {
  device_bytes_ += bytes;
  return DeviceBuffer(prefill_.device_, std::max<size_t>(bytes, 16));
}

// The model with every layer's cache pointers moved to one stream's cache.
ModelView BatchDecoder::stream_view(const ModelView &model, uint32_t stream) const {
  ModelView view = model;
  view.capacity = capacity_;
  auto *keys = static_cast<float *>(key_cache_->data());
  auto *values = static_cast<float *>(value_cache_->data());
  for (uint32_t layer = 0; layer < layers_; ++layer) {
    const size_t at = (size_t{stream} * layers_ + layer) * capacity_ * qd::kKvSize;
    view.layers[layer].key_cache = keys + at;
    view.layers[layer].value_cache = values + at;
  }
  return view;
}

void BatchDecoder::prefill_stream(const ModelView &model, uint32_t stream, const uint32_t *prompt,
                                  uint32_t count, Path path, uint64_t weights_generation) {
  if (stream >= streams_ || prompt == nullptr || count == 0 || count > capacity_) {
    throw std::invalid_argument("invalid stream prompt");
  }
  if (prompt[count - 1u] >= model.vocab) {
    throw std::invalid_argument("prompt token out of range");
  }
  prefill_.run(stream_view(model, stream), prompt, count - 1u, 0, path, weights_generation);
  positions_host_[stream] = count - 1u;
  next_host_[stream] = prompt[count - 1u];
  copy_to_device(*positions_, positions_host_.data(), sizeof(uint32_t) * streams_);
  copy_to_device(*next_tokens_, next_host_.data(), sizeof(uint32_t) * streams_);
}

// One greedy step of every stream (enqueued on the device's default queue).
void BatchDecoder::enqueue_step(const ModelView &model) {
  Prefill &p = prefill_;
  const uint32_t b = streams_;
  auto *hidden = static_cast<float *>(p.hidden_->data());
  auto *normalized = static_cast<float *>(p.normalized_->data());
  auto *normalized_lo = static_cast<float *>(p.normalized_lo_->data());
  auto *qkv = static_cast<float *>(p.qkv_->data());
  auto *attention = static_cast<float *>(p.attention_->data());
  auto *attention_lo = static_cast<float *>(p.attention_lo_->data());
  auto *activated = static_cast<float *>(p.activated_->data());
  auto *activated_lo = static_cast<float *>(p.activated_lo_->data());
  auto *positions = static_cast<uint32_t *>(positions_->data());
  const uint64_t stream_stride = uint64_t{layers_} * capacity_ * qd::kKvSize;
  auto finish = [&](const PartialTiles &partials, const float *norm_weight) {
    launch(p.finish_rows_.get(), rows_config(b, row_threads(b), staged_bytes(partials, kHidden)),
           FinishArgs{partials, hidden, b, model.epsilon, norm_weight, normalized, normalized_lo});
  };

  launch(p.embed_.get(), rows_config(b, 256),
         EmbedArgs{static_cast<const uint32_t *>(next_tokens_->data()), model.embeddings, hidden,
                   b, model.vocab});
  launch(p.rmsnorm_.get(), rows_config(b, 256),
         NormArgs{hidden, model.layers[0].attention_norm, normalized, normalized_lo, b,
                  model.epsilon});
  for (uint32_t layer = 0; layer < layers_; ++layer) {
    const LayerView &w = model.layers[layer];
    const Prefill::LayerMaps &maps = p.layer_maps_[layer];
    float *keys = static_cast<float *>(key_cache_->data()) + size_t{layer} * capacity_ * qd::kKvSize;
    float *values =
        static_cast<float *>(value_cache_->data()) + size_t{layer} * capacity_ * qd::kKvSize;
    const PartialTiles qkv_partials =
        p.tc_gemm(kQkvTile, p.normalized_maps_, maps.qkv, b, kQkv, kHidden, GemmEpilogue::bias,
                  qkv, nullptr, kQkv, w.qkv_bias, true);
    launch(p.rope_kv_.get(), rows_config(b, row_threads(b), staged_bytes(qkv_partials, kQkv)),
           RopeArgs{qkv, model.rope_cos, model.rope_sin, keys, values, b, 0, qkv_partials,
                    w.qkv_bias, positions, stream_stride});
    const DecodeAttentionArgs attend{qkv,
                                     keys,
                                     values,
                                     stream_stride,
                                     positions,
                                     static_cast<float *>(attention_partials_->data()),
                                     attention,
                                     attention_lo,
                                     b,
                                     splits_,
                                     chunk_,
                                     static_cast<uint32_t *>(attention_arrivals_->data())};
    launch(p.batch_attention_.get(),
           lr_launch_config_t{{splits_ * 256u, qd::kKvHeads, b}, {256, 1, 1}, kDecodeSharedBytes},
           attend);
    finish(p.tc_gemm(kHiddenTile, p.attention_maps_, maps.o, b, kHidden, kHidden,
                     GemmEpilogue::residual, hidden, nullptr, kHidden, nullptr, true),
           w.mlp_norm);
    p.tc_gemm(kGateUpTile, p.normalized_maps_, maps.gate_up, b, kIntermediate, kHidden,
              GemmEpilogue::swiglu, activated, activated_lo, kIntermediate, nullptr, false);
    // The last layer's residual finish applies the final norm for the LM head.
    finish(p.tc_gemm(kHiddenTile, p.activated_maps_, maps.down, b, kHidden, kIntermediate,
                     GemmEpilogue::residual, hidden, nullptr, kHidden, nullptr, true),
           layer + 1u < layers_ ? model.layers[layer + 1u].attention_norm : model.final_norm);
  }
  auto *logits = static_cast<float *>(logits_->data());
  p.tc_gemm(kGateUpTile, p.normalized_maps_, p.tail_maps_, b, model.vocab, kHidden,
            GemmEpilogue::store, logits, nullptr, model.vocab, nullptr, false);
  launch(p.batch_argmax_.get(),
         lr_launch_config_t{{kArgmaxPartitions * 1024u, b, 1}, {1024, 1, 1}, 0},
         ArgmaxArgs{logits, model.vocab, b, static_cast<uint32_t *>(next_tokens_->data()),
                    positions, static_cast<uint32_t *>(generated_->data()),
                    static_cast<uint32_t *>(tokens_->data()), max_tokens_,
                    static_cast<float *>(logit_values_->data()),
                    static_cast<float *>(candidate_values_->data()),
                    static_cast<uint32_t *>(candidate_indices_->data()),
                    static_cast<uint32_t *>(arrivals_->data())});
}

void BatchDecoder::capture_step(const ModelView &model) {
  check_cuda(cudaSetDevice(static_cast<int>(prefill_.device_.index())), "cudaSetDevice");
  void *native = nullptr;
  check(lr_queue_native_handle(prefill_.device_.get(), nullptr, &native),
        "lr_queue_native_handle");
  cudaStream_t stream = static_cast<cudaStream_t>(native);
  prefill_.device_.synchronize();
  check_cuda(cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal),
             "cudaStreamBeginCapture");
  cudaGraph_t graph = nullptr;
  try {
    enqueue_step(model);
  } catch (...) {
    cudaStreamEndCapture(stream, &graph);
    if (graph != nullptr) {
      cudaGraphDestroy(graph);
    }
    throw;
  }
  check_cuda(cudaStreamEndCapture(stream, &graph), "cudaStreamEndCapture");
  const cudaError_t instantiated = cudaGraphInstantiate(&graph_, graph, 0);
  cudaGraphDestroy(graph);
  check_cuda(instantiated, "cudaGraphInstantiate");
}

void BatchDecoder::decode(const ModelView &model, uint32_t steps, uint64_t weights_generation,
                          uint32_t *tokens, float *last_logits) {
  if (steps == 0 || steps > max_tokens_ || tokens == nullptr) {
    throw std::invalid_argument("batch decode needs 1..max_tokens steps and a token buffer");
  }
  for (uint32_t s = 0; s < streams_; ++s) {
    if (uint64_t{positions_host_[s]} + steps > capacity_) {
      throw std::invalid_argument("batch decode exceeds a stream's KV capacity");
    }
  }
  prefill_.device_.synchronize();
  prefill_.prepare_tensor_cores(model, weights_generation);
  prefill_.prepare_tail(model, weights_generation);
  const std::vector<uint32_t> zeros(streams_, 0);
  copy_to_device(*generated_, zeros.data(), sizeof(uint32_t) * streams_);
  const uint32_t zero = 0;
  check(lr_memcpy(prefill_.device_.get(), prefill_.error_->data(), &zero, sizeof(zero),
                  LR_MEMCPY_HOST_TO_DEVICE),
        "lr_memcpy batch error");
  if (graph_ == nullptr) {
    capture_step(model);
  }
  void *native = nullptr;
  check(lr_queue_native_handle(prefill_.device_.get(), nullptr, &native),
        "lr_queue_native_handle");
  for (uint32_t step = 0; step < steps; ++step) {
    check_cuda(cudaGraphLaunch(graph_, static_cast<cudaStream_t>(native)), "cudaGraphLaunch");
  }
  prefill_.device_.synchronize();
  uint32_t error = 0;
  check(lr_memcpy(prefill_.device_.get(), &error, prefill_.error_->data(), sizeof(error),
                  LR_MEMCPY_DEVICE_TO_HOST),
        "lr_memcpy batch error");
  if (error != 0) {
    throw std::runtime_error("batch decode: tensor-core GEMM gave up waiting (code " +
                             std::to_string(error) + ")");
  }
  std::vector<uint32_t> all(size_t{streams_} * max_tokens_);
  copy_to_host(all.data(), *tokens_, sizeof(uint32_t) * all.size());
  for (uint32_t s = 0; s < streams_; ++s) {
    std::copy_n(all.begin() + size_t{s} * max_tokens_, steps, tokens + size_t{s} * steps);
  }
  copy_to_host(positions_host_.data(), *positions_, sizeof(uint32_t) * streams_);
  copy_to_host(next_host_.data(), *next_tokens_, sizeof(uint32_t) * streams_);
  if (last_logits != nullptr) {
    copy_to_host(last_logits, *logit_values_, sizeof(float) * streams_);
  }
}

void BatchDecoder::write_cache(uint32_t stream, uint32_t layer, uint32_t first,
                               uint32_t positions, const float *keys, const float *values) {
  if (stream >= streams_ || layer >= layers_ || first > capacity_ ||
      positions > capacity_ - first) {
    throw std::invalid_argument("invalid cache write");
  }
  const size_t at = ((size_t{stream} * layers_ + layer) * capacity_ + first) * qd::kKvSize;
  const size_t bytes = sizeof(float) * positions * qd::kKvSize;
  if (keys != nullptr) {
    check(lr_memcpy(prefill_.device_.get(), static_cast<float *>(key_cache_->data()) + at, keys,
                    bytes, LR_MEMCPY_HOST_TO_DEVICE),
          "lr_memcpy cache");
  }
  if (values != nullptr) {
    check(lr_memcpy(prefill_.device_.get(), static_cast<float *>(value_cache_->data()) + at,
                    values, bytes, LR_MEMCPY_HOST_TO_DEVICE),
          "lr_memcpy cache");
  }
}

void BatchDecoder::set_next(uint32_t stream, uint32_t position, uint32_t token, uint32_t vocab) {
  if (stream >= streams_ || position >= capacity_ || token >= vocab) {
    throw std::invalid_argument("invalid stream position or token");
  }
  positions_host_[stream] = position;
  next_host_[stream] = token;
  copy_to_device(*positions_, positions_host_.data(), sizeof(uint32_t) * streams_);
  copy_to_device(*next_tokens_, next_host_.data(), sizeof(uint32_t) * streams_);
}

void BatchDecoder::read_cache(uint32_t stream, uint32_t layer, uint32_t positions, float *keys,
                              float *values) {
  if (stream >= streams_ || layer >= layers_ || positions > capacity_) {
    throw std::invalid_argument("invalid cache read");
  }
  const size_t at = (size_t{stream} * layers_ + layer) * capacity_ * qd::kKvSize;
  const size_t bytes = sizeof(float) * positions * qd::kKvSize;
  if (keys != nullptr) {
    check(lr_memcpy(prefill_.device_.get(), keys, static_cast<float *>(key_cache_->data()) + at,
                    bytes, LR_MEMCPY_DEVICE_TO_HOST),
          "lr_memcpy cache");
  }
  if (values != nullptr) {
    check(lr_memcpy(prefill_.device_.get(), values,
                    static_cast<float *>(value_cache_->data()) + at, bytes,
                    LR_MEMCPY_DEVICE_TO_HOST),
          "lr_memcpy cache");
  }
}

} // namespace lrrt::qwen::prefill
