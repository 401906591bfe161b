// Host side of the prompt prefill: chunk buffers, the 3xTF32 operand copies
// and tensor maps, and the launch sequence of one chunk through all layers.
#include "prefill.hpp"

#include "prefill_common.hpp"

#include <algorithm>

namespace lrrt::qwen::prefill {

using namespace detail;

Prefill::Prefill(Device device, const void *image, size_t image_size, uint32_t max_chunk_tokens)
    : device_(device), module_(device, image, image_size), embed_(module_.kernel("prefill_embed")),
      rmsnorm_(module_.kernel("prefill_rmsnorm")), rope_kv_(module_.kernel("prefill_rope_kv")),
      attend_(module_.kernel("prefill_attention")),
      attend_tc_(module_.kernel("prefill_attention_tc")), reduce_(module_.kernel("prefill_reduce")),
      split_(module_.kernel("prefill_split")), gemm_bias_(module_.kernel("prefill_gemm_bias")),
      gemm_residual_(module_.kernel("prefill_gemm_residual")),
      gemm_swiglu_(module_.kernel("prefill_gemm_swiglu")),
      tc_n192_(module_.kernel("prefill_tc_gemm_n192")),
      tc_n224_(module_.kernel("prefill_tc_gemm_n224")),
      tc_n256_(module_.kernel("prefill_tc_gemm_n256")),
      tc_pair288_(module_.kernel("prefill_tc_gemm_pair288")),
      tc_narrow_(module_.kernel("prefill_tc_narrow")),
      tc_narrow_pair_(module_.kernel("prefill_tc_narrow_pair")),
      tc_narrow_shared_sm_(module_.kernel("prefill_tc_narrow_shared_sm")),
      finish_rows_(module_.kernel("prefill_finish_rows")),
      batch_attention_(module_.kernel("batch_attention")),
      batch_argmax_(module_.kernel("batch_argmax")), chunk_(max_chunk_tokens) {
  if (chunk_ == 0 || chunk_ > 8192) {
    throw std::invalid_argument("prefill chunk must be 1..8192 tokens");
  }
  // Every kernel of the module waits for its predecessor before reading
  // device data (griddepcontrol.wait), so all of them may launch overlapped:
  // a kernel's prologue (barrier setup, TMEM allocation) runs while the
  // previous kernel drains.
  for (const Kernel *kernel :
       {&embed_, &rmsnorm_, &rope_kv_, &attend_, &attend_tc_, &reduce_, &split_, &gemm_bias_, &gemm_residual_,
        &gemm_swiglu_, &tc_n192_, &tc_n224_, &tc_n256_, &tc_pair288_, &tc_narrow_,
        &tc_narrow_pair_, &tc_narrow_shared_sm_,
        &finish_rows_, &batch_attention_, &batch_argmax_}) {
    check(lr_kernel_set_overlapped(kernel->get(), 1), "lr_kernel_set_overlapped");
  }
  const size_t c = chunk_;
  hidden_.emplace(allocate(sizeof(float) * c * kHidden));
  normalized_.emplace(allocate(sizeof(float) * c * kHidden));
  normalized_lo_.emplace(allocate(sizeof(float) * c * kHidden));
  qkv_.emplace(allocate(sizeof(float) * c * kQkv));
  attention_.emplace(allocate(sizeof(float) * c * kHidden));
  attention_lo_.emplace(allocate(sizeof(float) * c * kHidden));
  activated_.emplace(allocate(sizeof(float) * c * kIntermediate));
  activated_lo_.emplace(allocate(sizeof(float) * c * kIntermediate));
  // Split-K partials: at most one 128 x 256 tile per SM in flight.
  partials_.emplace(allocate(sizeof(float) * kSms * kTcTileM * kTcPairN));
  error_.emplace(allocate(sizeof(uint32_t)));
  // Attention: per (row tile, head) the key chunks' softmax states, and the
  // arrival counters (zero; the last chunk block resets its counter).
  // Sized for the larger of the two row tilings (64-row SIMT tiles,
  // 128-row tensor-core tiles); counters for the finer one.
  const size_t row_tiles = ceil_div(chunk_, kAttentionTileRows);
  const size_t tiled_rows = std::max<size_t>(row_tiles * kAttentionTileRows,
                                             ceil_div(chunk_, kTcAttentionRows) * kTcAttentionRows);
  attention_partials_.emplace(allocate(sizeof(float) * tiled_rows * qd::kAttentionHeads *
                                       kAttentionMaximumChunks * kAttentionPartialStride));
  attention_arrivals_.emplace(allocate(sizeof(uint32_t) * row_tiles * qd::kAttentionHeads));
  const std::vector<uint32_t> no_arrivals(row_tiles * qd::kAttentionHeads, 0u);
  check(lr_memcpy(device_.get(), attention_arrivals_->data(), no_arrivals.data(),
                  sizeof(uint32_t) * no_arrivals.size(), LR_MEMCPY_HOST_TO_DEVICE),
        "lr_memcpy attention arrivals");
}

DeviceBuffer Prefill::allocate(size_t bytes) {
  device_bytes_ += bytes;
  return DeviceBuffer(device_, std::max<size_t>(bytes, 16));
}

namespace {

// Maps of a (hi, lo) activation pair [rows][columns]: 128-row boxes (the
// wide kernels' A operand) and kNarrowRows-row boxes (the narrow kernels' B).
OperandMaps activation_maps(const float *hi, const float *lo, uint64_t rows,
                                     uint64_t columns) {
  OperandMaps maps;
  maps.wide[0] = map_2d(hi, rows, columns, kTcTileM);
  maps.wide[1] = map_2d(lo, rows, columns, kTcTileM);
  maps.narrow[0] = map_2d(hi, rows, columns, kNarrowRows);
  maps.narrow[1] = map_2d(lo, rows, columns, kNarrowRows);
  return maps;
}

// Maps of a weight matrix [rows][columns]: over its (hi, lo) pair, boxes of
// half a tile_columns-wide tile (the wide kernels' B operand); over the FP32
// weights themselves, kNarrowTileN-row boxes (the narrow kernels' A, which
// they split into the TF32 pair in shared memory).
OperandMaps weight_maps(const float *hi, const float *lo, const float *weights, uint64_t rows,
                        uint64_t columns, uint32_t tile_columns) {
  OperandMaps maps;
  maps.wide[0] = map_2d(hi, rows, columns, tile_columns / 2u);
  maps.wide[1] = map_2d(lo, rows, columns, tile_columns / 2u);
  maps.narrow[0] = map_2d(weights, rows, columns, kNarrowTileN);
  return maps;
}

} // namespace

// (Re)builds the TF32 (hi, lo) weight copies when the weights changed since
// the last split, and the tensor maps over them and the chunk operands.
void Prefill::prepare_tensor_cores(const ModelView &model, uint64_t weights_generation) {
  const size_t layers = model.layers.size();
  if (!split_weights_ || split_weights_->size() < sizeof(float) * 2 * kLayerFloats * layers) {
    split_weights_.reset();
    split_weights_.emplace(allocate(sizeof(float) * 2 * kLayerFloats * layers));
    split_generation_ = UINT64_MAX;
  }
  if (split_generation_ == weights_generation && split_source_ == model.layers[0].qkv &&
      layer_maps_.size() == layers) {
    return;
  }
  if (cudaSetDevice(static_cast<int>(device_.index())) != cudaSuccess) {
    throw std::runtime_error("cudaSetDevice failed");
  }
  const size_t c = chunk_;
  auto *hi_lo = static_cast<float *>(split_weights_->data());
  normalized_maps_ = activation_maps(static_cast<float *>(normalized_->data()),
                                     static_cast<float *>(normalized_lo_->data()), c, kHidden);
  attention_maps_ = activation_maps(static_cast<float *>(attention_->data()),
                                    static_cast<float *>(attention_lo_->data()), c, kHidden);
  activated_maps_ = activation_maps(static_cast<float *>(activated_->data()),
                                    static_cast<float *>(activated_lo_->data()), c, kIntermediate);
  layer_maps_.assign(layers, LayerMaps{});
  for (size_t layer = 0; layer < layers; ++layer) {
    const LayerView &w = model.layers[layer];
    float *hi = hi_lo + layer * 2 * kLayerFloats;
    float *lo = hi + kLayerFloats;
    const struct {
      const float *source;
      size_t offset, floats;
    } parts[] = {{w.qkv, 0, kQkvFloats},
                 {w.o, kQkvFloats, kOFloats},
                 {w.gate_up, kQkvFloats + kOFloats, kGateUpFloats},
                 {w.down, kQkvFloats + kOFloats + kGateUpFloats, kDownFloats}};
    for (const auto &part : parts) {
      const SplitArgs args{part.source, hi + part.offset, lo + part.offset, part.floats};
      launch(split_.get(), rows_config(std::min<uint32_t>(ceil_div(part.floats, 256), kSms * 8), 256),
             args);
    }
    LayerMaps &maps = layer_maps_[layer];
    const size_t gate_up = kQkvFloats + kOFloats, down = gate_up + kGateUpFloats;
    maps.qkv = weight_maps(hi, lo, w.qkv, kQkv, kHidden, kQkvTile);
    maps.o = weight_maps(hi + kQkvFloats, lo + kQkvFloats, w.o, kHidden, kHidden, kHiddenTile);
    maps.gate_up = weight_maps(hi + gate_up, lo + gate_up, w.gate_up, 2 * kIntermediate, kHidden,
                               kGateUpTile);
    maps.gate_up_pair =
        weight_maps(hi + gate_up, lo + gate_up, w.gate_up, 2 * kIntermediate, kHidden, kTcPairN);
    maps.down = weight_maps(hi + down, lo + down, w.down, kHidden, kIntermediate, kHiddenTile);
  }
  split_generation_ = weights_generation;
  split_source_ = model.layers[0].qkv;
}

void Prefill::prepare_tail(const ModelView &model, uint64_t weights_generation) {
  const uint64_t floats = uint64_t{model.vocab} * kHidden;
  if (!tail_split_ || tail_split_->size() < sizeof(float) * 2 * floats) {
    tail_split_.reset();
    tail_split_.emplace(allocate(sizeof(float) * 2 * floats));
    tail_generation_ = UINT64_MAX;
  }
  if (tail_generation_ == weights_generation && tail_source_ == model.lm_head) {
    return;
  }
  if (cudaSetDevice(static_cast<int>(device_.index())) != cudaSuccess) {
    throw std::runtime_error("cudaSetDevice failed");
  }
  auto *hi = static_cast<float *>(tail_split_->data());
  launch(split_.get(), rows_config(std::min<uint32_t>(ceil_div(floats, 256), kSms * 8), 256),
         SplitArgs{model.lm_head, hi, hi + floats, floats});
  tail_maps_ = weight_maps(hi, hi + floats, model.lm_head, model.vocab, kHidden, kGateUpTile);
  tail_generation_ = weights_generation;
  tail_source_ = model.lm_head;
}

// One 3xTF32 GEMM C = A . B^T over m chunk rows with tile_columns-wide
// tensor-core tiles. With `defer` and fewer tiles than SMs, every tile runs
// split along K into partial accumulators and the caller's next row kernel
// finishes them (the returned PartialTiles). Otherwise whole waves of kSms
// tiles run data-parallel with the epilogue in the GEMM, and the tiles of a
// last partial wave (or all tiles, when there are fewer than kSms) are split
// along K so that the launch fills the SMs, and prefill_reduce sums their
// partials in split order. At most kNarrowRows rows run the narrow
// (swapped-operand) kernels under the same schedule; tile_columns then
// follows from them.
PartialTiles Prefill::tc_gemm(uint32_t tile_columns, const OperandMaps &a, const OperandMaps &b,
                              uint32_t m, uint32_t n, uint32_t k, GemmEpilogue mode, float *c,
                              float *c_lo, uint32_t ldc, const float *bias, bool defer) {
  const bool swiglu = mode == GemmEpilogue::swiglu;
  // At most kNarrowRows rows: the swapped-operand kernels, whose tiles are
  // kNarrowTileN output columns (paired with the up columns for swiglu).
  const bool narrow = m <= kNarrowRows;
  if (narrow) {
    tile_columns = swiglu ? 2u * kNarrowTileN : kNarrowTileN;
  }
  const uint32_t tile_rows = narrow ? kNarrowRows : kTcTileM;
  const uint32_t out_columns = swiglu ? tile_columns / 2u : tile_columns;
  const uint32_t n_tiles = ceil_div(n, out_columns);
  const uint32_t tiles = n_tiles * ceil_div(m, tile_rows);
  const uint32_t k_tiles = k / kTcTileK;
  if (!narrow && tile_columns == kTcPairN && !swiglu) {
    throw std::invalid_argument("288-column tiles are gate/up pairs");
  }
  // Narrow launches of more than one wave of tiles (not swiglu) share SMs.
  const bool shared_sm = narrow && !swiglu && tiles > kSms;
  const Kernel &kernel = narrow ? (swiglu ? tc_narrow_pair_ : shared_sm ? tc_narrow_shared_sm_ : tc_narrow_)
                         : tile_columns == 192      ? tc_n192_
                         : tile_columns == 224      ? tc_n224_
                         : tile_columns == kTcPairN ? tc_pair288_
                                                    : tc_n256_;
  const uint32_t shared =
      narrow ? tc_narrow_shared_bytes(swiglu, shared_sm) : tc_shared_bytes(tile_columns);
  TcGemmArgs args{};
  // The narrow kernels take the weights as the MMA's A operand.
  args.a_hi = narrow ? b.narrow[0] : a.wide[0];
  args.a_lo = narrow ? TensorMap{} : a.wide[1]; // narrow: the kernel splits the weights
  args.b_hi = narrow ? a.narrow[0] : b.wide[0];
  args.b_lo = narrow ? a.narrow[1] : b.wide[1];
  args.m = m;
  args.n = n;
  args.k = k;
  args.ldc = ldc;
  args.n_tiles = n_tiles;
  args.n_gate_offset = swiglu ? n : 0u;
  args.wait_limit_ms = kWaitLimitMs;
  args.error = static_cast<uint32_t *>(error_->data());
  auto *partials = static_cast<float *>(partials_->data());
  auto run = [&](uint32_t offset, uint32_t count, uint32_t splits, bool finish) {
    const bool partial = splits > 1 || !finish;
    args.tile_offset = offset;
    args.tile_count = count;
    args.splits = splits;
    args.mode = static_cast<uint32_t>(partial ? GemmEpilogue::partial : mode);
    args.c = partial ? partials : c;
    args.c_lo = partial ? nullptr : c_lo;
    args.bias = bias;
    const lr_launch_config_t config{{count * kTcThreads, 1, splits}, {kTcThreads, 1, 1}, shared};
    launch(kernel.get(), config, args);
    if (partial && finish) {
      const ReduceArgs reduce{partials, bias,   c,      c_lo,   m,
                              n,        ldc,    static_cast<uint32_t>(mode),
                              offset,   count,  n_tiles, splits, tile_columns,
                              tile_rows};
      launch(reduce_.get(),
             rows_config(ceil_div(uint64_t{count} * tile_rows * out_columns, 256), 256), reduce);
    }
  };
  const uint32_t small_splits = std::max(
      1u, std::min({kSms / std::max(tiles, 1u), k_tiles / 4u, kMaximumDeferredSplits}));
  if (defer && !swiglu && tiles <= kSms) {
    run(0, tiles, small_splits, false);
    return PartialTiles{partials, small_splits, n_tiles, tiles, tile_columns, tile_rows};
  }
  if (tiles >= kSms) {
    const uint32_t full = tiles / kSms * kSms;
    run(0, full, 1, true);
    if (tiles > full) {
      // A few leftover tiles: split K to spread them over the SMs, keeping
      // each slice at least four K steps long (shorter slices spend their
      // time filling the pipeline and writing partials).
      const uint32_t rest = tiles - full;
      run(full, rest, std::max(1u, std::min(kSms / rest, k_tiles / 4u)), true);
    }
  } else {
    run(0, tiles, small_splits, true);
  }
  return PartialTiles{nullptr, 0, 0, 0, 0, 0};
}

void Prefill::run_chunk(const ModelView &model, uint32_t count, uint32_t first_position,
                        Path path) {
  const bool tc = path == Path::tf32x3;
  auto *hidden = static_cast<float *>(hidden_->data());
  auto *normalized = static_cast<float *>(normalized_->data());
  auto *normalized_lo = tc ? static_cast<float *>(normalized_lo_->data()) : nullptr;
  auto *qkv = static_cast<float *>(qkv_->data());
  auto *attention = static_cast<float *>(attention_->data());
  auto *attention_lo = tc ? static_cast<float *>(attention_lo_->data()) : nullptr;
  auto *activated = static_cast<float *>(activated_->data());
  auto *activated_lo = tc ? static_cast<float *>(activated_lo_->data()) : nullptr;
  const uint32_t m_tiles = ceil_div(count, 128);
  const PartialTiles direct{nullptr, 0, 0, 0, 0, 0};
  auto simt = [&](const Kernel &kernel, const GemmArgs &args, uint32_t n_tiles) {
    const lr_launch_config_t config{{n_tiles * 256u, m_tiles, 1}, {256, 1, 1}, 0};
    launch(kernel.get(), config, args);
  };
  // Residual finish of o_proj / down (from partial sums, when deferred) and
  // the next RMSNorm of the same rows.
  auto finish = [&](const PartialTiles &partials, const float *norm_weight) {
    launch(finish_rows_.get(),
           rows_config(count, row_threads(count), staged_bytes(partials, kHidden)),
           FinishArgs{partials, hidden, count, model.epsilon, norm_weight, normalized,
                      normalized_lo});
  };

  launch(rmsnorm_.get(), rows_config(count, 256),
         NormArgs{hidden, model.layers[0].attention_norm, normalized, normalized_lo, count,
                  model.epsilon});
  for (size_t layer = 0; layer < model.layers.size(); ++layer) {
    const LayerView &w = model.layers[layer];
    const float *next_norm =
        layer + 1 < model.layers.size() ? model.layers[layer + 1].attention_norm : nullptr;
    PartialTiles qkv_partials = direct;
    if (tc) {
      qkv_partials = tc_gemm(kQkvTile, normalized_maps_, layer_maps_[layer].qkv, count, kQkv,
                             kHidden, GemmEpilogue::bias, qkv, nullptr, kQkv, w.qkv_bias, true);
    } else {
      simt(gemm_bias_,
           GemmArgs{normalized, w.qkv, nullptr, w.qkv_bias, qkv, nullptr, count, kQkv, kHidden,
                    kHidden, kHidden, kQkv},
           ceil_div(kQkv, 128));
    }
    launch(rope_kv_.get(),
           rows_config(count, row_threads(count), staged_bytes(qkv_partials, kQkv)),
           RopeArgs{qkv, model.rope_cos, model.rope_sin, w.key_cache, w.value_cache, count,
                    first_position, qkv_partials, w.qkv_bias, nullptr, 0});
    // Attention blocks: a key chunk x 64 query rows x one head; chunks of
    // 128 positions (more when the context needs over kAttentionMaximumChunks).
    const uint32_t keys = first_position + count;
    const uint32_t chunk_keys =
        128u * std::max(1u, ceil_div(keys, 128u * kAttentionMaximumChunks));
    // The tf32x3 path runs the tensor-core kernel (128-row tiles).
    const uint32_t tile_rows = tc ? kTcAttentionRows : kAttentionTileRows;
    const uint32_t attention_threads = tc ? kTcAttentionThreads : kAttentionThreads;
    uint32_t attention_blocks = 0; // (row tile, key chunk) pairs with work
    for (uint32_t t0 = 0; t0 < count; t0 += tile_rows) {
      const uint32_t tile_last = first_position + std::min(count, t0 + tile_rows) - 1u;
      attention_blocks += tile_last / chunk_keys + 1u;
    }
    const lr_launch_config_t attention_config{
        {attention_blocks * attention_threads, qd::kAttentionHeads, 1},
        {attention_threads, 1, 1},
        tc ? kTcAttentionSharedBytes : kAttentionSharedBytes};
    launch(tc ? attend_tc_.get() : attend_.get(), attention_config,
           AttentionArgs{qkv, w.key_cache, w.value_cache, attention, attention_lo, count,
                         first_position, chunk_keys, kAttentionMaximumChunks,
                         static_cast<float *>(attention_partials_->data()),
                         static_cast<uint32_t *>(attention_arrivals_->data()), kWaitLimitMs,
                         static_cast<uint32_t *>(error_->data()),
                         tc ? attention_maps_.wide[0] : TensorMap{},
                         tc ? attention_maps_.wide[1] : TensorMap{}});
    if (tc) {
      finish(tc_gemm(kHiddenTile, attention_maps_, layer_maps_[layer].o, count, kHidden, kHidden,
                     GemmEpilogue::residual, hidden, nullptr, kHidden, nullptr, true),
             w.mlp_norm);
      // 144 + 144-column pair tiles: a 512-token chunk's gate/up is one wave.
      tc_gemm(count <= kNarrowRows ? kGateUpTile : kTcPairN, normalized_maps_,
              count <= kNarrowRows ? layer_maps_[layer].gate_up : layer_maps_[layer].gate_up_pair,
              count, kIntermediate, kHidden, GemmEpilogue::swiglu, activated, activated_lo,
              kIntermediate, nullptr, false);
      finish(tc_gemm(kHiddenTile, activated_maps_, layer_maps_[layer].down, count, kHidden,
                     kIntermediate, GemmEpilogue::residual, hidden, nullptr, kHidden, nullptr,
                     true),
             next_norm);
    } else {
      simt(gemm_residual_,
           GemmArgs{attention, w.o, nullptr, nullptr, hidden, nullptr, count, kHidden, kHidden,
                    kHidden, kHidden, kHidden},
           ceil_div(kHidden, 128));
      finish(direct, w.mlp_norm);
      const float *up = w.gate_up + size_t{kIntermediate} * kHidden;
      simt(gemm_swiglu_,
           GemmArgs{normalized, w.gate_up, up, nullptr, activated, nullptr, count, kIntermediate,
                    kHidden, kHidden, kHidden, kIntermediate},
           ceil_div(kIntermediate, 128));
      simt(gemm_residual_,
           GemmArgs{activated, w.down, nullptr, nullptr, hidden, nullptr, count, kHidden,
                    kIntermediate, kIntermediate, kIntermediate, kHidden},
           ceil_div(kHidden, 128));
      if (next_norm != nullptr) {
        finish(direct, next_norm);
      }
    }
  }
}

void Prefill::gemm_check(uint32_t tile_columns, GemmEpilogue mode, uint32_t m, uint32_t n,
                         uint32_t k, const float *a, const float *b, const float *bias,
                         float *c) {
  const bool swiglu = mode == GemmEpilogue::swiglu;
  if (m == 0 || n == 0 || k == 0 || k % kTcTileK != 0 || n % 32 != 0 || mode == GemmEpilogue::partial ||
      (tile_columns != 0 && tile_columns != 192 && tile_columns != 224 && tile_columns != 256 &&
       tile_columns != kTcPairN) ||
      (tile_columns == kTcPairN && !swiglu) ||
      (swiglu && tile_columns != 0 && tile_columns != kTcPairN && m > kNarrowRows &&
       (n % (tile_columns / 2u) != 0 || (tile_columns / 2u) % 32u != 0))) {
    throw std::invalid_argument("unsupported GEMM check shape");
  }
  const uint64_t rows_b = swiglu ? 2ull * n : n;
  DeviceBuffer a_dev(device_, sizeof(float) * m * k), b_dev(device_, sizeof(float) * rows_b * k);
  DeviceBuffer c_dev(device_, sizeof(float) * m * n);
  DeviceBuffer bias_dev(device_, sizeof(float) * n);
  copy_to_device(a_dev, a, a_dev.size());
  copy_to_device(b_dev, b, b_dev.size());
  copy_to_device(c_dev, c, c_dev.size());
  if (bias != nullptr) {
    copy_to_device(bias_dev, bias, bias_dev.size());
  }
  auto *bias_ptr = bias != nullptr ? static_cast<const float *>(bias_dev.data()) : nullptr;
  auto *cd = static_cast<float *>(c_dev.data());
  const uint32_t zero = 0;
  check(lr_memcpy(device_.get(), error_->data(), &zero, sizeof(zero), LR_MEMCPY_HOST_TO_DEVICE),
        "lr_memcpy gemm error");
  if (tile_columns == 0) {
    const auto *ad = static_cast<const float *>(a_dev.data());
    const auto *bd = static_cast<const float *>(b_dev.data());
    const GemmArgs args{ad, bd, swiglu ? bd + size_t{n} * k : nullptr, bias_ptr, cd, nullptr,
                        m, n, k, k, k, n};
    const Kernel &kernel = mode == GemmEpilogue::bias       ? gemm_bias_
                           : mode == GemmEpilogue::residual ? gemm_residual_
                                                            : gemm_swiglu_;
    const lr_launch_config_t config{{ceil_div(n, 128) * 256u, ceil_div(m, 128), 1}, {256, 1, 1}, 0};
    launch(kernel.get(), config, args);
  } else {
    if (cudaSetDevice(static_cast<int>(device_.index())) != cudaSuccess) {
      throw std::runtime_error("cudaSetDevice failed");
    }
    DeviceBuffer a_split(device_, 2 * a_dev.size()), b_split(device_, 2 * b_dev.size());
    auto *ah = static_cast<float *>(a_split.data());
    auto *bh = static_cast<float *>(b_split.data());
    const uint64_t a_floats = uint64_t{m} * k, b_floats = rows_b * k;
    launch(split_.get(), rows_config(std::min<uint32_t>(ceil_div(a_floats, 256), kSms * 8), 256),
           SplitArgs{static_cast<const float *>(a_dev.data()), ah, ah + a_floats, a_floats});
    launch(split_.get(), rows_config(std::min<uint32_t>(ceil_div(b_floats, 256), kSms * 8), 256),
           SplitArgs{static_cast<const float *>(b_dev.data()), bh, bh + b_floats, b_floats});
    tc_gemm(tile_columns, activation_maps(ah, ah + a_floats, m, k),
            weight_maps(bh, bh + b_floats, static_cast<const float *>(b_dev.data()), rows_b, k,
                        tile_columns),
            m, n, k, mode, cd, nullptr,
            n, bias_ptr, false);
  }
  device_.synchronize();
  copy_to_host(c, c_dev, c_dev.size());
  uint32_t error = 0;
  check(lr_memcpy(device_.get(), &error, error_->data(), sizeof(error), LR_MEMCPY_DEVICE_TO_HOST),
        "lr_memcpy gemm error");
  if (error != 0) {
    throw std::runtime_error("prefill tensor-core kernel gave up waiting (code " +
                             std::to_string(error) + ")");
  }
}

void Prefill::run(const ModelView &model, const uint32_t *tokens, uint32_t count,
                  uint32_t first_position, Path path, uint64_t weights_generation) {
  if (count == 0) {
    return;
  }
  if (uint64_t{first_position} + count > model.capacity) {
    throw std::invalid_argument("prefill exceeds the KV-cache capacity");
  }
  if (path != Path::simt && path != Path::tf32x3) {
    throw std::invalid_argument("unknown prefill path");
  }
  for (uint32_t i = 0; i < count; ++i) {
    if (tokens[i] >= model.vocab) {
      throw std::invalid_argument("prompt token out of range");
    }
  }
  if (!tokens_ || tokens_->size() < sizeof(uint32_t) * count) {
    tokens_.reset();
    tokens_.emplace(allocate(sizeof(uint32_t) * std::max<uint32_t>(count, chunk_)));
  }
  // The queue may still run an earlier prefill reading these buffers.
  device_.synchronize();
  check(lr_memcpy(device_.get(), tokens_->data(), tokens, sizeof(uint32_t) * count,
                  LR_MEMCPY_HOST_TO_DEVICE),
        "lr_memcpy prompt");
  const uint32_t zero = 0;
  check(lr_memcpy(device_.get(), error_->data(), &zero, sizeof(zero), LR_MEMCPY_HOST_TO_DEVICE),
        "lr_memcpy prefill error");
  if (path == Path::tf32x3) {
    prepare_tensor_cores(model, weights_generation);
  }
  for (uint32_t start = 0; start < count; start += chunk_) {
    const uint32_t n = std::min(chunk_, count - start);
    launch(embed_.get(), rows_config(n, 256),
           EmbedArgs{static_cast<const uint32_t *>(tokens_->data()) + start, model.embeddings,
                     static_cast<float *>(hidden_->data()), n, model.vocab});
    run_chunk(model, n, first_position + start, path);
  }
  device_.synchronize();
  uint32_t error = 0;
  check(lr_memcpy(device_.get(), &error, error_->data(), sizeof(error), LR_MEMCPY_DEVICE_TO_HOST),
        "lr_memcpy prefill error");
  if (error != 0) {
    throw std::runtime_error("prefill tensor-core kernel gave up waiting (code " +
                             std::to_string(error) + ")");
  }
}

} // namespace lrrt::qwen::prefill
