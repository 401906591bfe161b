// Host side of the prompt prefill (module qwen_prefill.cubin, kernels in
// csrc/kernels/qwen_prefill.cu): chunk buffers, the TF32 (hi, lo) weight
// copies and TMA tensor maps of the 3xTF32 path, and the per-layer launch
// sequence. The decode driver owns one Prefill per model and hands it views
// of the model's device arrays.
#ifndef LRRT_B200_QWEN_PREFILL_HPP_
#define LRRT_B200_QWEN_PREFILL_HPP_

#include "lrrt/lrrt.hpp"
#include "lrrt/qwen/prefill.hpp"

#include <cstdint>
#include <optional>
#include <vector>

namespace lrrt::qwen::prefill {

// Device pointers of one decoder layer. q, k, v (and their biases) are
// contiguous, as are gate and up, so QKV and gate/up are single B matrices.
struct LayerView {
  const float *attention_norm;
  const float *qkv;      // [1152][896]
  const float *qkv_bias; // [1152]
  const float *o;        // [896][896]
  const float *mlp_norm;
  const float *gate_up;  // [2 x 4864][896]
  const float *down;     // [896][4864]
  float *key_cache;      // [capacity][128]
  float *value_cache;
};

struct ModelView {
  uint32_t vocab;
  uint32_t capacity;
  float epsilon;
  const float *embeddings; // [vocab][896]
  const float *lm_head;    // [vocab][896] (the embeddings when tied)
  const float *final_norm; // [896]
  const float *rope_cos;   // [capacity][32]
  const float *rope_sin;
  std::vector<LayerView> layers;
};

enum class Path : uint32_t { simt = 0, tf32x3 = 1 };

class BatchDecoder;

// (hi, lo) tensor maps of one GEMM operand: `wide` boxes for the
// 128-row-band kernels (activations: 128 rows; weights: half a tile), and
// `narrow` boxes for the swapped-operand kernels of at most kNarrowRows rows
// (activations: kNarrowRows rows of the pair; weights: kNarrowTileN rows of
// the FP32 weights in narrow[0], which those kernels split themselves).
struct OperandMaps {
  TensorMap wide[2]{}, narrow[2]{};
};

class Prefill {
public:
  Prefill(Device device, const void *image, size_t image_size, uint32_t max_chunk_tokens);

  // Runs prompt tokens [0, count) through every layer at positions
  // first_position + i, writing their K/V rows. Enqueues on the device's
  // default queue, waits, and reports a device-side wait timeout.
  void run(const ModelView &model, const uint32_t *tokens, uint32_t count,
           uint32_t first_position, Path path, uint64_t weights_generation);

  // One GEMM C = epilogue(A . B^T) on host matrices through the same
  // scheduler and kernels as the prefill (numerics checks): A [m][k],
  // B [rows][k] (swiglu: gate rows [0, n), up rows [n, 2n)), c [m][n] in/out.
  // tile_columns 0 runs the SIMT kernels, else 192, 224 or 256 picks the
  // tensor-core tile width (288: gate/up pairs of 144 + 144, swiglu only).
  void gemm_check(uint32_t tile_columns, GemmEpilogue mode, uint32_t m, uint32_t n, uint32_t k,
                  const float *a, const float *b, const float *bias, float *c);

  uint64_t device_bytes() const { return device_bytes_; }
  uint32_t max_chunk_tokens() const { return chunk_; }

private:
  friend class BatchDecoder;

  // One layer's weights (gate_up_pair: the same rows in boxes of
  // kTcPairN / 2 for the prefill's pair tiles).
  struct LayerMaps {
    OperandMaps qkv, o, gate_up, gate_up_pair, down;
  };

  DeviceBuffer allocate(size_t bytes);
  void prepare_tensor_cores(const ModelView &model, uint64_t weights_generation);
  // TF32 (hi, lo) copy of the LM head and its tensor maps (batched decode).
  void prepare_tail(const ModelView &model, uint64_t weights_generation);
  void run_chunk(const ModelView &model, uint32_t count, uint32_t first_position, Path path);
  PartialTiles tc_gemm(uint32_t tile_columns, const OperandMaps &a, const OperandMaps &b,
                       uint32_t m, uint32_t n, uint32_t k, GemmEpilogue mode, float *c,
                       float *c_lo, uint32_t ldc, const float *bias, bool defer);

  Device device_;
  Module module_;
  Kernel embed_, rmsnorm_, rope_kv_, attend_, attend_tc_, reduce_, split_, gemm_bias_, gemm_residual_,
      gemm_swiglu_, tc_n192_, tc_n224_, tc_n256_, tc_pair288_, tc_narrow_, tc_narrow_pair_, tc_narrow_shared_sm_,
      finish_rows_, batch_attention_, batch_argmax_;
  uint32_t chunk_;
  uint64_t device_bytes_ = 0;

  std::optional<DeviceBuffer> tokens_, hidden_, normalized_, normalized_lo_, qkv_, attention_,
      attention_lo_, activated_, activated_lo_, partials_, error_, attention_partials_,
      attention_arrivals_;
  // 3xTF32 path: per-layer (hi, lo) weight copies and tensor maps.
  std::optional<DeviceBuffer> split_weights_;
  std::vector<LayerMaps> layer_maps_;
  OperandMaps normalized_maps_, attention_maps_, activated_maps_;
  uint64_t split_generation_ = UINT64_MAX;
  const void *split_source_ = nullptr;
  std::optional<DeviceBuffer> tail_split_;
  OperandMaps tail_maps_;
  uint64_t tail_generation_ = UINT64_MAX;
  const void *tail_source_ = nullptr;
};

} // namespace lrrt::qwen::prefill

#endif // LRRT_B200_QWEN_PREFILL_HPP_
