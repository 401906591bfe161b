// Per-operation FP32 decode kernels for the generic bundle executor
// (include/lrrt/executor/triton_executor.hpp): each kernel is one step of a
// Qwen2 decoder layer at batch 1, launched through an lrrt::Bundle whose
// manifest (decoder_ops.json, next to the cubin) declares its kernarg
// layout. They mirror the operation set of light-rocm-runtime's Triton
// mini decoder layer (examples/triton/mini_decoder_layer.hpp:117-175:
// rmsnorm, matvec, rope, kv_cache_update, attention_score, causal_softmax,
// value_aggregation, silu_mul, vector_add) with the decode step's arithmetic
// (benchmarks/qwen_stateful_graph_kernel.cpp: RMSNorm :665-701, row dot
// products :392-427, RoPE :517-552, attention :554-600, SwiGLU :494-515).
// They are simple one-pass kernels: this module exists for the bundle
// path's coverage, the resident kernel is the fast decode path.
#include <cstdint>

namespace {

constexpr unsigned kFullMask = 0xffffffffu;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (uint32_t offset = 16; offset != 0; offset >>= 1u) {
    v += __shfl_xor_sync(kFullMask, v, offset);
  }
  return v;
}

} // namespace

// out = x * (1 / sqrt(mean(x^2) + eps)) * weight; one block of 256 threads.
extern "C" __global__ void __launch_bounds__(256)
    ops_rmsnorm_f32(const float *x, const float *weight, float *out, uint32_t n, float eps) {
  __shared__ float partial[256];
  float sum = 0.0f;
  for (uint32_t i = threadIdx.x; i < n; i += 256u) {
    sum = fmaf(x[i], x[i], sum);
  }
  partial[threadIdx.x] = sum;
  __syncthreads();
  for (uint32_t stride = 128; stride != 0; stride >>= 1u) {
    if (threadIdx.x < stride) {
      partial[threadIdx.x] += partial[threadIdx.x + stride];
    }
    __syncthreads();
  }
  const float inverse = 1.0f / sqrtf(partial[0] / static_cast<float>(n) + eps);
  for (uint32_t i = threadIdx.x; i < n; i += 256u) {
    out[i] = x[i] * inverse * weight[i];
  }
}

// out[r] = sum_c w[r][c] * x[c] (+ bias[r]) (+ residual[r]); one warp per
// row, lane l summing columns l, l + 32, ... then a butterfly. bias and
// residual are optional (null).
extern "C" __global__ void __launch_bounds__(256)
    ops_matvec_f32(const float *w, const float *x, const float *bias, const float *residual,
                   float *out, uint32_t rows, uint32_t columns) {
  const uint32_t row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5u;
  const uint32_t lane = threadIdx.x & 31u;
  if (row >= rows) {
    return;
  }
  const float *w_row = w + static_cast<size_t>(row) * columns;
  float sum = 0.0f;
  for (uint32_t c = lane; c < columns; c += 32u) {
    sum = fmaf(w_row[c], x[c], sum);
  }
  sum = warp_sum(sum);
  if (lane == 0) {
    if (bias != nullptr) {
      sum += bias[row];
    }
    out[row] = residual != nullptr ? residual[row] + sum : sum;
  }
}

// Half-split RoPE in place on `heads` heads of `head_dim` at `position`:
// pairs (f, f + head_dim / 2) rotated by cos/sin[position][f].
extern "C" __global__ void __launch_bounds__(256)
    ops_rope_f32(float *x, const float *cos_table, const float *sin_table, uint32_t position,
                 uint32_t heads, uint32_t head_dim) {
  const uint32_t half = head_dim / 2u;
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= heads * half) {
    return;
  }
  const uint32_t head = i / half, f = i % half;
  float *base = x + static_cast<size_t>(head) * head_dim;
  const float c = cos_table[static_cast<size_t>(position) * half + f];
  const float s = sin_table[static_cast<size_t>(position) * half + f];
  const float x0 = base[f], x1 = base[f + half];
  base[f] = x0 * c - x1 * s;
  base[f + half] = x1 * c + x0 * s;
}

// k_cache[position][:] = k, v_cache[position][:] = v (rows of kv_dim).
extern "C" __global__ void __launch_bounds__(256)
    ops_kv_cache_update_f32(const float *k, const float *v, float *k_cache, float *v_cache,
                            uint32_t position, uint32_t kv_dim) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= kv_dim) {
    return;
  }
  k_cache[static_cast<size_t>(position) * kv_dim + i] = k[i];
  v_cache[static_cast<size_t>(position) * kv_dim + i] = v[i];
}

// scores[h][p] = scale * q[h] . k_cache[p][group(h)] for p < keys; one warp
// per (head, position), lanes over head dims.
extern "C" __global__ void __launch_bounds__(256)
    ops_attention_score_f32(const float *q, const float *k_cache, float *scores, uint32_t keys,
                            uint32_t heads, uint32_t kv_heads, uint32_t head_dim, float scale) {
  const uint32_t item = (blockIdx.x * blockDim.x + threadIdx.x) >> 5u;
  const uint32_t lane = threadIdx.x & 31u;
  if (item >= heads * keys) {
    return;
  }
  const uint32_t head = item / keys, p = item % keys;
  const uint32_t group = head / (heads / kv_heads);
  const float *qh = q + static_cast<size_t>(head) * head_dim;
  const float *kp = k_cache + (static_cast<size_t>(p) * kv_heads + group) * head_dim;
  float sum = 0.0f;
  for (uint32_t d = lane; d < head_dim; d += 32u) {
    sum = fmaf(qh[d], kp[d], sum);
  }
  sum = warp_sum(sum);
  if (lane == 0) {
    scores[item] = sum * scale;
  }
}

// probs[h][p] = exp(scores[h][p] - max) / sum over p < keys (expf, as the
// decode step); one block of 256 threads per head.
extern "C" __global__ void __launch_bounds__(256)
    ops_causal_softmax_f32(const float *scores, float *probs, uint32_t keys, uint32_t heads) {
  __shared__ float reduce[256];
  const uint32_t head = blockIdx.x;
  if (head >= heads) {
    return;
  }
  const float *row = scores + static_cast<size_t>(head) * keys;
  float maximum = -INFINITY;
  for (uint32_t p = threadIdx.x; p < keys; p += 256u) {
    maximum = fmaxf(maximum, row[p]);
  }
  reduce[threadIdx.x] = maximum;
  __syncthreads();
  for (uint32_t stride = 128; stride != 0; stride >>= 1u) {
    if (threadIdx.x < stride) {
      reduce[threadIdx.x] = fmaxf(reduce[threadIdx.x], reduce[threadIdx.x + stride]);
    }
    __syncthreads();
  }
  maximum = reduce[0];
  __syncthreads();
  float sum = 0.0f;
  for (uint32_t p = threadIdx.x; p < keys; p += 256u) {
    sum += expf(row[p] - maximum);
  }
  reduce[threadIdx.x] = sum;
  __syncthreads();
  for (uint32_t stride = 128; stride != 0; stride >>= 1u) {
    if (threadIdx.x < stride) {
      reduce[threadIdx.x] += reduce[threadIdx.x + stride];
    }
    __syncthreads();
  }
  const float inverse = 1.0f / reduce[0];
  for (uint32_t p = threadIdx.x; p < keys; p += 256u) {
    probs[static_cast<size_t>(head) * keys + p] = expf(row[p] - maximum) * inverse;
  }
}

// out[h][d] = sum_p probs[h][p] * v_cache[p][group(h)][d]; one thread per
// (head, dim).
extern "C" __global__ void __launch_bounds__(256)
    ops_value_aggregation_f32(const float *probs, const float *v_cache, float *out, uint32_t keys,
                              uint32_t heads, uint32_t kv_heads, uint32_t head_dim) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= heads * head_dim) {
    return;
  }
  const uint32_t head = i / head_dim, d = i % head_dim;
  const uint32_t group = head / (heads / kv_heads);
  const float *p_row = probs + static_cast<size_t>(head) * keys;
  float sum = 0.0f;
  for (uint32_t p = 0; p < keys; ++p) {
    sum = fmaf(p_row[p], v_cache[(static_cast<size_t>(p) * kv_heads + group) * head_dim + d], sum);
  }
  out[i] = sum;
}

// out = gate / (1 + exp(-gate)) * up.
extern "C" __global__ void __launch_bounds__(256)
    ops_silu_mul_f32(const float *gate, const float *up, float *out, uint32_t n) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) {
    const float g = gate[i];
    out[i] = g / (1.0f + expf(-g)) * up[i];
  }
}

// out = a + b.
extern "C" __global__ void __launch_bounds__(256)
    ops_vector_add_f32(const float *a, const float *b, float *out, uint32_t n) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) {
    out[i] = a[i] + b[i];
  }
}
