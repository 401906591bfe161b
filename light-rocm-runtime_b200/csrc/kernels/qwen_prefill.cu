// Prompt prefill of the Qwen2 FP32 decode path on sm_100a (module
// qwen_prefill.cubin). All tokens of a prompt chunk go through each layer
// together, so the projections become GEMMs over the chunk's rows:
// [T x 896].[896 x 1152] (QKV), [T x 896].[896 x 896] (o_proj),
// [T x 896].[896 x 2 x 4864] (gate/up), [T x 4864].[4864 x 896] (down).
// The results fill the KV cache the way single-token decode steps do (same
// token-major cache layout, same RoPE tables), after which decoding
// continues from the last prompt token.
//
// light-rocm-runtime has no prefill: its prompts run through the decode step
// one token at a time. The per-token arithmetic here follows that step
// (benchmarks/qwen_stateful_graph_kernel.cpp: RMSNorm :665-701, QKV + bias
// :392-427, RoPE + KV append :517-552, GQA :554-600, o_proj + residual
// :602-620, SwiGLU :494-515, down + residual :158-176).
//
// Two GEMM implementations share the per-token kernels:
//  * prefill_gemm_{bias,residual,swiglu}: FP32 FMA tiles on the CUDA cores
//    (exact FP32 products, the comparator);
//  * prefill_tc_gemm: 3xTF32 on the tcgen05 tensor cores. Operands are stored
//    as TF32 (hi, lo) pairs (include/lrrt/qwen/prefill.hpp), TMA moves
//    64-byte-swizzled tiles into shared memory, one thread issues
//    tcgen05.mma into a TMEM accumulator (hi.hi + hi.lo + lo.hi per K step)
//    and four warps read it back with tcgen05.ld for the epilogue. GEMMs of
//    at most 32 rows (prefill_tc_narrow*) swap the operands and stream the
//    FP32 weights, splitting them into TF32 pairs in shared memory.
// The causal attention has a CUDA-core kernel (prefill_attention, the SIMT
// path) and a tensor-core one (prefill_attention_tc, the 3xTF32 path).
#include "lrrt/persistent_graph/device_sync.cuh"
#include "lrrt/qwen/prefill.hpp"
#include "lrrt/qwen/stateful_graph_context.hpp"

#include <cstdint>

namespace qd = lrrt::qwen::stateful_graph;
namespace pf = lrrt::qwen::prefill;
namespace dev = lrrt::persistent_graph::device;

namespace {

constexpr unsigned kFullMask = 0xffffffffu;

// Round to TF32 (10 explicit mantissa bits), nearest with ties away from zero.
__device__ __forceinline__ float to_tf32(float x) {
  uint32_t bits;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(bits) : "f"(x));
  return __uint_as_float(bits);
}

// Writes v, or its (hi, lo) TF32 pair when lo is not null.
__device__ __forceinline__ void store_operand(float *out, float *lo, size_t index, float v) {
  if (lo == nullptr) {
    out[index] = v;
  } else {
    const float hi = to_tf32(v);
    out[index] = hi;
    lo[index] = to_tf32(v - hi);
  }
}

// Overlapped launches (lr_kernel_set_overlapped): every kernel of this
// module may start while its predecessor on the queue finishes. It waits for
// that grid (and so for every earlier one) before reading device data, then
// lets its own successor start.
__device__ __forceinline__ void dependent_launch_entry() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ float silu_times(float gate, float up) {
  return (gate / (1.0f + expf(-gate))) * up;
}

// ------------------------------------------------------------ SIMT GEMM --
//
// C[m][n] = sum_k A[m][k] * B[n][k]: A [M][K] (lda), B [N][K] (ldb), both
// K-contiguous. 128 x 128 output tiles per 256-thread block, K in steps of
// 16 staged in shared memory transposed to [k][m] / [k][n], 8 x 8 outputs
// per thread; the next K step is loaded into registers while the current
// one is multiplied. Requires K % 16 == 0 and lda, ldb % 4 == 0.

constexpr uint32_t kTileM = 128, kTileN = 128, kTileK = 16, kGemmThreads = 256;

template <pf::GemmEpilogue kMode>
__device__ __forceinline__ void simt_gemm(const pf::GemmArgs &p) {
  dependent_launch_entry();
  constexpr bool kTwo = kMode == pf::GemmEpilogue::swiglu;
  __shared__ __align__(16) float as[kTileK][kTileM + 4];
  __shared__ __align__(16) float bs[kTileK][kTileN + 4];
  __shared__ __align__(16) float b2s[kTwo ? kTileK : 1][kTwo ? kTileN + 4 : 4];
  const uint32_t tid = threadIdx.x;
  const uint32_t tx = tid % 16u, ty = tid / 16u;
  const uint32_t m0 = blockIdx.y * kTileM, n0 = blockIdx.x * kTileN;
  const uint32_t load_row = tid / 4u, load_k = (tid % 4u) * 4u;
  const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
  float4 a_next[2], b_next[2], b2_next[2];
  auto fetch = [&](uint32_t k0) {
#pragma unroll
    for (uint32_t h = 0; h < 2; ++h) {
      const uint32_t m = m0 + load_row + 64u * h;
      const uint32_t n = n0 + load_row + 64u * h;
      a_next[h] = m < p.m ? __ldg(reinterpret_cast<const float4 *>(p.a + size_t{m} * p.lda + k0 + load_k))
                          : zero;
      b_next[h] = n < p.n ? __ldg(reinterpret_cast<const float4 *>(p.b + size_t{n} * p.ldb + k0 + load_k))
                          : zero;
      if constexpr (kTwo) {
        b2_next[h] = n < p.n ? __ldg(reinterpret_cast<const float4 *>(p.b2 + size_t{n} * p.ldb + k0 +
                                                                      load_k))
                             : zero;
      }
    }
  };
  auto stage = [&]() {
#pragma unroll
    for (uint32_t h = 0; h < 2; ++h) {
      const uint32_t r = load_row + 64u * h;
      as[load_k + 0][r] = a_next[h].x;
      as[load_k + 1][r] = a_next[h].y;
      as[load_k + 2][r] = a_next[h].z;
      as[load_k + 3][r] = a_next[h].w;
      bs[load_k + 0][r] = b_next[h].x;
      bs[load_k + 1][r] = b_next[h].y;
      bs[load_k + 2][r] = b_next[h].z;
      bs[load_k + 3][r] = b_next[h].w;
      if constexpr (kTwo) {
        b2s[load_k + 0][r] = b2_next[h].x;
        b2s[load_k + 1][r] = b2_next[h].y;
        b2s[load_k + 2][r] = b2_next[h].z;
        b2s[load_k + 3][r] = b2_next[h].w;
      }
    }
  };
  float acc[8][8];
  float acc2[kTwo ? 8 : 1][kTwo ? 8 : 1];
#pragma unroll
  for (uint32_t i = 0; i < 8; ++i) {
#pragma unroll
    for (uint32_t j = 0; j < 8; ++j) {
      acc[i][j] = 0.0f;
      if constexpr (kTwo) {
        acc2[i][j] = 0.0f;
      }
    }
  }
  fetch(0);
  for (uint32_t k0 = 0; k0 < p.k; k0 += kTileK) {
    __syncthreads(); // the previous step's shared reads are done
    stage();
    __syncthreads();
    if (k0 + kTileK < p.k) {
      fetch(k0 + kTileK);
    }
#pragma unroll
    for (uint32_t kk = 0; kk < kTileK; ++kk) {
      float av[8], bv[8], b2v[kTwo ? 8 : 1];
      const float4 a0 = *reinterpret_cast<const float4 *>(&as[kk][ty * 4u]);
      const float4 a1 = *reinterpret_cast<const float4 *>(&as[kk][64u + ty * 4u]);
      const float4 b0 = *reinterpret_cast<const float4 *>(&bs[kk][tx * 4u]);
      const float4 b1 = *reinterpret_cast<const float4 *>(&bs[kk][64u + tx * 4u]);
      av[0] = a0.x; av[1] = a0.y; av[2] = a0.z; av[3] = a0.w;
      av[4] = a1.x; av[5] = a1.y; av[6] = a1.z; av[7] = a1.w;
      bv[0] = b0.x; bv[1] = b0.y; bv[2] = b0.z; bv[3] = b0.w;
      bv[4] = b1.x; bv[5] = b1.y; bv[6] = b1.z; bv[7] = b1.w;
      if constexpr (kTwo) {
        const float4 c0 = *reinterpret_cast<const float4 *>(&b2s[kk][tx * 4u]);
        const float4 c1 = *reinterpret_cast<const float4 *>(&b2s[kk][64u + tx * 4u]);
        b2v[0] = c0.x; b2v[1] = c0.y; b2v[2] = c0.z; b2v[3] = c0.w;
        b2v[4] = c1.x; b2v[5] = c1.y; b2v[6] = c1.z; b2v[7] = c1.w;
      }
#pragma unroll
      for (uint32_t i = 0; i < 8; ++i) {
#pragma unroll
        for (uint32_t j = 0; j < 8; ++j) {
          acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
          if constexpr (kTwo) {
            acc2[i][j] = fmaf(av[i], b2v[j], acc2[i][j]);
          }
        }
      }
    }
  }
  // Thread (ty, tx) owns tile rows ty*4 + {0..3}, 64 + ty*4 + {0..3} and
  // columns tx*4 + {0..3}, 64 + tx*4 + {0..3}.
#pragma unroll
  for (uint32_t i = 0; i < 8; ++i) {
    const uint32_t m = m0 + (i < 4 ? ty * 4u + i : 64u + ty * 4u + (i - 4u));
    if (m >= p.m) {
      continue;
    }
#pragma unroll
    for (uint32_t j = 0; j < 8; ++j) {
      const uint32_t n = n0 + (j < 4 ? tx * 4u + j : 64u + tx * 4u + (j - 4u));
      if (n >= p.n) {
        continue;
      }
      const size_t at = size_t{m} * p.ldc + n;
      if constexpr (kMode == pf::GemmEpilogue::bias) {
        p.c[at] = acc[i][j] + p.bias[n];
      } else if constexpr (kMode == pf::GemmEpilogue::residual) {
        p.c[at] = p.c[at] + acc[i][j];
      } else {
        store_operand(p.c, p.c_lo, at, silu_times(acc[i][j], acc2[i][j]));
      }
    }
  }
}

// ------------------------------------------------------ tcgen05 3xTF32 --

__device__ __forceinline__ void tma_load_2d(void *destination, const pf::TensorMap *map,
                                            uint32_t x, uint32_t y, uint64_t *barrier) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(dev::shared_address(destination)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(dev::shared_address(barrier))
      : "memory");
}

// Shared-memory matrix descriptor of a K-major tile stored as 64-byte rows
// with the 64-byte swizzle (the layout a TMA box of 16 fp32 x rows writes):
// 8-row atoms of 512 bytes, stride byte offset 512, descriptor version 1,
// layout type 4 (SWIZZLE_64B). Tiles start on 512-byte boundaries.
__device__ __forceinline__ uint64_t sw64_descriptor(const void *tile) {
  const uint64_t address = dev::shared_address(tile);
  return ((address & 0x3ffffu) >> 4) | (uint64_t{1} << 16) | (uint64_t{512 >> 4} << 32) |
         (uint64_t{1} << 46) | (uint64_t{4} << 61);
}

// Instruction descriptor: kind::tf32, FP32 accumulator, A and B K-major,
// M = 128, N = kN.
template <uint32_t kN> __host__ __device__ constexpr uint32_t tc_instruction() {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((kN >> 3) << 17) | ((pf::kTcTileM >> 4) << 24);
}

__device__ __forceinline__ void tc_mma(uint32_t tmem, uint64_t a, uint64_t b, uint32_t instruction,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n"
      ".reg .pred p;\n"
      "setp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n"
      "}\n" ::"r"(tmem),
      "l"(a), "l"(b), "r"(instruction), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void tc_commit(uint64_t *barrier) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          dev::shared_address(barrier))
      : "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

// 16 consecutive accumulator columns of this thread's TMEM lane.
__device__ __forceinline__ void tc_load16(uint32_t address, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(address));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (uint32_t i = 0; i < 16; ++i) {
    v[i] = __uint_as_float(r[i]);
  }
}

// 32 consecutive accumulator columns of this thread's TMEM lane.
__device__ __forceinline__ void tc_load32(uint32_t address, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, "
      "%28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(address));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (uint32_t i = 0; i < 32; ++i) {
    v[i] = __uint_as_float(r[i]);
  }
}

template <uint32_t kStages> struct TcShared {
  uint64_t full[kStages];
  uint64_t empty[kStages];
  uint64_t done;
  uint32_t tmem;
  uint32_t abort;
};

// Epilogue of one output element, shared by the GEMM and the split-K reduce.
__device__ __forceinline__ void finish_element(const float *bias, float *c, float *c_lo,
                                               size_t at, uint32_t column, uint32_t mode,
                                               float value, float up) {
  if (mode == static_cast<uint32_t>(pf::GemmEpilogue::store)) {
    c[at] = value;
  } else if (mode == static_cast<uint32_t>(pf::GemmEpilogue::bias)) {
    c[at] = value + bias[column];
  } else if (mode == static_cast<uint32_t>(pf::GemmEpilogue::residual)) {
    c[at] = c[at] + value;
  } else {
    store_operand(c, c_lo, at, silu_times(value, up));
  }
}

} // namespace

// ------------------------------------------------------------- kernels --

extern "C" __global__ void __launch_bounds__(kGemmThreads) prefill_gemm_bias(pf::GemmArgs p) {
  simt_gemm<pf::GemmEpilogue::bias>(p);
}

extern "C" __global__ void __launch_bounds__(kGemmThreads) prefill_gemm_residual(pf::GemmArgs p) {
  simt_gemm<pf::GemmEpilogue::residual>(p);
}

// c = silu(a . b^T) * (a . b2^T)
extern "C" __global__ void __launch_bounds__(kGemmThreads) prefill_gemm_swiglu(pf::GemmArgs p) {
  simt_gemm<pf::GemmEpilogue::swiglu>(p);
}

// One block per token; out-of-range token ids write a zero row (the host
// rejects them before launching).
extern "C" __global__ void __launch_bounds__(256) prefill_embed(pf::EmbedArgs p) {
  dependent_launch_entry();
  const uint32_t t = blockIdx.x;
  if (t >= p.count) {
    return;
  }
  const uint32_t token = p.tokens[t];
  float *out = p.hidden + size_t{t} * qd::kHiddenSize;
  for (uint32_t i = threadIdx.x; i < qd::kHiddenSize; i += blockDim.x) {
    out[i] = token < p.rows ? p.table[size_t{token} * qd::kHiddenSize + i] : 0.0f;
  }
}

// One block per token: the decode step's RMSNorm (per-thread strided sum of
// squares, shared-memory tree, 1/sqrt(mean + eps), x * inverse * weight).
extern "C" __global__ void __launch_bounds__(256) prefill_rmsnorm(pf::NormArgs p) {
  dependent_launch_entry();
  __shared__ float partial[256];
  const uint32_t t = blockIdx.x;
  if (t >= p.count) {
    return;
  }
  const float *x = p.hidden + size_t{t} * qd::kHiddenSize;
  float sum = 0.0f;
  for (uint32_t i = threadIdx.x; i < qd::kHiddenSize; i += 256u) {
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
  const float inverse = 1.0f / sqrtf(partial[0] / static_cast<float>(qd::kHiddenSize) + p.epsilon);
  for (uint32_t i = threadIdx.x; i < qd::kHiddenSize; i += 256u) {
    store_operand(p.out, p.out_lo, size_t{t} * qd::kHiddenSize + i, x[i] * inverse * p.weight[i]);
  }
}

// Copies the deferred GEMM's partial sums of row t, columns [0, columns),
// into shared memory stage[split][column]: 16-byte loads in batches of
// eight per thread, so that a row's loads of every split are in flight
// together (tile_columns and columns are multiples of 4).
__device__ __forceinline__ void stage_partials(const pf::PartialTiles &tiles, uint32_t t,
                                               uint32_t columns, float *stage) {
  const uint32_t vectors = columns / 4u;
  const uint32_t total = tiles.splits * vectors;
  const uint32_t band = t / tiles.tile_rows;
  const size_t tile_floats = size_t{tiles.tile_rows} * tiles.tile_columns;
  const size_t split_stride = size_t{tiles.tile_count} * tile_floats;
  const float *row = tiles.partials + size_t{t % tiles.tile_rows} * tiles.tile_columns;
  constexpr uint32_t kBatch = 8;
  for (uint32_t first = threadIdx.x; first < total; first += kBatch * blockDim.x) {
    float4 v[kBatch];
#pragma unroll
    for (uint32_t j = 0; j < kBatch; ++j) {
      const uint32_t i = first + j * blockDim.x;
      if (i < total) {
        const uint32_t split = i / vectors, column = (i % vectors) * 4u;
        const uint32_t tile = band * tiles.n_tiles + column / tiles.tile_columns;
        v[j] = __ldcg(reinterpret_cast<const float4 *>(row + split * split_stride +
                                                       tile * tile_floats +
                                                       column % tiles.tile_columns));
      }
    }
#pragma unroll
    for (uint32_t j = 0; j < kBatch; ++j) {
      const uint32_t i = first + j * blockDim.x;
      if (i < total) {
        const uint32_t split = i / vectors, column = (i % vectors) * 4u;
        *reinterpret_cast<float4 *>(stage + split * columns + column) = v[j];
      }
    }
  }
}

// Sum over splits, in split order, of a staged column.
__device__ __forceinline__ float staged_sum(const float *stage, uint32_t splits, uint32_t columns,
                                            uint32_t column) {
  float sum = stage[column];
  for (uint32_t s = 1; s < splits; ++s) {
    sum += stage[s * columns + column];
  }
  return sum;
}

// The decode step's RMSNorm of one 896-float row held in shared memory:
// per-thread strided sums of squares as the decode step's 256 threads form
// them (thread j adds x[j], x[j + 256], ...), the same shared tree, then
// 1/sqrt(mean + eps). Blocks of kRowThreads threads; threads >= 256 only
// help with the stores.
using pf::kRowThreads;

__device__ __forceinline__ void row_rmsnorm(const float *x, const float *weight, float epsilon,
                                            float *out, float *out_lo, size_t at,
                                            float *partial) {
  if (threadIdx.x < 256u) {
    float sum = 0.0f;
    for (uint32_t i = threadIdx.x; i < qd::kHiddenSize; i += 256u) {
      sum = fmaf(x[i], x[i], sum);
    }
    partial[threadIdx.x] = sum;
  }
  __syncthreads();
  for (uint32_t stride = 128; stride != 0; stride >>= 1u) {
    if (threadIdx.x < stride) {
      partial[threadIdx.x] += partial[threadIdx.x + stride];
    }
    __syncthreads();
  }
  const float inverse = 1.0f / sqrtf(partial[0] / static_cast<float>(qd::kHiddenSize) + epsilon);
  for (uint32_t i = threadIdx.x; i < qd::kHiddenSize; i += blockDim.x) {
    store_operand(out, out_lo, at + i, x[i] * inverse * weight[i]);
  }
}

// RoPE (pairs f and f + 32 of each head) on q and k of every chunk token at
// position first_position + t, then the cache append of k and v; one block
// per token. The row is first finished from the QKV GEMM's partial sums when
// those are given.
extern "C" __global__ void __launch_bounds__(kRowThreads) prefill_rope_kv(pf::RopeArgs p) {
  dependent_launch_entry();
  __shared__ float row[qd::kPackedQkvSize];
  extern __shared__ __align__(16) float stage[]; // [splits][1152] when deferred
  const uint32_t t = blockIdx.x;
  if (t >= p.count) {
    return;
  }
  const uint32_t position = p.positions != nullptr ? p.positions[t] : p.first_position + t;
  const size_t stream_offset = p.positions != nullptr ? t * p.stream_stride : 0;
  float *qkv = p.qkv + size_t{t} * qd::kPackedQkvSize;
  const bool deferred = p.qkv_partials.partials != nullptr;
  if (deferred) {
    stage_partials(p.qkv_partials, t, qd::kPackedQkvSize, stage);
    __syncthreads();
  }
  for (uint32_t i = threadIdx.x; i < qd::kPackedQkvSize; i += blockDim.x) {
    row[i] = deferred ? staged_sum(stage, p.qkv_partials.splits, qd::kPackedQkvSize, i) +
                            p.qkv_bias[i]
                      : qkv[i];
  }
  __syncthreads();
  const float *cos_row = p.rope_cos + size_t{position} * qd::kRotarySize;
  const float *sin_row = p.rope_sin + size_t{position} * qd::kRotarySize;
  float *key_row = p.key_cache + stream_offset + size_t{position} * qd::kKvSize;
  float *value_row = p.value_cache + stream_offset + size_t{position} * qd::kKvSize;
  for (uint32_t i = threadIdx.x; i < qd::kRotaryHeads * qd::kRotarySize; i += blockDim.x) {
    const uint32_t head = i / qd::kRotarySize, f = i % qd::kRotarySize;
    const uint32_t first = head * qd::kHeadSize + f;
    const float x0 = row[first], x1 = row[first + qd::kRotarySize];
    const float r0 = x0 * cos_row[f] - x1 * sin_row[f];
    const float r1 = x1 * cos_row[f] + x0 * sin_row[f];
    if (head < qd::kAttentionHeads) {
      qkv[first] = r0;
      qkv[first + qd::kRotarySize] = r1;
    } else {
      const uint32_t local = (head - qd::kAttentionHeads) * qd::kHeadSize + f;
      key_row[local] = r0;
      key_row[local + qd::kRotarySize] = r1;
    }
  }
  for (uint32_t i = threadIdx.x; i < qd::kKvSize; i += blockDim.x) {
    value_row[i] = row[qd::kQuerySize + qd::kKvSize + i];
  }
}

// Residual finish of o_proj / down from their partial sums, then the next
// RMSNorm of the same row (mlp norm, or the next layer's attention norm).
extern "C" __global__ void __launch_bounds__(kRowThreads) prefill_finish_rows(pf::FinishArgs p) {
  dependent_launch_entry();
  __shared__ float row[qd::kHiddenSize];
  __shared__ float partial[256];
  extern __shared__ __align__(16) float stage[]; // [splits][896] when deferred
  const uint32_t t = blockIdx.x;
  if (t >= p.count) {
    return;
  }
  float *hidden = p.hidden + size_t{t} * qd::kHiddenSize;
  const bool deferred = p.partials.partials != nullptr;
  for (uint32_t i = threadIdx.x; i < qd::kHiddenSize; i += blockDim.x) {
    row[i] = hidden[i];
  }
  if (deferred) {
    stage_partials(p.partials, t, qd::kHiddenSize, stage);
  }
  __syncthreads();
  for (uint32_t i = threadIdx.x; i < qd::kHiddenSize; i += blockDim.x) {
    const float value =
        deferred ? row[i] + staged_sum(stage, p.partials.splits, qd::kHiddenSize, i) : row[i];
    hidden[i] = value;
    row[i] = value;
  }
  __syncthreads();
  if (p.norm_weight != nullptr) {
    row_rmsnorm(row, p.norm_weight, p.epsilon, p.out, p.out_lo, size_t{t} * qd::kHiddenSize,
                partial);
  }
}

// 16 bytes global -> shared without registers; `bytes` 0 zero-fills.
__device__ __forceinline__ void copy16_async(void *destination, const void *source,
                                             uint32_t bytes) {
  const uint32_t address = static_cast<uint32_t>(__cvta_generic_to_shared(destination));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(address), "l"(source),
               "r"(bytes)
               : "memory");
}

template <uint32_t kPending> __device__ __forceinline__ void copy_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(kPending) : "memory");
}

// Causal GQA attention, register-blocked and split over key chunks. Block
// (x, h) serves, for the x-th (row tile r, key chunk c) pair that holds
// work, query rows t0 = 64r .. t0 + 63 of head h against cache positions
// [c * chunk_keys, (c + 1) * chunk_keys) up to each row's own position
// first_position + t. The chunk's 64-key tiles are copied with cp.async
// into two buffers (K and V row-major; tile t + 1 lands while tile t is
// computed). Thread (ty, tx) = (tid / 16, tid % 16) owns query rows
// 4ty..4ty+3 and, per tile, keys tx + 16j of S = Q.K^T / 8 (float4 reads
// along the rows of Q and K; 68-float row pitch keeps them conflict-free)
// and output dims 4tx..4tx+3 of O; a row's sixteen threads reduce with
// shuffles. The decode step's online softmax (expf) runs per tile. A tile
// row with a single chunk is written directly; otherwise each chunk writes
// (acc, maximum, sum) per row to `partials` and the last chunk block of
// (r, h) to finish merges them in chunk order. out[t][head * 64 + d].
constexpr uint32_t kAttentionRows = pf::kAttentionTileRows, kAttentionKeys = 64;
constexpr uint32_t kAttentionPitch = qd::kHeadSize + 4u;
static_assert(pf::kAttentionThreads == 4u * kAttentionRows, "16 x (rows / 4) thread tile");
static_assert(pf::kAttentionPartialStride % 4u == 0, "float4 partial-state rows");

struct AttentionShared {
  float q[kAttentionRows][kAttentionPitch];
  float k[2][kAttentionKeys][kAttentionPitch];
  float v[2][kAttentionKeys][qd::kHeadSize];
  float ps[kAttentionRows][kAttentionPitch]; // [row][key]
};

static_assert(sizeof(AttentionShared) == pf::kAttentionSharedBytes, "shared layout");

extern "C" __global__ void __launch_bounds__(pf::kAttentionThreads)
    prefill_attention(pf::AttentionArgs p) {
  dependent_launch_entry();
  extern __shared__ __align__(16) unsigned char attention_raw[];
  AttentionShared &sh = *reinterpret_cast<AttentionShared *>(attention_raw);
  const uint32_t tid = threadIdx.x, ty = tid / 16u, tx = tid % 16u;
  // blockIdx.x enumerates the (row tile, key chunk) pairs that hold work,
  // the last (heaviest) row tile first, chunks in order.
  const uint32_t head = blockIdx.y;
  const uint32_t row_tiles = (p.count + kAttentionRows - 1u) / kAttentionRows;
  auto chunks_of = [&](uint32_t tile) {
    const uint32_t tile_last = p.first_position + min(p.count, (tile + 1u) * kAttentionRows) - 1u;
    return tile_last / p.chunk_keys + 1u;
  };
  uint32_t r = row_tiles, chunk = blockIdx.x;
  while (r > 0u) {
    --r;
    const uint32_t n = chunks_of(r);
    if (chunk < n) {
      break;
    }
    chunk -= n;
  }
  const uint32_t kv_group = head / qd::kQueriesPerKvHead;
  const uint32_t t0 = r * kAttentionRows;
  const uint32_t chunks = chunks_of(r);
  if (t0 >= p.count || chunk >= chunks) {
    return; // past the enumeration (not launched by the host)
  }
  const uint32_t rows = min(kAttentionRows, p.count - t0);
  const uint32_t last = p.first_position + t0 + rows - 1u; // the tile's last position
  const uint32_t begin = chunk * p.chunk_keys;
  const uint32_t end = min(begin + p.chunk_keys, last + 1u);
  const uint32_t tiles = (end - begin + kAttentionKeys - 1u) / kAttentionKeys;
  const size_t kv_offset = size_t{kv_group} * qd::kHeadSize;
  // 16-byte copies; rows past `end` (or past count, for Q) become 0.
  auto issue = [&](uint32_t buffer, uint32_t base) {
#pragma unroll
    for (uint32_t j = 0; j < kAttentionKeys * 16u / pf::kAttentionThreads; ++j) {
      const uint32_t i = tid + pf::kAttentionThreads * j, key = i / 16u, c = (i % 16u) * 4u;
      const bool valid = base + key < end;
      const size_t row = size_t{valid ? base + key : begin} * qd::kKvSize + kv_offset + c;
      copy16_async(&sh.k[buffer][key][c], p.key_cache + row, valid ? 16u : 0u);
      copy16_async(&sh.v[buffer][key][c], p.value_cache + row, valid ? 16u : 0u);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
#pragma unroll
  for (uint32_t j = 0; j < kAttentionRows * 16u / pf::kAttentionThreads; ++j) {
    const uint32_t i = tid + pf::kAttentionThreads * j, row = i / 16u, c = (i % 16u) * 4u;
    const bool valid = row < rows;
    copy16_async(&sh.q[row][c],
                 p.qkv + size_t{t0 + (valid ? row : 0u)} * qd::kPackedQkvSize +
                     head * qd::kHeadSize + c,
                 valid ? 16u : 0u);
  }
  issue(0, begin); // with Q in the same group
  if (tiles > 1u) {
    issue(1, begin + kAttentionKeys);
  }
  uint32_t position[4];
  float maximum[4], denominator[4], acc[4][4];
#pragma unroll
  for (uint32_t i = 0; i < 4; ++i) {
    position[i] = p.first_position + t0 + 4u * ty + i;
    maximum[i] = -INFINITY;
    denominator[i] = 0.0f;
#pragma unroll
    for (uint32_t j = 0; j < 4; ++j) {
      acc[i][j] = 0.0f;
    }
  }
  for (uint32_t t = 0; t < tiles; ++t) {
    const uint32_t buffer = t & 1u, base = begin + t * kAttentionKeys;
    if (t + 1u < tiles) {
      copy_wait<1>();
    } else {
      copy_wait<0>();
    }
    __syncthreads();
    float score[4][4];
#pragma unroll
    for (uint32_t i = 0; i < 4; ++i) {
#pragma unroll
      for (uint32_t j = 0; j < 4; ++j) {
        score[i][j] = 0.0f;
      }
    }
#pragma unroll 4
    for (uint32_t d = 0; d < qd::kHeadSize; d += 4u) {
      float4 q[4], k[4];
#pragma unroll
      for (uint32_t i = 0; i < 4; ++i) {
        q[i] = *reinterpret_cast<const float4 *>(&sh.q[4u * ty + i][d]);
        k[i] = *reinterpret_cast<const float4 *>(&sh.k[buffer][tx + 16u * i][d]);
      }
#pragma unroll
      for (uint32_t i = 0; i < 4; ++i) {
#pragma unroll
        for (uint32_t j = 0; j < 4; ++j) {
          score[i][j] = fmaf(q[i].x, k[j].x, score[i][j]);
          score[i][j] = fmaf(q[i].y, k[j].y, score[i][j]);
          score[i][j] = fmaf(q[i].z, k[j].z, score[i][j]);
          score[i][j] = fmaf(q[i].w, k[j].w, score[i][j]);
        }
      }
    }
    float scale[4];
#pragma unroll
    for (uint32_t i = 0; i < 4; ++i) {
      float tile_maximum = -INFINITY;
#pragma unroll
      for (uint32_t j = 0; j < 4; ++j) {
        const uint32_t key = base + tx + 16u * j;
        score[i][j] = key <= position[i] && key < end ? score[i][j] * 0.125f : -INFINITY;
        tile_maximum = fmaxf(tile_maximum, score[i][j]);
      }
#pragma unroll
      for (uint32_t offset = 1; offset < 16; offset <<= 1u) {
        tile_maximum = fmaxf(tile_maximum, __shfl_xor_sync(kFullMask, tile_maximum, offset));
      }
      // Rows whose positions all precede this tile's keys keep their state:
      // scale 1, weights 0 (also while their maximum is still -inf).
      const float next = fmaxf(maximum[i], tile_maximum);
      const bool live = next != -INFINITY;
      scale[i] = live ? expf(maximum[i] - next) : 1.0f;
      float sum = 0.0f;
#pragma unroll
      for (uint32_t j = 0; j < 4; ++j) {
        const float w = live ? expf(score[i][j] - next) : 0.0f;
        sh.ps[4u * ty + i][tx + 16u * j] = w;
        sum += w;
      }
#pragma unroll
      for (uint32_t offset = 1; offset < 16; offset <<= 1u) {
        sum += __shfl_xor_sync(kFullMask, sum, offset);
      }
      denominator[i] = denominator[i] * scale[i] + sum;
      maximum[i] = next;
    }
#pragma unroll
    for (uint32_t i = 0; i < 4; ++i) {
#pragma unroll
      for (uint32_t j = 0; j < 4; ++j) {
        acc[i][j] *= scale[i];
      }
    }
    __syncwarp(); // a row's weights come from the sixteen threads of its warp half
#pragma unroll 2
    for (uint32_t key = 0; key < kAttentionKeys; key += 4) {
      float pv[4][4];
#pragma unroll
      for (uint32_t i = 0; i < 4; ++i) {
        const float4 w = *reinterpret_cast<const float4 *>(&sh.ps[4u * ty + i][key]);
        pv[i][0] = w.x;
        pv[i][1] = w.y;
        pv[i][2] = w.z;
        pv[i][3] = w.w;
      }
#pragma unroll
      for (uint32_t e = 0; e < 4; ++e) {
        const float4 v = *reinterpret_cast<const float4 *>(&sh.v[buffer][key + e][4u * tx]);
        const float vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (uint32_t i = 0; i < 4; ++i) {
#pragma unroll
          for (uint32_t j = 0; j < 4; ++j) {
            acc[i][j] = fmaf(pv[i][e], vv[j], acc[i][j]);
          }
        }
      }
    }
    __syncthreads(); // buffer `buffer` and the weights are free again
    if (t + 2u < tiles) {
      issue(buffer, base + 2u * kAttentionKeys);
    }
  }
  auto store_row = [&](uint32_t row, const float (&o)[4]) {
    if (row < rows) {
      const size_t at = size_t{t0 + row} * qd::kQuerySize + head * qd::kHeadSize + 4u * tx;
#pragma unroll
      for (uint32_t j = 0; j < 4; ++j) {
        store_operand(p.out, p.out_lo, at + j, o[j]);
      }
    }
  };
  if (chunks == 1u) {
#pragma unroll
    for (uint32_t i = 0; i < 4; ++i) {
      const float inverse = 1.0f / denominator[i];
      const float o[4] = {acc[i][0] * inverse, acc[i][1] * inverse, acc[i][2] * inverse,
                          acc[i][3] * inverse};
      store_row(4u * ty + i, o);
    }
    return;
  }
  // Partial state of this chunk: [r][head][chunk][row][kAttentionPartialStride].
  const size_t tile_state = size_t{r} * qd::kAttentionHeads + head;
  float *states = p.partials + tile_state * p.max_chunks * kAttentionRows *
                                   pf::kAttentionPartialStride;
#pragma unroll
  for (uint32_t i = 0; i < 4; ++i) {
    float *row = states + (size_t{chunk} * kAttentionRows + 4u * ty + i) *
                              pf::kAttentionPartialStride;
    *reinterpret_cast<float4 *>(row + 4u * tx) =
        make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
    if (tx == 0) {
      row[64] = maximum[i];     // -inf: no key of this chunk precedes the row
      row[65] = denominator[i]; // 0 then
    }
  }
  __shared__ bool finisher;
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    finisher = atomicAdd(&p.arrivals[tile_state], 1u) == chunks - 1u;
  }
  __syncthreads();
  if (!finisher) {
    return;
  }
  __threadfence();
  // Merge in chunk order: per row, the common maximum, then the rescaled
  // sums and accumulators.
#pragma unroll
  for (uint32_t i = 0; i < 4; ++i) {
    const uint32_t row = 4u * ty + i;
    const float *first = states + size_t{row} * pf::kAttentionPartialStride;
    const size_t chunk_stride = size_t{kAttentionRows} * pf::kAttentionPartialStride;
    float common = -INFINITY;
    for (uint32_t c = 0; c < chunks; ++c) {
      common = fmaxf(common, __ldcg(first + c * chunk_stride + 64));
    }
    float total = 0.0f, o[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    for (uint32_t c = 0; c < chunks; ++c) {
      const float m = __ldcg(first + c * chunk_stride + 64);
      if (m == -INFINITY) {
        continue;
      }
      const float weight = expf(m - common);
      total += __ldcg(first + c * chunk_stride + 65) * weight;
      const float4 a = __ldcg(reinterpret_cast<const float4 *>(first + c * chunk_stride + 4u * tx));
      o[0] += a.x * weight;
      o[1] += a.y * weight;
      o[2] += a.z * weight;
      o[3] += a.w * weight;
    }
#pragma unroll
    for (uint32_t j = 0; j < 4; ++j) {
      o[j] /= total;
    }
    store_row(row, o);
  }
  if (tid == 0) {
    p.arrivals[tile_state] = 0; // ready for the next layer
  }
}

// ------------------------------------------------ tensor-core attention --

// The same causal GQA attention on the tensor cores (3xTF32), for the
// tf32x3 path. Block (x, h) serves query rows t0 = 128r .. t0 + 127 of head
// h against key positions [c * chunk_keys, (c + 1) * chunk_keys) for the
// x-th (row tile r, key chunk c) pair with work (the last row tile first, as
// prefill_attention), in sub-tiles of 64 keys:
//   S = Q.K^T (M = 128 rows, N = 64 keys, K = 64 dims) into TMEM columns
//   [0, 64), then P = exp(S / 8 - running maximum) into shared memory and
//   O = P.V (N = 64 dims, K = 64 keys) into TMEM columns [64, 128); the
//   running output stays in registers, rescaled per sub-tile (the decode
//   step's online softmax, expf).
// Every product is hi.hi + hi.lo + lo.hi of TF32 pairs that the block splits
// while staging Q, K and V^T (transposed on the way) from global memory into
// K-major slabs of 16 fp32 (64-byte rows, 64-byte swizzle; the layout the
// GEMMs' TMA boxes write). Thread (warp w, lane l) owns query row
// 32 (w % 4) + l, its TMEM lane, and column half w / 4 of S and O; the two
// threads of a row combine maxima and sums through shared memory. The key
// and value rows of sub-tile j + 1 are loaded into registers while sub-tile
// j is on the tensor cores. A row tile split over several chunks merges
// their partial states in the last chunk block to finish, in chunk order.
// Every mbarrier wait is bounded; on expiry the block records
// kTcErrorWaitTimeout, stores nothing and frees its TMEM.
constexpr uint32_t kTaRows = pf::kTcAttentionRows, kTaKeys = pf::kTcAttentionKeys;
constexpr uint32_t kTaSlabs = qd::kHeadSize / 16u; // 16-fp32 slabs along the head dims
constexpr uint32_t kTaKeySlabs = kTaKeys / 16u;    // 16-fp32 slabs along the keys
constexpr uint32_t kTaTmemColumns = 128;           // S [0, 64), O [64, 128)
static_assert(pf::kTcAttentionThreads == 2u * kTaRows && kTaRows == pf::kTcTileM,
              "two threads per row, one 128-lane accumulator");
static_assert(kTaKeys == 64u && qd::kHeadSize == 64u, "32-column halves of S and O");

struct TcAttentionShared {
  float q[2][kTaSlabs][kTaRows][16];           // [hi / lo][dim slab][row]
  float k[2][kTaSlabs][kTaKeys][16];           // [hi / lo][dim slab][key]
  float vt[2][kTaKeySlabs][qd::kHeadSize][16]; // [hi / lo][key slab][dim]
  float p[2][kTaKeySlabs][kTaRows][16];        // [hi / lo][key slab][row]
  float maximum[2][kTaRows];                   // [column half][row]
  float sum[2][kTaRows];
  uint64_t s_done, o_done;
  uint32_t tmem;
  uint32_t finisher;
};
static_assert(sizeof(TcAttentionShared) + 1024u <= pf::kTcAttentionSharedBytes, "shared layout");
static_assert(offsetof(TcAttentionShared, k) % 1024u == 0 &&
                  offsetof(TcAttentionShared, vt) % 1024u == 0 &&
                  offsetof(TcAttentionShared, p) % 1024u == 0,
              "slabs on swizzle-pattern boundaries");

// Byte offset of 16-byte chunk `chunk` (0..3) of row `row` in a
// 64-byte-swizzled slab: address bits [4, 6) XOR bits [7, 9).
__device__ __forceinline__ uint32_t sw64_offset(uint32_t row, uint32_t chunk) {
  return row * 64u + ((chunk ^ ((row >> 1) & 3u)) << 4);
}

// TF32 pair by truncation: hi keeps the sign, exponent and top 10 mantissa
// bits, lo = x - hi is exact, and the MMA reads lo's top 10 mantissa bits
// (relative error of hi + lo below 2^-20, no conversion instructions).
__device__ __forceinline__ float tf32_high(float x) {
  return __uint_as_float(__float_as_uint(x) & 0xffffe000u);
}

__device__ __forceinline__ void store_pair4(float *hi_slab, float *lo_slab, uint32_t offset,
                                            float4 x) {
  const float4 hi = make_float4(tf32_high(x.x), tf32_high(x.y), tf32_high(x.z), tf32_high(x.w));
  *reinterpret_cast<float4 *>(reinterpret_cast<unsigned char *>(hi_slab) + offset) = hi;
  *reinterpret_cast<float4 *>(reinterpret_cast<unsigned char *>(lo_slab) + offset) =
      make_float4(x.x - hi.x, x.y - hi.y, x.z - hi.z, x.w - hi.w);
}

__device__ __forceinline__ void proxy_fence_shared() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void tma_store_2d(const pf::TensorMap *map, const void *source,
                                             uint32_t x, uint32_t y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(dev::shared_address(source)), "r"(x), "r"(y)
               : "memory");
}

extern "C" __global__ void __launch_bounds__(pf::kTcAttentionThreads, 1)
    prefill_attention_tc(const __grid_constant__ pf::AttentionArgs p) {
  extern __shared__ __align__(1024) unsigned char ta_raw[];
  TcAttentionShared &sh = *reinterpret_cast<TcAttentionShared *>(
      (reinterpret_cast<uintptr_t>(ta_raw) + 1023u) & ~uintptr_t{1023});
  const uint32_t tid = threadIdx.x, warp = tid >> 5u, lane = tid & 31u;
  const uint32_t quadrant = warp & 3u, half = warp >> 2u;
  const uint32_t row = quadrant * 32u + lane; // this thread's query row and TMEM lane
  const uint32_t head = blockIdx.y;
  const uint32_t row_tiles = (p.count + kTaRows - 1u) / kTaRows;
  auto chunks_of = [&](uint32_t tile) {
    const uint32_t tile_last = p.first_position + min(p.count, (tile + 1u) * kTaRows) - 1u;
    return tile_last / p.chunk_keys + 1u;
  };
  uint32_t r = row_tiles, chunk = blockIdx.x;
  while (r > 0u) {
    --r;
    const uint32_t n = chunks_of(r);
    if (chunk < n) {
      break;
    }
    chunk -= n;
  }
  const uint32_t t0 = r * kTaRows;
  const uint32_t chunks = chunks_of(r);
  if (t0 >= p.count || chunk >= chunks) {
    return; // past the enumeration (not launched by the host)
  }
  const uint32_t rows = min(kTaRows, p.count - t0);
  const uint32_t last = p.first_position + t0 + rows - 1u;
  const uint32_t begin = chunk * p.chunk_keys;
  const uint32_t end = min(begin + p.chunk_keys, last + 1u);
  const uint32_t tiles = (end - begin + kTaKeys - 1u) / kTaKeys;
  const size_t kv_offset = size_t{head / qd::kQueriesPerKvHead} * qd::kHeadSize;

  if (tid == 0) {
    dev::mbarrier_init(&sh.s_done, 1);
    dev::mbarrier_init(&sh.o_done, 1);
    dev::mbarrier_init_fence();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     dev::shared_address(&sh.tmem)),
                 "r"(kTaTmemColumns)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh.tmem;
  const uint32_t lane_address = tmem + ((quadrant * 32u) << 16);
  dependent_launch_entry(); // barriers and TMEM are ready; qkv and the cache come next

  // Q and K rows are copied two rows per warp instruction (coalesced): lane
  // l takes chunk 4 (l / 8) + l % 4 of row 2 i + (l / 4) % 2, so that each
  // quarter-warp stores both rows' 64-byte piece of one slab (all 32 banks).
  const uint32_t pair_row = (lane >> 2u) & 1u, pair_chunk = (lane >> 3u) * 4u + (lane & 3u);
  // V: thread (key 16 (w % 4) + l % 16, chunks 8 (w / 4) + 4 (l / 16) ..)
  // loads four chunks and writes them down the columns of V^T; lanes 16..31
  // take the elements in the order 1, 0, 3, 2 so that the two half-warps
  // write rows of opposite parity (other banks).
  const uint32_t v_key = (warp & 3u) * 16u + (lane & 15u);
  const uint32_t v_chunk = (warp >> 2u) * 8u + (lane >> 4u) * 4u;
  const uint32_t v_swap = lane >> 4u;
  float4 k_next[4], v_next[4];
  auto load_tile = [&](uint32_t base) {
#pragma unroll
    for (uint32_t j = 0; j < 4; ++j) {
      const uint32_t key = 2u * (warp + 8u * j) + pair_row;
      k_next[j] = base + key < end
                      ? reinterpret_cast<const float4 *>(p.key_cache + size_t{base + key} * qd::kKvSize +
                                                         kv_offset)[pair_chunk]
                      : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    }
    const bool v_valid = base + v_key < end;
    const float4 *v_source = reinterpret_cast<const float4 *>(
        p.value_cache + size_t{v_valid ? base + v_key : begin} * qd::kKvSize + kv_offset +
        v_chunk * 4u);
#pragma unroll
    for (uint32_t j = 0; j < 4; ++j) {
      v_next[j] = v_valid ? v_source[j] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    }
  };
  load_tile(begin); // in flight while Q is staged
  {
    float4 x[8];
#pragma unroll
    for (uint32_t j = 0; j < 8; ++j) {
      const uint32_t q_row = 2u * (warp + 8u * j) + pair_row;
      x[j] = q_row < rows ? reinterpret_cast<const float4 *>(
                                p.qkv + size_t{t0 + q_row} * qd::kPackedQkvSize +
                                head * qd::kHeadSize)[pair_chunk]
                          : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    }
#pragma unroll
    for (uint32_t j = 0; j < 8; ++j) {
      const uint32_t q_row = 2u * (warp + 8u * j) + pair_row;
      store_pair4(&sh.q[0][pair_chunk / 4u][0][0], &sh.q[1][pair_chunk / 4u][0][0],
                  sw64_offset(q_row, pair_chunk % 4u), x[j]);
    }
  }
  auto stage_tile = [&]() {
#pragma unroll
    for (uint32_t j = 0; j < 4; ++j) {
      store_pair4(&sh.k[0][pair_chunk / 4u][0][0], &sh.k[1][pair_chunk / 4u][0][0],
                  sw64_offset(2u * (warp + 8u * j) + pair_row, pair_chunk % 4u), k_next[j]);
    }
    const uint32_t slab = v_key / 16u, column = v_key % 16u;
#pragma unroll
    for (uint32_t j = 0; j < 4; ++j) {
      const float4 v = v_next[j];
      const float in_order[4] = {v.x, v.y, v.z, v.w};
      const float swapped[4] = {v.y, v.x, v.w, v.z};
#pragma unroll
      for (uint32_t e = 0; e < 4; ++e) {
        const uint32_t dim = (v_chunk + j) * 4u + (e ^ v_swap);
        const float x = v_swap != 0u ? swapped[e] : in_order[e];
        const uint32_t offset = sw64_offset(dim, column / 4u) + (column % 4u) * 4u;
        const float hi = tf32_high(x);
        *reinterpret_cast<float *>(reinterpret_cast<unsigned char *>(&sh.vt[0][slab][0][0]) +
                                   offset) = hi;
        *reinterpret_cast<float *>(reinterpret_cast<unsigned char *>(&sh.vt[1][slab][0][0]) +
                                   offset) = x - hi;
      }
    }
  };

  constexpr uint32_t kInstruction = tc_instruction<kTaKeys>(); // M = 128, N = 64
  static_assert(kTaKeys == qd::kHeadSize, "one instruction for S and O");
  // Descriptor units (16 bytes) between consecutive slabs.
  constexpr uint64_t kRowSlab = kTaRows * 64u / 16u, kKeySlab = kTaKeys * 64u / 16u;
  auto issue = [&](uint32_t accumulator, const float *a_hi, const float *a_lo, uint64_t a_slab,
                   const float *b_hi, const float *b_lo, uint64_t b_slab, uint64_t *done) {
    tc_fence_after();
    const uint64_t ah = sw64_descriptor(a_hi), al = sw64_descriptor(a_lo);
    const uint64_t bh = sw64_descriptor(b_hi), bl = sw64_descriptor(b_lo);
#pragma unroll
    for (uint32_t s = 0; s < 4u; ++s) {
#pragma unroll
      for (uint32_t kk = 0; kk < 2u; ++kk) {
        const uint64_t a = s * a_slab + kk * 2u, b = s * b_slab + kk * 2u;
        tc_mma(accumulator, ah + a, bh + b, kInstruction, (s | kk) != 0u ? 1u : 0u);
        tc_mma(accumulator, ah + a, bl + b, kInstruction, 1u);
        tc_mma(accumulator, al + a, bh + b, kInstruction, 1u);
      }
    }
    tc_commit(done);
  };

  const uint32_t position = p.first_position + t0 + row;
  float maximum = -INFINITY, denominator = 0.0f, acc[32];
#pragma unroll
  for (uint32_t i = 0; i < 32; ++i) {
    acc[i] = 0.0f;
  }
  const dev::Deadline deadline(p.wait_limit_ms);
  bool failed = false;
  for (uint32_t t = 0; t < tiles; ++t) {
    const uint32_t base = begin + t * kTaKeys;
    stage_tile();
    proxy_fence_shared();
    tc_fence_before();
    failed = __syncthreads_or(failed); // also: the previous sub-tile's O is read
    if (failed) {
      break;
    }
    if (tid == 0) {
      issue(tmem, &sh.q[0][0][0][0], &sh.q[1][0][0][0], kRowSlab, &sh.k[0][0][0][0],
            &sh.k[1][0][0][0], kKeySlab, &sh.s_done);
    }
    if (t + 1u < tiles) {
      load_tile(base + kTaKeys);
    }
    failed |= !dev::mbarrier_wait(&sh.s_done, t & 1u, deadline);
    __syncwarp(); // the warp-collective TMEM load below runs converged
    tc_fence_after();
    float s[32];
    tc_load32(lane_address + half * 32u, s);
    float tile_maximum = -INFINITY;
#pragma unroll
    for (uint32_t i = 0; i < 32; ++i) {
      const uint32_t key = base + half * 32u + i;
      s[i] = key <= position && key < end ? s[i] * 0.125f : -INFINITY;
      tile_maximum = fmaxf(tile_maximum, s[i]);
    }
    sh.maximum[half][row] = tile_maximum;
    asm volatile("bar.sync %0, 64;" ::"r"(1u + quadrant) : "memory"); // warps q and q + 4
    tile_maximum = fmaxf(tile_maximum, sh.maximum[half ^ 1u][row]);
    // Rows whose positions all precede this sub-tile's keys keep their
    // state: scale 1, weights 0 (also while their maximum is still -inf).
    const float next = fmaxf(maximum, tile_maximum);
    const bool live = next != -INFINITY;
    const float scale = live ? expf(maximum - next) : 1.0f;
    float sum = 0.0f;
#pragma unroll
    for (uint32_t i = 0; i < 32; ++i) {
      s[i] = live ? expf(s[i] - next) : 0.0f;
      sum += s[i];
    }
#pragma unroll
    for (uint32_t c = 0; c < 8; ++c) {
      const uint32_t slab = half * 2u + c / 4u;
      store_pair4(&sh.p[0][slab][0][0], &sh.p[1][slab][0][0], sw64_offset(row, c % 4u),
                  make_float4(s[4u * c], s[4u * c + 1u], s[4u * c + 2u], s[4u * c + 3u]));
    }
    sh.sum[half][row] = sum;
    proxy_fence_shared();
    tc_fence_before();
    failed = __syncthreads_or(failed); // P complete; S read by every warp
    denominator = denominator * scale + sum + sh.sum[half ^ 1u][row];
    maximum = next;
    if (failed) {
      break;
    }
    if (tid == 0) {
      issue(tmem + kTaKeys, &sh.p[0][0][0][0], &sh.p[1][0][0][0], kRowSlab, &sh.vt[0][0][0][0],
            &sh.vt[1][0][0][0], kKeySlab, &sh.o_done);
    }
    failed |= !dev::mbarrier_wait(&sh.o_done, t & 1u, deadline);
    __syncwarp();
    tc_fence_after();
    float o[32];
    tc_load32(lane_address + kTaKeys + half * 32u, o);
#pragma unroll
    for (uint32_t i = 0; i < 32; ++i) {
      acc[i] = fmaf(acc[i], scale, o[i]);
    }
    tc_fence_before();
  }
  failed = __syncthreads_or(failed);
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(kTaTmemColumns)
                 : "memory");
  }
  if (failed) {
    if (tid == 0) {
      atomicExch(p.error, pf::kTcErrorWaitTimeout);
    }
    return;
  }

  // Output rows o * scale as TF32 pairs into the Q slabs (free now, the
  // layout of the out maps' 16-column boxes), then thread 0 stores the
  // head's four boxes per buffer with TMA (rows past the chunk's count land
  // in unused rows of the buffer; the box is clipped at its end).
  auto store_rows = [&](const float (&o)[32], float scale) {
#pragma unroll
    for (uint32_t c = 0; c < 8u; ++c) {
      const uint32_t slab = half * 2u + c / 4u;
      const float4 x = make_float4(o[4u * c] * scale, o[4u * c + 1u] * scale,
                                   o[4u * c + 2u] * scale, o[4u * c + 3u] * scale);
      const float4 hi = make_float4(to_tf32(x.x), to_tf32(x.y), to_tf32(x.z), to_tf32(x.w));
      const uint32_t offset = sw64_offset(row, c % 4u);
      *reinterpret_cast<float4 *>(reinterpret_cast<unsigned char *>(&sh.q[0][slab][0][0]) +
                                  offset) = hi;
      *reinterpret_cast<float4 *>(reinterpret_cast<unsigned char *>(&sh.q[1][slab][0][0]) +
                                  offset) =
          make_float4(to_tf32(x.x - hi.x), to_tf32(x.y - hi.y), to_tf32(x.z - hi.z),
                      to_tf32(x.w - hi.w));
    }
    proxy_fence_shared();
    __syncthreads();
    if (tid == 0) {
#pragma unroll
      for (uint32_t s = 0; s < kTaSlabs; ++s) {
        tma_store_2d(&p.out_map, &sh.q[0][s][0][0], head * qd::kHeadSize + 16u * s, t0);
        tma_store_2d(&p.out_lo_map, &sh.q[1][s][0][0], head * qd::kHeadSize + 16u * s, t0);
      }
      asm volatile("cp.async.bulk.commit_group;" ::: "memory");
      asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
    }
  };
  if (chunks == 1u) {
    store_rows(acc, 1.0f / denominator);
    return;
  }
  // Partial state of this chunk, in column quads so that a warp's 32 rows
  // are 512 contiguous bytes: [r][head][chunk] then acc [16][128 rows][4],
  // maximum [128], sum [128] (within kAttentionPartialStride x 128 floats).
  const size_t tile_state = size_t{r} * qd::kAttentionHeads + head;
  const size_t chunk_stride = size_t{kTaRows} * pf::kAttentionPartialStride;
  static_assert(pf::kAttentionPartialStride >= qd::kHeadSize + 2u, "acc, maximum, sum");
  float *states = p.partials + tile_state * p.max_chunks * chunk_stride;
  {
    float *state = states + chunk * chunk_stride;
#pragma unroll
    for (uint32_t i = 0; i < 8u; ++i) {
      *reinterpret_cast<float4 *>(state + ((half * 8u + i) * kTaRows + row) * 4u) =
          make_float4(acc[4u * i], acc[4u * i + 1u], acc[4u * i + 2u], acc[4u * i + 3u]);
    }
    if (half == 0u) {
      state[64u * kTaRows + row] = maximum;     // -inf: no key of this chunk precedes the row
      state[65u * kTaRows + row] = denominator; // 0 then
    }
  }
  // The block's stores, then one release-acquire count per block: the CTA
  // barrier orders every thread's stores before thread 0's release, and the
  // finisher's acquire (with the barrier after it) orders its loads after
  // the other blocks' stores.
  __syncthreads();
  if (tid == 0) {
    uint32_t previous;
    asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], 1;"
                 : "=r"(previous)
                 : "l"(p.arrivals + tile_state)
                 : "memory");
    sh.finisher = previous == chunks - 1u ? 1u : 0u;
  }
  __syncthreads();
  if (sh.finisher == 0u) {
    return;
  }
  // Merge in chunk order: the common maximum, then the rescaled sums and
  // accumulators. All chunks' maxima and sums are loaded at once, the
  // accumulators four chunks at a time.
  constexpr uint32_t kChunks = pf::kAttentionMaximumChunks;
  float weight[kChunks], chunk_sum[kChunks];
#pragma unroll
  for (uint32_t c = 0; c < kChunks; ++c) {
    const float *state = states + c * chunk_stride + row;
    weight[c] = c < chunks ? __ldcg(state + 64u * kTaRows) : -INFINITY;
    chunk_sum[c] = c < chunks ? __ldcg(state + 65u * kTaRows) : 0.0f;
  }
  float common = -INFINITY;
#pragma unroll
  for (uint32_t c = 0; c < kChunks; ++c) {
    common = fmaxf(common, weight[c]);
  }
  float total = 0.0f;
#pragma unroll
  for (uint32_t c = 0; c < kChunks; ++c) {
    // A chunk without keys before the row (maximum -inf) adds nothing.
    weight[c] = weight[c] == -INFINITY ? 0.0f : expf(weight[c] - common);
    total += chunk_sum[c] * weight[c];
  }
#pragma unroll
  for (uint32_t i = 0; i < 32; ++i) {
    acc[i] = 0.0f;
  }
#pragma unroll
  for (uint32_t c0 = 0; c0 < kChunks; c0 += 4u) {
    if (c0 < chunks) {
      float4 a[4][8];
#pragma unroll
      for (uint32_t cc = 0; cc < 4u; ++cc) {
        const float4 *state = reinterpret_cast<const float4 *>(states + (c0 + cc) * chunk_stride);
#pragma unroll
        for (uint32_t i = 0; i < 8u; ++i) {
          a[cc][i] = c0 + cc < chunks ? __ldcg(state + (half * 8u + i) * kTaRows + row)
                                      : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        }
      }
#pragma unroll
      for (uint32_t cc = 0; cc < 4u; ++cc) {
#pragma unroll
        for (uint32_t i = 0; i < 8u; ++i) {
          acc[4u * i] += a[cc][i].x * weight[c0 + cc];
          acc[4u * i + 1u] += a[cc][i].y * weight[c0 + cc];
          acc[4u * i + 2u] += a[cc][i].z * weight[c0 + cc];
          acc[4u * i + 3u] += a[cc][i].w * weight[c0 + cc];
        }
      }
    }
  }
  store_rows(acc, 1.0f / total);
  __syncthreads();
  if (tid == 0) {
    p.arrivals[tile_state] = 0; // ready for the next layer
  }
}

// Finishes split-K tiles: one thread per output element of tiles
// [tile_offset, tile_offset + tile_count); partial sums are added in split
// order, so the result does not depend on which CTA finished first.
extern "C" __global__ void __launch_bounds__(256) prefill_reduce(pf::ReduceArgs p) {
  dependent_launch_entry();
  const bool swiglu = p.mode == static_cast<uint32_t>(pf::GemmEpilogue::swiglu);
  const uint32_t out_columns = swiglu ? p.tile_columns / 2u : p.tile_columns;
  const uint64_t i = uint64_t{blockIdx.x} * blockDim.x + threadIdx.x;
  if (i >= uint64_t{p.tile_count} * p.tile_rows * out_columns) {
    return;
  }
  const uint32_t local = static_cast<uint32_t>(i / (uint64_t{p.tile_rows} * out_columns));
  const uint32_t r = static_cast<uint32_t>((i / out_columns) % p.tile_rows);
  const uint32_t column_in_tile = static_cast<uint32_t>(i % out_columns);
  const uint32_t tile = p.tile_offset + local;
  const uint32_t row = (tile / p.n_tiles) * p.tile_rows + r;
  const uint32_t column = (tile % p.n_tiles) * out_columns + column_in_tile;
  if (row >= p.m || column >= p.n) {
    return;
  }
  const size_t tile_floats = size_t{p.tile_rows} * p.tile_columns;
  const float *partial = p.partials + local * tile_floats + size_t{r} * p.tile_columns +
                         column_in_tile;
  const size_t split_stride = size_t{p.tile_count} * tile_floats;
  // Loads four splits at a time, sums in split order.
  float value = partial[0];
  float up = swiglu ? partial[out_columns] : 0.0f;
  uint32_t s = 1;
  for (; s + 4u <= p.splits; s += 4u) {
    float v[4], u[4];
#pragma unroll
    for (uint32_t j = 0; j < 4; ++j) {
      v[j] = partial[(s + j) * split_stride];
      u[j] = swiglu ? partial[(s + j) * split_stride + out_columns] : 0.0f;
    }
#pragma unroll
    for (uint32_t j = 0; j < 4; ++j) {
      value += v[j];
      up += u[j];
    }
  }
  for (; s < p.splits; ++s) {
    value += partial[s * split_stride];
    if (swiglu) {
      up += partial[s * split_stride + out_columns];
    }
  }
  finish_element(p.bias, p.c, p.c_lo, size_t{row} * p.ldc + column, column, p.mode, value, up);
}

// TF32 (hi, lo) split of an FP32 array (weights, once per weight change).
extern "C" __global__ void __launch_bounds__(256) prefill_split(pf::SplitArgs p) {
  dependent_launch_entry();
  const uint64_t stride = uint64_t{gridDim.x} * blockDim.x;
  for (uint64_t i = uint64_t{blockIdx.x} * blockDim.x + threadIdx.x; i < p.count; i += stride) {
    const float x = p.x[i];
    const float hi = to_tf32(x);
    p.hi[i] = hi;
    p.lo[i] = to_tf32(x - hi);
  }
}

// 3xTF32 GEMM tile on the tensor cores: CTA (x, 0, z) computes output tile
// tile_offset + x (n tile fastest: 128 rows x kN accumulator columns, which
// are kN output columns, or kN / 2 for swiglu with gate in the first half and
// up in the second) over K slice z. Warp 0 lane 0 issues the TMA loads into a
// ring of kStages (A_hi, A_lo, B_hi, B_lo) stages, warp 1 owns the TMEM
// allocation and its lane 0 issues the MMAs, then all four warps run the
// epilogue, one accumulator row per thread. Every mbarrier wait is bounded;
// on expiry the kernel records kTcErrorWaitTimeout, skips its stores, waits
// (bounded) for its copies and MMAs in flight, frees TMEM and returns.
// Pair tiles wider than one MMA (kN = kTcPairN, gate/up pairs only) issue
// each product as two MMAs of N = kN / 2 into the two halves of the
// accumulator.
template <uint32_t kN>
__device__ __forceinline__ void tc_gemm(const pf::TcGemmArgs &p) {
  constexpr bool kSplitMma = kN > pf::kTcMaximumN;
  constexpr uint32_t kMmaN = kSplitMma ? kN / 2u : kN;
  constexpr uint32_t kTmemColumns = kSplitMma ? pf::kTcPairTmemColumns : pf::kTcTmemColumns;
  constexpr uint32_t kStages = pf::tc_stages(kN);
  constexpr uint32_t kStageBytes = pf::tc_stage_bytes(kN);
  constexpr uint32_t kBytesA = pf::kTcTileM * pf::kTcTileK * 4u;
  constexpr uint32_t kBytesB = kN * pf::kTcTileK * 4u;
  constexpr uint32_t kInstruction = tc_instruction<kMmaN>();
  static_assert(kN % 32 == 0 && kMmaN % 16 == 0 && kMmaN <= pf::kTcMaximumN &&
                    kN <= kTmemColumns,
                "accumulator width");
  // The swiglu epilogue reads gate/up column pairs in chunks of 32; widths
  // whose halves are not multiples of 32 (224) serve only the other modes.
  static_assert(kBytesA % 512 == 0 && (kBytesB / 2) % 512 == 0, "swizzle atom alignment");
  extern __shared__ __align__(1024) unsigned char raw_shared[];
  unsigned char *tiles = reinterpret_cast<unsigned char *>(
      (reinterpret_cast<uintptr_t>(raw_shared) + 1023u) & ~uintptr_t{1023});
  auto &s = *reinterpret_cast<TcShared<kStages> *>(tiles + kStages * kStageBytes);
  auto a_hi = [&](uint32_t st) { return tiles + st * kStageBytes; };
  auto a_lo = [&](uint32_t st) { return a_hi(st) + kBytesA; };
  auto b_hi = [&](uint32_t st) { return a_lo(st) + kBytesA; };
  auto b_lo = [&](uint32_t st) { return b_hi(st) + kBytesB; };

  const uint32_t warp = threadIdx.x >> 5u, lane = threadIdx.x & 31u;
  const bool swiglu = p.mode == static_cast<uint32_t>(pf::GemmEpilogue::swiglu);
  const uint32_t tile = p.tile_offset + blockIdx.x;
  const uint32_t m0 = (tile / p.n_tiles) * pf::kTcTileM;
  const uint32_t n_tile = tile % p.n_tiles;
  const uint32_t k_tiles = p.k / pf::kTcTileK;
  const uint32_t first_tile = blockIdx.z * k_tiles / p.splits;
  const uint32_t count = (blockIdx.z + 1u) * k_tiles / p.splits - first_tile;
  const dev::Deadline deadline(p.wait_limit_ms);

  if (threadIdx.x == 0) {
    for (uint32_t i = 0; i < kStages; ++i) {
      dev::mbarrier_init(&s.full[i], 1);
      dev::mbarrier_init(&s.empty[i], 1);
    }
    dev::mbarrier_init(&s.done, 1);
    s.abort = 0;
    dev::mbarrier_init_fence();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     dev::shared_address(&s.tmem)),
                 "r"(kTmemColumns)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s.tmem;
  dependent_launch_entry(); // barriers and TMEM are ready; operands come next

  auto fail = [&]() {
    s.abort = 1;
    atomicExch(p.error, pf::kTcErrorWaitTimeout);
  };

  if (warp == 0 && lane == 0) {
    // Producer. B rows: [n0, n0 + kN/2) and the next half, or, for a gate/up
    // pair (n_gate_offset set; also in split mode, whose epilogue is
    // `partial`), kN/2 gate rows and the matching kN/2 up rows.
    const uint32_t half = kN / 2u;
    const bool paired = p.n_gate_offset != 0;
    const uint32_t n_first = paired ? n_tile * half : n_tile * kN;
    const uint32_t n_second = paired ? p.n_gate_offset + n_tile * half : n_first + half;
    uint32_t issued = 0;
    for (uint32_t i = 0; i < count && s.abort == 0; ++i) {
      const uint32_t st = i % kStages;
      if (i >= kStages && !dev::mbarrier_wait(&s.empty[st], ((i / kStages) + 1u) & 1u, deadline)) {
        fail();
        break;
      }
      const uint32_t k0 = (first_tile + i) * pf::kTcTileK;
      dev::mbarrier_arrive_expect_tx(&s.full[st], kStageBytes);
      tma_load_2d(a_hi(st), &p.a_hi, k0, m0, &s.full[st]);
      tma_load_2d(a_lo(st), &p.a_lo, k0, m0, &s.full[st]);
      tma_load_2d(b_hi(st), &p.b_hi, k0, n_first, &s.full[st]);
      tma_load_2d(b_hi(st) + kBytesB / 2u, &p.b_hi, k0, n_second, &s.full[st]);
      tma_load_2d(b_lo(st), &p.b_lo, k0, n_first, &s.full[st]);
      tma_load_2d(b_lo(st) + kBytesB / 2u, &p.b_lo, k0, n_second, &s.full[st]);
      ++issued;
    }
    // Wait for the newest load of every stage (already consumed when
    // nothing failed) so that no copy lands after the exit.
    const dev::Deadline drain(p.wait_limit_ms);
    for (uint32_t i = issued > kStages ? issued - kStages : 0; i < issued; ++i) {
      if (!dev::mbarrier_wait(&s.full[i % kStages], (i / kStages) & 1u, drain)) {
        fail();
      }
    }
  } else if (warp == 1 && lane == 0) {
    // MMA issuer: per stage two K = 8 steps, three products each.
    for (uint32_t i = 0; i < count; ++i) {
      const uint32_t st = i % kStages;
      if (!dev::mbarrier_wait(&s.full[st], (i / kStages) & 1u, deadline)) {
        fail();
        break;
      }
      tc_fence_after();
      const uint64_t ah = sw64_descriptor(a_hi(st)), al = sw64_descriptor(a_lo(st));
      const uint64_t bh = sw64_descriptor(b_hi(st)), bl = sw64_descriptor(b_lo(st));
#pragma unroll
      for (uint32_t kk = 0; kk < pf::kTcTileK / 8u; ++kk) {
        const uint64_t step = kk * 2u; // 32 bytes, in 16-byte descriptor units
        const uint32_t first = (i | kk) != 0 ? 1u : 0u;
        tc_mma(tmem, ah + step, bh + step, kInstruction, first);
        tc_mma(tmem, ah + step, bl + step, kInstruction, 1u);
        tc_mma(tmem, al + step, bh + step, kInstruction, 1u);
        if constexpr (kSplitMma) {
          // The second half of B (the up rows, 512-byte aligned) into
          // accumulator columns kMmaN..kN - 1.
          constexpr uint64_t kHalf = (kBytesB / 2u) >> 4u; // descriptor units
          tc_mma(tmem + kMmaN, ah + step, bh + kHalf + step, kInstruction, first);
          tc_mma(tmem + kMmaN, ah + step, bl + kHalf + step, kInstruction, 1u);
          tc_mma(tmem + kMmaN, al + step, bh + kHalf + step, kInstruction, 1u);
        }
      }
      tc_commit(&s.empty[st]);
    }
    tc_commit(&s.done);
  }
  __syncwarp();

  // Epilogue: thread (warp, lane) reads accumulator row 32 * warp + lane
  // from TMEM, 32 columns at a time; the warp stages the 32 x 32 chunk in
  // shared memory (the consumed stage ring) and stores it row by row, eight
  // lanes per 128-byte row segment.
  const dev::Deadline finish(p.wait_limit_ms);
  const bool ready = dev::mbarrier_wait(&s.done, 0, finish);
  if (!ready) {
    fail();
  }
  __syncwarp(); // the warp-collective TMEM loads below run converged
  tc_fence_after();
  const uint32_t lane_address = tmem + ((warp * 32u) << 16);
  const uint32_t row_base = m0 + warp * 32u;
  // Warps whose 32 rows all lie past m (short batches) store nothing.
  const bool store = ready && s.abort == 0 && count != 0 && row_base < p.m;
  float *stage = reinterpret_cast<float *>(tiles) + warp * 32u * 33u; // [32][33] per warp
  const bool partial = p.mode == static_cast<uint32_t>(pf::GemmEpilogue::partial);
  // Writes this thread's 32 values into the staging rows, then each lane
  // emits float4 (row, column) pieces through `emit`. A tile with at most 32
  // valid rows (short batches: warp 0 alone stores) skips the staging: each
  // thread emits its own row, whose eight float4s already fill whole lines.
  const bool direct_rows = p.m <= m0 + 32u;
  auto staged = [&](const float (&v)[32], auto emit) {
    if (direct_rows) {
#pragma unroll
      for (uint32_t c = 0; c < 32u; c += 4u) {
        emit(lane, c, make_float4(v[c], v[c + 1u], v[c + 2u], v[c + 3u]));
      }
      return;
    }
#pragma unroll
    for (uint32_t j = 0; j < 32; ++j) {
      stage[lane * 33u + j] = v[j];
    }
    __syncwarp();
#pragma unroll
    for (uint32_t it = 0; it < 8; ++it) {
      const uint32_t r = it * 4u + lane / 8u, c = (lane % 8u) * 4u;
      const float4 x = make_float4(stage[r * 33u + c], stage[r * 33u + c + 1u],
                                   stage[r * 33u + c + 2u], stage[r * 33u + c + 3u]);
      emit(r, c, x);
    }
    __syncwarp();
  };
  if (partial) {
    float *out = p.c + (size_t{blockIdx.z} * p.tile_count + blockIdx.x) * pf::kTcTileM * kN +
                 size_t{warp * 32u} * kN;
#pragma unroll 1
    for (uint32_t chunk = 0; chunk < kN / 32u; ++chunk) {
      float v[32];
      tc_load32(lane_address + chunk * 32u, v);
      if (store) {
        staged(v, [&](uint32_t r, uint32_t c, float4 x) {
          if (row_base + r < p.m) {
            *reinterpret_cast<float4 *>(out + size_t{r} * kN + chunk * 32u + c) = x;
          }
        });
      }
    }
  } else if (swiglu) {
    // Gate columns [0, kN / 2), up columns [kN / 2, kN): whole 32-column
    // chunks, then (kN / 2 = 144) a 16-column tail.
#pragma unroll 1
    for (uint32_t chunk = 0; chunk < kN / 64u; ++chunk) {
      float gate[32], up[32];
      tc_load32(lane_address + chunk * 32u, gate);
      tc_load32(lane_address + kN / 2u + chunk * 32u, up);
      const uint32_t column = n_tile * (kN / 2u) + chunk * 32u;
      if (store && column < p.n) {
#pragma unroll
        for (uint32_t j = 0; j < 32; ++j) {
          gate[j] = silu_times(gate[j], up[j]);
        }
        staged(gate, [&](uint32_t r, uint32_t c, float4 x) {
          if (row_base + r < p.m && column + c < p.n) {
            const size_t at = size_t{row_base + r} * p.ldc + column + c;
            if (p.c_lo == nullptr) {
              *reinterpret_cast<float4 *>(p.c + at) = x;
            } else {
              const float4 hi = make_float4(to_tf32(x.x), to_tf32(x.y), to_tf32(x.z), to_tf32(x.w));
              *reinterpret_cast<float4 *>(p.c + at) = hi;
              *reinterpret_cast<float4 *>(p.c_lo + at) =
                  make_float4(to_tf32(x.x - hi.x), to_tf32(x.y - hi.y), to_tf32(x.z - hi.z),
                              to_tf32(x.w - hi.w));
            }
          }
        });
      }
    }
    if constexpr ((kN / 2u) % 32u != 0u) {
      static_assert((kN / 2u) % 32u == 16u, "a 16-column tail");
      constexpr uint32_t kTail = kN / 2u - 16u;
      float gate[16], up[16];
      tc_load16(lane_address + kTail, gate);
      tc_load16(lane_address + kN / 2u + kTail, up);
      const uint32_t row = row_base + lane;
      const uint32_t column = n_tile * (kN / 2u) + kTail;
      if (store && row < p.m) {
#pragma unroll
        for (uint32_t c = 0; c < 16u; c += 4u) {
          if (column + c < p.n) {
            const size_t at = size_t{row} * p.ldc + column + c;
            const float4 x = make_float4(silu_times(gate[c], up[c]), silu_times(gate[c + 1u], up[c + 1u]),
                                         silu_times(gate[c + 2u], up[c + 2u]),
                                         silu_times(gate[c + 3u], up[c + 3u]));
            if (p.c_lo == nullptr) {
              *reinterpret_cast<float4 *>(p.c + at) = x;
            } else {
              const float4 hi = make_float4(to_tf32(x.x), to_tf32(x.y), to_tf32(x.z), to_tf32(x.w));
              *reinterpret_cast<float4 *>(p.c + at) = hi;
              *reinterpret_cast<float4 *>(p.c_lo + at) =
                  make_float4(to_tf32(x.x - hi.x), to_tf32(x.y - hi.y), to_tf32(x.z - hi.z),
                              to_tf32(x.w - hi.w));
            }
          }
        }
      }
    }
  } else {
#pragma unroll 1
    for (uint32_t chunk = 0; chunk < kN / 32u; ++chunk) {
      float v[32];
      tc_load32(lane_address + chunk * 32u, v);
      const uint32_t column = n_tile * kN + chunk * 32u;
      if (store && column < p.n) {
        staged(v, [&](uint32_t r, uint32_t c, float4 x) {
          if (row_base + r < p.m) {
            const size_t at = size_t{row_base + r} * p.ldc + column + c;
            const float values[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
            for (uint32_t e = 0; e < 4; ++e) {
              finish_element(p.bias, p.c, p.c_lo, at + e, column + c + e, p.mode, values[e],
                             0.0f);
            }
          }
        });
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(kTmemColumns)
                 : "memory");
  }
}

extern "C" __global__ void __launch_bounds__(pf::kTcThreads, 1)
    prefill_tc_gemm_n192(const __grid_constant__ pf::TcGemmArgs p) {
  tc_gemm<192>(p);
}

extern "C" __global__ void __launch_bounds__(pf::kTcThreads, 1)
    prefill_tc_gemm_n224(const __grid_constant__ pf::TcGemmArgs p) {
  tc_gemm<224>(p);
}

extern "C" __global__ void __launch_bounds__(pf::kTcThreads, 1)
    prefill_tc_gemm_n256(const __grid_constant__ pf::TcGemmArgs p) {
  tc_gemm<256>(p);
}

// Gate/up pairs of 144 + 144 columns (swiglu, or its split-K partials).
extern "C" __global__ void __launch_bounds__(pf::kTcThreads, 1)
    prefill_tc_gemm_pair288(const __grid_constant__ pf::TcGemmArgs p) {
  tc_gemm<pf::kTcPairN>(p);
}

// Narrow 3xTF32 GEMM (m <= kNarrowRows rows) with the operands swapped:
// CTA (x, 0, z) computes output columns [n0, n0 + 128), n0 = 128 *
// (tile_offset + x), over K slice z as D^T = W . X^T: the 128 weight rows
// (TMA map a_hi over the FP32 weights, box 16 x 128) are the MMA's A
// operand (M = 128) and the 32 activation rows (b_hi / b_lo, box 16 x 32;
// rows past m are never stored) its B operand (N = 32), so the tensor cores
// spend nothing on padding rows and each weight byte is read from HBM once
// per step, as FP32: warps 2 and 3 split every landed weight tile in place
// into its TF32 pair (hi = the top 10 mantissa bits, lo = w - hi exactly,
// written beside it) and release the stage to the MMA warp. kPaired
// (swiglu): a second accumulator takes the up rows n_gate_offset + n0...;
// the gate/up pair lands on the same thread. Same ring and bounded waits as
// tc_gemm; thread (warp, lane) owns output column n0 + 32 * warp + lane and
// walks the rows, so each row's 32 columns per warp are one 128-byte store.
// Partial tiles: [split][tile][kNarrowRows][128 or 256].
template <uint32_t kStages> struct NarrowShared {
  uint64_t full[kStages];      // TMA landed
  uint64_t converted[kStages]; // weight tiles split (64 converter arrivals)
  uint64_t empty[kStages];     // MMAs done
  uint64_t done;
  uint32_t tmem;
  uint32_t abort;
};
static_assert(sizeof(NarrowShared<8>) <= 256u, "within the 256 bytes the host adds");

template <bool kPaired, bool kSharedSm = false>
__device__ __forceinline__ void tc_narrow(const pf::TcGemmArgs &p) {
  constexpr uint32_t kStages = pf::tc_narrow_stages(kPaired, kSharedSm);
  constexpr uint32_t kStageBytes = pf::tc_narrow_stage_bytes(kPaired);
  constexpr uint32_t kWeightBytes = pf::kNarrowTileN * pf::kTcTileK * 4u;
  constexpr uint32_t kRowBytes = pf::kNarrowRows * pf::kTcTileK * 4u;
  constexpr uint32_t kWeights = kPaired ? 2u : 1u;
  constexpr uint32_t kTileColumns = kWeights * pf::kNarrowTileN;
  constexpr uint32_t kInstruction = tc_instruction<pf::kNarrowRows>();
  constexpr uint32_t kConverters = 64;                         // warps 2 and 3
  constexpr uint32_t kLoadBytes = kStageBytes - kWeights * kWeightBytes; // no W_lo
  static_assert(pf::kTcThreads == 128u && kWeightBytes % (16u * kConverters) == 0,
                "two converter warps, whole float4s each");
  static_assert(kWeightBytes % 512 == 0 && kRowBytes % 512 == 0, "swizzle atom alignment");
  extern __shared__ __align__(1024) unsigned char raw_shared[];
  unsigned char *tiles = reinterpret_cast<unsigned char *>(
      (reinterpret_cast<uintptr_t>(raw_shared) + 1023u) & ~uintptr_t{1023});
  auto &s = *reinterpret_cast<NarrowShared<kStages> *>(tiles + kStages * kStageBytes);
  // Stage: W_hi, W_lo (then the up rows' W_hi, W_lo), X_hi, X_lo. TMA fills
  // W_hi with the FP32 weights; the converters rewrite it as hi and fill W_lo.
  auto w_hi = [&](uint32_t st, uint32_t w) { return tiles + st * kStageBytes + 2u * w * kWeightBytes; };
  auto w_lo = [&](uint32_t st, uint32_t w) { return w_hi(st, w) + kWeightBytes; };
  auto x_hi = [&](uint32_t st) { return tiles + st * kStageBytes + 2u * kWeights * kWeightBytes; };
  auto x_lo = [&](uint32_t st) { return x_hi(st) + kRowBytes; };

  const uint32_t warp = threadIdx.x >> 5u, lane = threadIdx.x & 31u;
  const uint32_t tile = p.tile_offset + blockIdx.x;
  const uint32_t n0 = tile * pf::kNarrowTileN;
  const uint32_t k_tiles = p.k / pf::kTcTileK;
  const uint32_t first_tile = blockIdx.z * k_tiles / p.splits;
  const uint32_t count = (blockIdx.z + 1u) * k_tiles / p.splits - first_tile;
  const dev::Deadline deadline(p.wait_limit_ms);

  if (threadIdx.x == 0) {
    for (uint32_t i = 0; i < kStages; ++i) {
      dev::mbarrier_init(&s.full[i], 1);
      dev::mbarrier_init(&s.converted[i], kConverters);
      dev::mbarrier_init(&s.empty[i], 1);
    }
    dev::mbarrier_init(&s.done, 1);
    s.abort = 0;
    dev::mbarrier_init_fence();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     dev::shared_address(&s.tmem)),
                 "r"(pf::kNarrowTmemColumns)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s.tmem;
  dependent_launch_entry(); // barriers and TMEM are ready; operands come next

  auto fail = [&]() {
    s.abort = 1;
    atomicExch(p.error, pf::kTcErrorWaitTimeout);
  };

  if (warp == 0 && lane == 0) {
    uint32_t issued = 0;
    for (uint32_t i = 0; i < count && s.abort == 0; ++i) {
      const uint32_t st = i % kStages;
      if (i >= kStages && !dev::mbarrier_wait(&s.empty[st], ((i / kStages) + 1u) & 1u, deadline)) {
        fail();
        break;
      }
      const uint32_t k0 = (first_tile + i) * pf::kTcTileK;
      dev::mbarrier_arrive_expect_tx(&s.full[st], kLoadBytes);
#pragma unroll
      for (uint32_t w = 0; w < kWeights; ++w) {
        const uint32_t row = w == 0 ? n0 : p.n_gate_offset + n0;
        tma_load_2d(w_hi(st, w), &p.a_hi, k0, row, &s.full[st]);
      }
      tma_load_2d(x_hi(st), &p.b_hi, k0, 0, &s.full[st]);
      tma_load_2d(x_lo(st), &p.b_lo, k0, 0, &s.full[st]);
      ++issued;
    }
    const dev::Deadline drain(p.wait_limit_ms);
    for (uint32_t i = issued > kStages ? issued - kStages : 0; i < issued; ++i) {
      if (!dev::mbarrier_wait(&s.full[i % kStages], (i / kStages) & 1u, drain)) {
        fail();
      }
    }
  } else if (warp >= 2) {
    // Converters: per landed stage, w -> (hi, lo) for every weight tile
    // (elementwise, so the swizzled layout is kept), then release it.
    const uint32_t t = threadIdx.x - 64u;
    for (uint32_t i = 0; i < count; ++i) {
      const uint32_t st = i % kStages;
      if (!dev::mbarrier_wait(&s.full[st], (i / kStages) & 1u, deadline)) {
        fail();
        break;
      }
#pragma unroll
      for (uint32_t w = 0; w < kWeights; ++w) {
        float4 *hi = reinterpret_cast<float4 *>(w_hi(st, w));
        float4 *lo = reinterpret_cast<float4 *>(w_lo(st, w));
#pragma unroll
        for (uint32_t j = 0; j < kWeightBytes / (16u * kConverters); ++j) {
          const float4 x = hi[t + kConverters * j];
          const float4 h =
              make_float4(tf32_high(x.x), tf32_high(x.y), tf32_high(x.z), tf32_high(x.w));
          hi[t + kConverters * j] = h;
          lo[t + kConverters * j] = make_float4(x.x - h.x, x.y - h.y, x.z - h.z, x.w - h.w);
        }
      }
      proxy_fence_shared();
      asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(
                       dev::shared_address(&s.converted[st]))
                   : "memory");
    }
  } else if (warp == 1 && lane == 0) {
    // Per stage two K = 8 steps, three products per accumulator each.
    for (uint32_t i = 0; i < count; ++i) {
      const uint32_t st = i % kStages;
      if (!dev::mbarrier_wait(&s.converted[st], (i / kStages) & 1u, deadline)) {
        fail();
        break;
      }
      tc_fence_after();
      const uint64_t xh = sw64_descriptor(x_hi(st)), xl = sw64_descriptor(x_lo(st));
#pragma unroll
      for (uint32_t w = 0; w < kWeights; ++w) {
        const uint64_t wh = sw64_descriptor(w_hi(st, w)), wl = sw64_descriptor(w_lo(st, w));
        const uint32_t d = tmem + w * pf::kNarrowRows;
#pragma unroll
        for (uint32_t kk = 0; kk < pf::kTcTileK / 8u; ++kk) {
          const uint64_t step = kk * 2u; // 32 bytes, in 16-byte descriptor units
          tc_mma(d, wh + step, xh + step, kInstruction, (i | kk) != 0 ? 1u : 0u);
          tc_mma(d, wh + step, xl + step, kInstruction, 1u);
          tc_mma(d, wl + step, xh + step, kInstruction, 1u);
        }
      }
      tc_commit(&s.empty[st]);
    }
    tc_commit(&s.done);
  }
  __syncwarp();

  const dev::Deadline finish(p.wait_limit_ms);
  const bool ready = dev::mbarrier_wait(&s.done, 0, finish);
  if (!ready) {
    fail();
  }
  __syncwarp(); // the warp-collective TMEM loads below run converged
  tc_fence_after();
  const uint32_t lane_address = tmem + ((warp * 32u) << 16);
  const uint32_t local = warp * 32u + lane; // column within the tile
  const uint32_t column = n0 + local;
  const bool store = ready && s.abort == 0 && count != 0;
  float v[32];
  tc_load32(lane_address, v);
  float up[32];
  if (kPaired) {
    tc_load32(lane_address + pf::kNarrowRows, up);
  }
  if (store) {
    if (p.mode == static_cast<uint32_t>(pf::GemmEpilogue::partial)) {
      float *out = p.c + (size_t{blockIdx.z} * p.tile_count + blockIdx.x) * pf::kNarrowRows *
                             kTileColumns +
                   local;
#pragma unroll
      for (uint32_t r = 0; r < pf::kNarrowRows; ++r) {
        if (r < p.m) {
          out[r * kTileColumns] = v[r];
          if (kPaired) {
            out[r * kTileColumns + pf::kNarrowTileN] = up[r];
          }
        }
      }
    } else if (column < p.n) {
#pragma unroll
      for (uint32_t r = 0; r < pf::kNarrowRows; ++r) {
        if (r < p.m) {
          const size_t at = size_t{r} * p.ldc + column;
          if (kPaired) {
            store_operand(p.c, p.c_lo, at, silu_times(v[r], up[r]));
          } else {
            finish_element(p.bias, p.c, p.c_lo, at, column, p.mode, v[r], 0.0f);
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(pf::kNarrowTmemColumns)
                 : "memory");
  }
}

extern "C" __global__ void __launch_bounds__(pf::kTcThreads, 1)
    prefill_tc_narrow(const __grid_constant__ pf::TcGemmArgs p) {
  tc_narrow<false>(p);
}

extern "C" __global__ void __launch_bounds__(pf::kTcThreads, 1)
    prefill_tc_narrow_pair(const __grid_constant__ pf::TcGemmArgs p) {
  tc_narrow<true>(p);
}

// The same with a half-size ring, two CTAs per SM (launches of more than
// one wave of tiles).
extern "C" __global__ void __launch_bounds__(pf::kTcThreads, 2)
    prefill_tc_narrow_shared_sm(const __grid_constant__ pf::TcGemmArgs p) {
  tc_narrow<false, true>(p);
}

// ------------------------------------------------------- batched decode --

// Decode attention of one query row per stream, split over key positions;
// the last split block of a (stream, KV group) merges the splits.
// Block (s, g, b) serves the 7 query heads 7g..7g+6 of KV head g of stream b
// over key positions [s * chunk, min((s + 1) * chunk, positions[b] + 1)), in
// tiles of kDecodeTileKeys keys copied into shared memory with cp.async into
// two buffers: tile t + 1 (K, then V, as two groups; positions past the
// range zero-filled) is in flight while tile t is computed. Each staged
// element is read once per block for all 7 heads:
//   scores: warp w sums dims 8w..8w+7 of keys l and l + 32 (lane l, float4
//           reads along the key rows) for all 7 heads; the 8 dim-slice
//           partials are summed in slice order by warp h (head h), which
//           runs the decode step's online softmax (scale 1/8, expf);
//   P.V:    warp w accumulates keys 8w..8w+7 into dims 2l, 2l + 1 of all 7
//           heads; the 8 key-slice sums are added in slice order after the
//           last tile.
using pf::kDecodeTileKeys;
constexpr uint32_t kDecodeSlices = 8; // warps
constexpr uint32_t kDecodeKeyPitch = qd::kHeadSize + 4u; // conflict-free float4 column reads

struct DecodeBuffer {
  // The tile's K rows; after the score sums, the same bytes hold the
  // dim-slice partial scores.
  union {
    float ks[kDecodeTileKeys][kDecodeKeyPitch];
    float scores[kDecodeSlices][qd::kQueriesPerKvHead][kDecodeTileKeys];
  };
  float vs[kDecodeTileKeys][qd::kHeadSize]; // [key][d]
};

struct DecodeShared {
  union {
    DecodeBuffer buffer[2];
    // After the last tile: the key slices' partial P.V sums.
    float sums[kDecodeSlices][qd::kQueriesPerKvHead][qd::kHeadSize];
  };
  float q[qd::kQueriesPerKvHead][qd::kHeadSize];
  float probability[qd::kQueriesPerKvHead][kDecodeTileKeys]; // the tile's softmax weights
  float rescale[kDecodeSlices];                              // per head, [7] unused
  float weight[qd::kQueriesPerKvHead][32];                   // merge: per (head, split) scale
  float total[qd::kQueriesPerKvHead];
};

static_assert(sizeof(DecodeShared) == pf::kDecodeSharedBytes, "decode shared layout");

extern "C" __global__ void __launch_bounds__(256) batch_attention(pf::DecodeAttentionArgs p) {
  dependent_launch_entry();
  extern __shared__ __align__(16) unsigned char decode_raw[];
  DecodeShared &sh = *reinterpret_cast<DecodeShared *>(decode_raw);
  const uint32_t split = blockIdx.x, group = blockIdx.y, b = blockIdx.z;
  const uint32_t warp = threadIdx.x >> 5u, lane = threadIdx.x & 31u;
  const uint32_t last = p.positions[b];
  const uint32_t begin = split * p.chunk;
  const uint32_t end = min(begin + p.chunk, last + 1u);
  if (threadIdx.x < qd::kQueriesPerKvHead * qd::kHeadSize / 4u) {
    reinterpret_cast<float4 *>(&sh.q[0][0])[threadIdx.x] = reinterpret_cast<const float4 *>(
        p.qkv + size_t{b} * qd::kPackedQkvSize +
        group * qd::kQueriesPerKvHead * qd::kHeadSize)[threadIdx.x];
  }
  const float *keys = p.key_cache + b * p.stream_stride + size_t{group} * qd::kHeadSize;
  const float *values = p.value_cache + b * p.stream_stride + size_t{group} * qd::kHeadSize;
  // Thread t copies 16-byte chunks t + 256j of the tile (row = chunk / 16):
  // coalesced 256-byte row reads; rows at or past `end` read nothing and
  // become 0. K and V are committed as two groups.
  auto issue = [&](DecodeBuffer &buffer, uint32_t base) {
    constexpr uint32_t kChunks = kDecodeTileKeys * qd::kHeadSize / 4u / 256u;
#pragma unroll
    for (uint32_t j = 0; j < kChunks; ++j) {
      const uint32_t i = threadIdx.x + 256u * j, key = i / 16u, c = (i % 16u) * 4u;
      const bool valid = base + key < end;
      copy16_async(&buffer.ks[key][c], keys + size_t{valid ? base + key : base} * qd::kKvSize + c,
                   valid ? 16u : 0u);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
#pragma unroll
    for (uint32_t j = 0; j < kChunks; ++j) {
      const uint32_t i = threadIdx.x + 256u * j, key = i / 16u, c = (i % 16u) * 4u;
      const bool valid = base + key < end;
      copy16_async(&buffer.vs[key][c], values + size_t{valid ? base + key : base} * qd::kKvSize + c,
                   valid ? 16u : 0u);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  // Warp h < 7: head h's running maximum and denominator (all lanes alike).
  float maximum = -INFINITY, denominator = 0.0f;
  float acc[qd::kQueriesPerKvHead][2] = {};
  if (begin < end) {
    issue(sh.buffer[0], begin);
  }
  uint32_t t = 0;
  for (uint32_t base = begin; base < end; base += kDecodeTileKeys, ++t) {
    DecodeBuffer &buffer = sh.buffer[t & 1u];
    __syncthreads(); // the previous tile's reads are done (and q is written)
    const bool next = base + kDecodeTileKeys < end;
    if (next) {
      issue(sh.buffer[(t + 1u) & 1u], base + kDecodeTileKeys);
      copy_wait<3>(); // this thread's K chunks of tile t
    } else {
      copy_wait<1>();
    }
    __syncthreads();
    // Dim slice `warp` of the 7 x 2 scores of keys l + 32j.
    float score[qd::kQueriesPerKvHead][2] = {};
#pragma unroll
    for (uint32_t half = 0; half < 2u; ++half) {
      const uint32_t d0 = kDecodeSlices * warp + 4u * half;
      float4 key4[2];
#pragma unroll
      for (uint32_t j = 0; j < 2u; ++j) {
        key4[j] = *reinterpret_cast<const float4 *>(&buffer.ks[lane + 32u * j][d0]);
      }
#pragma unroll
      for (uint32_t h = 0; h < qd::kQueriesPerKvHead; ++h) {
        const float4 q = *reinterpret_cast<const float4 *>(&sh.q[h][d0]);
#pragma unroll
        for (uint32_t j = 0; j < 2u; ++j) {
          score[h][j] = fmaf(q.x, key4[j].x, score[h][j]);
          score[h][j] = fmaf(q.y, key4[j].y, score[h][j]);
          score[h][j] = fmaf(q.z, key4[j].z, score[h][j]);
          score[h][j] = fmaf(q.w, key4[j].w, score[h][j]);
        }
      }
    }
    __syncthreads(); // K reads are done: its bytes take the partial scores
#pragma unroll
    for (uint32_t h = 0; h < qd::kQueriesPerKvHead; ++h) {
#pragma unroll
      for (uint32_t j = 0; j < 2u; ++j) {
        buffer.scores[warp][h][lane + 32u * j] = score[h][j];
      }
    }
    __syncthreads();
    if (warp < qd::kQueriesPerKvHead) {
      float s2[2];
#pragma unroll
      for (uint32_t j = 0; j < 2u; ++j) {
        s2[j] = buffer.scores[0][warp][lane + 32u * j];
      }
#pragma unroll
      for (uint32_t slice = 1; slice < kDecodeSlices; ++slice) {
#pragma unroll
        for (uint32_t j = 0; j < 2u; ++j) {
          s2[j] += buffer.scores[slice][warp][lane + 32u * j];
        }
      }
      float tile_maximum = -INFINITY;
#pragma unroll
      for (uint32_t j = 0; j < 2u; ++j) {
        s2[j] = base + lane + 32u * j < end ? s2[j] * 0.125f : -INFINITY;
        tile_maximum = fmaxf(tile_maximum, s2[j]);
      }
#pragma unroll
      for (uint32_t offset = 16; offset != 0; offset >>= 1u) {
        tile_maximum = fmaxf(tile_maximum, __shfl_xor_sync(kFullMask, tile_maximum, offset));
      }
      const float next_maximum = fmaxf(maximum, tile_maximum); // finite: key `base` is in range
      const float scale = expf(maximum - next_maximum);
      float sum = 0.0f;
#pragma unroll
      for (uint32_t j = 0; j < 2u; ++j) {
        const float w = expf(s2[j] - next_maximum);
        sh.probability[warp][lane + 32u * j] = w;
        sum += w;
      }
#pragma unroll
      for (uint32_t offset = 16; offset != 0; offset >>= 1u) {
        sum += __shfl_xor_sync(kFullMask, sum, offset);
      }
      denominator = denominator * scale + sum;
      maximum = next_maximum;
      if (lane == 0) {
        sh.rescale[warp] = scale;
      }
    }
    if (next) {
      copy_wait<2>(); // this thread's V chunks of tile t
    } else {
      copy_wait<0>();
    }
    __syncthreads();
    // Key slice `warp` (keys 8w..8w+7) into dims 2l, 2l + 1 of the 7 heads.
#pragma unroll
    for (uint32_t h = 0; h < qd::kQueriesPerKvHead; ++h) {
      const float scale = sh.rescale[h];
      acc[h][0] *= scale;
      acc[h][1] *= scale;
    }
#pragma unroll
    for (uint32_t c = 0; c < 2u; ++c) {
      const uint32_t key0 = 8u * warp + 4u * c;
      float4 weight[qd::kQueriesPerKvHead];
#pragma unroll
      for (uint32_t h = 0; h < qd::kQueriesPerKvHead; ++h) {
        weight[h] = *reinterpret_cast<const float4 *>(&sh.probability[h][key0]);
      }
#pragma unroll
      for (uint32_t j = 0; j < 4u; ++j) {
        const float2 v2 = *reinterpret_cast<const float2 *>(&buffer.vs[key0 + j][2u * lane]);
#pragma unroll
        for (uint32_t h = 0; h < qd::kQueriesPerKvHead; ++h) {
          const float pj =
              j == 0 ? weight[h].x : j == 1 ? weight[h].y : j == 2 ? weight[h].z : weight[h].w;
          acc[h][0] = fmaf(pj, v2.x, acc[h][0]);
          acc[h][1] = fmaf(pj, v2.y, acc[h][1]);
        }
      }
    }
  }
  __syncthreads(); // the last tile's reads are done: its bytes take the sums
#pragma unroll
  for (uint32_t h = 0; h < qd::kQueriesPerKvHead; ++h) {
    *reinterpret_cast<float2 *>(&sh.sums[warp][h][2u * lane]) = make_float2(acc[h][0], acc[h][1]);
  }
  __syncthreads();
  const float *group_partials = p.partials + (size_t{b} * qd::kKvHeads + group) * p.splits *
                                                 qd::kQueriesPerKvHead * pf::kDecodePartialStride;
  const size_t split_stride = size_t{qd::kQueriesPerKvHead} * pf::kDecodePartialStride;
  float *own = const_cast<float *>(group_partials) + split * split_stride;
  for (uint32_t i = threadIdx.x; i < qd::kQueriesPerKvHead * qd::kHeadSize; i += 256u) {
    const uint32_t h = i / qd::kHeadSize, d = i % qd::kHeadSize;
    float value = sh.sums[0][h][d];
#pragma unroll
    for (uint32_t slice = 1; slice < kDecodeSlices; ++slice) {
      value += sh.sums[slice][h][d];
    }
    own[size_t{h} * pf::kDecodePartialStride + d] = value;
  }
  if (warp < qd::kQueriesPerKvHead && lane == 0) {
    own[size_t{warp} * pf::kDecodePartialStride + 64] = maximum;     // -inf: the split holds
    own[size_t{warp} * pf::kDecodePartialStride + 65] = denominator; // no key of this stream
  }
  // The last split block of (b, group) to arrive combines the splits: per
  // head, rescale to the common maximum, sum, divide.
  __shared__ bool finisher;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint32_t arrived = atomicAdd(&p.arrivals[b * qd::kKvHeads + group], 1u);
    finisher = arrived == p.splits - 1u;
  }
  __syncthreads();
  if (!finisher) {
    return;
  }
  __threadfence();
  if (warp < qd::kQueriesPerKvHead) {
    // Warp h: the head's per-split maxima and sums (lane = split).
    const float *first = group_partials + size_t{warp} * pf::kDecodePartialStride;
    const float m = lane < p.splits ? __ldcg(first + lane * split_stride + 64) : -INFINITY;
    const float l = lane < p.splits ? __ldcg(first + lane * split_stride + 65) : 0.0f;
    float common = m;
#pragma unroll
    for (uint32_t offset = 16; offset != 0; offset >>= 1u) {
      common = fmaxf(common, __shfl_xor_sync(kFullMask, common, offset));
    }
    const float weight = m != -INFINITY ? expf(m - common) : 0.0f;
    sh.weight[warp][lane] = weight;
    // Sum in split order (lane 0 walks the lanes' terms).
    float total = 0.0f;
    for (uint32_t s2 = 0; s2 < p.splits; ++s2) {
      total += __shfl_sync(kFullMask, l * weight, s2);
    }
    if (lane == 0) {
      sh.total[warp] = total;
    }
  }
  __syncthreads();
  for (uint32_t i = threadIdx.x; i < qd::kQueriesPerKvHead * qd::kHeadSize; i += blockDim.x) {
    const uint32_t local = i / qd::kHeadSize, d = i % qd::kHeadSize;
    const float *first = group_partials + size_t{local} * pf::kDecodePartialStride + d;
    float value = 0.0f;
    uint32_t s2 = 0;
    for (; s2 + 4u <= p.splits; s2 += 4u) {
      const float a0 = __ldcg(first + s2 * split_stride);
      const float a1 = __ldcg(first + (s2 + 1u) * split_stride);
      const float a2 = __ldcg(first + (s2 + 2u) * split_stride);
      const float a3 = __ldcg(first + (s2 + 3u) * split_stride);
      value += a0 * sh.weight[local][s2];
      value += a1 * sh.weight[local][s2 + 1u];
      value += a2 * sh.weight[local][s2 + 2u];
      value += a3 * sh.weight[local][s2 + 3u];
    }
    for (; s2 < p.splits; ++s2) {
      value += __ldcg(first + s2 * split_stride) * sh.weight[local][s2];
    }
    const uint32_t head = group * qd::kQueriesPerKvHead + local;
    store_operand(p.out, p.out_lo, size_t{b} * qd::kQuerySize + head * qd::kHeadSize + d,
                  value / sh.total[local]);
  }
  if (threadIdx.x == 0) {
    p.arrivals[b * qd::kKvHeads + group] = 0; // ready for the next step
  }
}

// Greedy token of each stream row. Block (part, b) scans columns
// [part * width, (part + 1) * width) of row b (per-thread best over a strided
// range, loads issued four at a time), then warp and block reductions keep
// the larger logit and, on equal logits, the lower index (the decode step's
// better_top1 rule); the block's winner goes to the row's candidate slot. The
// last block of the row to finish (per-row arrival counter, reset by that
// block) reduces the candidates in partition order and publishes the token.
__device__ __forceinline__ bool better_top1(float va, uint32_t ia, float vb, uint32_t ib) {
  return vb > va || (vb == va && ib < ia);
}

__device__ __forceinline__ void block_top1(float &value, uint32_t &index, float *values,
                                           uint32_t *indices) {
  const uint32_t warp = threadIdx.x >> 5u, lane = threadIdx.x & 31u;
#pragma unroll
  for (uint32_t offset = 16; offset != 0; offset >>= 1u) {
    const float v = __shfl_xor_sync(kFullMask, value, offset);
    const uint32_t i = __shfl_xor_sync(kFullMask, index, offset);
    if (better_top1(value, index, v, i)) {
      value = v;
      index = i;
    }
  }
  if (lane == 0) {
    values[warp] = value;
    indices[warp] = index;
  }
  __syncthreads();
  if (warp == 0) {
    value = lane < blockDim.x / 32u ? values[lane] : -INFINITY;
    index = lane < blockDim.x / 32u ? indices[lane] : UINT32_MAX;
#pragma unroll
    for (uint32_t offset = 16; offset != 0; offset >>= 1u) {
      const float v = __shfl_xor_sync(kFullMask, value, offset);
      const uint32_t i = __shfl_xor_sync(kFullMask, index, offset);
      if (better_top1(value, index, v, i)) {
        value = v;
        index = i;
      }
    }
  }
}

extern "C" __global__ void __launch_bounds__(1024) batch_argmax(pf::ArgmaxArgs p) {
  dependent_launch_entry();
  __shared__ float values[32];
  __shared__ uint32_t indices[32];
  __shared__ bool finisher;
  const uint32_t part = blockIdx.x, b = blockIdx.y;
  const uint32_t width = (p.vocab + gridDim.x - 1u) / gridDim.x;
  const uint32_t begin = part * width, end = min(begin + width, p.vocab);
  const float *row = p.logits + size_t{b} * p.vocab;
  float value = -INFINITY;
  uint32_t index = UINT32_MAX;
  uint32_t i = begin + threadIdx.x;
  for (; i + 3u * blockDim.x < end; i += 4u * blockDim.x) {
    const float x0 = row[i], x1 = row[i + blockDim.x];
    const float x2 = row[i + 2u * blockDim.x], x3 = row[i + 3u * blockDim.x];
    const float xs[4] = {x0, x1, x2, x3};
#pragma unroll
    for (uint32_t j = 0; j < 4; ++j) {
      if (xs[j] > value || index == UINT32_MAX) {
        value = xs[j];
        index = i + j * blockDim.x;
      }
    }
  }
  for (; i < end; i += blockDim.x) {
    if (row[i] > value || index == UINT32_MAX) {
      value = row[i];
      index = i;
    }
  }
  block_top1(value, index, values, indices);
  if (threadIdx.x == 0) {
    p.candidate_values[b * gridDim.x + part] = value;
    p.candidate_indices[b * gridDim.x + part] = index;
    __threadfence();
    const uint32_t arrived = atomicAdd(&p.arrivals[b], 1u);
    finisher = arrived == gridDim.x - 1u;
  }
  __syncthreads();
  if (!finisher) {
    return;
  }
  __threadfence();
  if (threadIdx.x < 32u) {
    value = -INFINITY;
    index = UINT32_MAX;
    for (uint32_t c = threadIdx.x; c < gridDim.x; c += 32u) {
      const float v = __ldcg(&p.candidate_values[b * gridDim.x + c]);
      const uint32_t x = __ldcg(&p.candidate_indices[b * gridDim.x + c]);
      if (better_top1(value, index, v, x)) {
        value = v;
        index = x;
      }
    }
#pragma unroll
    for (uint32_t offset = 16; offset != 0; offset >>= 1u) {
      const float v = __shfl_xor_sync(kFullMask, value, offset);
      const uint32_t x = __shfl_xor_sync(kFullMask, index, offset);
      if (better_top1(value, index, v, x)) {
        value = v;
        index = x;
      }
    }
    if (threadIdx.x == 0) {
      const uint32_t slot = p.generated[b];
      p.tokens[size_t{b} * p.token_stride + slot] = index;
      p.generated[b] = slot + 1u;
      p.positions[b] += 1u;
      p.next_tokens[b] = index;
      p.logit_values[b] = value;
      p.arrivals[b] = 0; // ready for the next step
    }
  }
}
