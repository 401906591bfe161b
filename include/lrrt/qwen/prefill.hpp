// Kernel arguments of the prompt prefill module (qwen_prefill.cubin), shared
// by the device code and the host driver. Every kernel takes one of these
// structs by value, so the host launches them through lr_launch with the
// struct as the packed argument blob.
//
// Prefill runs one chunk of prompt tokens through all layers at once: the
// projections become GEMMs C[m][n] = A[m][k] . B[n][k] over the chunk's
// token rows (B is an nn.Linear weight, row-major [out][in]). There is no
// counterpart in light-rocm-runtime, whose prompts go through the decode step
// one token at a time; the per-token arithmetic is the decode step's.
//
// 3xTF32 operands: for the tensor-core GEMM every operand x is stored as two
// float arrays, hi = x rounded to TF32 and lo = (x - hi) rounded to TF32, and
// C = A_hi.B_hi + A_hi.B_lo + A_lo.B_hi accumulates in FP32. Producers of
// GEMM inputs write (hi, lo) pairs when `*_lo` is not null and plain FP32
// otherwise.
#ifndef LRRT_QWEN_PREFILL_HPP_
#define LRRT_QWEN_PREFILL_HPP_

#include <cstdint>

#if defined(__CUDACC__)
#define LRRT_PREFILL_HD __host__ __device__
#else
#define LRRT_PREFILL_HD
#endif

namespace lrrt::qwen::prefill {

// hidden[t] = table[tokens[t]]
struct EmbedArgs {
  const uint32_t *tokens;
  const float *table; // [rows][896]
  float *hidden;      // [count][896]
  uint32_t count;
  uint32_t rows;      // table rows; out-of-range tokens write zeros
};

// out[t] = hidden[t] * rsqrt(mean(hidden[t]^2) + epsilon) * weight
struct NormArgs {
  const float *hidden;
  const float *weight;
  float *out;    // FP32, or the TF32 hi part when out_lo is set
  float *out_lo; // optional TF32 lo part
  uint32_t count;
  float epsilon;
};

enum class GemmEpilogue : uint32_t {
  bias = 0,     // c = acc + bias[n]                            (QKV)
  residual = 1, // c += acc                                      (o_proj, down)
  swiglu = 2,   // c = silu(acc(gate)) * acc(up)                 (gate/up)
  partial = 3,  // compact split-K partial accumulators, finished by prefill_reduce
  store = 4,    // c = acc                                        (LM-head logits)
};

// SIMT FP32 GEMM (mode bias, residual or swiglu): A [m][k] (lda),
// B [n][k] (ldb), B2 the second weight for swiglu; c [m][ldc].
struct GemmArgs {
  const float *a;
  const float *b;
  const float *b2;
  const float *bias;
  float *c;
  float *c_lo; // swiglu only: optional TF32 lo part of the output
  uint32_t m, n, k, lda, ldb, ldc;
};

// Finishes split-K tiles of the tensor-core GEMM: for tiles
// [tile_offset, tile_offset + tile_count) of the output's tile grid
// (n_tiles per 128-row band), sums the `splits` compact partial
// accumulators [split][tile][128][tile_columns] in split order and applies
// the epilogue `mode` (bias, residual or swiglu) as the GEMM would have.
struct ReduceArgs {
  const float *partials;
  const float *bias;
  float *c;
  float *c_lo;
  uint32_t m, n, ldc;
  uint32_t mode;          // GemmEpilogue (not partial)
  uint32_t tile_offset, tile_count, n_tiles, splits;
  uint32_t tile_columns;  // accumulator columns per tile (swiglu: gate + up)
  uint32_t tile_rows;     // rows per tile: kTcTileM, or kNarrowRows
};

// Split-K partial accumulators of a tensor-core GEMM whose finish is left
// to the next row kernel: tiles [0, tile_count) of the output's tile grid
// (n_tiles per band of tile_rows rows), [split][tile][tile_rows][tile_columns].
struct PartialTiles {
  const float *partials; // null: the GEMM wrote its output directly
  uint32_t splits, n_tiles, tile_count, tile_columns, tile_rows;
};

// RoPE on the q and k parts of qkv rows [count][1152] at positions
// first_position + t, then k and v appended to the cache rows. With
// qkv_partials set, each row is first finished from the QKV GEMM's partial
// sums plus qkv_bias and written to qkv.
struct RopeArgs {
  float *qkv;
  const float *rope_cos; // [capacity][32]
  const float *rope_sin;
  float *key_cache;      // [capacity][128]
  float *value_cache;
  uint32_t count;
  uint32_t first_position;
  PartialTiles qkv_partials;
  const float *qkv_bias;
  // Batched decode: row t is stream t at position positions[t], whose cache
  // rows start stream_stride floats after stream t - 1's (null: prompt rows
  // at first_position + t of one cache).
  const uint32_t *positions;
  uint64_t stream_stride;
};

// Row finish of a residual GEMM: hidden[t] += (partial sums of row t), then,
// when norm_weight is set, out[t] = RMSNorm(hidden[t]) * norm_weight (TF32
// hi/lo pair when out_lo is set). One block per row (also for
// prefill_rope_kv) of 256 threads or kRowThreads: both kernels work for any
// block size of at least 256.
struct FinishArgs {
  PartialTiles partials;
  float *hidden; // [count][896]
  uint32_t count;
  float epsilon;
  const float *norm_weight;
  float *out;
  float *out_lo;
};

// An encoded CUtensorMap, passed by value in kernel arguments.
struct alignas(64) TensorMap {
  uint64_t opaque[16];
};

// Causal GQA attention: query row t attends to cache positions
// 0..first_position + t. out [count][896] (hi part when out_lo is set).
// Launch: blocks of kAttentionThreads threads over (the (row tile, key
// chunk) pairs with work, 14) with kAttentionSharedBytes of dynamic shared
// memory; a row tile of kAttentionTileRows rows holds the chunks up to its
// last position;
// chunk_keys * max_chunks covers first_position + count positions.
struct AttentionArgs {
  const float *qkv;
  const float *key_cache;
  const float *value_cache;
  float *out;
  float *out_lo;
  uint32_t count;
  uint32_t first_position;
  uint32_t chunk_keys;   // key positions per block (a multiple of 64)
  uint32_t max_chunks;   // partial-state slots per (row tile, head)
  float *partials;       // per (row tile, head, chunk): rows x kAttentionPartialStride floats
  uint32_t *arrivals;    // [row tile][14], zero between launches
  uint32_t wait_limit_ms; // prefill_attention_tc: per mbarrier wait
  uint32_t *error;        // prefill_attention_tc: kTcErrorWaitTimeout when a wait gives up
  // prefill_attention_tc: tensor maps of out and out_lo ([rows][896], boxes
  // of 16 columns x 128 rows, 64-byte swizzle) for its TMA stores.
  TensorMap out_map, out_lo_map;
};

// Batched decode attention: one query row per stream. Block (s, g, b)
// covers key positions [s * chunk, (s + 1) * chunk) of stream b's cache for
// the seven query heads of KV group g and writes a partial softmax state
// (maximum, sum, acc[64]) per head to `partials`
// [b][g][split][7][kDecodePartialStride]; the last block of (b, g) to finish
// (arrivals[b * 2 + g], reset by that block) combines the splits into
// out[b][head * 64 + d] (TF32 pair when out_lo is set).
constexpr uint32_t kDecodePartialStride = 66;
constexpr uint32_t kDecodeMaximumSplits = 32;
// Keys per batch_attention tile; each block streams its key range through
// two tile buffers, and the batch sizes its splits so that all blocks fit
// one wave of kDecodeBlocksPerSm blocks per SM.
constexpr uint32_t kDecodeTileKeys = 64;
constexpr uint32_t kDecodeBlocksPerSm = 3;
// Dynamic shared memory of batch_attention: two tile buffers of K[64][68]
// (reused for the partial scores) and V[64][64] (both reused for the final
// sums), queries [7][64], softmax weights [7][64], rescales [8], merge
// weights [7][32] and totals [7].
constexpr uint32_t kDecodeSharedBytes =
    4u * (2u * (64u * 68u + 64u * 64u) + 7u * 64u + 7u * 64u + 8u + 7u * 32u + 7u);
struct DecodeAttentionArgs {
  const float *qkv;         // [streams][1152], q rotated
  const float *key_cache;   // stream b's cache at key_cache + b * stream_stride
  const float *value_cache;
  uint64_t stream_stride;
  const uint32_t *positions; // attend to 0..positions[b]
  float *partials;
  float *out;
  float *out_lo;
  uint32_t streams, splits, chunk;
  uint32_t *arrivals; // [streams][2], zero between steps
};

// Greedy step end: per stream row, the first index of the largest logit
// (lower index on ties, as the decode step's reduce), appended to
// tokens[b * token_stride + generated[b]] and stored as the stream's next
// input token; positions[b] and generated[b] advance.
struct ArgmaxArgs {
  const float *logits;       // [streams][vocab]
  uint32_t vocab, streams;
  uint32_t *next_tokens;     // [streams]
  uint32_t *positions;
  uint32_t *generated;
  uint32_t *tokens;
  uint32_t token_stride;
  float *logit_values;       // [streams]: the chosen logit
  float *candidate_values;   // [streams][partitions] per-block winners
  uint32_t *candidate_indices;
  uint32_t *arrivals;        // [streams], zero between steps
};

constexpr uint32_t kArgmaxPartitions = 8; // blocks per stream row
constexpr uint32_t kRowThreads = 1024;     // prefill_rope_kv, prefill_finish_rows
// At most this many K splits for a GEMM whose partials the next row kernel
// finishes (it stages splits x columns floats of shared memory per row).
constexpr uint32_t kMaximumDeferredSplits = 24;

constexpr uint32_t kAttentionTileRows = 64; // query rows per block
constexpr uint32_t kAttentionThreads = 256;
// Shared memory of prefill_attention: Q [64][68], K [2][64][68], V [2][64][64]
// and the tile's softmax weights [64][68].
constexpr uint32_t kAttentionSharedBytes = 4u * (64u * 68u + 2u * 64u * 68u + 2u * 64u * 64u + 64u * 68u);
constexpr uint32_t kAttentionPartialStride = 68; // acc[64], maximum, sum, 2 pad: 16-byte rows
constexpr uint32_t kAttentionMaximumChunks = 16;
// prefill_attention_tc (the 3xTF32 path): kTcAttentionRows query rows per
// block, keys in sub-tiles of kTcAttentionKeys on the tensor cores; the same
// arguments and (row tile, key chunk) enumeration as prefill_attention.
// Shared memory: Q, K, V^T and the softmax weights P as TF32 (hi, lo) pairs
// in 64-byte-swizzled slabs (Q [2][128][64], K [2][64][64], V^T [2][64][64],
// P [2][128][64] floats), the row maxima and sums of both column halves
// [2][2][128], two mbarriers and flags, and 1 KB to align the slabs.
constexpr uint32_t kTcAttentionRows = 128;
constexpr uint32_t kTcAttentionKeys = 64;
constexpr uint32_t kTcAttentionThreads = 256;
constexpr uint32_t kTcAttentionSharedBytes =
    1024u + 4u * (2u * 128u * 64u + 2u * 64u * 64u + 2u * 64u * 64u + 2u * 128u * 64u) +
    4u * 4u * 128u + 64u;

// hi[i] = tf32(x[i]), lo[i] = tf32(x[i] - hi[i]) for i < count.
struct SplitArgs {
  const float *x;
  float *hi;
  float *lo;
  uint64_t count;
};

// Tensor-core 3xTF32 GEMM. Each CTA computes one 128 x N output tile
// (N = 192, 224 or 256 accumulator columns, one kernel per width) over one
// K slice: linear tile index tile_offset + blockIdx.x (n tile fastest),
// K slice blockIdx.z of `splits`. A is [m][k], B is [rows][k]; the tensor maps
// are 2-D fp32 maps with 64-byte swizzle and boxes of 16 columns x 128 rows
// (A) or N / 2 rows (B: each B tile loads as two half boxes, so swiglu takes
// N / 2 gate rows and N / 2 up rows starting at n_gate_offset).
struct TcGemmArgs {
  TensorMap a_hi, a_lo, b_hi, b_lo;
  const float *bias;
  float *c;               // output, or the compact partials when mode == partial
  float *c_lo;
  uint32_t m, n, k, ldc;
  uint32_t mode;          // GemmEpilogue
  uint32_t tile_offset, n_tiles, tile_count, splits;
  uint32_t n_gate_offset; // swiglu: row of the first up row in B
  uint32_t wait_limit_ms; // per mbarrier wait
  uint32_t *error;        // set to kTcErrorWaitTimeout when a wait gives up
};

constexpr uint32_t kTcTileM = 128;
constexpr uint32_t kTcTileK = 16;   // one 64-byte swizzle row of fp32
constexpr uint32_t kTcThreads = 128;
constexpr uint32_t kTcMaximumN = 256;     // one MMA's N
constexpr uint32_t kTcTmemColumns = 256;
// Gate/up pair tiles wider than one MMA: kTcPairN accumulator columns (gate
// then up, kTcPairN / 2 each, two MMAs per product), 512 TMEM columns. 4864
// gate/up columns make 34 such tiles per 128-row band: the 511 rows of a
// 512-token chunk fit one wave of 148 SMs (136 tiles) where 128 + 128 tiles
// need 152.
constexpr uint32_t kTcPairN = 288;
constexpr uint32_t kTcPairTmemColumns = 512;

LRRT_PREFILL_HD constexpr uint32_t tc_stage_bytes(uint32_t n) { return 2u * (kTcTileM + n) * kTcTileK * 4u; }
// Up to 200 KB of stages (213 KB for the pair tiles: four 52 KB stages).
LRRT_PREFILL_HD constexpr uint32_t tc_stage_budget(uint32_t n) {
  return (n > kTcMaximumN ? 213u : 200u) * 1024u;
}
LRRT_PREFILL_HD constexpr uint32_t tc_stages(uint32_t n) {
  return tc_stage_budget(n) / tc_stage_bytes(n) > 8u ? 8u : tc_stage_budget(n) / tc_stage_bytes(n);
}
LRRT_PREFILL_HD constexpr uint32_t tc_shared_bytes(uint32_t n) {
  return tc_stages(n) * tc_stage_bytes(n) + 1024u /* alignment */ + 256u /* barriers */;
}
static_assert(tc_stages(kTcPairN) == 4 && tc_shared_bytes(kTcPairN) <= 227u * 1024u,
              "pair tiles: four stages within one block's shared memory");

// Narrow GEMMs (at most kNarrowRows rows: batched decode, short chunks) swap
// the operands: a tile is kNarrowTileN weight rows (the MMA's M) times the
// kNarrowRows activation rows (its N). Paired tiles (swiglu) hold the gate
// rows and the matching up rows in two accumulators.
constexpr uint32_t kNarrowRows = 32;
constexpr uint32_t kNarrowTileN = 128;
constexpr uint32_t kNarrowTmemColumns = 64;
LRRT_PREFILL_HD constexpr uint32_t tc_narrow_stage_bytes(bool paired) {
  return 2u * ((paired ? 2u : 1u) * kNarrowTileN + kNarrowRows) * kTcTileK * 4u;
}
// Up to 200 KB of stages (one CTA per SM); `shared_sm` narrow launches of
// more than one wave of tiles (prefill_tc_narrow_shared_sm: the LM head of
// a batched step) take 100 KB, so that two CTAs share an SM and one's
// pipeline fill and epilogue overlap the other's weight stream.
LRRT_PREFILL_HD constexpr uint32_t tc_narrow_stages(bool paired, bool shared_sm = false) {
  return ((shared_sm ? 100u : 200u) * 1024u) / tc_narrow_stage_bytes(paired) > 8u
             ? 8u
             : ((shared_sm ? 100u : 200u) * 1024u) / tc_narrow_stage_bytes(paired);
}
LRRT_PREFILL_HD constexpr uint32_t tc_narrow_shared_bytes(bool paired, bool shared_sm = false) {
  return tc_narrow_stages(paired, shared_sm) * tc_narrow_stage_bytes(paired) + 1024u + 256u;
}
static_assert(2u * tc_narrow_shared_bytes(false, true) <= 227u * 1024u,
              "two shared-SM narrow CTAs per SM");

constexpr uint32_t kTcErrorWaitTimeout = 1;

} // namespace lrrt::qwen::prefill

#endif // LRRT_QWEN_PREFILL_HPP_
