/*
 * C ABI of the Qwen2 FP32 resident decode driver (liblrrt_qwen.so).
 *
 * This is the B200 counterpart of the host side of light-rocm-runtime's
 * Qwen stateful-graph path, benchmarks/qwen_stateful_graph.cpp:
 *   lrq_build_program_table  <- make_qwen_decoder_programs (:368-485)
 *   lrq_rope_tables          <- RoPE table loop (:912-929)
 *   lrq_model_create         <- device weights, buffers, Context/TailContext
 *                               arrays and ResidentExecutors (:730-1118)
 *   lrq_decode / _launch     <- initialize_decode_state + executor initialize
 *                               + launch + synchronize (:1256-1340, :1364-1384)
 *   LRQ_PATH_HOST_STEP       <- launch_host_decode (:1161-1172)
 *   lrq_model_read           <- the read-backs of the cross-path verification
 *                               (:1613-1746)
 * The reference drives these through the lr_* and lrrt:: C++ APIs; this C
 * ABI wraps the same sequence for callers in other languages (the test suite
 * and bench.py use it through ctypes). The device code is the sm_100a module
 * built from light-rocm-runtime_b200/csrc/kernels/qwen_stateful_graph.cu and
 * loaded with lr_module_load_hsaco.
 *
 * All functions return lr_status_t; lrq_last_error() describes the last
 * failure of this library in the calling process.
 */
#ifndef LRRT_QWEN_H_
#define LRRT_QWEN_H_

#include "lrrt/lrrt.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct lrq_model_t lrq_model_t;

typedef struct lrq_task_t {
  uint32_t opcode, dependency_mask, begin, end, argument0, argument1,
      dependency_mask_high, reserved;
} lrq_task_t;

typedef struct lrq_program_t {
  uint32_t task_offset, task_count, next_program, flags, branch_program,
      reserved[3];
} lrq_program_t;

typedef struct lrq_model_config_t {
  uint32_t layer_count;        /* decoder layers */
  uint32_t vocab_size;         /* LM-head / embedding rows */
  uint32_t cache_capacity;     /* KV positions per layer (and RoPE rows) */
  uint32_t lm_head_partitions; /* 1..32; 0 = min(vocab, 32, workers) */
  uint32_t worker_count;       /* 0 = one resident block per SM */
  uint32_t max_tokens_per_run; /* output buffer and phase-state sizing */
  float rope_theta;            /* 1e6 for Qwen2.5 */
  float rms_epsilon;           /* 1e-6 */
  uint32_t tied_embeddings;    /* 1: the LM head is the embedding table */
  uint32_t disable_fused_path; /* 1: leave the workspace unbound (generic path) */
} lrq_model_config_t;

/* Host pointers to one decoder layer, row-major [out][in] (nn.Linear). */
typedef struct lrq_layer_weights_t {
  const float *attention_norm; /* [896] */
  const float *q;              /* [896][896] */
  const float *k;              /* [128][896] */
  const float *v;              /* [128][896] */
  const float *q_bias;         /* [896] */
  const float *k_bias;         /* [128] */
  const float *v_bias;         /* [128] */
  const float *o;              /* [896][896] */
  const float *mlp_norm;       /* [896] */
  const float *gate;           /* [4864][896] */
  const float *up;             /* [4864][896] */
  const float *down;           /* [896][4864] */
} lrq_layer_weights_t;

typedef enum lrq_path_t {
  LRQ_PATH_COMPILED = 0,          /* compiled resident kernel (fused when possible) */
  LRQ_PATH_DYNAMIC = 1,           /* dynamic-claim resident kernel */
  LRQ_PATH_HOST_STEP = 2,         /* 9 launches per layer + 4 per token */
  LRQ_PATH_SCHEDULER_PROFILE = 3, /* control-only compiled run */
  LRQ_PATH_STAGE_PROFILE = 4,     /* compiled run with per-stage ticks */
  LRQ_PATH_GRAPH = 5              /* CUDA graph of one matched-step launch per compiled
                                     stage, replayed per token (fixed count, no EOS) */
} lrq_path_t;

typedef struct lrq_decode_request_t {
  uint32_t token_position; /* first position to write (== kv_length) */
  uint32_t maximum_tokens; /* tokens to generate in this run */
  uint32_t eos_token;      /* UINT32_MAX = none */
  uint32_t path;           /* lrq_path_t */
  uint32_t max_steps;      /* 0 = 2 * maximum_tokens * layers */
  uint32_t stop_value;     /* 0 = 1 */
  uint32_t wait_limit_ms;  /* 0 = default */
  uint32_t launch_workers; /* 0 = the model's worker count (test hook) */
} lrq_decode_request_t;

/* Final State (persistent_graph State fields) and DecodeState of a run. */
typedef struct lrq_run_state_t {
  uint32_t status, phase, step, max_steps, stop_value, error_code, worker_count,
      predicate_value, branch_value, reserved;
  uint64_t executed_tasks;
  uint32_t token_position, kv_length, sampled_token, eos_token, generated_tokens,
      maximum_tokens, stop_reason;
  float sampled_logit;
  uint32_t fused_path; /* 1 fused, 2 generic, 0 unknown (non-compiled path) */
  uint32_t reserved2;
} lrq_run_state_t;

typedef enum lrq_buffer_t {
  LRQ_BUFFER_HIDDEN = 0,
  LRQ_BUFFER_ATTENTION_NORMALIZED = 1,
  LRQ_BUFFER_QUERY = 2,
  LRQ_BUFFER_KEY = 3,
  LRQ_BUFFER_VALUE = 4,
  LRQ_BUFFER_KEY_CACHE = 5,   /* layer's [capacity][128] */
  LRQ_BUFFER_VALUE_CACHE = 6, /* layer's [capacity][128] */
  LRQ_BUFFER_MLP_NORMALIZED = 7,
  LRQ_BUFFER_ACTIVATED = 8,
  LRQ_BUFFER_PROJECTED = 9,
  LRQ_BUFFER_FINAL_NORMALIZED = 10,
  LRQ_BUFFER_PARTIAL_VALUES = 11,
  LRQ_BUFFER_PARTIAL_INDICES = 12,
  LRQ_BUFFER_OUTPUT_TOKENS = 13,
  LRQ_BUFFER_ROPE_COS = 14,
  LRQ_BUFFER_ROPE_SIN = 15,
  LRQ_BUFFER_LOGITS = 16      /* [vocab] last step's LM-head rows (logit capture) */
} lrq_buffer_t;

/* The reference task/Program table for the decode graph. Capacities in
 * entries; *task_count / *program_count receive the sizes (needed sizes when
 * the capacity is too small, with LR_ERROR_INVALID_ARGUMENT). */
LRRT_API lr_status_t lrq_build_program_table(uint32_t vocab_size,
                                             uint32_t lm_head_partitions,
                                             lrq_task_t *tasks, uint32_t task_capacity,
                                             uint32_t *task_count,
                                             lrq_program_t *programs,
                                             uint32_t program_capacity,
                                             uint32_t *program_count);

/* cos/sin tables [positions][32], float arithmetic as the reference host. */
LRRT_API lr_status_t lrq_rope_tables(uint32_t positions, float theta,
                                     float *cos_table, float *sin_table);

/* Bytes of device memory a model with this configuration allocates. */
LRRT_API lr_status_t lrq_model_device_bytes(const lrq_model_config_t *config,
                                            uint32_t worker_count, uint64_t *bytes);

LRRT_API lr_status_t lrq_model_create(lr_device_t device, const void *module_image,
                                      size_t module_image_size,
                                      const lrq_model_config_t *config,
                                      lrq_model_t **model);
LRRT_API lr_status_t lrq_model_destroy(lrq_model_t *model);

LRRT_API lr_status_t lrq_model_set_layer(lrq_model_t *model, uint32_t layer,
                                         const lrq_layer_weights_t *weights);
/* embeddings may be NULL when the model was created with tied embeddings. */
LRRT_API lr_status_t lrq_model_set_tail(lrq_model_t *model, const float *final_norm,
                                        const float *lm_head, const float *embeddings);
/* Writes cache rows [first_position, first_position + positions) of one layer
 * from host arrays [positions][128]. */
/* Loads one decoder layer / the model tail from the reference's FP32 weight
 * bundles ("lrrt.mini_decoder_weights" v2, "lrrt.mini_model_tail_weights"
 * v1; include/lrrt/qwen/weight_bundle.hpp) into the model: the manifests'
 * shapes and rope_theta must match the model configuration (reference
 * benchmarks/qwen_stateful_graph.cpp:760-880 reads the same files). */
LRRT_API lr_status_t lrq_model_load_layer_bundle(lrq_model_t *model, uint32_t layer,
                                                 const char *manifest_path);
LRRT_API lr_status_t lrq_model_load_tail_bundle(lrq_model_t *model, const char *manifest_path);

LRRT_API lr_status_t lrq_model_set_kv(lrq_model_t *model, uint32_t layer,
                                      uint32_t first_position, uint32_t positions,
                                      const float *keys, const float *values);
/* Copies the same device layer into every layer slot (synthetic benchmarks). */
LRRT_API lr_status_t lrq_model_replicate_layer(lrq_model_t *model, uint32_t source_layer);
/* Initial hidden vector for the next runs: from the host, or an embedding row. */
LRRT_API lr_status_t lrq_model_set_hidden(lrq_model_t *model, const float *hidden);
LRRT_API lr_status_t lrq_model_set_hidden_from_token(lrq_model_t *model, uint32_t token);

/* Enqueues one run on the device's default queue: device-side copies reset
 * State, MaskStates, DecodeState and hidden from their staged images, then
 * the path's kernel(s) launch. Returns without waiting. */
LRRT_API lr_status_t lrq_decode_launch(lrq_model_t *model,
                                       const lrq_decode_request_t *request);
/* lrq_decode_launch + synchronize + read back the run state and, when
 * tokens is not NULL, the generated tokens (capacity token_capacity). */
LRRT_API lr_status_t lrq_decode(lrq_model_t *model, const lrq_decode_request_t *request,
                                lrq_run_state_t *state, uint32_t *tokens,
                                uint32_t token_capacity);
/* Reads the state of the last run (synchronizes first). */
LRRT_API lr_status_t lrq_model_read_state(lrq_model_t *model, lrq_run_state_t *state);

/*
 * Prompt ingestion by single-token decode steps: positions 0..count-2 run as
 * one-token compiled decodes fed with prompt[i] (their sampled tokens are
 * discarded), then hidden is staged from prompt[count-1] so the next
 * lrq_decode with token_position = count-1 produces the first new token.
 */
LRRT_API lr_status_t lrq_model_ingest_prompt(lrq_model_t *model, const uint32_t *prompt,
                                             uint32_t count);

/*
 * Batched prompt prefill (no counterpart in the reference, which ingests
 * prompts one decode step at a time). The prefill kernels
 * live in their own sm_100a module (qwen_prefill.cubin, built from
 * light-rocm-runtime_b200/csrc/kernels/qwen_prefill.cu).
 *
 * lrq_model_enable_prefill loads that module and sizes its buffers for
 * chunks of up to max_chunk_tokens tokens (0 = 512); longer prompts run in
 * chunks. With LRQ_PREFILL_TF32X3 the first prefill after a weight upload
 * also builds TF32 (hi, lo) copies of every layer's GEMM weights (2 x 59.6 MB
 * per layer).
 *
 * lrq_model_prefill has lrq_model_ingest_prompt's contract: positions
 * 0..count-2 are computed from prompt[0..count-2] (K/V rows written for
 * every layer), then hidden is staged from prompt[count-1], so the next
 * lrq_decode with token_position = count-1 produces the first new token.
 * The projections run as GEMMs over all prompt rows:
 *   LRQ_PREFILL_SIMT    FP32 FMA tiles on the CUDA cores;
 *   LRQ_PREFILL_TF32X3  3xTF32 on the tcgen05 tensor cores (FP32 accuracy:
 *                       each operand split into TF32 hi + lo, three products;
 *                       the causal attention too). GEMMs of at most 32 rows
 *                       read the FP32 weights and split them on chip.
 * Results match single-token ingestion to FP32 rounding (summation order
 * differs), not bit for bit. Waits for the device before returning.
 *
 * lrq_model_prefill_at computes `count` tokens at positions
 * first_position.. (K/V rows only, no hidden staging); positions before
 * first_position must already hold the context's K/V rows.
 */
typedef enum lrq_prefill_path_t {
  LRQ_PREFILL_SIMT = 0,
  LRQ_PREFILL_TF32X3 = 1
} lrq_prefill_path_t;

LRRT_API lr_status_t lrq_model_enable_prefill(lrq_model_t *model, const void *module_image,
                                              size_t module_image_size,
                                              uint32_t max_chunk_tokens);
LRRT_API lr_status_t lrq_model_prefill(lrq_model_t *model, const uint32_t *prompt,
                                       uint32_t count, uint32_t path);
LRRT_API lr_status_t lrq_model_prefill_at(lrq_model_t *model, const uint32_t *tokens,
                                          uint32_t count, uint32_t first_position,
                                          uint32_t path);

/*
 * Numerics check of one prefill GEMM on host matrices, through the prefill's
 * own scheduler and kernels: c = epilogue(A . B^T) with A [m][k], B [n][k]
 * row-major (mode 2, swiglu: B [2n][k], gate rows then up rows), c [m][n]
 * read and written (mode 0: c = acc + bias; 1: c += acc; 2: c = silu(gate) *
 * up). tile_columns 0 runs the FP32 SIMT kernels; 192, 224 or 256 runs the
 * 3xTF32 tensor-core kernel of that accumulator width (k a multiple of 16,
 * n of 32; swiglu: tile_columns 192 or 256 and n a multiple of half of it,
 * or 288, the prefill's 144 + 144 gate/up pairs, for any n), except that
 * m <= 32 rows run the narrow swapped-operand kernels whatever the
 * tensor-core width (swiglu then takes any n).
 * Needs
 * lrq_model_enable_prefill; waits for the device.
 */
LRRT_API lr_status_t lrq_prefill_gemm_check(lrq_model_t *model, uint32_t tile_columns,
                                            uint32_t mode, uint32_t m, uint32_t n, uint32_t k,
                                            const float *a, const float *b, const float *bias,
                                            float *c);

/*
 * Batched multi-stream greedy decode on one GPU (BASELINE config 4's
 * per-GPU batch; no counterpart in the reference, whose ABI decodes one
 * stream per DecodeState). `streams` independent streams (at most the
 * prefill chunk size) each own a KV cache of `capacity` positions (at most
 * the model's cache_capacity), a position and a next input token; they
 * share the model's weights, so one decode step streams the weights once
 * for every stream. A step runs the prefill module's kernels over one row
 * per stream (3xTF32 GEMMs, RoPE + KV append, split decode attention over
 * each stream's own cache, the LM head and a greedy argmax with the
 * lower-index tie rule) as one CUDA graph replayed per token. Needs
 * lrq_model_enable_prefill; destroy batches before re-enabling the prefill
 * (lrq_model_destroy destroys any that remain).
 *
 * lrq_batch_prefill: stream's prompt, lrq_model_prefill's contract
 *   (positions 0..count-2 into the stream's cache; prompt[count-1] is the
 *   stream's next input token, at position count-1).
 * lrq_batch_decode: `steps` (<= max_tokens) greedy tokens of every stream,
 *   tokens[stream * steps + i]; last_logits (optional, [streams]) receives
 *   each stream's last chosen logit. Positions advance by `steps`; a stream
 *   never prefilled starts from token 0 at position 0. Waits for the device.
 * Logits match single-stream decoding to FP32 rounding (GEMM summation
 * order), not bit for bit.
 */
typedef struct lrq_batch_t lrq_batch_t;

LRRT_API lr_status_t lrq_batch_create(lrq_model_t *model, uint32_t streams, uint32_t capacity,
                                      uint32_t max_tokens, lrq_batch_t **batch);
LRRT_API lr_status_t lrq_batch_destroy(lrq_batch_t *batch);
LRRT_API lr_status_t lrq_batch_prefill(lrq_batch_t *batch, uint32_t stream,
                                       const uint32_t *prompt, uint32_t count, uint32_t path);
LRRT_API lr_status_t lrq_batch_decode(lrq_batch_t *batch, uint32_t steps, uint32_t *tokens,
                                      float *last_logits);
/* Cache rows [0, positions) of one stream and layer, [positions][128] each
 * (keys or values may be NULL). */
LRRT_API lr_status_t lrq_batch_read_cache(lrq_batch_t *batch, uint32_t stream, uint32_t layer,
                                          uint32_t positions, float *keys, float *values);
/* Cache rows [first_position, first_position + positions) of one stream and
 * layer from host arrays [positions][128] (keys or values may be NULL), and a
 * stream's next position and input token: a context set up without running
 * its prompt (the stream's cache must then hold rows 0..position-1). */
LRRT_API lr_status_t lrq_batch_write_cache(lrq_batch_t *batch, uint32_t stream, uint32_t layer,
                                           uint32_t first_position, uint32_t positions,
                                           const float *keys, const float *values);
LRRT_API lr_status_t lrq_batch_set_next(lrq_batch_t *batch, uint32_t stream, uint32_t position,
                                        uint32_t token);
LRRT_API lr_status_t lrq_batch_position(lrq_batch_t *batch, uint32_t stream,
                                        uint32_t *position);

/*
 * End-to-end generate from host memory: copies the host hidden vector (or,
 * when hidden is NULL, stages the embedding of start_token) to the device,
 * runs the compiled path and copies the generated tokens back into `tokens`.
 */
LRRT_API lr_status_t lrq_generate(lrq_model_t *model, const float *hidden,
                                  uint32_t start_token, uint32_t token_position,
                                  uint32_t maximum_tokens, uint32_t eos_token,
                                  uint32_t *tokens, lrq_run_state_t *state);

LRRT_API lr_status_t lrq_model_read(lrq_model_t *model, uint32_t buffer, uint32_t layer,
                                    void *destination, size_t bytes);

/*
 * Fused-path workspace for callers that build the Context / TailContext
 * arrays themselves, as the reference driver does
 * (benchmarks/qwen_stateful_graph.cpp:730-1118), and launch through
 * ResidentExecutor. The sm_100a compiled kernel takes its fast path only when
 * TailContext::workspace (bytes 88-95, the reference's tail padding) points
 * to an initialised workspace and the launch has the fused path's dynamic
 * shared memory (ResidentConfig::dynamic_shared_memory_bytes =
 * lrrt::qwen::stateful_graph::resident::kFusedSharedBytes, also given to
 * admit_resident_workers); otherwise it runs the reference's per-task path.
 *  - lrq_workspace_bytes: bytes of a workspace for `worker_count` blocks.
 *  - lrq_workspace_init: zero-fills the device allocation `workspace`
 *    (256-byte aligned, `bytes` from lrq_workspace_bytes) and writes its
 *    header and the KV caches' tensor maps from `contexts`, the host copy of
 *    the caller's Context array (layer_count entries; key_cache, value_cache
 *    and cache_capacity as on the device). Call it again after moving a KV
 *    cache.
 *  - lrq_workspace_path: which path the last launch with this workspace
 *    took: 1 fused, 2 per-task (0 none yet).
 */
LRRT_API lr_status_t lrq_workspace_bytes(uint32_t worker_count, uint64_t *bytes);
LRRT_API lr_status_t lrq_workspace_init(lr_device_t device, void *workspace, uint64_t bytes,
                                        uint32_t worker_count, const void *contexts,
                                        uint32_t layer_count);
LRRT_API lr_status_t lrq_workspace_path(lr_device_t device, const void *workspace,
                                        uint32_t *path);

/* Logit capture (a B200 test aid with no reference counterpart): with
 * enable != 0 the fused path also stores every LM-head row it computes, so
 * LRQ_BUFFER_LOGITS holds all vocab_size logits of the last decode step
 * (the reference's resident kernel only keeps per-partition maxima). Off by
 * default; enabling allocates vocab_size floats. */
LRRT_API lr_status_t lrq_model_set_logit_capture(lrq_model_t *model, uint32_t enable);

typedef struct lrq_model_info_t {
  uint32_t worker_count, lm_head_partitions, layer_count, vocab_size, cache_capacity,
      dynamic_shared_bytes, phase_state_count, task_count;
  uint64_t device_bytes;
  uint64_t weight_bytes_per_token; /* algorithmic weight stream per decode step */
} lrq_model_info_t;

LRRT_API lr_status_t lrq_model_info(lrq_model_t *model, lrq_model_info_t *info);

/* Per-stage device nanoseconds of the last LRQ_PATH_STAGE_PROFILE run
 * (13 entries, reference ProfileStage order) and their counts. */
LRRT_API lr_status_t lrq_model_stage_profile(lrq_model_t *model, uint64_t *ticks,
                                             uint64_t *counts);

/*
 * Runs a caller-supplied task/Program table on the model's device context with
 * the dynamic (path = LRQ_PATH_DYNAMIC) or compiled (LRQ_PATH_COMPILED)
 * resident kernel, then restores the decode graph. This is how the
 * reference's pre-timing self checks run (qwen_stateful_graph.cpp:1272-1311:
 * the 64-task chain and the cyclic-graph rejection). DecodeState and hidden
 * are staged from (token_position, maximum_tokens, eos_token) as for a decode.
 */
LRRT_API lr_status_t lrq_model_run_graph(lrq_model_t *model, const lrq_task_t *tasks,
                                         uint32_t task_count, const lrq_program_t *programs,
                                         uint32_t program_count, uint32_t path,
                                         uint32_t program_index, uint32_t max_steps,
                                         uint32_t stop_value, uint32_t token_position,
                                         uint32_t maximum_tokens, lrq_run_state_t *state);

/* Per-block barrier trace of LRQ_PATH_STAGE_PROFILE runs: with `entries` > 0
 * every block records (arrive_ns, leave_ns) %globaltimer stamps of each grid
 * barrier at entries[barrier * workers + worker]; 0 turns tracing off. */
LRRT_API lr_status_t lrq_model_set_trace(lrq_model_t *model, uint32_t entries);
/* Copies `capacity` (arrive, leave) pairs (2 x u64 each) of the last trace. */
LRRT_API lr_status_t lrq_model_read_trace(lrq_model_t *model, uint64_t *entries,
                                          uint32_t capacity);

/*
 * Greedy LM-head top-1 that allocates no device memory. No counterpart in the
 * reference: it is a variant of the LM-head partition + reduce tasks whose
 * per-block candidates live in a file-scope static device array of
 * LRQ_STATIC_TOP1_MAX_BLOCKS entries (8 KB) instead of partial buffers the
 * caller allocates. It serves callers whose device memory belongs to another
 * allocator (a serving stack that reserves HBM up front) and callers that
 * cannot take cudaMalloc/cudaFree's implicit device-wide synchronisation on
 * the decode path.
 *
 * token = argmax over rows r < `rows` of lm_head[r] . hidden (row-major
 * [rows][columns], device pointers), ties to the lower row; logit = that dot
 * product. Rows use the partitioned path's dot-product order, so both match
 * it exactly.
 *  - `blocks` is the grid size (0 = 2 x SMs); more than
 *    LRQ_STATIC_TOP1_MAX_BLOCKS returns LR_ERROR_INVALID_ARGUMENT.
 *  - Runs on `queue` (NULL = the device's default queue), waits for it and
 *    writes token and logit to host memory.
 *  - The first call on a device looks up the scratch address
 *    (cudaGetSymbolAddress) and the SM count; make that first call before any
 *    stream capture begins on the device.
 *  - The scratch's arrival counter must be zero when a launch starts; every
 *    call clears it on `queue` before launching.
 *  - All calls on a device share the one scratch: calls that overlap in time
 *    (other threads, other queues) race, and the caller must serialise them.
 */
#define LRQ_STATIC_TOP1_MAX_BLOCKS 1024u
LRRT_API lr_status_t lrq_lm_head_top1_static(lr_device_t device, lr_queue_t *queue,
                                             const float *lm_head, const float *hidden,
                                             uint32_t rows, uint32_t columns,
                                             uint32_t blocks, uint32_t *token,
                                             float *logit);

LRRT_API const char *lrq_last_error(void);

#ifdef __cplusplus
}
#endif

#endif /* LRRT_QWEN_H_ */
