/*
 * CPU oracle for the Persistent Graph Qwen2 FP32 decode path.
 *
 * TEST INFRASTRUCTURE ONLY. This is a plain-C restatement of
 * light-rocm-runtime's scheduler semantics and Qwen task arithmetic, used by
 * tests/ as the checker, by __graft_entry__.smoke() as the checker, and by
 * bench.py as the timed CPU baseline. Nothing in the product path links or
 * calls it.
 *
 * What it restates (files of the reference project):
 *   scheduler:  include/lrrt/persistent_graph/device_scheduler.hpp:65-131
 *               (validate_programs) and compiled_scheduler.hpp:69-99
 *               (finish_program); stage order from resident_executor.hpp:227-263
 *   workload:   benchmarks/qwen_stateful_graph_kernel.cpp
 *               valid_qwen_task :47-77, valid_qwen_contexts :79-120,
 *               wave_sum :122-127, matvec/two-row matvec :129-176,
 *               better_top1 :225-229, LM-head partition :231-337,
 *               reduce_top1 :339-356, embedding_feedback :358-390,
 *               QKV :392-492, gate/up/SiLU :494-515, RoPE + KV :517-552,
 *               GQA :554-600, o_proj + residual :602-659, RMSNorm and
 *               residual_advance :661-761, layer selection :776-783
 *   fixture:    tests/stateful_graph_device_kernel.cpp:46-136 (synthetic
 *               scheduler workload) with goldens in
 *               tests/stateful_graph_device.cpp:103-136
 *
 * Dot products reproduce the reference's reduction order: 32 lane partial sums
 * (lane l accumulates columns l, l+32, ... with fmaf), then the shfl_down tree
 * with offsets 16, 8, 4, 2, 1. Build with -ffp-contract=off.
 */
#ifndef LRRT_ORACLE_H_
#define LRRT_ORACLE_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct or_task_t {
  uint32_t opcode, dependency_mask, begin, end, argument0, argument1,
      dependency_mask_high, reserved;
} or_task_t;

typedef struct or_program_t {
  uint32_t task_offset, task_count, next_program, flags, branch_program,
      reserved[3];
} or_program_t;

typedef struct or_state_t {
  uint32_t abi_version, status, phase, step, max_steps, stop_value, error_code,
      worker_count;
  uint64_t executed_tasks;
  uint32_t predicate_value, branch_value, reserved[4];
} or_state_t;

enum {
  OR_STATUS_READY = 0,
  OR_STATUS_RUNNING = 1,
  OR_STATUS_COMPLETE = 2,
  OR_STATUS_MAX_STEPS = 3,
  OR_STATUS_INVALID = 4,
};
enum {
  OR_ADVANCES_STEP = 1u,
  OR_EVALUATES_PREDICATE = 2u,
  OR_BRANCHES_ON_STATE = 4u,
};

/* Workload hooks (the reference's valid_context / valid_task / execute). */
typedef struct or_workload_t {
  int (*valid_context)(const or_state_t *state, void *context);
  int (*valid_task)(const or_task_t *task, void *context);
  void (*execute)(const or_task_t *task, or_state_t *state, void *context);
} or_workload_t;

/* Fills *state like ResidentExecutor::initialize. */
void or_initialize_state(or_state_t *state, uint32_t abi_version,
                         uint32_t program_index, uint32_t max_steps,
                         uint32_t stop_value, uint32_t worker_count);

/* Device-side validation of the reference (returns 1 when valid).
 * maximum_workers is the ABI's worker cap. */
int or_validate_programs(const or_state_t *state, const or_task_t *tasks,
                         const or_program_t *programs, uint32_t program_count,
                         uint32_t task_count, uint32_t phase_state_count,
                         uint32_t abi_version, uint32_t maximum_workers,
                         const or_workload_t *workload, void *context);

/* Runs the graph to completion: validation, then Programs in phase order with
 * tasks in compiled-stage (table) order, then the finish_program transition.
 * Leaves the final State in *state exactly as the resident kernels do. */
void or_run(or_state_t *state, const or_task_t *tasks,
            const or_program_t *programs, uint32_t program_count,
            uint32_t task_count, uint32_t phase_state_count,
            uint32_t abi_version, uint32_t maximum_workers,
            const or_workload_t *workload, void *context);

/* ---------------- Qwen2 decode workload (opcodes 1-13) ---------------- */

typedef struct or_decode_state_t {
  uint32_t token_position, kv_length, sampled_token, eos_token,
      generated_tokens, maximum_tokens, stop_reason;
  float sampled_logit;
} or_decode_state_t;

typedef struct or_qwen_tail_t {
  const float *final_norm_weight;
  const float *lm_head_weight;
  const float *token_embeddings;
  float *final_normalized;
  float *partial_max_values;
  uint32_t *partial_max_indices;
  or_decode_state_t *decode_state;
  uint32_t *output_tokens;
  uint32_t vocab_size, partition_count, embedding_count;
  /* Optional diagnostics (may be NULL): logits of the last LM-head pass
   * [vocab_size], and per generated token the gap between the best and the
   * second-best logit [maximum_tokens]. */
  float *logits;
  float *top2_gaps;
} or_qwen_tail_t;

typedef struct or_qwen_layer_t {
  float *hidden;
  const float *attention_norm_weight, *q_weight, *k_weight, *v_weight, *q_bias,
      *k_bias, *v_bias, *out_weight, *mlp_norm_weight, *gate_weight,
      *up_weight, *down_weight;
  float *attention_normalized, *query, *key, *value;
  const float *rope_cos, *rope_sin;
  float *key_cache, *value_cache, *mlp_normalized, *activated, *projected;
  or_qwen_tail_t *tail;
  uint32_t hidden_size, query_size, kv_size, intermediate_size, cache_capacity,
      layer_count;
} or_qwen_layer_t;

/* The Qwen workload; its context is an array of layer_count or_qwen_layer_t. */
const or_workload_t *or_qwen_workload(void);

/* Reference-order dot product of two length-n vectors (n % 32 == 0). */
float or_wave_dot(const float *x, const float *w, uint32_t n);

/* RoPE tables as the reference host driver builds them
 * (benchmarks/qwen_stateful_graph.cpp:912-929): [positions][32] each. */
void or_rope_tables(uint32_t positions, float theta, float *cos_table,
                    float *sin_table);

/* Number of OpenMP threads the Qwen workload may use (1 = scalar). */
void or_set_threads(int threads);
int or_max_threads(void);

/* ---------------- synthetic scheduler fixture workload ---------------- */

typedef struct or_fixture_context_t {
  uint32_t magic, value_count;
  uint32_t *values, *step_checksums, *branch_steps, *task_executions,
      *validation_calls;
} or_fixture_context_t;

const or_workload_t *or_fixture_workload(void);

#ifdef __cplusplus
}
#endif

#endif /* LRRT_ORACLE_H_ */
