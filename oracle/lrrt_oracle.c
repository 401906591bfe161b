/*
 * CPU oracle (test infrastructure only; see lrrt_oracle.h for what it restates
 * and which reference lines each function follows).
 */
#include "lrrt_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

#define OR_KERNEL_THREADS 256u
#define OR_MAX_TASKS 64u
#define OR_MAX_PROGRAMS 256u
#define OR_PROGRAM_BITS 8u

static int g_threads = 1;

void or_set_threads(int threads) { g_threads = threads < 1 ? 1 : threads; }

int or_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

static uint32_t make_phase(uint32_t generation, uint32_t program) {
  return (generation << OR_PROGRAM_BITS) | program;
}
static uint32_t phase_generation(uint32_t phase) { return phase >> OR_PROGRAM_BITS; }
static uint32_t phase_program(uint32_t phase) {
  return phase & ((1u << OR_PROGRAM_BITS) - 1u);
}
static uint64_t task_dependencies(const or_task_t *task) {
  return (uint64_t)task->dependency_mask |
         ((uint64_t)task->dependency_mask_high << 32u);
}
static uint64_t all_tasks_mask(uint32_t count) {
  return count >= OR_MAX_TASKS ? UINT64_MAX : (((uint64_t)1 << count) - 1u);
}

void or_initialize_state(or_state_t *state, uint32_t abi_version,
                         uint32_t program_index, uint32_t max_steps,
                         uint32_t stop_value, uint32_t worker_count) {
  memset(state, 0, sizeof(*state));
  state->abi_version = abi_version;
  state->status = OR_STATUS_READY;
  state->phase = make_phase(0, program_index);
  state->max_steps = max_steps;
  state->stop_value = stop_value;
  state->worker_count = worker_count;
}

/* device_scheduler.hpp:65-131 */
int or_validate_programs(const or_state_t *state, const or_task_t *tasks,
                         const or_program_t *programs, uint32_t program_count,
                         uint32_t task_count, uint32_t phase_state_count,
                         uint32_t abi_version, uint32_t maximum_workers,
                         const or_workload_t *workload, void *context) {
  if (state->abi_version != abi_version || program_count == 0 ||
      task_count == 0 || program_count > OR_MAX_PROGRAMS ||
      phase_program(state->phase) >= program_count ||
      phase_generation(state->phase) >= phase_state_count ||
      state->max_steps == 0 || tasks == NULL || programs == NULL ||
      phase_state_count == 0 || state->worker_count == 0 ||
      state->worker_count > maximum_workers ||
      !workload->valid_context(state, context)) {
    return 0;
  }
  for (uint32_t p = 0; p < program_count; ++p) {
    const or_program_t *program = &programs[p];
    if (program->task_count == 0 || program->task_count > OR_MAX_TASKS ||
        program->task_offset > task_count ||
        program->task_count > task_count - program->task_offset ||
        program->next_program >= program_count ||
        (program->flags & ~(uint32_t)(OR_ADVANCES_STEP | OR_EVALUATES_PREDICATE |
                                      OR_BRANCHES_ON_STATE)) != 0 ||
        ((program->flags & OR_BRANCHES_ON_STATE) != 0 &&
         program->branch_program >= program_count)) {
      return 0;
    }
    const or_task_t *local = tasks + program->task_offset;
    const uint64_t valid = all_tasks_mask(program->task_count);
    for (uint32_t t = 0; t < program->task_count; ++t) {
      const uint64_t deps = task_dependencies(&local[t]);
      if (!workload->valid_task(&local[t], context) || (deps & ~valid) != 0 ||
          (deps & ((uint64_t)1 << t)) != 0) {
        return 0;
      }
    }
    uint64_t reachable = 0;
    for (uint32_t pass = 0; pass < program->task_count; ++pass) {
      for (uint32_t t = 0; t < program->task_count; ++t) {
        const uint64_t bit = (uint64_t)1 << t;
        const uint64_t deps = task_dependencies(&local[t]);
        if ((reachable & bit) == 0 && (deps & reachable) == deps) {
          reachable |= bit;
        }
      }
    }
    if (reachable != valid) {
      return 0;
    }
  }
  return 1;
}

/* compiled_scheduler.hpp:69-99 (identical transition in
 * device_scheduler.hpp:260-295). */
static void finish_program(or_state_t *state, const or_program_t *program,
                           uint32_t generation, uint32_t phase_state_count) {
  const uint32_t next_step =
      state->step + ((program->flags & OR_ADVANCES_STEP) != 0 ? 1u : 0u);
  state->step = next_step;
  state->executed_tasks += program->task_count;
  const int predicate = (program->flags & OR_EVALUATES_PREDICATE) != 0 &&
                        state->predicate_value >= state->stop_value;
  if (predicate) {
    state->status = OR_STATUS_COMPLETE;
  } else if (next_step >= state->max_steps) {
    state->status = OR_STATUS_MAX_STEPS;
  } else if (generation + 1u >= phase_state_count) {
    state->error_code = 2;
    state->status = OR_STATUS_INVALID;
  } else {
    uint32_t next = program->next_program;
    if ((program->flags & OR_BRANCHES_ON_STATE) != 0 && state->branch_value != 0) {
      next = program->branch_program;
    }
    state->phase = make_phase(generation + 1u, next);
  }
}

void or_run(or_state_t *state, const or_task_t *tasks,
            const or_program_t *programs, uint32_t program_count,
            uint32_t task_count, uint32_t phase_state_count,
            uint32_t abi_version, uint32_t maximum_workers,
            const or_workload_t *workload, void *context) {
  if (!or_validate_programs(state, tasks, programs, program_count, task_count,
                            phase_state_count, abi_version, maximum_workers,
                            workload, context)) {
    state->error_code = 1;
    state->status = OR_STATUS_INVALID;
    return;
  }
  state->status = OR_STATUS_RUNNING;
  while (state->status == OR_STATUS_RUNNING) {
    const uint32_t phase = state->phase;
    const uint32_t generation = phase_generation(phase);
    const or_program_t *program = &programs[phase_program(phase)];
    const or_task_t *local = tasks + program->task_offset;
    /* Greedy stage order (resident_executor.hpp:227-263): each stage is the
     * longest run of tasks whose dependencies earlier stages satisfied; tasks
     * of one stage touch disjoint outputs, so running them in table order is
     * equivalent to running them concurrently. */
    uint64_t done = 0;
    uint32_t next = 0;
    while (next < program->task_count) {
      uint32_t end = next;
      while (end < program->task_count) {
        const uint64_t deps = task_dependencies(&local[end]);
        if ((deps & done) != deps) {
          break;
        }
        ++end;
      }
      if (end == next) { /* unreachable after validation */
        state->error_code = 1;
        state->status = OR_STATUS_INVALID;
        return;
      }
      for (uint32_t t = next; t < end; ++t) {
        workload->execute(&local[t], state, context);
      }
      done |= all_tasks_mask(end - next) << next;
      next = end;
    }
    finish_program(state, program, generation, phase_state_count);
  }
}

/* ======================= Qwen2 decode workload ======================= */

enum {
  OP_ATTENTION_RMSNORM = 1,
  OP_QKV = 2,
  OP_ROPE_KV = 3,
  OP_GQA = 4,
  OP_ATTENTION_OUTPUT = 5,
  OP_MLP_RMSNORM = 6,
  OP_GATE_UP_SILU = 7,
  OP_DOWN = 8,
  OP_RESIDUAL_ADVANCE = 9,
  OP_FINAL_RMSNORM = 10,
  OP_LM_HEAD = 11,
  OP_TOP1_REDUCE = 12,
  OP_EMBEDDING_FEEDBACK = 13,
};

#define Q_HIDDEN 896u
#define Q_HEADS 14u
#define Q_KV_HEADS 2u
#define Q_HEAD 64u
#define Q_ROTARY 32u
#define Q_ROTARY_HEADS 16u
#define Q_QUERY 896u
#define Q_KV 128u
#define Q_PACKED 1152u
#define Q_INTERMEDIATE 4864u
#define Q_MAX_LM_PARTITIONS 32u

/* wave_sum over 32 lane partials (qwen_stateful_graph_kernel.cpp:122-127). */
static float lane_tree(float *lane) {
  for (uint32_t offset = 16; offset != 0; offset >>= 1u) {
    for (uint32_t l = 0; l < offset; ++l) {
      lane[l] += lane[l + offset];
    }
  }
  return lane[0];
}

float or_wave_dot(const float *x, const float *w, uint32_t n) {
  float lane[32];
  for (uint32_t l = 0; l < 32; ++l) {
    lane[l] = 0.0f;
  }
  for (uint32_t c = 0; c < n; c += 32u) {
    for (uint32_t l = 0; l < 32; ++l) {
      lane[l] = fmaf(x[c + l], w[c + l], lane[l]);
    }
  }
  return lane_tree(lane);
}

void or_rope_tables(uint32_t positions, float theta, float *cos_table,
                    float *sin_table) {
  for (uint32_t p = 0; p < positions; ++p) {
    for (uint32_t f = 0; f < Q_ROTARY; ++f) {
      const float exponent = -2.0f * (float)f / (float)Q_HEAD;
      const float angle = (float)p * powf(theta, exponent);
      cos_table[(size_t)p * Q_ROTARY + f] = cosf(angle);
      sin_table[(size_t)p * Q_ROTARY + f] = sinf(angle);
    }
  }
}

static int better_top1(float value, uint32_t index, float best_value,
                       uint32_t best_index) {
  return value > best_value || (value == best_value && index < best_index);
}

/* :47-77 */
static int qwen_valid_task(const or_task_t *task, void *opaque) {
  const or_qwen_layer_t *context = (const or_qwen_layer_t *)opaque;
  switch (task->opcode) {
  case OP_ATTENTION_RMSNORM:
  case OP_MLP_RMSNORM:
  case OP_FINAL_RMSNORM:
  case OP_DOWN:
    return task->begin < task->end && task->end <= context->hidden_size;
  case OP_QKV:
    return task->begin < task->end && task->end <= Q_PACKED;
  case OP_ROPE_KV:
    return task->begin == 0 && task->end == Q_ROTARY_HEADS;
  case OP_GQA:
    return task->begin < task->end && task->end <= Q_HEADS;
  case OP_ATTENTION_OUTPUT:
    return task->begin < task->end && task->end <= context->hidden_size;
  case OP_RESIDUAL_ADVANCE:
    return task->begin < task->end && task->end <= context->hidden_size &&
           task->argument0 != 0;
  case OP_GATE_UP_SILU:
    return task->begin < task->end && task->end <= context->intermediate_size;
  case OP_LM_HEAD:
    return task->begin < task->end && task->end <= context->tail->vocab_size &&
           task->argument0 < context->tail->partition_count;
  case OP_TOP1_REDUCE:
    return task->begin == 0 && task->end == context->tail->partition_count;
  case OP_EMBEDDING_FEEDBACK:
    return task->begin == 0 && task->end == context->hidden_size;
  default:
    return 0;
  }
}

/* :79-120 */
static int qwen_valid_context(const or_state_t *state, void *opaque) {
  (void)state;
  const or_qwen_layer_t *contexts = (const or_qwen_layer_t *)opaque;
  const or_qwen_layer_t *c = contexts;
  if (contexts == NULL || c->layer_count == 0 || c->hidden_size != Q_HIDDEN ||
      c->query_size != Q_QUERY || c->kv_size != Q_KV ||
      c->intermediate_size != Q_INTERMEDIATE || c->tail == NULL ||
      c->tail->final_norm_weight == NULL || c->tail->lm_head_weight == NULL ||
      c->tail->token_embeddings == NULL || c->tail->final_normalized == NULL ||
      c->tail->partial_max_values == NULL ||
      c->tail->partial_max_indices == NULL || c->tail->decode_state == NULL ||
      c->tail->output_tokens == NULL || c->tail->vocab_size == 0 ||
      c->tail->partition_count == 0 ||
      c->tail->partition_count > Q_MAX_LM_PARTITIONS ||
      c->tail->embedding_count != c->tail->vocab_size ||
      c->tail->decode_state->maximum_tokens == 0 ||
      c->tail->decode_state->maximum_tokens > c->cache_capacity ||
      c->tail->decode_state->token_position != c->tail->decode_state->kv_length ||
      c->tail->decode_state->token_position >= c->cache_capacity) {
    return 0;
  }
  for (uint32_t layer = 1; layer < c->layer_count; ++layer) {
    const or_qwen_layer_t *other = &contexts[layer];
    if (other->hidden_size != c->hidden_size ||
        other->query_size != c->query_size || other->kv_size != c->kv_size ||
        other->intermediate_size != c->intermediate_size ||
        other->cache_capacity != c->cache_capacity ||
        other->layer_count != c->layer_count || other->tail != c->tail) {
      return 0;
    }
  }
  return 1;
}

/* RMSNorm task (:665-701): 256 strided per-thread partial sums of squares, a
 * shared-memory tree, x * rsqrt(mean + eps) * w. rsqrt is taken as a correctly
 * rounded 1/sqrt. */
static void qwen_rmsnorm(const or_task_t *task, or_qwen_layer_t *c) {
  float partial[OR_KERNEL_THREADS];
  for (uint32_t t = 0; t < OR_KERNEL_THREADS; ++t) {
    float sum = 0.0f;
    for (uint32_t i = task->begin + t; i < task->end; i += OR_KERNEL_THREADS) {
      const float value = c->hidden[i];
      sum = fmaf(value, value, sum);
    }
    partial[t] = sum;
  }
  for (uint32_t stride = OR_KERNEL_THREADS / 2u; stride != 0; stride >>= 1u) {
    for (uint32_t t = 0; t < stride; ++t) {
      partial[t] += partial[t + stride];
    }
  }
  float epsilon;
  memcpy(&epsilon, &task->argument0, sizeof(epsilon));
  const float inverse_rms =
      1.0f / sqrtf(partial[0] / (float)(task->end - task->begin) + epsilon);
  const float *weight = c->tail->final_norm_weight;
  float *out = c->tail->final_normalized;
  if (task->opcode == OP_ATTENTION_RMSNORM) {
    weight = c->attention_norm_weight;
    out = c->attention_normalized;
  } else if (task->opcode == OP_MLP_RMSNORM) {
    weight = c->mlp_norm_weight;
    out = c->mlp_normalized;
  }
  for (uint32_t i = task->begin; i < task->end; ++i) {
    out[i] = c->hidden[i] * inverse_rms * weight[i];
  }
}

/* :392-427 packed rows: [0,896) q, [896,1024) k, [1024,1152) v, with bias. */
static void qwen_qkv(const or_task_t *task, or_qwen_layer_t *c) {
  const int64_t begin = task->begin, end = task->end;
#pragma omp parallel for schedule(static) num_threads(g_threads) if (g_threads > 1)
  for (int64_t packed = begin; packed < end; ++packed) {
    const float *weight = c->q_weight;
    const float *bias = c->q_bias;
    float *out = c->query;
    uint32_t row = (uint32_t)packed;
    if (row >= c->query_size + c->kv_size) {
      weight = c->v_weight;
      bias = c->v_bias;
      out = c->value;
      row -= c->query_size + c->kv_size;
    } else if (row >= c->query_size) {
      weight = c->k_weight;
      bias = c->k_bias;
      out = c->key;
      row -= c->query_size;
    }
    const float sum = or_wave_dot(c->attention_normalized,
                                  weight + (size_t)row * c->hidden_size,
                                  c->hidden_size);
    out[row] = sum + bias[row];
  }
}

/* :517-552 half-split RoPE at token_position on 14 q heads + 2 k heads, then
 * append rotated k and v to this layer's cache row token_position. */
static void qwen_rope_kv(or_qwen_layer_t *c) {
  const uint32_t position = c->tail->decode_state->token_position;
  const size_t rope = (size_t)position * Q_ROTARY;
  for (uint32_t pair = 0; pair < Q_ROTARY_HEADS * Q_ROTARY; ++pair) {
    const uint32_t head = pair / Q_ROTARY;
    const uint32_t f = pair % Q_ROTARY;
    const int is_query = head < Q_HEADS;
    const uint32_t local = is_query ? head : head - Q_HEADS;
    float *vector = is_query ? c->query : c->key;
    const uint32_t first = local * Q_HEAD + f;
    const uint32_t second = first + Q_ROTARY;
    const float x0 = vector[first];
    const float x1 = vector[second];
    const float cosine = c->rope_cos[rope + f];
    const float sine = c->rope_sin[rope + f];
    const float r0 = x0 * cosine - x1 * sine;
    const float r1 = x1 * cosine + x0 * sine;
    vector[first] = r0;
    vector[second] = r1;
    if (!is_query) {
      const size_t row = (size_t)position * c->kv_size;
      c->key_cache[row + first] = r0;
      c->key_cache[row + second] = r1;
    }
  }
  const size_t row = (size_t)position * c->kv_size;
  for (uint32_t i = 0; i < c->kv_size; ++i) {
    c->value_cache[row + i] = c->value[i];
  }
}

/* :554-600 one query head per wave, online softmax over positions
 * 0..kv_length inclusive, output written over the head's query slice. Lane l
 * owns dims l and l+32. */
static void qwen_gqa(const or_task_t *task, or_qwen_layer_t *c) {
  const uint32_t kv_length = c->tail->decode_state->kv_length;
  const float scale = 1.0f / sqrtf((float)Q_HEAD);
#pragma omp parallel for schedule(static) num_threads(g_threads) if (g_threads > 1)
  for (int64_t hq = task->begin; hq < (int64_t)task->end; ++hq) {
    const uint32_t head = (uint32_t)hq;
    const uint32_t kv_head = head / (Q_HEADS / Q_KV_HEADS);
    const float *q = c->query + head * Q_HEAD;
    float acc[Q_HEAD];
    for (uint32_t d = 0; d < Q_HEAD; ++d) {
      acc[d] = 0.0f;
    }
    float maximum = -INFINITY;
    float denominator = 0.0f;
    for (uint32_t position = 0; position <= kv_length; ++position) {
      const float *k = c->key_cache + (size_t)position * c->kv_size + kv_head * Q_HEAD;
      const float *v = c->value_cache + (size_t)position * c->kv_size + kv_head * Q_HEAD;
      float lane[32];
      for (uint32_t l = 0; l < 32; ++l) {
        lane[l] = q[l] * k[l] + q[l + 32] * k[l + 32];
      }
      const float score = lane_tree(lane) * scale;
      const float next_maximum = fmaxf(maximum, score);
      const float previous_scale = expf(maximum - next_maximum);
      const float score_scale = expf(score - next_maximum);
      denominator = denominator * previous_scale + score_scale;
      for (uint32_t d = 0; d < Q_HEAD; ++d) {
        acc[d] = acc[d] * previous_scale + score_scale * v[d];
      }
      maximum = next_maximum;
    }
    float *out = c->query + head * Q_HEAD;
    for (uint32_t d = 0; d < Q_HEAD; ++d) {
      out[d] = acc[d] / denominator;
    }
  }
}

/* :602-659 hidden[r] += O[r,:] . attention */
static void qwen_attention_output(const or_task_t *task, or_qwen_layer_t *c) {
#pragma omp parallel for schedule(static) num_threads(g_threads) if (g_threads > 1)
  for (int64_t r = task->begin; r < (int64_t)task->end; ++r) {
    c->hidden[r] += or_wave_dot(c->query, c->out_weight + (size_t)r * c->query_size,
                                c->query_size);
  }
}

/* :494-515 act = (g / (1 + exp(-g))) * u */
static void qwen_gate_up(const or_task_t *task, or_qwen_layer_t *c) {
#pragma omp parallel for schedule(static) num_threads(g_threads) if (g_threads > 1)
  for (int64_t r = task->begin; r < (int64_t)task->end; ++r) {
    const size_t offset = (size_t)r * c->hidden_size;
    const float gate = or_wave_dot(c->mlp_normalized, c->gate_weight + offset,
                                   c->hidden_size);
    const float up = or_wave_dot(c->mlp_normalized, c->up_weight + offset,
                                 c->hidden_size);
    c->activated[r] = (gate / (1.0f + expf(-gate))) * up;
  }
}

/* :158-223 projected[r] = D[r,:] . act */
static void qwen_down(const or_task_t *task, or_qwen_layer_t *c) {
#pragma omp parallel for schedule(static) num_threads(g_threads) if (g_threads > 1)
  for (int64_t r = task->begin; r < (int64_t)task->end; ++r) {
    c->projected[r] = or_wave_dot(
        c->activated, c->down_weight + (size_t)r * c->intermediate_size,
        c->intermediate_size);
  }
}

/* :749-760 */
static void qwen_residual_advance(const or_task_t *task, or_state_t *state,
                                  or_qwen_layer_t *c) {
  for (uint32_t i = task->begin; i < task->end; ++i) {
    c->hidden[i] += c->projected[i];
  }
  const int boundary =
      task->argument1 == 0 || (state->step + 1u) % c->layer_count == 0;
  if (boundary && task->argument1 == 0) {
    state->predicate_value += task->argument0;
  }
  state->branch_value = (uint32_t)boundary;
}

/* :231-337 per-partition top-1 with lower-index tie break. */
static void qwen_lm_head(const or_task_t *task, or_qwen_layer_t *c) {
  or_qwen_tail_t *tail = c->tail;
  const int64_t begin = task->begin, end = task->end;
  const int64_t count = end - begin;
  float *logits = tail->logits != NULL ? tail->logits + begin
                                       : (float *)malloc((size_t)count * sizeof(float));
#pragma omp parallel for schedule(static) num_threads(g_threads) if (g_threads > 1)
  for (int64_t r = begin; r < end; ++r) {
    logits[r - begin] = or_wave_dot(tail->final_normalized,
                                    tail->lm_head_weight + (size_t)r * c->hidden_size,
                                    c->hidden_size);
  }
  float best_value = -INFINITY;
  uint32_t best_index = UINT32_MAX;
  for (int64_t r = begin; r < end; ++r) {
    if (better_top1(logits[r - begin], (uint32_t)r, best_value, best_index)) {
      best_value = logits[r - begin];
      best_index = (uint32_t)r;
    }
  }
  tail->partial_max_values[task->argument0] = best_value;
  tail->partial_max_indices[task->argument0] = best_index;
  if (tail->logits == NULL) {
    free(logits);
  }
}

/* :339-356 */
static void qwen_reduce_top1(or_qwen_layer_t *c) {
  or_qwen_tail_t *tail = c->tail;
  float best_value = tail->partial_max_values[0];
  uint32_t best_index = tail->partial_max_indices[0];
  for (uint32_t p = 1; p < tail->partition_count; ++p) {
    if (better_top1(tail->partial_max_values[p], tail->partial_max_indices[p],
                    best_value, best_index)) {
      best_value = tail->partial_max_values[p];
      best_index = tail->partial_max_indices[p];
    }
  }
  tail->decode_state->sampled_logit = best_value;
  tail->decode_state->sampled_token = best_index;
  if (tail->logits != NULL && tail->top2_gaps != NULL &&
      tail->decode_state->generated_tokens < tail->decode_state->maximum_tokens) {
    float second = -INFINITY;
    for (uint32_t r = 0; r < tail->vocab_size; ++r) {
      if (r != best_index && tail->logits[r] > second) {
        second = tail->logits[r];
      }
    }
    tail->top2_gaps[tail->decode_state->generated_tokens] = best_value - second;
  }
}

/* :358-390 */
static void qwen_embedding_feedback(or_qwen_layer_t *c, or_state_t *state) {
  or_decode_state_t *decode = c->tail->decode_state;
  const uint32_t index = decode->generated_tokens;
  const uint32_t token = decode->sampled_token;
  c->tail->output_tokens[index] = token;
  decode->generated_tokens = index + 1u;
  const int eos = token == decode->eos_token;
  const int limit = decode->generated_tokens >= decode->maximum_tokens;
  if (eos || limit) {
    decode->stop_reason = eos ? 2u : 1u;
    state->predicate_value = 1;
  } else {
    ++decode->token_position;
    ++decode->kv_length;
  }
  if (state->predicate_value == 0) {
    const float *row = c->tail->token_embeddings + (size_t)token * c->hidden_size;
    memcpy(c->hidden, row, c->hidden_size * sizeof(float));
  }
}

static void qwen_execute(const or_task_t *task, or_state_t *state, void *opaque) {
  or_qwen_layer_t *contexts = (or_qwen_layer_t *)opaque;
  or_qwen_layer_t *c = &contexts[state->step % contexts[0].layer_count];
  switch (task->opcode) {
  case OP_ATTENTION_RMSNORM:
  case OP_MLP_RMSNORM:
  case OP_FINAL_RMSNORM:
    qwen_rmsnorm(task, c);
    return;
  case OP_QKV:
    qwen_qkv(task, c);
    return;
  case OP_ROPE_KV:
    qwen_rope_kv(c);
    return;
  case OP_GQA:
    qwen_gqa(task, c);
    return;
  case OP_ATTENTION_OUTPUT:
    qwen_attention_output(task, c);
    return;
  case OP_GATE_UP_SILU:
    qwen_gate_up(task, c);
    return;
  case OP_DOWN:
    qwen_down(task, c);
    return;
  case OP_LM_HEAD:
    qwen_lm_head(task, c);
    return;
  case OP_TOP1_REDUCE:
    qwen_reduce_top1(c);
    return;
  case OP_EMBEDDING_FEEDBACK:
    qwen_embedding_feedback(c, state);
    return;
  default:
    qwen_residual_advance(task, state, c);
    return;
  }
}

static const or_workload_t k_qwen_workload = {qwen_valid_context, qwen_valid_task,
                                              qwen_execute};

const or_workload_t *or_qwen_workload(void) { return &k_qwen_workload; }

/* ================== synthetic scheduler fixture workload ================== */
/* tests/stateful_graph_device_kernel.cpp:46-136 of the reference. */

#define FX_MAGIC 0x53504754u
#define FX_VALUES 8u
#define FX_MAX_STEPS 8u
#define FX_TASKS 5u

static int fixture_valid_context(const or_state_t *state, void *opaque) {
  (void)state;
  or_fixture_context_t *c = (or_fixture_context_t *)opaque;
  if (c != NULL && c->validation_calls != NULL) {
    ++*c->validation_calls;
  }
  return c != NULL && c->magic == FX_MAGIC && c->value_count == FX_VALUES &&
         c->values != NULL && c->step_checksums != NULL &&
         c->branch_steps != NULL && c->task_executions != NULL &&
         c->validation_calls != NULL;
}

static int fixture_valid_task(const or_task_t *task, void *opaque) {
  (void)opaque;
  if (task->argument1 >= FX_TASKS) {
    return 0;
  }
  switch (task->opcode) {
  case 0:
    return task->begin < task->end && task->end <= FX_VALUES && task->argument0 != 0;
  case 1:
    return task->begin == 0 && task->end == FX_VALUES;
  case 2:
  case 3:
    return task->begin == 0 && task->end == 1 && task->argument0 != 0;
  default:
    return 0;
  }
}

static void fixture_execute(const or_task_t *task, or_state_t *state, void *opaque) {
  or_fixture_context_t *c = (or_fixture_context_t *)opaque;
  ++c->task_executions[task->argument1];
  switch (task->opcode) {
  case 0:
    for (uint32_t i = task->begin; i < task->end; ++i) {
      c->values[i] += task->argument0 + state->step;
    }
    return;
  case 1: {
    uint32_t checksum = 0;
    for (uint32_t i = task->begin; i < task->end; ++i) {
      checksum += c->values[i];
    }
    if (state->step < FX_MAX_STEPS) {
      c->step_checksums[state->step] = checksum;
    }
    return;
  }
  case 2:
    state->branch_value = (uint32_t)((state->step + 1u) % task->argument0 == 0);
    return;
  case 3:
    if (state->predicate_value < FX_MAX_STEPS) {
      c->branch_steps[state->predicate_value] = state->step;
    }
    state->predicate_value += task->argument0;
    return;
  default:
    return;
  }
}

static const or_workload_t k_fixture_workload = {
    fixture_valid_context, fixture_valid_task, fixture_execute};

const or_workload_t *or_fixture_workload(void) { return &k_fixture_workload; }
