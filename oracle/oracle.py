"""Python side of the CPU oracle (TEST INFRASTRUCTURE ONLY).

Loads oracle/_build/liblrrt_oracle.so (built by oracle/Makefile) and exposes
the reference's decode graph and Qwen task arithmetic on host arrays. Only
tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import this
module; the product path never does.

make_program_table restates light-rocm-runtime
benchmarks/qwen_stateful_graph.cpp:368-485 independently of the product's
C++ builder so the two can be compared.
"""
from __future__ import annotations

import ctypes as C
import struct
import subprocess
from pathlib import Path

import numpy as np

ORACLE_DIR = Path(__file__).resolve().parent
LIBRARY = ORACLE_DIR / "_build" / "liblrrt_oracle.so"

ABI_VERSION = 10          # B200 persistent-graph ABI revision
MAXIMUM_WORKERS = 256     # B200 kMaximumResidentWorkers
HIDDEN, QUERY, KV, INTERMEDIATE = 896, 896, 128, 4864
PACKED_QKV, HEADS, ROTARY_HEADS = 1152, 14, 16
NO_TOKEN = 0xFFFFFFFF

u32, u64, f32, vp = C.c_uint32, C.c_uint64, C.c_float, C.c_void_p


class Task(C.Structure):
    _fields_ = [(n, u32) for n in ("opcode", "dependency_mask", "begin", "end",
                                   "argument0", "argument1", "dependency_mask_high",
                                   "reserved")]


class Program(C.Structure):
    _fields_ = [("task_offset", u32), ("task_count", u32), ("next_program", u32),
                ("flags", u32), ("branch_program", u32), ("reserved", u32 * 3)]


class State(C.Structure):
    _fields_ = [("abi_version", u32), ("status", u32), ("phase", u32), ("step", u32),
                ("max_steps", u32), ("stop_value", u32), ("error_code", u32),
                ("worker_count", u32), ("executed_tasks", u64), ("predicate_value", u32),
                ("branch_value", u32), ("reserved", u32 * 4)]


class DecodeState(C.Structure):
    _fields_ = [("token_position", u32), ("kv_length", u32), ("sampled_token", u32),
                ("eos_token", u32), ("generated_tokens", u32), ("maximum_tokens", u32),
                ("stop_reason", u32), ("sampled_logit", f32)]


class Tail(C.Structure):
    _fields_ = [("final_norm_weight", vp), ("lm_head_weight", vp), ("token_embeddings", vp),
                ("final_normalized", vp), ("partial_max_values", vp),
                ("partial_max_indices", vp), ("decode_state", vp), ("output_tokens", vp),
                ("vocab_size", u32), ("partition_count", u32), ("embedding_count", u32),
                ("logits", vp), ("top2_gaps", vp)]


LAYER_POINTERS = ("hidden", "attention_norm_weight", "q_weight", "k_weight", "v_weight",
                  "q_bias", "k_bias", "v_bias", "out_weight", "mlp_norm_weight",
                  "gate_weight", "up_weight", "down_weight", "attention_normalized",
                  "query", "key", "value", "rope_cos", "rope_sin", "key_cache",
                  "value_cache", "mlp_normalized", "activated", "projected")


class Layer(C.Structure):
    _fields_ = [(n, vp) for n in LAYER_POINTERS] + [
        ("tail", C.POINTER(Tail)), ("hidden_size", u32), ("query_size", u32),
        ("kv_size", u32), ("intermediate_size", u32), ("cache_capacity", u32),
        ("layer_count", u32)]


class FixtureContext(C.Structure):
    _fields_ = [("magic", u32), ("value_count", u32), ("values", vp),
                ("step_checksums", vp), ("branch_steps", vp), ("task_executions", vp),
                ("validation_calls", vp)]


class Workload(C.Structure):
    _fields_ = [("valid_context", vp), ("valid_task", vp), ("execute", vp)]


_lib = None


def library() -> C.CDLL:
    global _lib
    if _lib is None:
        if not LIBRARY.exists():
            subprocess.run(["make", "-s", "-C", str(ORACLE_DIR)], check=True)
        lib = C.CDLL(str(LIBRARY))
        lib.or_initialize_state.argtypes = [C.POINTER(State), u32, u32, u32, u32, u32]
        lib.or_run.argtypes = [C.POINTER(State), C.POINTER(Task), C.POINTER(Program), u32,
                               u32, u32, u32, u32, vp, vp]
        lib.or_validate_programs.argtypes = [C.POINTER(State), C.POINTER(Task),
                                             C.POINTER(Program), u32, u32, u32, u32, u32,
                                             vp, vp]
        lib.or_validate_programs.restype = C.c_int
        lib.or_qwen_workload.restype = vp
        lib.or_fixture_workload.restype = vp
        lib.or_wave_dot.argtypes = [vp, vp, u32]
        lib.or_wave_dot.restype = f32
        lib.or_rope_tables.argtypes = [u32, f32, vp, vp]
        lib.or_set_threads.argtypes = [C.c_int]
        lib.or_max_threads.restype = C.c_int
        _lib = lib
    return _lib


def set_threads(threads: int) -> None:
    library().or_set_threads(threads)


def max_threads() -> int:
    return library().or_max_threads()


def float_bits(value: float) -> int:
    return struct.unpack("<I", struct.pack("<f", value))[0]


def make_task(opcode, dependencies, begin, end, argument0=0, argument1=0):
    return (opcode, dependencies & 0xFFFFFFFF, begin, end, argument0, argument1,
            dependencies >> 32, 0)


def make_program_table(vocab: int, partitions: int):
    """Reference decode graph (qwen_stateful_graph.cpp:368-485) as tuples."""
    eps = float_bits(1.0e-6)
    tasks, programs = [], []
    tasks.append(make_task(1, 0, 0, HIDDEN, eps))
    qkv = 0
    for p in range(8):
        qkv |= 1 << len(tasks)
        tasks.append(make_task(2, 1, PACKED_QKV * p // 8, PACKED_QKV * (p + 1) // 8))
    rope = 1 << len(tasks)
    tasks.append(make_task(3, qkv, 0, ROTARY_HEADS))
    attention = 0
    for p in range(7):
        attention |= 1 << len(tasks)
        tasks.append(make_task(4, rope, HEADS * p // 7, HEADS * (p + 1) // 7))
    for p in range(8):
        tasks.append(make_task(5, attention, HIDDEN * p // 8, HIDDEN * (p + 1) // 8))
    programs.append((0, len(tasks), 1, 0, 0))
    ffn = len(tasks)
    tasks.append(make_task(6, 0, 0, HIDDEN, eps))
    activated = 0
    for p in range(20):
        activated |= 1 << (len(tasks) - ffn)
        tasks.append(make_task(7, 1, INTERMEDIATE * p // 20, INTERMEDIATE * (p + 1) // 20))
    down = 0
    for p in range(32):
        down |= 1 << (len(tasks) - ffn)
        tasks.append(make_task(8, activated, HIDDEN * p // 32, HIDDEN * (p + 1) // 32))
    tasks.append(make_task(9, down, 0, HIDDEN, 1, 1))
    programs.append((ffn, len(tasks) - ffn, 0, 1 | 4, 2))
    tail = len(tasks)
    tasks.append(make_task(10, 0, 0, HIDDEN, eps))
    candidates = 0
    for p in range(partitions):
        candidates |= 1 << (len(tasks) - tail)
        tasks.append(make_task(11, 1, vocab * p // partitions, vocab * (p + 1) // partitions, p))
    reduce = 1 << (len(tasks) - tail)
    tasks.append(make_task(12, candidates, 0, partitions))
    tasks.append(make_task(13, reduce, 0, HIDDEN))
    programs.append((tail, partitions + 3, 0, 2, 0))
    return tasks, programs


def task_array(tasks):
    array = (Task * len(tasks))()
    for i, t in enumerate(tasks):
        array[i] = Task(*t)
    return array


def program_array(programs):
    array = (Program * len(programs))()
    for i, p in enumerate(programs):
        array[i] = Program(p[0], p[1], p[2], p[3], p[4], (u32 * 3)(0, 0, 0))
    return array


def run_graph(state: State, tasks, programs, phase_state_count, workload, context) -> State:
    t, p = task_array(tasks), program_array(programs)
    library().or_run(C.byref(state), t, p, len(programs), len(tasks), phase_state_count,
                     ABI_VERSION, MAXIMUM_WORKERS, workload, context)
    return state


def initial_state(program: int, max_steps: int, stop_value: int, workers: int) -> State:
    state = State()
    library().or_initialize_state(C.byref(state), ABI_VERSION, program, max_steps,
                                  stop_value, workers)
    return state


def wave_dot(x: np.ndarray, w: np.ndarray) -> float:
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    return float(library().or_wave_dot(x.ctypes.data, w.ctypes.data, x.size))


def rope_tables(positions: int, theta: float):
    cos = np.zeros((positions, 32), np.float32)
    sin = np.zeros((positions, 32), np.float32)
    library().or_rope_tables(positions, theta, cos.ctypes.data, sin.ctypes.data)
    return cos, sin


class OracleModel:
    """Host-memory restatement of the decode model, run through or_run with
    the reference task table."""

    def __init__(self, layers, tail, cache_capacity, partitions, workers=148,
                 theta=1.0e6, max_tokens=128, keep_logits=True):
        self.layer_weights = [{k: np.ascontiguousarray(v, np.float32) for k, v in w.items()}
                              for w in layers]
        self.tail_weights = {k: np.ascontiguousarray(v, np.float32) for k, v in tail.items()}
        self.layers = len(layers)
        self.vocab = self.tail_weights["lm_head"].shape[0]
        self.capacity = cache_capacity
        self.partitions = partitions
        self.workers = workers
        self.max_tokens = max_tokens
        z = lambda n, dt=np.float32: np.zeros(n, dt)  # noqa: E731
        self.hidden = z(HIDDEN)
        self.attention_normalized = z(HIDDEN)
        self.query, self.key, self.value = z(QUERY), z(KV), z(KV)
        self.mlp_normalized, self.activated, self.projected = z(HIDDEN), z(INTERMEDIATE), z(HIDDEN)
        self.final_normalized = z(HIDDEN)
        self.partial_values = z(32)
        self.partial_indices = z(32, np.uint32)
        self.output_tokens = z(max_tokens, np.uint32)
        self.logits = z(self.vocab) if keep_logits else None
        self.top2_gaps = z(max_tokens)
        self.key_cache = [np.zeros((cache_capacity, KV), np.float32) for _ in range(self.layers)]
        self.value_cache = [np.zeros((cache_capacity, KV), np.float32) for _ in range(self.layers)]
        self.rope_cos, self.rope_sin = rope_tables(cache_capacity, theta)
        self.decode_state = DecodeState()
        self.tail = Tail(self.tail_weights["final_norm"].ctypes.data,
                         self.tail_weights["lm_head"].ctypes.data,
                         self.tail_weights.get("embeddings", self.tail_weights["lm_head"]).ctypes.data,
                         self.final_normalized.ctypes.data, self.partial_values.ctypes.data,
                         self.partial_indices.ctypes.data, C.addressof(self.decode_state),
                         self.output_tokens.ctypes.data, self.vocab, partitions, self.vocab,
                         self.logits.ctypes.data if keep_logits else None,
                         self.top2_gaps.ctypes.data)
        names = {"attention_norm_weight": "attention_norm", "q_weight": "q", "k_weight": "k",
                 "v_weight": "v", "q_bias": "q_bias", "k_bias": "k_bias", "v_bias": "v_bias",
                 "out_weight": "o", "mlp_norm_weight": "mlp_norm", "gate_weight": "gate",
                 "up_weight": "up", "down_weight": "down"}
        self.contexts = (Layer * self.layers)()
        for i, w in enumerate(self.layer_weights):
            c = self.contexts[i]
            c.hidden = self.hidden.ctypes.data
            for field, key in names.items():
                setattr(c, field, w[key].ctypes.data)
            c.attention_normalized = self.attention_normalized.ctypes.data
            c.query, c.key, c.value = (self.query.ctypes.data, self.key.ctypes.data,
                                       self.value.ctypes.data)
            c.rope_cos, c.rope_sin = self.rope_cos.ctypes.data, self.rope_sin.ctypes.data
            c.key_cache = self.key_cache[i].ctypes.data
            c.value_cache = self.value_cache[i].ctypes.data
            c.mlp_normalized = self.mlp_normalized.ctypes.data
            c.activated, c.projected = self.activated.ctypes.data, self.projected.ctypes.data
            c.tail = C.pointer(self.tail)
            c.hidden_size, c.query_size, c.kv_size = HIDDEN, QUERY, KV
            c.intermediate_size, c.cache_capacity, c.layer_count = (INTERMEDIATE,
                                                                    cache_capacity,
                                                                    self.layers)
        self.tasks, self.programs = make_program_table(self.vocab, partitions)

    def set_kv(self, layer, first, keys, values):
        self.key_cache[layer][first:first + len(keys)] = keys
        self.value_cache[layer][first:first + len(values)] = values

    def decode(self, hidden, token_position, maximum_tokens, eos=NO_TOKEN):
        self.hidden[:] = hidden
        self.decode_state.token_position = token_position
        self.decode_state.kv_length = token_position
        self.decode_state.sampled_token = 0
        self.decode_state.eos_token = eos
        self.decode_state.generated_tokens = 0
        self.decode_state.maximum_tokens = maximum_tokens
        self.decode_state.stop_reason = 0
        self.decode_state.sampled_logit = 0.0
        phase_states = maximum_tokens * 2 * (2 * self.layers + 1) + 1
        state = initial_state(0, 2 * maximum_tokens * self.layers, 1, self.workers)
        run_graph(state, self.tasks, self.programs, phase_states,
                  library().or_qwen_workload(), C.cast(self.contexts, vp))
        return state

    def embedding(self, token):
        table = self.tail_weights.get("embeddings", self.tail_weights["lm_head"])
        return table[token].copy()


__all__ = ["OracleModel", "make_program_table", "run_graph", "initial_state", "wave_dot",
           "rope_tables", "set_threads", "max_threads", "FixtureContext", "library",
           "NO_TOKEN"]
