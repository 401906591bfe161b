"""Qwen2 FP32 resident decode model on one B200 (wraps include/lrrt_qwen.h).

Mirrors the host flow of light-rocm-runtime benchmarks/qwen_stateful_graph.cpp:
build the decode graph, upload weights and KV caches, stage the initial hidden
vector and DecodeState, run the resident kernel, read results back.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from typing import Optional

import numpy as np

from . import native as N

HIDDEN = 896
HEADS = 14
KV_HEADS = 2
HEAD_DIM = 64
KV = KV_HEADS * HEAD_DIM
INTERMEDIATE = 4864
NO_TOKEN = 0xFFFFFFFF

PATH_COMPILED = 0
PATH_DYNAMIC = 1
PATH_HOST_STEP = 2
PATH_SCHEDULER_PROFILE = 3
PATH_STAGE_PROFILE = 4
PATH_GRAPH = 5

PREFILL_SIMT = 0    # FP32 FMA GEMM tiles on the CUDA cores
PREFILL_TF32X3 = 1  # 3xTF32 tcgen05 tensor-core GEMMs

BUFFERS = {
    "hidden": (0, HIDDEN, np.float32),
    "attention_normalized": (1, HIDDEN, np.float32),
    "query": (2, HEADS * HEAD_DIM, np.float32),
    "key": (3, KV, np.float32),
    "value": (4, KV, np.float32),
    "key_cache": (5, None, np.float32),
    "value_cache": (6, None, np.float32),
    "mlp_normalized": (7, HIDDEN, np.float32),
    "activated": (8, INTERMEDIATE, np.float32),
    "projected": (9, HIDDEN, np.float32),
    "final_normalized": (10, HIDDEN, np.float32),
    "partial_values": (11, None, np.float32),
    "partial_indices": (12, None, np.uint32),
    "output_tokens": (13, None, np.uint32),
    "rope_cos": (14, None, np.float32),
    "rope_sin": (15, None, np.float32),
    "logits": (16, None, np.float32),
}

STATUS_NAMES = {0: "ready", 1: "running", 2: "complete", 3: "max_steps", 4: "invalid_program"}


def _f32(array: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(array, dtype=np.float32)


def _ptr(array: np.ndarray) -> int:
    return array.ctypes.data


class Runtime:
    """Process-wide lr_init / lr_shutdown pair."""

    _initialized = False

    @classmethod
    def ensure(cls) -> None:
        if not cls._initialized:
            status = N.runtime().lr_init()
            if status not in (N.LR_SUCCESS, N.LR_ERROR_ALREADY_INITIALIZED):
                N.check(status, "lr_init")
            cls._initialized = True

    @classmethod
    def device_count(cls) -> int:
        cls.ensure()
        count = C.c_uint32()
        N.check(N.runtime().lr_device_count(C.byref(count)), "lr_device_count")
        return count.value

    @classmethod
    def open_device(cls, index: int) -> N.Device:
        cls.ensure()
        device = N.Device()
        N.check(N.runtime().lr_device_open(index, C.byref(device)), "lr_device_open")
        return device


@dataclass
class ModelConfig:
    layer_count: int = 24
    vocab_size: int = 151936
    cache_capacity: int = 256
    lm_head_partitions: int = 0
    worker_count: int = 0
    max_tokens_per_run: int = 128
    rope_theta: float = 1.0e6
    rms_epsilon: float = 1.0e-6
    tied_embeddings: bool = True
    disable_fused_path: bool = False

    def native(self) -> N.ModelConfig:
        return N.ModelConfig(self.layer_count, self.vocab_size, self.cache_capacity,
                             self.lm_head_partitions, self.worker_count,
                             self.max_tokens_per_run, self.rope_theta, self.rms_epsilon,
                             int(self.tied_embeddings), int(self.disable_fused_path))


def program_table(vocab_size: int, partitions: int):
    """The reference decode graph as (tasks, programs) numpy structured views."""
    tasks = (N.Task * 128)()
    programs = (N.Program * 4)()
    task_count, program_count = C.c_uint32(), C.c_uint32()
    N.check(N.driver().lrq_build_program_table(vocab_size, partitions, tasks, 128,
                                               C.byref(task_count), programs, 4,
                                               C.byref(program_count)),
            "lrq_build_program_table")
    return list(tasks[:task_count.value]), list(programs[:program_count.value])


def rope_tables(positions: int, theta: float = 1.0e6):
    cos = np.zeros((positions, HEAD_DIM // 2), np.float32)
    sin = np.zeros_like(cos)
    N.check(N.driver().lrq_rope_tables(positions, theta,
                                       cos.ctypes.data_as(C.POINTER(C.c_float)),
                                       sin.ctypes.data_as(C.POINTER(C.c_float))),
            "lrq_rope_tables")
    return cos, sin


class Model:
    """One decode model resident on one device."""

    def __init__(self, config: ModelConfig, device_index: int = 0,
                 cubin: Optional[bytes] = None):
        Runtime.ensure()
        self.config = config
        self.device = Runtime.open_device(device_index)
        image = cubin if cubin is not None else N.QWEN_CUBIN.read_bytes()
        self._image = C.create_string_buffer(image, len(image))
        handle = C.c_void_p()
        native_config = config.native()
        N.check(N.driver().lrq_model_create(self.device, self._image, len(image),
                                            C.byref(native_config), C.byref(handle)),
                "lrq_model_create")
        self.handle = handle
        info = N.ModelInfo()
        N.check(N.driver().lrq_model_info(self.handle, C.byref(info)), "lrq_model_info")
        self.info = info

    def close(self) -> None:
        if getattr(self, "handle", None):
            N.check(N.driver().lrq_model_destroy(self.handle), "lrq_model_destroy")
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    # ---- uploads -----------------------------------------------------------
    def set_layer(self, layer: int, weights: dict) -> None:
        arrays = {name: _f32(weights[name]) for name in N.LAYER_FIELDS}
        native = N.LayerWeights(*[_ptr(arrays[name]) for name in N.LAYER_FIELDS])
        N.check(N.driver().lrq_model_set_layer(self.handle, layer, C.byref(native)),
                "lrq_model_set_layer")

    def replicate_layer(self, source: int = 0) -> None:
        N.check(N.driver().lrq_model_replicate_layer(self.handle, source),
                "lrq_model_replicate_layer")

    def load_layer_bundle(self, layer: int, manifest: str) -> None:
        """Uploads decoder layer `layer` from an FP32 weight bundle
        ("lrrt.mini_decoder_weights" v2, see lrrt_b200.weight_bundle)."""
        N.check(N.driver().lrq_model_load_layer_bundle(self.handle, layer,
                                                       str(manifest).encode()),
                "lrq_model_load_layer_bundle")

    def load_tail_bundle(self, manifest: str) -> None:
        """Uploads the final norm and LM head (and, for an untied model, the
        embedding table) from a "lrrt.mini_model_tail_weights" v1 bundle."""
        N.check(N.driver().lrq_model_load_tail_bundle(self.handle, str(manifest).encode()),
                "lrq_model_load_tail_bundle")

    def set_tail(self, final_norm: np.ndarray, lm_head: np.ndarray,
                 embeddings: Optional[np.ndarray] = None) -> None:
        final_norm, lm_head = _f32(final_norm), _f32(lm_head)
        emb = _f32(embeddings) if embeddings is not None else None
        N.check(N.driver().lrq_model_set_tail(self.handle, _ptr(final_norm), _ptr(lm_head),
                                              _ptr(emb) if emb is not None else None),
                "lrq_model_set_tail")

    def set_kv(self, layer: int, first_position: int, keys: np.ndarray,
               values: np.ndarray) -> None:
        keys, values = _f32(keys).reshape(-1, KV), _f32(values).reshape(-1, KV)
        N.check(N.driver().lrq_model_set_kv(self.handle, layer, first_position,
                                            keys.shape[0], _ptr(keys), _ptr(values)),
                "lrq_model_set_kv")

    def set_hidden(self, hidden: np.ndarray) -> None:
        hidden = _f32(hidden)
        N.check(N.driver().lrq_model_set_hidden(self.handle, _ptr(hidden)),
                "lrq_model_set_hidden")

    def set_hidden_from_token(self, token: int) -> None:
        N.check(N.driver().lrq_model_set_hidden_from_token(self.handle, token),
                "lrq_model_set_hidden_from_token")

    def ingest_prompt(self, prompt) -> None:
        tokens = (C.c_uint32 * len(prompt))(*prompt)
        N.check(N.driver().lrq_model_ingest_prompt(self.handle, tokens, len(prompt)),
                "lrq_model_ingest_prompt")

    def enable_prefill(self, max_chunk_tokens: int = 512,
                       cubin: Optional[bytes] = None) -> None:
        """Loads the prefill module (lib/qwen_prefill.cubin) into the model."""
        image = cubin if cubin is not None else N.PREFILL_CUBIN.read_bytes()
        self._prefill_image = C.create_string_buffer(image, len(image))
        N.check(N.driver().lrq_model_enable_prefill(self.handle, self._prefill_image,
                                                    len(image), max_chunk_tokens),
                "lrq_model_enable_prefill")

    def prefill(self, prompt, path: int = PREFILL_TF32X3) -> None:
        """Batched prompt ingestion, same contract as ingest_prompt."""
        tokens = (C.c_uint32 * len(prompt))(*[int(t) for t in prompt])
        N.check(N.driver().lrq_model_prefill(self.handle, tokens, len(prompt), path),
                "lrq_model_prefill")

    def prefill_at(self, tokens, first_position: int, path: int = PREFILL_TF32X3) -> None:
        """K/V rows of `tokens` at positions first_position.. (no hidden staging)."""
        array = (C.c_uint32 * max(len(tokens), 1))(*[int(t) for t in tokens])
        N.check(N.driver().lrq_model_prefill_at(self.handle, array, len(tokens),
                                                first_position, path),
                "lrq_model_prefill_at")

    def prefill_gemm_check(self, tile_columns: int, mode: int, a: np.ndarray, b: np.ndarray,
                           c: np.ndarray, bias: Optional[np.ndarray] = None) -> np.ndarray:
        """One prefill GEMM on host arrays (see lrq_prefill_gemm_check)."""
        a, b = _f32(a), _f32(b)
        out = _f32(c).copy()
        m, k = a.shape
        n = out.shape[1]
        bias_array = _f32(bias) if bias is not None else None
        N.check(N.driver().lrq_prefill_gemm_check(
            self.handle, tile_columns, mode, m, n, k, _ptr(a), _ptr(b),
            _ptr(bias_array) if bias_array is not None else None, _ptr(out)),
            "lrq_prefill_gemm_check")
        return out

    # ---- runs --------------------------------------------------------------
    @staticmethod
    def request(token_position: int, maximum_tokens: int, eos_token: int = NO_TOKEN,
                path: int = PATH_COMPILED, max_steps: int = 0, stop_value: int = 0,
                wait_limit_ms: int = 0, launch_workers: int = 0) -> N.DecodeRequest:
        return N.DecodeRequest(token_position, maximum_tokens, eos_token, path, max_steps,
                               stop_value, wait_limit_ms, launch_workers)

    def launch(self, request: N.DecodeRequest) -> None:
        N.check(N.driver().lrq_decode_launch(self.handle, C.byref(request)),
                "lrq_decode_launch")

    def decode(self, token_position: int, maximum_tokens: int, **kwargs):
        request = self.request(token_position, maximum_tokens, **kwargs)
        state = N.RunState()
        tokens = (C.c_uint32 * self.config.max_tokens_per_run)()
        N.check(N.driver().lrq_decode(self.handle, C.byref(request), C.byref(state), tokens,
                                      self.config.max_tokens_per_run), "lrq_decode")
        return state, np.frombuffer(tokens, dtype=np.uint32)[:state.generated_tokens].copy()

    def read_state(self) -> N.RunState:
        state = N.RunState()
        N.check(N.driver().lrq_model_read_state(self.handle, C.byref(state)),
                "lrq_model_read_state")
        return state

    def generate(self, token_position: int, maximum_tokens: int, hidden=None,
                 start_token: int = 0, eos_token: int = NO_TOKEN, tokens=None):
        """End-to-end: host hidden in, host tokens out (one C-ABI call)."""
        out = tokens if tokens is not None else np.zeros(maximum_tokens, np.uint32)
        state = N.RunState()
        h = _f32(hidden) if hidden is not None else None
        N.check(N.driver().lrq_generate(self.handle, _ptr(h) if h is not None else None,
                                        start_token, token_position, maximum_tokens,
                                        eos_token, out.ctypes.data_as(C.POINTER(C.c_uint32)),
                                        C.byref(state)), "lrq_generate")
        return state, out

    def read(self, name: str, layer: int = 0, count: Optional[int] = None) -> np.ndarray:
        code, default_count, dtype = BUFFERS[name]
        if count is None:
            if name in ("key_cache", "value_cache"):
                count = self.config.cache_capacity * KV
            elif name in ("partial_values", "partial_indices"):
                count = self.info.lm_head_partitions
            elif name == "output_tokens":
                count = self.config.max_tokens_per_run
            elif name == "logits":
                count = self.config.vocab_size
            elif name in ("rope_cos", "rope_sin"):
                count = self.config.cache_capacity * HEAD_DIM // 2
            else:
                count = default_count
        out = np.zeros(count, dtype)
        N.check(N.driver().lrq_model_read(self.handle, code, layer, _ptr(out), out.nbytes),
                "lrq_model_read")
        return out

    def stage_profile(self):
        ticks = (C.c_uint64 * 13)()
        counts = (C.c_uint64 * 13)()
        N.check(N.driver().lrq_model_stage_profile(self.handle, ticks, counts),
                "lrq_model_stage_profile")
        return list(ticks), list(counts)

    def set_logit_capture(self, enable: bool = True) -> None:
        """Keep every LM-head row of the last decode step (read("logits"))."""
        N.check(N.driver().lrq_model_set_logit_capture(self.handle, 1 if enable else 0),
                "lrq_model_set_logit_capture")

    def set_trace(self, entries: int) -> None:
        N.check(N.driver().lrq_model_set_trace(self.handle, entries), "lrq_model_set_trace")

    def read_trace(self, entries: int) -> np.ndarray:
        out = np.zeros((entries, 2), np.uint64)
        N.check(N.driver().lrq_model_read_trace(
            self.handle, out.ctypes.data_as(C.POINTER(C.c_uint64)), entries),
            "lrq_model_read_trace")
        return out

    def synchronize(self) -> None:
        N.check(N.runtime().lr_synchronize(self.device), "lr_synchronize")


class EventTimer:
    """Device-time interval on the default queue via lr_event_*."""

    def __init__(self, device: N.Device):
        self.device = device
        self.start, self.end = C.c_void_p(), C.c_void_p()
        N.check(N.runtime().lr_event_create(device, C.byref(self.start)), "lr_event_create")
        N.check(N.runtime().lr_event_create(device, C.byref(self.end)), "lr_event_create")

    def record_start(self) -> None:
        N.check(N.runtime().lr_event_record(self.start), "lr_event_record")

    def record_end(self) -> None:
        N.check(N.runtime().lr_event_record(self.end), "lr_event_record")

    def elapsed_ns(self) -> int:
        value = C.c_uint64()
        N.check(N.runtime().lr_event_elapsed_time_ns(self.start, self.end, C.byref(value)),
                "lr_event_elapsed_time_ns")
        return value.value

    def close(self) -> None:
        for event in (self.start, self.end):
            if event:
                N.runtime().lr_event_destroy(event)
        self.start = self.end = None


class Batch:
    """Batched multi-stream greedy decode on one GPU (lrq_batch_* C ABI):
    `streams` independent streams with their own KV caches share the model's
    weights; every decode step produces one token per stream."""

    def __init__(self, model: Model, streams: int, capacity: int, max_tokens: int):
        self.model = model
        self.streams = streams
        self.max_tokens = max_tokens
        handle = C.c_void_p()
        N.check(N.driver().lrq_batch_create(model.handle, streams, capacity, max_tokens,
                                            C.byref(handle)), "lrq_batch_create")
        self.handle = handle

    def close(self) -> None:
        if self.handle:
            N.check(N.driver().lrq_batch_destroy(self.handle), "lrq_batch_destroy")
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def prefill(self, stream: int, prompt, path: int = PREFILL_TF32X3) -> None:
        tokens = (C.c_uint32 * len(prompt))(*[int(t) for t in prompt])
        N.check(N.driver().lrq_batch_prefill(self.handle, stream, tokens, len(prompt), path),
                "lrq_batch_prefill")

    def decode(self, steps: int):
        """(tokens [streams, steps], last chosen logit per stream)."""
        tokens = np.zeros((self.streams, steps), np.uint32)
        logits = np.zeros(self.streams, np.float32)
        N.check(N.driver().lrq_batch_decode(self.handle, steps, _ptr(tokens), _ptr(logits)),
                "lrq_batch_decode")
        return tokens, logits

    def write_cache(self, stream: int, layer: int, first: int, keys, values) -> None:
        k, v = _f32(keys), _f32(values)
        N.check(N.driver().lrq_batch_write_cache(self.handle, stream, layer, first, len(k),
                                                 _ptr(k), _ptr(v)), "lrq_batch_write_cache")

    def set_next(self, stream: int, position: int, token: int) -> None:
        N.check(N.driver().lrq_batch_set_next(self.handle, stream, position, token),
                "lrq_batch_set_next")

    def read_cache(self, stream: int, layer: int, positions: int):
        keys = np.zeros((positions, 128), np.float32)
        values = np.zeros((positions, 128), np.float32)
        N.check(N.driver().lrq_batch_read_cache(self.handle, stream, layer, positions,
                                                _ptr(keys), _ptr(values)),
                "lrq_batch_read_cache")
        return keys, values

    def position(self, stream: int) -> int:
        value = C.c_uint32()
        N.check(N.driver().lrq_batch_position(self.handle, stream, C.byref(value)),
                "lrq_batch_position")
        return value.value
