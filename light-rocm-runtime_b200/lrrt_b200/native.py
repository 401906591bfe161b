"""ctypes declarations of the package's two C ABIs.

liblrrt.so       -- the lr_* runtime ABI (include/lrrt/lrrt.h)
liblrrt_qwen.so  -- the Qwen decode driver ABI (include/lrrt_qwen.h)

Both libraries are built in-tree by ``build.py``; loading fails loudly when
they are missing, there is no fallback implementation.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent.parent
LIB = PACKAGE / "lib"
RUNTIME_PATH = LIB / "liblrrt.so"
DRIVER_PATH = LIB / "liblrrt_qwen.so"
QWEN_CUBIN = LIB / "qwen_stateful_graph.cubin"
PREFILL_CUBIN = LIB / "qwen_prefill.cubin"
FIXTURE_CUBIN = PACKAGE / "_build" / "tests" / "stateful_graph_fixture.cubin"

u32, u64, f32, vp, cp, sz = C.c_uint32, C.c_uint64, C.c_float, C.c_void_p, C.c_char_p, C.c_size_t

LR_SUCCESS = 0
LR_ERROR_INVALID_ARGUMENT = 1
LR_ERROR_NOT_INITIALIZED = 2
LR_ERROR_ALREADY_INITIALIZED = 3
LR_ERROR_NOT_SUPPORTED = 4
LR_ERROR_RUNTIME = 5
LR_ERROR_DEVICE_FAULT = 6

LR_MEMCPY_HOST_TO_DEVICE = 0
LR_MEMCPY_DEVICE_TO_HOST = 1
LR_MEMCPY_DEVICE_TO_DEVICE = 2


class Device(C.Structure):
    _fields_ = [("index", u32)]


class Dim3(C.Structure):
    _fields_ = [("x", u32), ("y", u32), ("z", u32)]


class LaunchConfig(C.Structure):
    _fields_ = [("grid", Dim3), ("block", Dim3), ("shared_memory_bytes", u32)]


class MemoryStats(C.Structure):
    _fields_ = [(name, u64) for name in (
        "live_bytes", "peak_live_bytes", "total_allocated_bytes", "total_freed_bytes",
        "allocation_count", "free_count", "h2d_copy_bytes", "d2h_copy_bytes",
        "d2d_copy_bytes", "memcpy_count", "pinned_host_live_bytes",
        "pinned_host_peak_live_bytes", "pinned_host_total_allocated_bytes",
        "pinned_host_total_freed_bytes", "pinned_host_allocation_count",
        "pinned_host_free_count")]


class DeviceProperties(C.Structure):
    _fields_ = [("compute_unit_count", u32), ("wavefront_size", u32),
                ("maximum_waves_per_compute_unit", u32), ("maximum_workgroup_size", u32),
                ("group_segment_size", u64), ("shader_engine_count", u32)]


class KernelProperties(C.Structure):
    _fields_ = [("kernarg_size", u32), ("group_segment_size", u32),
                ("private_segment_size", u32)]


class Task(C.Structure):
    _fields_ = [(name, u32) for name in (
        "opcode", "dependency_mask", "begin", "end", "argument0", "argument1",
        "dependency_mask_high", "reserved")]


class Program(C.Structure):
    _fields_ = [("task_offset", u32), ("task_count", u32), ("next_program", u32),
                ("flags", u32), ("branch_program", u32), ("reserved", u32 * 3)]


class ModelConfig(C.Structure):
    _fields_ = [("layer_count", u32), ("vocab_size", u32), ("cache_capacity", u32),
                ("lm_head_partitions", u32), ("worker_count", u32),
                ("max_tokens_per_run", u32), ("rope_theta", f32), ("rms_epsilon", f32),
                ("tied_embeddings", u32), ("disable_fused_path", u32)]


LAYER_FIELDS = ("attention_norm", "q", "k", "v", "q_bias", "k_bias", "v_bias", "o",
                "mlp_norm", "gate", "up", "down")


class LayerWeights(C.Structure):
    _fields_ = [(name, vp) for name in LAYER_FIELDS]


class DecodeRequest(C.Structure):
    _fields_ = [(name, u32) for name in (
        "token_position", "maximum_tokens", "eos_token", "path", "max_steps",
        "stop_value", "wait_limit_ms", "launch_workers")]


class RunState(C.Structure):
    _fields_ = [("status", u32), ("phase", u32), ("step", u32), ("max_steps", u32),
                ("stop_value", u32), ("error_code", u32), ("worker_count", u32),
                ("predicate_value", u32), ("branch_value", u32), ("reserved", u32),
                ("executed_tasks", u64), ("token_position", u32), ("kv_length", u32),
                ("sampled_token", u32), ("eos_token", u32), ("generated_tokens", u32),
                ("maximum_tokens", u32), ("stop_reason", u32), ("sampled_logit", f32),
                ("fused_path", u32), ("reserved2", u32)]


class ModelInfo(C.Structure):
    _fields_ = [("worker_count", u32), ("lm_head_partitions", u32), ("layer_count", u32),
                ("vocab_size", u32), ("cache_capacity", u32), ("dynamic_shared_bytes", u32),
                ("phase_state_count", u32), ("task_count", u32), ("device_bytes", u64),
                ("weight_bytes_per_token", u64)]


P = C.POINTER

# name -> (restype, argtypes)
RUNTIME_FUNCTIONS = {
    "lr_status_string": (cp, [u32]),
    "lr_init": (u32, []),
    "lr_shutdown": (u32, []),
    "lr_device_count": (u32, [P(u32)]),
    "lr_device_open": (u32, [u32, P(Device)]),
    "lr_device_name": (u32, [Device, C.c_char_p, sz]),
    "lr_device_get_properties": (u32, [Device, P(DeviceProperties)]),
    "lr_get_memory_stats": (u32, [Device, P(MemoryStats)]),
    "lr_reset_memory_stats": (u32, [Device]),
    "lr_queue_create": (u32, [Device, P(vp)]),
    "lr_queue_destroy": (u32, [vp]),
    "lr_queue_synchronize": (u32, [vp]),
    "lr_event_create": (u32, [Device, P(vp)]),
    "lr_event_destroy": (u32, [vp]),
    "lr_event_record": (u32, [vp]),
    "lr_event_record_on_queue": (u32, [vp, vp]),
    "lr_event_synchronize": (u32, [vp]),
    "lr_event_elapsed_time_ns": (u32, [vp, vp, P(u64)]),
    "lr_event_duration_ns": (u32, [vp, P(u64)]),
    "lr_malloc": (u32, [Device, sz, P(vp)]),
    "lr_free": (u32, [Device, vp]),
    "lr_host_malloc": (u32, [Device, sz, P(vp)]),
    "lr_host_free": (u32, [Device, vp]),
    "lr_memcpy": (u32, [Device, vp, vp, sz, u32]),
    "lr_memcpy_async": (u32, [Device, vp, vp, sz, u32, vp]),
    "lr_memcpy_async_with_dependencies": (u32, [Device, vp, vp, sz, u32, vp, P(vp), sz]),
    "lr_module_load_hsaco": (u32, [Device, vp, sz, P(vp)]),
    "lr_module_destroy": (u32, [vp]),
    "lr_kernel_get": (u32, [vp, cp, P(vp)]),
    "lr_kernel_get_properties": (u32, [vp, P(KernelProperties)]),
    "lr_launch": (u32, [vp, P(LaunchConfig), vp, sz]),
    "lr_launch_with_dependencies": (u32, [vp, P(LaunchConfig), vp, sz, P(vp), sz]),
    "lr_launch_on_queue": (u32, [vp, vp, P(LaunchConfig), vp, sz]),
    "lr_launch_on_queue_with_dependencies": (u32, [vp, vp, P(LaunchConfig), vp, sz, P(vp),
                                                   sz]),
    "lr_synchronize": (u32, [Device]),
    "lr_kernel_set_resident": (u32, [vp, u32]),
    "lr_kernel_set_overlapped": (u32, [vp, u32]),
    "lr_kernel_max_resident_blocks": (u32, [vp, u32, u32, P(u32)]),
    "lr_queue_native_handle": (u32, [Device, vp, P(vp)]),
    "lr_last_error_detail": (u32, [C.c_char_p, sz]),
}

DRIVER_FUNCTIONS = {
    "lrq_build_program_table": (u32, [u32, u32, P(Task), u32, P(u32), P(Program), u32,
                                      P(u32)]),
    "lrq_rope_tables": (u32, [u32, f32, P(f32), P(f32)]),
    "lrq_model_device_bytes": (u32, [P(ModelConfig), u32, P(u64)]),
    "lrq_model_create": (u32, [Device, vp, sz, P(ModelConfig), P(vp)]),
    "lrq_model_destroy": (u32, [vp]),
    "lrq_model_set_layer": (u32, [vp, u32, P(LayerWeights)]),
    "lrq_model_set_tail": (u32, [vp, vp, vp, vp]),
    "lrq_model_load_layer_bundle": (u32, [vp, u32, cp]),
    "lrq_model_load_tail_bundle": (u32, [vp, cp]),
    "lrq_model_set_kv": (u32, [vp, u32, u32, u32, vp, vp]),
    "lrq_model_replicate_layer": (u32, [vp, u32]),
    "lrq_model_set_hidden": (u32, [vp, vp]),
    "lrq_model_set_hidden_from_token": (u32, [vp, u32]),
    "lrq_decode_launch": (u32, [vp, P(DecodeRequest)]),
    "lrq_decode": (u32, [vp, P(DecodeRequest), P(RunState), P(u32), u32]),
    "lrq_model_read_state": (u32, [vp, P(RunState)]),
    "lrq_model_ingest_prompt": (u32, [vp, P(u32), u32]),
    "lrq_model_enable_prefill": (u32, [vp, vp, sz, u32]),
    "lrq_model_prefill": (u32, [vp, P(u32), u32, u32]),
    "lrq_model_prefill_at": (u32, [vp, P(u32), u32, u32, u32]),
    "lrq_prefill_gemm_check": (u32, [vp, u32, u32, u32, u32, u32, vp, vp, vp, vp]),
    "lrq_batch_create": (u32, [vp, u32, u32, u32, P(vp)]),
    "lrq_batch_destroy": (u32, [vp]),
    "lrq_batch_prefill": (u32, [vp, u32, P(u32), u32, u32]),
    "lrq_batch_decode": (u32, [vp, u32, vp, vp]),
    "lrq_batch_read_cache": (u32, [vp, u32, u32, u32, vp, vp]),
    "lrq_batch_position": (u32, [vp, u32, P(u32)]),
    "lrq_batch_write_cache": (u32, [vp, u32, u32, u32, u32, vp, vp]),
    "lrq_batch_set_next": (u32, [vp, u32, u32, u32]),
    "lrq_generate": (u32, [vp, vp, u32, u32, u32, u32, P(u32), P(RunState)]),
    "lrq_model_read": (u32, [vp, u32, u32, vp, sz]),
    "lrq_model_info": (u32, [vp, P(ModelInfo)]),
    "lrq_model_stage_profile": (u32, [vp, P(u64), P(u64)]),
    "lrq_model_run_graph": (u32, [vp, P(Task), u32, P(Program), u32, u32, u32, u32, u32,
                                  u32, u32, P(RunState)]),
    "lrq_model_set_trace": (u32, [vp, u32]),
    "lrq_model_set_logit_capture": (u32, [vp, u32]),
    "lrq_model_read_trace": (u32, [vp, P(u64), u32]),
    "lrq_last_error": (cp, []),
}

_runtime = None
_driver = None


def _declare(library: C.CDLL, table: dict) -> C.CDLL:
    for name, (restype, argtypes) in table.items():
        function = getattr(library, name)
        function.restype = restype
        function.argtypes = argtypes
    return library


def runtime() -> C.CDLL:
    """The lr_* runtime library (loaded once per process)."""
    global _runtime
    if _runtime is None:
        if not RUNTIME_PATH.exists():
            raise RuntimeError(f"{RUNTIME_PATH} is missing: run light-rocm-runtime_b200/build.py")
        _runtime = _declare(C.CDLL(str(RUNTIME_PATH), mode=C.RTLD_GLOBAL), RUNTIME_FUNCTIONS)
    return _runtime


def driver() -> C.CDLL:
    """The Qwen decode driver library."""
    global _driver
    if _driver is None:
        runtime()
        if not DRIVER_PATH.exists():
            raise RuntimeError(f"{DRIVER_PATH} is missing: run light-rocm-runtime_b200/build.py")
        _driver = _declare(C.CDLL(str(DRIVER_PATH)), DRIVER_FUNCTIONS)
    return _driver


class LrrtError(RuntimeError):
    def __init__(self, status: int, operation: str, detail: str = ""):
        name = runtime().lr_status_string(status).decode()
        super().__init__(f"{operation} failed: {name}" + (f" ({detail})" if detail else ""))
        self.status = status


def check(status: int, operation: str) -> None:
    if status != LR_SUCCESS:
        buffer = C.create_string_buffer(512)
        runtime().lr_last_error_detail(buffer, len(buffer))
        detail = buffer.value.decode(errors="replace")
        if operation.startswith("lrq_"):
            detail = driver().lrq_last_error().decode(errors="replace") or detail
        raise LrrtError(status, operation, detail)
