"""lrq_lm_head_top1_static: the LM-head top-1 whose scratch is a static
device array. It must return exactly the token and logit of the existing
partitioned LM-head path (the sampled token and logit of a decode run on the
same final-normalized vector), on two calls in a row, and reject a grid
larger than its scratch. The test allocates its own input buffers; the entry
point allocates nothing."""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from helpers import build_pair, ingest_prompt
from lrrt_b200 import native as N
from lrrt_b200 import qwen as Q
from lrrt_b200 import synthetic as S

HOST_TO_DEVICE = 0
NO_TOKEN = 0xFFFFFFFF


def _bind():
    driver = N.driver()
    function = driver.lrq_lm_head_top1_static
    function.restype = C.c_uint32
    function.argtypes = [N.Device, C.c_void_p, C.c_void_p, C.c_void_p, C.c_uint32,
                         C.c_uint32, C.c_uint32, C.POINTER(C.c_uint32),
                         C.POINTER(C.c_float)]
    return function


def _upload(device, array: np.ndarray) -> C.c_void_p:
    runtime = N.runtime()
    pointer = C.c_void_p()
    N.check(runtime.lr_malloc(device, array.nbytes, C.byref(pointer)), "lr_malloc")
    N.check(runtime.lr_memcpy(device, pointer, array.ctypes.data, array.nbytes,
                              HOST_TO_DEVICE), "lr_memcpy")
    return pointer


def _device_memory():
    """(free device bytes, the runtime's allocation count)."""
    import torch
    free, _ = torch.cuda.mem_get_info(0)
    stats = N.MemoryStats()
    N.check(N.runtime().lr_get_memory_stats(N.Device(0), C.byref(stats)),
            "lr_get_memory_stats")
    return free, stats.allocation_count


@pytest.mark.gpu
def test_static_top1_matches_partitioned_lm_head_on_two_calls(gpu):
    vocab = 8192
    model, oracle, _, tail = build_pair(seed=11, layers=2, vocab=vocab, capacity=24,
                                        max_tokens=4)
    prompt = S.prompt(11, 6, vocab)
    ingest_prompt(model, oracle, prompt)
    # The existing path: a one-token decode through the host-driven tasks
    # (lm_head_top1_partition + top1_reduce into allocated partial buffers).
    state, tokens = model.decode(len(prompt) - 1, 1, path=Q.PATH_HOST_STEP)
    # Host-driven kernels publish no status; the run is checked by its
    # predicate, error code and token as the GPU parity tests do.
    assert state.predicate_value == 1 and state.error_code == 0
    assert tokens.tolist() == [state.sampled_token]
    # ... which itself agrees with the CPU oracle's run of the same step.
    oracle.decode(oracle.embedding(int(prompt[-1])), len(prompt) - 1, 1)
    assert state.sampled_token == oracle.decode_state.sampled_token
    assert abs(state.sampled_logit - oracle.decode_state.sampled_logit) <= \
        1.0e-4 * max(1.0, abs(oracle.decode_state.sampled_logit))
    normalized = model.read("final_normalized").astype(np.float32)
    lm_head = np.ascontiguousarray(tail["lm_head"], dtype=np.float32)
    top1 = _bind()
    runtime = N.runtime()
    device = model.device
    lm_head_device = _upload(device, lm_head)
    hidden_device = _upload(device, normalized)
    try:
        for call in range(2):
            before = _device_memory() if call == 1 else None
            token = C.c_uint32(NO_TOKEN)
            logit = C.c_float(float("nan"))
            N.check(top1(device, None, lm_head_device, hidden_device, vocab, 896, 0,
                         C.byref(token), C.byref(logit)), "lrq_lm_head_top1_static")
            assert token.value == state.sampled_token, (call, token.value)
            assert np.float32(logit.value).tobytes() == np.float32(state.sampled_logit).tobytes(), \
                (call, logit.value, state.sampled_logit)
            if before is not None:
                # The second call (set-up done) changes neither the device's
                # free memory nor the runtime's allocation count.
                assert _device_memory() == before
        # A grid larger than the static scratch is refused with a message.
        token = C.c_uint32(0)
        logit = C.c_float(0.0)
        status = top1(device, None, lm_head_device, hidden_device, vocab, 896, 1025,
                      C.byref(token), C.byref(logit))
        assert status == N.LR_ERROR_INVALID_ARGUMENT
        message = N.driver().lrq_last_error().decode()
        assert "1025 blocks" in message and "1024" in message, message
        # Still correct after the refusal, with an explicit grid.
        N.check(top1(device, None, lm_head_device, hidden_device, vocab, 896, 37,
                     C.byref(token), C.byref(logit)), "lrq_lm_head_top1_static")
        assert token.value == state.sampled_token
        # On a queue the caller created; and 256 rows over 1024 blocks, so
        # most blocks own no row and publish an empty candidate.
        queue = C.c_void_p()
        N.check(runtime.lr_queue_create(device, C.byref(queue)), "lr_queue_create")
        try:
            rows = 256
            N.check(top1(device, queue, lm_head_device, hidden_device, rows, 896, 1024,
                         C.byref(token), C.byref(logit)), "lrq_lm_head_top1_static")
        finally:
            runtime.lr_queue_destroy(queue)
        scores = lm_head[:rows].astype(np.float64) @ normalized.astype(np.float64)
        assert token.value == int(np.argmax(scores))
        assert abs(logit.value - scores[token.value]) <= 1.0e-4 * max(1.0, abs(scores[token.value]))
    finally:
        runtime.lr_free(device, lm_head_device)
        runtime.lr_free(device, hidden_device)
        model.close()
