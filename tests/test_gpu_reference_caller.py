"""A reference-style caller on a B200 (tests/cpp/reference_caller_test.cpp):
Context / TailContext arrays built by the caller and launched through
ResidentExecutor, as the reference driver does, with the workspace from
lrq_workspace_init and the fused path's dynamic shared memory. The run must
take the fused path and produce the oracle's greedy tokens."""
import subprocess

import numpy as np
import pytest

import oracle as O
from lrrt_b200 import native as N
from lrrt_b200 import synthetic as S


@pytest.mark.gpu
def test_reference_built_contexts_take_the_fused_path(gpu, built, tmp_path):
    layers, vocab, position, tokens = 2, 4096, 5, 12
    weights, tail = S.model(17, layers, vocab)
    hidden = S.hidden(17)
    np.array([layers, vocab, position, tokens], np.uint32).tofile(tmp_path / "meta")
    for i, layer in enumerate(weights):
        for name, array in layer.items():
            np.ascontiguousarray(array, np.float32).tofile(tmp_path / f"l{i}_{name}")
    np.ascontiguousarray(tail["lm_head"], np.float32).tofile(tmp_path / "lm_head")
    np.ascontiguousarray(tail["final_norm"], np.float32).tofile(tmp_path / "final_norm")
    hidden.astype(np.float32).tofile(tmp_path / "hidden")
    result = subprocess.run([str(built["test:reference_caller_test"]), str(N.QWEN_CUBIN),
                             str(tmp_path)], capture_output=True, text=True, timeout=300)
    assert result.returncode == 0, result.stderr + result.stdout
    status, error, path, sampled = np.fromfile(tmp_path / "result", np.uint32).tolist()
    assert (status, error) == (2, 0), result.stdout
    assert path == 1, "reference-built contexts did not take the fused sm_100a path"
    capacity = position + tokens + 8
    partitions = min(vocab, 32, 148)
    reference = O.OracleModel(weights, tail, capacity, partitions, workers=148, max_tokens=tokens)
    reference.decode(hidden, position, tokens)
    got = np.fromfile(tmp_path / "tokens", np.uint32)
    assert got.tolist() == reference.output_tokens[:tokens].tolist()
    assert sampled == reference.decode_state.sampled_token
