"""lrrt::Bundle on a B200: loads the test bundle (manifest + sm_100a cubin),
packs kernargs and launches through every Bundle::launch overload."""
import subprocess

import numpy as np
import pytest

import oracle as O
from helpers import max_relative_error
from lrrt_b200 import synthetic as S


@pytest.mark.gpu
def test_bundle_launches_on_device(gpu, built):
    binary = built["test:bundle_device_test"]
    result = subprocess.run([str(binary), str(built["bundle_manifest"])], capture_output=True,
                            text=True, timeout=120)
    assert result.returncode == 0, result.stderr + result.stdout
    assert "bundle device checks: ok" in result.stdout


@pytest.mark.gpu
def test_executor_decode_layer_on_device(gpu, built):
    """Generic bundle executor (BundleSet, arena BufferSet, named launch
    arguments, the reference's error texts) and one Qwen2 layer's decode step
    composed from per-operation bundles, against double precision."""
    binary = built["test:decode_layer_test"]
    result = subprocess.run([str(binary), str(built["decoder_ops_manifest"])],
                            capture_output=True, text=True, timeout=300)
    assert result.returncode == 0, result.stderr + result.stdout
    assert "decode layer checks: ok" in result.stdout
    print(result.stdout)


@pytest.mark.gpu
def test_executor_decode_layer_matches_oracle(gpu, built, tmp_path):
    """The same per-operation decode layer on BASELINE config 1's seeded
    inputs (weights of synthetic.model(0, 1, ...), KV rows 0..127 and hidden
    of seed 0), against the CPU oracle's decode step of that layer: layer
    output and the appended (rotated) key row within 1e-4."""
    weights, tail = S.model(0, 1, 64)
    layer = weights[0]
    keys, values = S.kv_prefill(0, 1, 128)[0]
    hidden = S.hidden(0)
    for name, array in list(layer.items()) + [("cache_keys", keys), ("cache_values", values),
                                               ("hidden", hidden)]:
        np.ascontiguousarray(array, np.float32).tofile(tmp_path / name)
    result = subprocess.run([str(built["test:decode_layer_test"]),
                             str(built["decoder_ops_manifest"]), str(tmp_path)],
                            capture_output=True, text=True, timeout=300)
    assert result.returncode == 0, result.stderr + result.stdout
    oracle = O.OracleModel(weights, tail, 256, 4, workers=148, max_tokens=1)
    oracle.set_kv(0, 0, keys, values)
    oracle.decode(hidden, 128, 1)
    out = np.fromfile(tmp_path / "out.f32", np.float32)
    key = np.fromfile(tmp_path / "key.f32", np.float32)
    assert max_relative_error(out, oracle.hidden) <= 1.0e-4
    assert max_relative_error(key, oracle.key_cache[0][128]) <= 1.0e-4
