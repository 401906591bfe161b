"""lrrt::Bundle on a B200: loads the test bundle (manifest + sm_100a cubin),
packs kernargs and launches through every Bundle::launch overload."""
import subprocess

import pytest


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
