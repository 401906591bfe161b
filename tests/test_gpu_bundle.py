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
