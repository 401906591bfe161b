import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
for path in (REPO / "light-rocm-runtime_b200", REPO / "oracle", REPO / "tests"):
    if str(path) not in sys.path:
        sys.path.insert(0, str(path))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an NVIDIA B200 (sm_100a)")


@pytest.fixture(scope="session")
def built():
    """Native libraries, cubins, C++ test programs and the CPU oracle."""
    import build
    outputs = build.build()
    outputs["oracle"] = build.build_oracle()
    return outputs


@pytest.fixture(scope="session")
def gpu(built):
    """The first B200; a GPU test fails (never skips) when none is visible."""
    from lrrt_b200.qwen import Runtime
    count = Runtime.device_count()
    assert count > 0, "GPU test ran without a visible CUDA device"
    return 0
