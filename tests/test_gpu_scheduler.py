"""Both resident schedulers on the B200 against the reference's scheduler
fixture goldens (tests/stateful_graph_device.cpp:103-176 of the reference)."""
import json
import subprocess
from pathlib import Path

import pytest

from lrrt_b200 import native as N

GOLDEN = json.loads((Path(__file__).parent / "golden" / "scheduler_fixture.json").read_text())


@pytest.mark.gpu
def test_fixture_on_both_schedulers(gpu, built):
    binary = built["test:stateful_graph_device_test"]
    result = subprocess.run([str(binary), str(N.FIXTURE_CUBIN)], capture_output=True,
                            text=True, timeout=120)
    assert result.returncode == 0, result.stderr
    observed = json.loads(result.stdout)
    assert "skipped" not in observed
    for path in ("dynamic", "compiled"):
        runs = observed[path]
        assert len(runs) == 3
        for run, calls in zip(runs, GOLDEN["expected_validation_calls_per_run"]):
            for key, want in GOLDEN["expected_state"].items():
                assert run[key] == want, (path, key, run)
            assert run["values"] == GOLDEN["expected_values"], path
            assert run["checksums"] == GOLDEN["expected_checksums"], path
            assert run["branch_steps"] == GOLDEN["expected_branch_steps"], path
            assert run["task_executions"] == GOLDEN["expected_task_executions"], path
            assert run["validation_calls"] == calls, (path, run["validation_calls"])
