"""CPU tests of the host side: the C ABI libraries load and export every
declared entry point, the decode graph and RoPE tables match the reference
restatement, and the C++ host checks pass."""
import ctypes as C
import re
import subprocess
from pathlib import Path

import numpy as np

import oracle as O
from lrrt_b200 import native as N
from lrrt_b200 import qwen as Q

REPO = Path(__file__).resolve().parents[1]


def declared(header: Path):
    text = header.read_text()
    return sorted(set(re.findall(r"LRRT_API\s+[\w\s\*]+?\b(l[rq]{1,2}_\w+)\s*\(", text)))


def test_runtime_library_exports_every_declared_symbol(built):
    library = N.runtime()
    names = declared(REPO / "include" / "lrrt" / "lrrt.h")
    assert len(names) == 40  # 35 reference entry points + 5 B200 additions
    for name in names:
        assert hasattr(library, name), name


def test_driver_library_exports_every_declared_symbol(built):
    library = N.driver()
    names = declared(REPO / "include" / "lrrt_qwen.h")
    assert len(names) >= 20
    for name in names:
        assert hasattr(library, name), name


def test_abi_struct_sizes():
    assert C.sizeof(N.Task) == 32 and C.sizeof(N.Program) == 32
    assert C.sizeof(O.State) == 64
    assert C.sizeof(N.LaunchConfig) == 28
    assert C.sizeof(N.MemoryStats) == 128


def test_cpp_resident_executor_checks(built):
    binary = built["test:resident_executor_test"]
    result = subprocess.run([str(binary)], capture_output=True, text=True, timeout=60)
    assert result.returncode == 0, result.stderr
    assert "ok" in result.stdout


def test_cpp_runtime_api_contract(built):
    binary = built["test:runtime_api_test"]
    result = subprocess.run([str(binary)], capture_output=True, text=True, timeout=120)
    assert result.returncode == 0, result.stderr + result.stdout
    assert "runtime api: ok" in result.stdout


def test_program_table_matches_reference_restatement(built):
    for vocab, partitions in ((151936, 32), (4096, 20), (64, 4), (3, 1)):
        tasks, programs = Q.program_table(vocab, partitions)
        want_tasks, want_programs = O.make_program_table(vocab, partitions)
        got_tasks = [tuple(getattr(t, f) for f, _ in N.Task._fields_) for t in tasks]
        assert got_tasks == [tuple(t) for t in want_tasks]
        got_programs = [(p.task_offset, p.task_count, p.next_program, p.flags,
                         p.branch_program) for p in programs]
        assert got_programs == [tuple(p) for p in want_programs]
    assert len(tasks) == 79 + 1 + 3


def test_program_table_rejects_bad_partitioning(built):
    for vocab, partitions in ((0, 1), (64, 0), (64, 33), (4, 8)):
        tasks = (N.Task * 128)()
        programs = (N.Program * 4)()
        n, m = C.c_uint32(), C.c_uint32()
        status = N.driver().lrq_build_program_table(vocab, partitions, tasks, 128, C.byref(n),
                                                    programs, 4, C.byref(m))
        assert status == N.LR_ERROR_INVALID_ARGUMENT


def test_rope_tables_match_reference_arithmetic(built):
    cos, sin = Q.rope_tables(4352, 1.0e6)
    want_cos, want_sin = O.rope_tables(4352, 1.0e6)
    assert np.array_equal(cos, want_cos) and np.array_equal(sin, want_sin)


def test_runtime_without_devices_reports_zero(built):
    # On a GPU-less host lr_init succeeds and reports no devices; on a GPU box
    # this still passes (count > 0).
    assert Q.Runtime.device_count() >= 0


def test_cpp_resident_schedule_checks(built):
    """Fused-path partition and weight-stream order (producer == consumer)."""
    binary = built["test:resident_schedule_test"]
    result = subprocess.run([str(binary)], capture_output=True, text=True, timeout=300)
    assert result.returncode == 0, result.stderr
    assert "ok" in result.stdout


def test_cpp_bundle_checks(built):
    """lrrt::bundle manifest parsing, launch configuration and kernarg packing
    with the reference's error texts (no device needed)."""
    binary = built["test:bundle_test"]
    result = subprocess.run([str(binary)], capture_output=True, text=True, timeout=60)
    assert result.returncode == 0, result.stderr
    assert "bundle checks: ok" in result.stdout


def test_cpp_weight_bundle_checks(built, tmp_path):
    """FP32 weight bundles: the fixture written by the reference's converter
    loads, our writer round-trips, malformed manifests fail with the
    reference's messages."""
    binary = built["test:weight_bundle_test"]
    fixture = Path(__file__).parent / "golden" / "weight_bundles"
    result = subprocess.run([str(binary), str(fixture), str(tmp_path)], capture_output=True,
                            text=True, timeout=60)
    assert result.returncode == 0, result.stderr
    assert "weight bundle checks: ok" in result.stdout
