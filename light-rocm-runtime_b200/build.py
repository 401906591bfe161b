"""Builds every native artefact of the package in-tree.

Outputs (git-ignored, shipped with the working tree):
  lib/liblrrt.so                  lr_* C ABI over the CUDA driver API
  lib/liblrrt_qwen.so             Qwen decode driver (include/lrrt_qwen.h)
  lib/qwen_stateful_graph.cubin   sm_100a decode megakernels
  lib/qwen_prefill.cubin          sm_100a prompt prefill kernels
  lib/decoder_ops.cubin + .json   per-operation decode kernels as an lrrt::bundle
  _build/tests/stateful_graph_fixture.cubin  sm_100a scheduler fixture kernels (tests)
  _build/tests/*                  C++ host tests (tests/cpp)

Rebuilds a target only when one of its inputs is newer than it.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
REPO = PACKAGE.parent
INCLUDE = REPO / "include"
LIB = PACKAGE / "lib"
BUILD = PACKAGE / "_build"
CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
NVCC = str(CUDA_HOME / "bin" / "nvcc")
CXX = shutil.which("g++") or "g++"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CXXFLAGS = ["-std=c++17", "-O2", "-fPIC", "-Wall", "-Wextra", f"-I{INCLUDE}",
            f"-I{CUDA_HOME / 'include'}"]
NVCCFLAGS = ["-std=c++17", "-O3", *ARCH, "-lineinfo", f"-I{INCLUDE}"]


def _headers() -> list[Path]:
    return (sorted(INCLUDE.rglob("*.h*")) + sorted(INCLUDE.rglob("*.cuh")) +
            sorted((PACKAGE / "csrc" / "common").glob("*.hpp")))


def _stale(target: Path, inputs: list[Path]) -> bool:
    if not target.exists():
        return True
    stamp = target.stat().st_mtime
    return any(path.stat().st_mtime > stamp for path in inputs)


def _run(command: list[str], verbose: bool) -> None:
    if verbose:
        print("+", " ".join(command), flush=True)
    subprocess.run(command, check=True)


def build(verbose: bool = False) -> dict[str, Path]:
    LIB.mkdir(exist_ok=True)
    BUILD.mkdir(exist_ok=True)
    headers = _headers()
    csrc = PACKAGE / "csrc"
    outputs: dict[str, Path] = {}

    runtime = LIB / "liblrrt.so"
    runtime_sources = sorted((csrc / "runtime").glob("*.cpp"))
    runtime_inputs = runtime_sources + sorted((csrc / "runtime").glob("*.hpp")) + headers
    if _stale(runtime, runtime_inputs):
        _run([CXX, *CXXFLAGS, "-shared", "-fvisibility=hidden",
              *map(str, runtime_sources), "-o", str(runtime), "-ldl"], verbose)
    outputs["runtime"] = runtime

    driver = LIB / "liblrrt_qwen.so"
    driver_sources = sorted((csrc / "qwen").glob("*.cpp"))
    driver_headers = sorted((csrc / "qwen").glob("*.hpp"))
    # CUDA runtime code of the driver (the static-scratch LM-head top-1),
    # compiled to an object and linked with the static CUDA runtime.
    static_top1 = csrc / "qwen" / "lm_head_top1_static.cu"
    static_top1_object = BUILD / "lm_head_top1_static.o"
    static_inputs = [static_top1, csrc / "qwen" / "lm_head_top1_static.hpp"] + headers
    if _stale(static_top1_object, static_inputs):
        _run([NVCC, *NVCCFLAGS, "-c", "-Xcompiler", "-fPIC,-fvisibility=hidden",
              str(static_top1), "-o", str(static_top1_object)], verbose)
    if _stale(driver, driver_sources + driver_headers + static_inputs +
              [static_top1_object, runtime]):
        _run([CXX, *CXXFLAGS, "-shared", "-fvisibility=hidden",
              *map(str, driver_sources), str(static_top1_object), "-o", str(driver),
              f"-L{LIB}", "-llrrt", f"-L{CUDA_HOME / 'lib64'}", "-lcudart_static",
              "-lrt", "-ldl", "-lpthread", "-Wl,-rpath,$ORIGIN"], verbose)
    outputs["driver"] = driver

    for name in ("qwen_stateful_graph", "qwen_prefill", "decoder_ops"):
        source = csrc / "kernels" / f"{name}.cu"
        cubin = LIB / f"{name}.cubin"
        if _stale(cubin, [source] + headers):
            _run([NVCC, *NVCCFLAGS, "-cubin", str(source), "-o", str(cubin)], verbose)
        outputs[name] = cubin
    # Per-operation decode kernels as a bundle: manifest next to its cubin.
    ops_manifest = LIB / "decoder_ops.json"
    shutil.copyfile(csrc / "kernels" / "decoder_ops.json", ops_manifest)
    outputs["decoder_ops_manifest"] = ops_manifest

    tests_dir = REPO / "tests" / "cpp"
    test_build = BUILD / "tests"
    test_build.mkdir(exist_ok=True)
    # Scheduler fixture kernels (test infrastructure: the reference test's
    # synthetic workload, replayed on both schedulers against its goldens).
    fixture_source = tests_dir / "stateful_graph_fixture.cu"
    fixture = test_build / "stateful_graph_fixture.cubin"
    if _stale(fixture, [fixture_source] + headers):
        _run([NVCC, *NVCCFLAGS, "-cubin", str(fixture_source), "-o", str(fixture)], verbose)
    outputs["stateful_graph_fixture"] = fixture
    # Test bundle for lrrt::Bundle: manifest + sm_100a cubin side by side.
    bundle_dir = test_build / "bundle"
    bundle_dir.mkdir(exist_ok=True)
    bundle_cubin = bundle_dir / "bundle_kernels.cubin"
    if _stale(bundle_cubin, [tests_dir / "bundle_kernels.cu"]):
        _run([NVCC, *NVCCFLAGS, "-cubin", str(tests_dir / "bundle_kernels.cu"), "-o",
              str(bundle_cubin)], verbose)
    bundle_manifest = bundle_dir / "manifest.json"
    shutil.copyfile(tests_dir / "bundle_manifest.json", bundle_manifest)
    outputs["bundle_manifest"] = bundle_manifest
    for source in sorted(tests_dir.glob("*.cpp")):
        binary = test_build / source.stem
        if _stale(binary, [source] + headers + [runtime, driver]):
            _run([CXX, *CXXFLAGS, str(source), "-o", str(binary), f"-L{LIB}", "-llrrt_qwen",
                  "-llrrt", "-Wl,-rpath,$ORIGIN/../../lib"], verbose)
        outputs[f"test:{source.stem}"] = binary
    return outputs


def build_oracle(verbose: bool = False) -> Path:
    """Compiles the CPU oracle (test infrastructure) with its own Makefile."""
    oracle = REPO / "oracle"
    _run(["make", "-s", "-C", str(oracle)], verbose)
    return oracle / "_build" / "liblrrt_oracle.so"


if __name__ == "__main__":
    for key, path in build(verbose="-v" in sys.argv).items():
        print(f"{key}: {path}")
    print("oracle:", build_oracle(verbose="-v" in sys.argv))
