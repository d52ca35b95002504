"""The drop-ins for the reference's operator layer and engine: the
reference's own hip/ops.hpp compiled with include/lfm3_gpu_ops.inl
(hipStream_t mapped to cudaStream_t by tests/shim/hip/hip_runtime.h), and
its engine.hpp with include/lfm3_engine.inl (plus its weights.cpp and
config.cpp), each linked against liblfm3_cuda.so. The link proves every
function and member those headers declare has a definition of exactly its
signature; the programs then check what needs no GPU. CPU only; skipped
where the reference tree is absent."""
import os
import shutil
import subprocess

import pytest

from helpers import ROOT, lfm3



def _reference_tree():
    """The reference tree the oracle's Makefile builds from (its REFERENCE
    variable: the environment's, else its default)."""
    import subprocess
    out = subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "oracle"),
                          "print-reference"], capture_output=True, text=True)
    return out.stdout.strip()


REFERENCE = _reference_tree()


def test_reference_ops_header_links_against_library(tmp_path):
    if not os.path.exists(os.path.join(REFERENCE, "hip", "ops.hpp")):
        pytest.skip("reference tree absent")
    if not shutil.which("g++"):
        pytest.skip("no g++")
    lib_dir = os.path.dirname(lfm3.abi.LIBRARY)
    lfm3.library()  # the library is built
    exe = str(tmp_path / "ops_shim_check")
    cmd = ["g++", "-std=c++20", "-Wall", "-Wextra", "-Wno-unused-parameter",
           "-I", os.path.join(ROOT, "tests", "shim"),
           "-I", os.path.join(ROOT, "oracle", "stubs"),
           "-I", REFERENCE, "-I", os.path.join(ROOT, "include"),
           "-I", "/usr/local/cuda/include",
           os.path.join(ROOT, "tests", "shim", "ops_shim_check.cpp"),
           "-L", lib_dir, "-llfm3_cuda", "-Wl,-rpath," + lib_dir,
           "-Wl,--allow-shlib-undefined", "-o", exe]
    build = subprocess.run(cmd, capture_output=True, text=True)
    assert build.returncode == 0, build.stdout + build.stderr
    run = subprocess.run([exe], capture_output=True, text=True, timeout=60)
    assert run.returncode == 0, run.stdout + run.stderr
    assert "missing 0 failures 0" in run.stdout


def test_reference_engine_header_links_against_library(tmp_path):
    if not os.path.exists(os.path.join(REFERENCE, "engine.hpp")):
        pytest.skip("reference tree absent")
    if not shutil.which("g++"):
        pytest.skip("no g++")
    lib_dir = os.path.dirname(lfm3.abi.LIBRARY)
    lfm3.library()
    exe = str(tmp_path / "engine_shim_check")
    cmd = ["g++", "-std=c++20", "-Wall", "-Wextra", "-Wno-unused-parameter",
           "-I", os.path.join(ROOT, "oracle", "stubs"),
           "-I", REFERENCE, "-I", os.path.join(ROOT, "include"),
           os.path.join(ROOT, "tests", "shim", "engine_shim_check.cpp"),
           os.path.join(REFERENCE, "weights.cpp"),
           os.path.join(REFERENCE, "config.cpp"),
           "-L", lib_dir, "-llfm3_cuda", "-Wl,-rpath," + lib_dir,
           "-Wl,--allow-shlib-undefined", "-o", exe]
    build = subprocess.run(cmd, capture_output=True, text=True)
    assert build.returncode == 0, build.stdout + build.stderr
    run = subprocess.run([exe], capture_output=True, text=True, timeout=60)
    assert run.returncode == 0, run.stdout + run.stderr
    assert "failures 0" in run.stdout
