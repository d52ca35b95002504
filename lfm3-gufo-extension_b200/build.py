"""Builds lib/liblfm3_cuda.so for sm_100a: every kernel, the host engine, the
C ABI and the synthetic-weight generator, compiled in-tree with nvcc
(relocatable device code, one device link) so the library travels with the
repository.

    python build.py            # incremental
    python build.py --clean    # rebuild everything
"""
import argparse
import concurrent.futures
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "lib", "liblfm3_cuda.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CUDA_FLAGS = ARCH + [
    "-std=c++20", "-O3", "-lineinfo", "-rdc=true", "-Xcompiler", "-fPIC",
    "-Xcompiler", "-Wall", "-diag-suppress", "20044", "-I", INCLUDE,
    "--expt-relaxed-constexpr",
]
SOURCES = [
    "abi.cu", "attention_decode.cu", "attention_prompt.cu",
    "attention_prompt_tc.cu", "conv.cu",
    "device_error.cu", "engine.cpp", "noalloc.cu", "norm.cu", "q8_decode.cu",
    "q8_gemv.cu",
    "q8_prefill.cu", "sampling.cu", "scheduler.cpp",
    "tensor_map.cpp",
]
HOST_C = ["host/synth.c"]


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _headers():
    out = []
    for root in (CSRC, INCLUDE):
        for dirpath, _, files in os.walk(root):
            out += [os.path.join(dirpath, f) for f in files
                    if f.endswith((".cuh", ".hpp", ".h"))]
    return out


def _run(cmd):
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(" ".join(cmd) + "\n" + proc.stdout + proc.stderr)
    return proc.stdout + proc.stderr


def build(clean=False, verbose=False, jobs=None):
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(os.path.dirname(LIB), exist_ok=True)
    headers = _headers()
    objects, commands = [], []
    for src in SOURCES:
        path = os.path.join(CSRC, src)
        obj = os.path.join(BUILD, src.replace("/", "_") + ".o")
        objects.append(obj)
        if clean or _stale(obj, [path] + headers):
            lang = ["-x", "cu"] if src.endswith(".cpp") else []
            commands.append([NVCC] + CUDA_FLAGS + lang + ["-c", path, "-o", obj])
    for src in HOST_C:
        path = os.path.join(CSRC, src)
        obj = os.path.join(BUILD, os.path.basename(src) + ".o")
        objects.append(obj)
        if clean or _stale(obj, [path] + headers):
            commands.append(["gcc", "-std=c11", "-O2", "-fPIC", "-Wall",
                             "-pthread", "-I", INCLUDE, "-c", path, "-o", obj])
    with concurrent.futures.ThreadPoolExecutor(jobs or os.cpu_count()) as pool:
        for out in pool.map(_run, commands):
            if verbose and out.strip():
                print(out)
    if clean or commands or not os.path.exists(LIB):
        dlink = os.path.join(BUILD, "dlink.o")
        cu_objects = [o for o in objects if not o.endswith("synth.c.o")]
        _run([NVCC] + ARCH + ["-Xcompiler", "-fPIC", "-dlink"] + cu_objects +
             ["-o", dlink])
        _run([NVCC] + ARCH + ["-shared", "-Xcompiler", "-fPIC"] + objects +
             [dlink, "-o", LIB, "-lcudart", "-lpthread", "-lm"])
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--clean", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    args = ap.parse_args()
    try:
        print(build(args.clean, args.verbose))
    except RuntimeError as e:
        print(e, file=sys.stderr)
        sys.exit(1)
