"""In-tree build of the native libraries (no JIT cache: the .so files travel
with the source tree).

    python -m huggingfaceeacp_b200.build          # product libraries
    python -m huggingfaceeacp_b200.build --all    # plus the test oracle

libhf_cuda.so : csrc/hf_cuda.cu for sm_100a (nvcc -gencode arch=compute_100a,code=sm_100a)
libhf_host.so : host/int8_blocks.cpp + host/synthetic.cpp (F16C, pthreads)
libhf.so      : host/hf_decoder.cpp, the C++ HF:: surface over the two above
"""
from __future__ import annotations

import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
LIB = os.path.join(PKG, "lib")
INCLUDE = os.path.join(ROOT, "include")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _run(cmd):
    print("+", " ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)


def _stale(target, sources):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(s) > t for s in sources)


def build_host(force=False):
    os.makedirs(LIB, exist_ok=True)
    sources = [os.path.join(PKG, "host", f) for f in ("int8_blocks.cpp", "synthetic.cpp", "safetensors.cpp")]
    target = os.path.join(LIB, "libhf_host.so")
    if force or _stale(target, sources + [os.path.join(INCLUDE, "hf_host.h"), os.path.join(PKG, "host", "safetensors.h")]):
        _run(["g++", "-std=c++17", "-O3", "-mf16c", "-fPIC", "-shared", "-pthread", f"-I{INCLUDE}", *sources,
              "-o", target])
    return target


def build_cuda(force=False):
    os.makedirs(LIB, exist_ok=True)
    csrc = os.path.join(PKG, "csrc")
    sources = [os.path.join(csrc, f) for f in os.listdir(csrc) if f.endswith((".cu", ".cuh"))]
    target = os.path.join(LIB, "libhf_cuda.so")
    if force or _stale(target, sources + [os.path.join(INCLUDE, "hf_cuda.h"), os.path.join(PKG, "host", "safetensors.h")]):
        _run([NVCC, *ARCH, "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC", "-shared", f"-I{INCLUDE}",
              os.path.join(csrc, "hf_cuda.cu"), "-o", target])
    return target


def build_cpp_surface(force=False):
    source = os.path.join(PKG, "host", "hf_decoder.cpp")
    if not os.path.exists(source):
        return None
    target = os.path.join(LIB, "libhf.so")
    headers = [os.path.join(INCLUDE, "HF", f) for f in os.listdir(os.path.join(INCLUDE, "HF"))] if os.path.isdir(
        os.path.join(INCLUDE, "HF")) else []
    if force or _stale(target, [source, os.path.join(PKG, "host", "safetensors.h"), *headers]):
        _run(["g++", "-std=c++20", "-O2", "-fPIC", "-shared", f"-I{INCLUDE}", source, f"-L{LIB}", "-lhf_cuda",
              "-lhf_host", "-Wl,-rpath,$ORIGIN", "-o", target])
    return target


def reference_root():
    """The reference project's checkout that oracle/build_ref.sh compiles from:
    $HF_REFERENCE_ROOT, else a directory named `reference` beside this
    repository, else None."""
    root = os.environ.get("HF_REFERENCE_ROOT") or os.path.join(os.path.dirname(ROOT), "reference")
    return root if os.path.isdir(os.path.join(root, "Lib", "HuggingFaceEACP")) else None


def build_oracle():
    """Test infrastructure: the C oracle, and oracle/_ref when the reference tree is present."""
    _run(["sh", os.path.join(ROOT, "oracle", "build.sh")])
    ref = reference_root()
    if ref:
        _run(["sh", os.path.join(ROOT, "oracle", "build_ref.sh"), ref])


def build(force=False, oracle=True):
    build_host(force)
    build_cuda(force)
    build_cpp_surface(force)
    if oracle:
        build_oracle()


if __name__ == "__main__":
    build(force="--force" in sys.argv, oracle="--all" in sys.argv)
