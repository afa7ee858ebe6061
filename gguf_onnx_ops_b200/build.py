"""Build libgguf_onnx_ops.so in-tree for sm_100a (nvcc, static CUDA runtime).

    python -m gguf_onnx_ops_b200.build            # or: python gguf_onnx_ops_b200/build.py

Output: gguf_onnx_ops_b200/lib/libgguf_onnx_ops.so (+ libbolt_ops.so symlink, the reference's
library name, CMakeLists.txt:18-20).  When ORT_INCLUDE_DIR names a directory holding
onnxruntime_c_api.h, the ONNX Runtime custom-op shim (csrc/ort_ops.cc, exporting
RegisterCustomOps) is compiled into the same library, as the reference's CMakeLists.txt:4-7
requires; otherwise the library exports the C ABI of include/gguf_ops.h only.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIBDIR = os.path.join(HERE, "lib")
LIB = os.path.join(LIBDIR, "libgguf_onnx_ops.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC,-fvisibility=hidden",
              "-Xptxas", "-warn-spills"]


def nvcc() -> str:
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found")


def sources() -> list[str]:
    return [os.path.join(CSRC, f) for f in sorted(os.listdir(CSRC)) if f.endswith((".cu", ".cuh", ".h", ".cc"))] + [
        os.path.join(ROOT, "include", "gguf_ops.h")]


def up_to_date() -> bool:
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    return all(os.path.getmtime(s) <= t for s in sources())


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and up_to_date():
        return LIB
    os.makedirs(LIBDIR, exist_ok=True)
    objs = []
    tmp = os.path.join(LIBDIR, "_obj")
    os.makedirs(tmp, exist_ok=True)
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, "-I", os.path.join(ROOT, "include"), "-c", os.path.join(CSRC, "gguf_ops.cu"),
           "-o", os.path.join(tmp, "gguf_ops.o")]
    if verbose:
        cmd += ["-Xptxas", "-v"]
    subprocess.run(cmd, check=True)
    objs.append(os.path.join(tmp, "gguf_ops.o"))
    host_flags = ["-O2", "-std=c++17", "-fPIC", "-fvisibility=hidden", "-pthread", "-Wall", "-I",
                  os.path.join(ROOT, "include"), "-I", os.path.join(os.path.dirname(os.path.dirname(nvcc())), "include")]
    subprocess.run(["g++", *host_flags, "-c", os.path.join(CSRC, "gguf_file.cc"), "-o", os.path.join(tmp, "gguf_file.o")],
                   check=True)
    objs.append(os.path.join(tmp, "gguf_file.o"))
    ort_inc = os.environ.get("ORT_INCLUDE_DIR", "")
    if ort_inc and os.path.exists(os.path.join(ort_inc, "onnxruntime_c_api.h")):
        cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-fvisibility=hidden", "-I", ort_inc, "-I", os.path.join(ROOT, "include"),
               "-I", "/usr/local/cuda/include", "-c", os.path.join(CSRC, "ort_ops.cc"), "-o", os.path.join(tmp, "ort_ops.o")]
        subprocess.run(cmd, check=True)
        objs.append(os.path.join(tmp, "ort_ops.o"))
    out_tmp = LIB + ".tmp"
    subprocess.run([nvcc(), *ARCH, "-shared", "-o", out_tmp, *objs, "-lrt", "-lpthread", "-ldl"], check=True)
    os.replace(out_tmp, LIB)
    link = os.path.join(LIBDIR, "libbolt_ops.so")
    if os.path.lexists(link):
        os.remove(link)
    os.symlink("libgguf_onnx_ops.so", link)
    shutil.rmtree(tmp, ignore_errors=True)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
