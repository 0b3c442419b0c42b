"""Builds the B200 backend in-tree: kraken-infer_b200/lib/libkib.so (sm_100a),
and lib/libkib_gguf.so, the host-only GGUF tools (synthetic model writer and
K-quant quantisers, no device code) for processes that must not map the CUDA
backend.

Usage: python kraken-infer_b200/build.py [--force]
The CUDA sources are compiled with nvcc for sm_100a only; the host C++ (GGUF
reader/writer) with the same nvcc invocation.  Output stays in the source tree
so it travels with the repository snapshot.
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB_DIR = os.path.join(HERE, "lib")
LIB = os.path.join(LIB_DIR, "libkib.so")
SOURCES = ["ops.cu", "ops_seam.cu", "engine.cu", "noalloc.cu", "gguf.cpp", "gguf_tools.cpp", "prefix_cache.cpp", "tokenizer.cpp"]
TOOLS_LIB = os.path.join(LIB_DIR, "libkib_gguf.so")
TOOLS_SOURCES = ["gguf.cpp", "gguf_tools.cpp", "prefix_cache.cpp", "tokenizer.cpp"]
HEADERS = ["tokenizer.hpp", "prefix_cache.hpp", "kq_skinny.cuh", "batch_kernels.cuh", "gdn_chunk.cuh", "gemm_tc.cuh", "kib_common.cuh", "kquant.cuh", "kquant_gemv.cuh", "kquant_gemv2.cuh", "decode_persistent.cuh", "layer_kernels.cuh", "kib_ctx.cuh", "gguf.hpp"]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-pthread",
         "--expt-relaxed-constexpr", "-I" + os.path.join(HERE, "..", "include")]


def _stale():
    if not os.path.exists(LIB) or not os.path.exists(TOOLS_LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = [os.path.join(CSRC, f) for f in SOURCES + HEADERS]
    deps.append(os.path.join(HERE, "..", "include", "kib.h"))
    gw = os.path.join(HERE, "gateway")
    deps += [os.path.join(gw, f) for f in ("gw_core.cpp", "gw_abi.cpp", "gw_server.cpp", "gw_core.hpp", "gw_json.hpp")]
    if not os.path.exists(os.path.join(gw, "_build", "kib_gateway")):
        return True
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def build(force=False, verbose=False, ptxas_info=False):
    if not force and not _stale():
        return LIB
    os.makedirs(LIB_DIR, exist_ok=True)
    objs, cmds = [], []
    for src in SOURCES:
        obj = os.path.join(LIB_DIR, src + ".o")
        cmd = [NVCC] + ARCH + FLAGS + ["-c", os.path.join(CSRC, src), "-o", obj]
        if ptxas_info and src.endswith(".cu"):
            cmd += ["-Xptxas", "-v"]
        if verbose:
            print(" ".join(cmd))
        cmds.append(cmd)
        objs.append(obj)
    # the translation units are independent: compile them side by side
    procs = [subprocess.Popen(c) for c in cmds]
    codes = [p.wait() for p in procs]
    for c, rc in zip(cmds, codes):
        if rc:
            raise subprocess.CalledProcessError(rc, c)
    cmd = [NVCC] + ARCH + ["-shared", "-o", LIB] + objs
    if verbose:
        print(" ".join(cmd))
    subprocess.check_call(cmd)
    for o in objs:
        os.remove(o)
    cmd = [os.environ.get("CXX", "g++"), "-O3", "-std=c++17", "-fPIC", "-pthread", "-shared",
           "-I" + os.path.join(HERE, "..", "include"), "-o", TOOLS_LIB] + [os.path.join(CSRC, f) for f in TOOLS_SOURCES]
    if verbose:
        print(" ".join(cmd))
    subprocess.check_call(cmd)
    # the OpenAI-compatible gateway (host C++ over libkib.so)
    subprocess.check_call(["make", "-s", "-C", os.path.join(HERE, "gateway")])
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True, ptxas_info="--ptxas" in sys.argv)
