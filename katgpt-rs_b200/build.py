"""Build libkgcuda.so (sm_100a) in-tree: katgpt-rs_b200/lib/libkgcuda.so.

Files that restate the reference's CPU operation order (kg_micro.cu, kg_tq.cu)
are compiled with -fmad=false so nvcc never contracts a*b+c; explicit fmaf()
calls still emit FMA. Host table code is compiled with -ffp-contract=off.
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OBJ = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "lib")
LIBPATH = os.path.join(LIB, "libkgcuda.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_COMMON = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
                      "-Xcompiler", "-ffp-contract=off", "-Xptxas", "-v"]
EXACT = {"kg_micro.cu", "kg_tq.cu"}
CU_FILES = ["kg_micro.cu", "kg_tq.cu", "kg_api.cu", "kg_bf16.cu", "kg_attn.cu", "kg_tqattn.cu", "kg_big.cu", "kg_umma.cu",
            "kg_sample.cu", "kg_tcattn.cu", "kg_comm.cu", "kg_paged.cu", "kg_selftest.cu"]
CPP_FILES = ["kg_tables.cpp", "kg_sq.cpp"]


def _nvcc():
    for c in ("/usr/local/cuda/bin/nvcc", "nvcc"):
        if os.path.exists(c) or c == "nvcc":
            return c
    raise RuntimeError("nvcc not found")


def _run(cmd, log):
    r = subprocess.run(cmd, capture_output=True, text=True)
    log.append(" ".join(cmd) + "\n" + r.stdout + r.stderr)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("build step failed: " + " ".join(cmd))


def _stale(src, obj, deps):
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    return any(os.path.getmtime(d) > t for d in [src] + deps)


def build(verbose=False, force=False):
    os.makedirs(OBJ, exist_ok=True)
    os.makedirs(LIB, exist_ok=True)
    nvcc = _nvcc()
    headers = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))]
    headers.append(os.path.join(HERE, "..", "include", "kg_abi.h"))
    log, objs = [], []
    for f in CU_FILES:
        src, obj = os.path.join(CSRC, f), os.path.join(OBJ, f + ".o")
        objs.append(obj)
        if force or _stale(src, obj, headers):
            flags = list(NVCC_COMMON) + (["-fmad=false"] if f in EXACT else [])
            _run([nvcc] + flags + ["-c", src, "-o", obj], log)
    for f in CPP_FILES:
        src, obj = os.path.join(CSRC, f), os.path.join(OBJ, f + ".o")
        objs.append(obj)
        if force or _stale(src, obj, headers):
            _run(["g++", "-O2", "-std=c++17", "-fPIC", "-ffp-contract=off", "-fno-fast-math",
                  "-c", src, "-o", obj], log)
    if force or not os.path.exists(LIBPATH) or any(
            os.path.getmtime(o) > os.path.getmtime(LIBPATH) for o in objs):
        _run([nvcc] + ARCH + ["-shared", "-cudart", "static", "-o", LIBPATH] + objs, log)
    with open(os.path.join(OBJ, "build.log"), "w") as fh:
        fh.write("\n".join(log))
    if verbose:
        print("\n".join(log))
    return LIBPATH


if __name__ == "__main__":
    build(verbose="-v" in sys.argv, force="-f" in sys.argv)
