"""Builds libs1kv.so (sm_100a) and the C++ reference-interface shim in-tree.

    python s1-infer_b200/build.py [--verbose-ptxas] [--force]

Outputs (git-ignored, shipped with the tree):
    s1-infer_b200/lib/libs1kv.so        C-ABI engine (include/s1kv.h)
    s1-infer_b200/lib/libs1kv_shim.so   KVBlockPool / GQA_attention_paged /
                                        apply_rope with the reference's C++
                                        signatures, on top of libs1kv.so
Objects go to s1-infer_b200/_build/.  Only stale objects are rebuilt.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
SHIM = os.path.join(PKG, "shim")
BUILD = os.path.join(PKG, "_build")
LIBDIR = os.path.join(PKG, "lib")
LIB = os.path.join(LIBDIR, "libs1kv.so")
SHIM_LIB = os.path.join(LIBDIR, "libs1kv_shim.so")
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA, "bin", "nvcc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
INC = ["-I", os.path.join(ROOT, "include"), "-I", CSRC]
# -ffp-contract=off on the host side: the RoPE table must be the plain
# float expression of the reference (no fused multiply-add contraction).
HOST_FLAGS = ["-O2", "-fPIC", "-std=c++17", "-ffp-contract=off", "-fno-fast-math", "-Wall", "-Wno-unused-function"]


def _stale(out, deps):
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    return any(os.path.getmtime(d) > t for d in deps)


def _headers(d):
    return [os.path.join(d, f) for f in os.listdir(d) if f.endswith(".h")]


def _run(cmd):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(" ".join(cmd) + "\n" + r.stdout + r.stderr)
        raise RuntimeError("compile failed: " + os.path.basename(cmd[-1]))
    return r.stdout + r.stderr


def build(verbose_ptxas=False, force=False, jobs=None):
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(LIBDIR, exist_ok=True)
    hdrs = _headers(CSRC) + [os.path.join(ROOT, "include", "s1kv.h")]
    jobs_list = []
    objs = []
    for f in sorted(os.listdir(CSRC)):
        src = os.path.join(CSRC, f)
        if f.endswith(".cu"):
            obj = os.path.join(BUILD, f + ".o")
            cmd = [NVCC] + ARCH + ["-lineinfo", "-O3", "-std=c++17", "--expt-relaxed-constexpr",
                                   "-Xcompiler", ",".join(["-fPIC", "-ffp-contract=off"])] + INC
            if verbose_ptxas:
                cmd += ["-Xptxas", "-v"]
            cmd += ["-c", "-o", obj, src]
        elif f.endswith(".cpp"):
            obj = os.path.join(BUILD, f + ".o")
            cmd = ["g++"] + HOST_FLAGS + INC + ["-I", os.path.join(CUDA, "include"), "-c", "-o", obj, src]
        else:
            continue
        objs.append(obj)
        if force or _stale(obj, [src] + hdrs):
            jobs_list.append(cmd)
    logs = []
    if jobs_list:
        with cf.ThreadPoolExecutor(max_workers=jobs or os.cpu_count()) as ex:
            logs = list(ex.map(_run, jobs_list))
    if force or jobs_list or _stale(LIB, objs):
        _run([NVCC] + ARCH + ["-shared", "-o", LIB] + objs + ["-cudart", "static", "-lrt", "-ldl", "-lpthread"])
    # C++ shim with the reference's interface, linked against libs1kv.so.
    shim_srcs = [os.path.join(SHIM, "src", f) for f in sorted(os.listdir(os.path.join(SHIM, "src")))
                 if f.endswith(".cpp")] if os.path.isdir(os.path.join(SHIM, "src")) else []
    if shim_srcs:
        shim_hdrs = []
        for dp, _, fs in os.walk(os.path.join(SHIM, "include")):
            shim_hdrs += [os.path.join(dp, f) for f in fs if f.endswith(".h")]
        if force or _stale(SHIM_LIB, shim_srcs + shim_hdrs + [LIB]):
            _run(["g++"] + HOST_FLAGS +
                 ["-shared", "-I", os.path.join(SHIM, "include"), "-I", os.path.join(CUDA, "include"),
                  "-I", os.path.join(ROOT, "include"), "-o", SHIM_LIB] + shim_srcs +
                 ["-L", LIBDIR, "-ls1kv", "-L", os.path.join(CUDA, "lib64"), "-lcudart", "-Wl,--no-undefined",
                  "-Wl,-rpath,$ORIGIN", "-Wl,-rpath," + os.path.join(CUDA, "lib64")])
    return "\n".join(l for l in logs if l.strip())


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose-ptxas", action="store_true")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    out = build(a.verbose_ptxas, a.force)
    if out:
        print(out)
    print("built", LIB)
