"""Build libwgkv.so (all CUDA sources of csrc/) for sm_100a, in-tree.

    python wg-kv_b200/build.py [--debug]

Each .cu is compiled to an object in wg-kv_b200/_build/ (in parallel), then
linked into wg-kv_b200/wgkv/libwgkv.so against the CUDA runtime only (the
driver entry point for tensor-map encoding is fetched at run time).
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(PKG, "csrc")
# WGKV_LIB_OUT / WGKV_BUILD_DIR / WGKV_EXTRA_NVCC redirect a build (e.g. a variant with extra -D flags)
OUT = os.environ.get("WGKV_LIB_OUT", os.path.join(PKG, "wgkv", "libwgkv.so"))
BUILD = os.environ.get("WGKV_BUILD_DIR", os.path.join(PKG, "_build"))
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc():
    home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    p = os.path.join(home, "bin", "nvcc")
    return p if os.path.exists(p) else (shutil.which("nvcc") or "nvcc")


def flags(debug=False):
    f = ["-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
         "--expt-relaxed-constexpr", "-Xptxas", "-v" if os.environ.get("WGKV_PTXAS_V") else "-O3"]
    if debug:
        f += ["-DWGKV_DEBUG=1"]
    f += os.environ.get("WGKV_EXTRA_NVCC", "").split()
    return ARCH + f


def compile_one(src, debug):
    obj = os.path.join(BUILD, os.path.basename(src) + ".o")
    if os.path.exists(obj) and os.path.getmtime(obj) >= max(
            os.path.getmtime(src), *(os.path.getmtime(os.path.join(CSRC, h)) for h in os.listdir(CSRC)
                                    if h.endswith((".cuh", ".h"))),
            os.path.getmtime(os.path.join(os.path.dirname(PKG), "include", "wgkv.h"))):
        return obj, ""
    cmd = [nvcc()] + flags(debug) + ["-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    return obj, r.stderr


def build(debug=False, verbose=False):
    os.makedirs(BUILD, exist_ok=True)
    srcs = sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        res = list(ex.map(lambda s: compile_one(s, debug), srcs))
    if verbose:
        for _, log in res:
            if log:
                print(log)
    objs = [o for o, _ in res]
    tmp = OUT + ".tmp"
    cmd = [nvcc()] + ARCH + ["-shared", "-cudart", "static", "-o", tmp] + objs
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    print(build(debug="--debug" in sys.argv, verbose="-v" in sys.argv))
