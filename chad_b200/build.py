"""Build libqkv.so (the sm_100a kernels + C ABI) in-tree with nvcc.

    python -m chad_b200.build          # incremental
    python -m chad_b200.build --force  # rebuild everything

Translation units compile in parallel to objects under chad_b200/_build/, then link into
chad_b200/libqkv.so (static CUDA runtime, no torch dependency). The CPython bindings of the
per-layer entry points (csrc/qkv_pyext.c) build with gcc into chad_b200/_qkvext*.so.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libqkv.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O2", "--expt-relaxed-constexpr"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def headers():
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    hs.append(os.path.join(os.path.dirname(HERE), "include", "qkv.h"))
    return hs


def _compile(src: str, force: bool, extra) -> str:
    obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
    newest_dep = max(os.path.getmtime(p) for p in [src, *headers(), __file__])
    if not force and os.path.exists(obj) and os.path.getmtime(obj) >= newest_dep:
        return obj
    cmd = [nvcc(), *ARCH, *FLAGS, *extra, "-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src}:\n{r.stdout}\n{r.stderr}")
    return obj


def build(force: bool = False, verbose: bool = False, extra=()) -> str:
    os.makedirs(BUILD, exist_ok=True)
    srcs = sources()
    with cf.ThreadPoolExecutor(max_workers=max(1, min(len(srcs), os.cpu_count() or 4))) as ex:
        objs = list(ex.map(lambda s: _compile(s, force, list(extra)), srcs))
    newest = max(os.path.getmtime(o) for o in objs)
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < newest:
        cmd = [nvcc(), *ARCH, "-shared", "-o", LIB, *objs, "-cudart", "static", "-lpthread"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    build_ext(force)
    if verbose:
        print(LIB)
    return LIB


EXT_SRC = os.path.join(CSRC, "qkv_pyext.c")


def ext_path() -> str:
    import sysconfig

    return os.path.join(HERE, "_qkvext" + sysconfig.get_config_var("EXT_SUFFIX"))


def build_ext(force: bool = False) -> str:
    """The CPython bindings of the per-layer entry points (chad_b200._qkvext), with gcc."""
    import sysconfig

    out = ext_path()
    deps = [EXT_SRC, os.path.join(os.path.dirname(HERE), "include", "qkv.h"), __file__]
    if not force and os.path.exists(out) and os.path.getmtime(out) >= max(map(os.path.getmtime, deps)):
        return out
    cc = os.environ.get("CC") or shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        raise RuntimeError("no C compiler for the Python bindings")
    cmd = [cc, "-O2", "-fPIC", "-shared", "-std=gnu11", "-Wall",
           "-I" + sysconfig.get_paths()["include"], EXT_SRC, "-o", out]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"bindings build failed:\n{r.stdout}\n{r.stderr}")
    return out


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-v", action="store_true", help="print register/smem usage")
    args = ap.parse_args()
    extra = ["-Xptxas", "-v"] if args.ptxas_v else []
    try:
        build(force=args.force or args.ptxas_v, verbose=True, extra=extra)
    except RuntimeError as e:
        print(e, file=sys.stderr)
        sys.exit(1)
