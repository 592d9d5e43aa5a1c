"""Build recipe for libneuratensor_native.so (sm_100a only).

    python -m neuratensor_b200.build [--verbose] [--ptxas-info]

Compiles every ``csrc/*.cu`` with nvcc for ``sm_100a`` into objects under
``neuratensor_b200/_build/`` and links them into
``neuratensor_b200/lib/libneuratensor_native.so``.  The CUDA runtime is
linked statically; the driver entry points are resolved at run time, so the
library needs only ``libcuda.so`` from the GPU driver.  nvcc cross-compiles
without a GPU.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(PKG, "_build")
LIBDIR = os.path.join(PKG, "lib")
LIB = os.path.join(LIBDIR, "libneuratensor_native.so")
INCLUDE = os.path.join(os.path.dirname(PKG), "include")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
              "-I" + INCLUDE, "-I" + CSRC]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def _deps_mtime() -> float:
    paths = [os.path.join(CSRC, f) for f in os.listdir(CSRC)] + [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE)]
    return max(os.path.getmtime(p) for p in paths)


def up_to_date() -> bool:
    """Every object is newer than its source and every header, and the library
    newer than every source, header and object."""
    if not os.path.exists(LIB):
        return False
    headers = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if not f.endswith(".cu")] + \
        [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE)]
    hdr = max(os.path.getmtime(p) for p in headers)
    objs = []
    for src in sources():
        obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
        if not os.path.exists(obj) or os.path.getmtime(obj) < max(os.path.getmtime(src), hdr):
            return False
        objs.append(obj)
    newest = max([_deps_mtime()] + [os.path.getmtime(o) for o in objs])
    return os.path.getmtime(LIB) >= newest


def build(verbose: bool = False, ptxas_info: bool = False, force: bool = False) -> str:
    if not force and up_to_date():
        return LIB
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(LIBDIR, exist_ok=True)
    cc = nvcc()
    extra = ["-Xptxas", "-v"] if ptxas_info else []

    headers = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if not f.endswith(".cu")] + \
        [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE)]
    hdr_mtime = max(os.path.getmtime(p) for p in headers)

    def compile_one(src):
        obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
        # an object newer than its source and every header is reused (not with --force / --ptxas-info)
        if (not force and not ptxas_info and os.path.exists(obj) and
                os.path.getmtime(obj) >= max(os.path.getmtime(src), hdr_mtime)):
            return obj
        cmd = [cc, *ARCH, *NVCC_FLAGS, *extra, "-c", src, "-o", obj]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
        if verbose or ptxas_info:
            sys.stderr.write(r.stdout + r.stderr)
        return obj

    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(compile_one, sources()))
    tmp = LIB + ".tmp"
    cmd = [cc, *ARCH, "-shared", "-Xcompiler", "-fPIC", "-o", tmp, *objs]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB)
    return LIB


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(build(verbose=a.verbose, ptxas_info=a.ptxas_info, force=a.force or a.ptxas_info))


if __name__ == "__main__":
    main()
