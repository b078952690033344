"""Build libkq.so (the sm_100a kernels behind include/kq.h) in-tree.

    python k-search_b200/kq/build.py [--force] [-v]

Every .cu under k-search_b200/csrc is compiled by nvcc for sm_100a
(-gencode arch=compute_100a,code=sm_100a -lineinfo -O3) in parallel, then
linked into k-search_b200/kq/libkq.so. Objects go to k-search_b200/_build/.
Rebuilds only what changed (a header change rebuilds everything).
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG_DIR)                      # k-search_b200/
REPO = os.path.dirname(ROOT)
CSRC = os.path.join(ROOT, "csrc")
INCLUDE = os.path.join(REPO, "include")
BUILD = os.path.join(ROOT, "_build")
LIB = os.path.join(PKG_DIR, "libkq.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC,-O3", "--expt-relaxed-constexpr",
                     f"-I{INCLUDE}", f"-I{CSRC}"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _newest(paths) -> float:
    return max((os.path.getmtime(p) for p in paths), default=0.0)


def build(force: bool = False, verbose: bool = False, extra_flags: list[str] | None = None) -> str:
    os.makedirs(BUILD, exist_ok=True)
    sources = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    headers = glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh")) + \
        glob.glob(os.path.join(INCLUDE, "*.h"))
    hdr_time = _newest(headers + [os.path.abspath(__file__)])
    flags = NVCC_FLAGS + (extra_flags or [])
    jobs = []
    objs = []
    for src in sources:
        obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
        objs.append(obj)
        if force or not os.path.exists(obj) or os.path.getmtime(obj) < max(os.path.getmtime(src), hdr_time):
            jobs.append((src, obj))

    def compile_one(job):
        src, obj = job
        cmd = [nvcc()] + flags + ["-c", src, "-o", obj]
        r = subprocess.run(cmd, capture_output=True, text=True)
        return src, r.returncode, r.stdout + r.stderr

    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(len(jobs), os.cpu_count() or 4)) as ex:
            for src, rc, out in ex.map(compile_one, jobs):
                if verbose or rc != 0:
                    sys.stderr.write(out)
                if rc != 0:
                    raise RuntimeError(f"nvcc failed on {os.path.basename(src)}")
    if jobs or not os.path.exists(LIB) or os.path.getmtime(LIB) < _newest(objs):
        cmd = [nvcc()] + ARCH + ["-shared", "-o", LIB] + objs
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            sys.stderr.write(r.stdout + r.stderr)
            raise RuntimeError("link of libkq.so failed")
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    ap.add_argument("--ptxas-v", action="store_true", help="print register / smem usage")
    a = ap.parse_args()
    extra = ["-Xptxas", "-v"] if a.ptxas_v else None
    print(build(force=a.force or a.ptxas_v, verbose=a.verbose or a.ptxas_v, extra_flags=extra))


if __name__ == "__main__":
    main()
