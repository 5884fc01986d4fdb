"""Build the sm_100a CUDA library ``libnkimoe.so`` in-tree.

    python -m nki_moe_b200.build            # incremental
    python -m nki_moe_b200.build --force    # rebuild everything

nvcc cross-compiles for ``sm_100a`` without a GPU.  The library has no torch
dependency: it exports the C ABI declared in ``include/nkimoe.h`` and links
the CUDA runtime statically.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(REPO, "_build")
LIB = os.path.join(PKG, "libnkimoe.so")
SOURCES = ["norm.cu", "router.cu", "permute.cu", "pack.cu", "grouped_gemm.cu", "ep_peer.cu", "capi.cu",
           "noalloc.cu", "attention.cu", "linear.cu"]
HEADERS = ["common.cuh", "kernels.h", "rope.cuh", "permute_small.cuh"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def flags() -> list[str]:
    return [
        "-gencode", "arch=compute_100a,code=sm_100a",
        "-O3", "-lineinfo", "-std=c++17",
        "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
        "--expt-relaxed-constexpr",
        "-I", os.path.join(REPO, "include"), "-I", CSRC,
    ]


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    cc = nvcc()
    hdrs = [os.path.join(CSRC, h) for h in HEADERS] + [os.path.join(REPO, "include", "nkimoe.h")]
    jobs = []
    objs = []
    for src in SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(BUILD, src.replace(".cu", ".o"))
        objs.append(o)
        if force or _stale(o, [s] + hdrs):
            jobs.append([cc, *flags(), "-c", s, "-o", o])

    def run(cmd):
        r = subprocess.run(cmd, capture_output=True, text=True)
        if verbose or r.returncode != 0:
            sys.stderr.write(r.stdout + r.stderr)
        if r.returncode != 0:
            raise RuntimeError("nvcc failed: " + " ".join(cmd))

    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(len(jobs), os.cpu_count() or 4)) as ex:
            list(ex.map(run, jobs))
    if force or jobs or _stale(LIB, objs):
        # export only the C ABI: the kernels have hidden visibility
        run([cc, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-Xcompiler", "-fPIC",
             *objs, "-o", LIB, "-cudart", "static", "-ldl", "-lrt", "-lpthread"])
    return LIB


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))


if __name__ == "__main__":
    main()
