"""Build step for the ferrite B200 C-ABI library (``libferrite_b200.so``).

Compiles every ``csrc/*.cu`` for sm_100a with nvcc (one object per translation
unit, in parallel) and links them into ``ferrite/_lib/libferrite_b200.so``
in-tree, so the built library travels with the source tree.  Objects are rebuilt
only when a source or header is newer than the object.

Usage: ``python ferrite-tpu_b200/build.py [--force] [-j N]``.
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
INCLUDE = os.path.join(os.path.dirname(HERE), "include")
OBJDIR = os.path.join(HERE, "_build")
LIBDIR = os.path.join(HERE, "ferrite", "_lib")
LIB = os.path.join(LIBDIR, "libferrite_b200.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    *ARCH,
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xcompiler",
    "-fPIC,-O2,-fvisibility=hidden",
    "-I" + INCLUDE,
    "-DFERRITE_BUILD",
]


def nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _sources() -> list[str]:
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def _headers() -> list[str]:
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    hs += [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE) if f.endswith(".h")]
    return hs


def _stale(obj: str, src: str, headers: list[str]) -> bool:
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    return any(os.path.getmtime(p) > t for p in [src, *headers])


def _compile(src: str, obj: str, extra: list[str], verbose_ptxas: bool) -> tuple[str, str]:
    cmd = [nvcc(), *NVCC_FLAGS, *extra, "-c", src, "-o", obj]
    if verbose_ptxas:
        cmd.insert(1, "-Xptxas=-v")
    p = subprocess.run(cmd, capture_output=True, text=True)
    if p.returncode != 0:
        raise RuntimeError(f"nvcc failed for {os.path.basename(src)}:\n{p.stderr}\n{' '.join(cmd)}")
    return src, p.stderr


def build(force: bool = False, jobs: int | None = None, verbose_ptxas: bool = False, extra: list[str] | None = None) -> str:
    """Compile and link the library; returns the path of the shared object."""
    os.makedirs(OBJDIR, exist_ok=True)
    os.makedirs(LIBDIR, exist_ok=True)
    headers = _headers()
    srcs = _sources()
    objs = [os.path.join(OBJDIR, os.path.basename(s)[:-3] + ".o") for s in srcs]
    todo = [(s, o) for s, o in zip(srcs, objs) if force or verbose_ptxas or _stale(o, s, headers)]
    logs = []
    if todo:
        with cf.ThreadPoolExecutor(max_workers=jobs or min(len(todo), os.cpu_count() or 4)) as ex:
            futs = [ex.submit(_compile, s, o, extra or [], verbose_ptxas) for s, o in todo]
            for f in futs:
                logs.append(f.result())
    if todo or not os.path.exists(LIB):
        cmd = [nvcc(), *ARCH, "-shared", "-o", LIB, *objs, "-lcudart_static", "-lrt", "-ldl", "-lpthread"]
        p = subprocess.run(cmd, capture_output=True, text=True)
        if p.returncode != 0:
            raise RuntimeError(f"link failed:\n{p.stderr}\n{' '.join(cmd)}")
    if verbose_ptxas:
        for src, err in logs:
            print(f"== {os.path.basename(src)}\n{err}")
    return LIB


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", "--jobs", type=int, default=None)
    ap.add_argument("--ptxas-v", action="store_true", help="print register/smem usage")
    a = ap.parse_args(argv)
    print(build(force=a.force, jobs=a.jobs, verbose_ptxas=a.ptxas_v))


if __name__ == "__main__":
    sys.exit(main())
