"""Builds libspecdec_b200.so (sm_100a) in-tree with nvcc.

The library is self-contained CUDA C++ (no PyTorch).  csrc/engine.cu holds the
host engine and the C ABI declared in include/specdec.h and includes most
kernel headers; the other csrc/*.cu files are kernels with their own host
launch wrappers.  Each translation unit compiles to an object under _build/
(in parallel, and only when it or a header it includes changed), then one
link step makes the shared library.
"""
from __future__ import annotations

import os
import re
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "specdec_b200", "libspecdec_b200.so")
OBJ_DIR = os.path.join(HERE, "_build")
INCLUDE = os.path.join(ROOT, "include")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
                     "-Xptxas", "-v"]


def nvcc() -> str:
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if c and (os.path.exists(c) or c == "nvcc"):
            return c
    raise RuntimeError("nvcc not found")


def sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


_INC = re.compile(r'^\s*#\s*include\s+"([^"]+)"', re.M)


def deps(path: str, seen=None) -> set:
    """The file and every quoted include it reaches."""
    seen = set() if seen is None else seen
    path = os.path.normpath(path)
    if path in seen or not os.path.exists(path):
        return seen
    seen.add(path)
    with open(path) as f:
        for inc in _INC.findall(f.read()):
            deps(os.path.join(os.path.dirname(path), inc), seen)
    return seen


def obj_of(src: str) -> str:
    return os.path.join(OBJ_DIR, os.path.basename(src)[:-3] + ".o")


def stale(target: str, dep_files) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in dep_files if os.path.exists(d))


def needs_build() -> bool:
    srcs = sources()
    return any(stale(obj_of(s), deps(s)) for s in srcs) or stale(OUT, [obj_of(s) for s in srcs])


def _compile(src: str):
    cmd = [nvcc()] + NVCC_FLAGS + ["-I", INCLUDE, "-c", "-o", obj_of(src), src]
    r = subprocess.run(cmd, capture_output=True, text=True)
    return src, r


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(OBJ_DIR, exist_ok=True)
    srcs = sources()
    todo = [s for s in srcs if force or stale(obj_of(s), deps(s))]
    reports = []
    if todo:
        with ThreadPoolExecutor(max_workers=len(todo)) as ex:
            for src, r in ex.map(_compile, todo):
                if r.returncode != 0:
                    sys.stderr.write(r.stdout + r.stderr)
                    raise RuntimeError(f"nvcc failed on {os.path.basename(src)}")
                reports.append(f"== {os.path.basename(src)}\n{r.stderr}")
        with open(os.path.join(OBJ_DIR, "ptxas_report.txt"), "w") as f:
            f.write("\n".join(reports))
        if verbose:
            sys.stderr.write("\n".join(reports))
    objs = [obj_of(s) for s in srcs]
    if force or todo or stale(OUT, objs):
        cmd = [nvcc()] + ARCH + ["-shared", "-o", OUT] + objs + ["-ldl"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            sys.stderr.write(r.stdout + r.stderr)
            raise RuntimeError("nvcc link failed")
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
