"""Build libomc.so in-tree: CUDA kernels for sm_100a + the C host runtime.

    python -m overhang_b200.build            # or overhang_b200.build.build()

nvcc cross-compiles sm_100a without a GPU, so this runs on a CPU-only box.
The result is ``overhang_b200/libomc.so`` (git-ignored, shipped with the tree).
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libomc.so")

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
# the image's CC wrapper lacks libgomp/specs; use the system gcc from PATH
HOSTCC = shutil.which("gcc") or "gcc"
GENCODE = ["-gencode", "arch=compute_100a,code=sm_100a"]
INCLUDES = ["-I" + os.path.join(ROOT, "include"), "-I" + CSRC]
NVFLAGS = GENCODE + ["-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
                     "-Xcompiler", "-fPIC", "-Xptxas", "-v"] + INCLUDES
CFLAGS = ["-O2", "-fPIC", "-std=gnu11", "-Wall", "-Wno-unused-function",
          "-I/usr/local/cuda/include"] + INCLUDES


def _sources():
    cu = sorted(f for f in os.listdir(CSRC) if f.endswith(".cu"))
    c = sorted(f for f in os.listdir(CSRC) if f.endswith(".c"))
    return cu, c


def _newer(src_paths, out):
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    return any(os.path.getmtime(p) > t for p in src_paths)


def _headers():
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))]
    inc = os.path.join(ROOT, "include")
    hs += [os.path.join(inc, f) for f in os.listdir(inc) if f.endswith(".h")]
    return hs


def _run(cmd, log):
    p = subprocess.run(cmd, capture_output=True, text=True)
    with open(log, "w") as f:
        f.write(" ".join(cmd) + "\n" + p.stdout + p.stderr)
    if p.returncode:
        raise RuntimeError(f"build failed: {' '.join(cmd)}\n{p.stdout}{p.stderr}")
    return p.stdout + p.stderr


def build(verbose: bool = False, force: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    cu, c = _sources()
    hdrs = _headers()
    jobs = []
    objs = []
    for f in cu:
        src = os.path.join(CSRC, f)
        obj = os.path.join(BUILD, f + ".o")
        objs.append(obj)
        if force or _newer([src] + hdrs, obj):
            jobs.append(([NVCC] + NVFLAGS + ["-c", src, "-o", obj], obj + ".log"))
    for f in c:
        src = os.path.join(CSRC, f)
        obj = os.path.join(BUILD, f + ".o")
        objs.append(obj)
        if force or _newer([src] + hdrs, obj):
            jobs.append(([HOSTCC] + CFLAGS + ["-c", src, "-o", obj], obj + ".log"))
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        outs = list(ex.map(lambda j: _run(*j), jobs))
    if verbose:
        for o in outs:
            sys.stdout.write(o)
    if force or jobs or _newer(objs, LIB):
        tmp = LIB + ".tmp"
        _run([NVCC] + GENCODE + ["-shared", "-o", tmp] + objs + ["-ldl", "-lpthread", "-lm"],
             os.path.join(BUILD, "link.log"))
        os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, force="-f" in sys.argv))
