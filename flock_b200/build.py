"""Build libflock_cuda.so in-tree for sm_100a (B200).

    python -m flock_b200.build          # incremental
    python -m flock_b200.build --force  # rebuild everything

Each .cu under csrc/ compiles to an object under csrc/_build/ in parallel and
the objects link into flock_b200/libflock_cuda.so.  --fmad=false keeps every
multiply and add that the sources write separately as separately rounded
operations (the kernels spell out their FMAs with __fmaf_rn).
"""
from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OBJ = os.path.join(CSRC, "_build")
LIB = os.path.join(HERE, "libflock_cuda.so")
ROOT = os.path.dirname(HERE)

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "--fmad=false", "-Xcompiler", "-fPIC",
              "-Xcompiler", "-fvisibility=hidden", "-Xcompiler", "-Wall",
              "-DFLOCK_BUILD", f"-I{os.path.join(ROOT, 'include')}"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _deps_newer(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False, ptxas_v: bool = False) -> str:
    os.makedirs(OBJ, exist_ok=True)
    sources = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    headers = sorted(glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h"))
                     + [os.path.join(ROOT, "include", "flock_cuda.h")])
    objs, jobs = [], []
    for src in sources:
        obj = os.path.join(OBJ, os.path.basename(src).replace(".cu", ".o"))
        objs.append(obj)
        if force or _deps_newer(obj, [src] + headers):
            cmd = [nvcc(), *ARCH, *NVCC_FLAGS, "-c", src, "-o", obj]
            if ptxas_v:
                cmd += ["-Xptxas", "-v"]
            jobs.append(cmd)

    def run(cmd):
        r = subprocess.run(cmd, capture_output=True, text=True)
        return cmd, r

    with cf.ThreadPoolExecutor(max_workers=min(8, max(1, len(jobs)))) as ex:
        for cmd, r in ex.map(run, jobs):
            if verbose or r.returncode != 0 or ptxas_v:
                sys.stderr.write(" ".join(cmd) + "\n" + r.stdout + r.stderr)
            if r.returncode != 0:
                raise RuntimeError(f"nvcc failed on {cmd[-3]}")
    if force or jobs or _deps_newer(LIB, objs):
        cmd = [nvcc(), *ARCH, "-shared", "-o", LIB, *objs, "-lcuda", "-ldl"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("link failed:\n" + r.stdout + r.stderr)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv,
          ptxas_v="--ptxas" in sys.argv)
    print(LIB)
