"""Build the sm_100a shared library ``toy_b200/libtoyb200.so`` with nvcc.

The library is built in-tree so it travels with the source tree; object files
go to ``toy_b200/_build``. Every CUDA translation unit is compiled for
``compute_100a``/``sm_100a`` only. Rebuilds are incremental on file mtimes.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libtoyb200.so")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O3", "--expt-relaxed-constexpr",
                     "-I", CSRC, "-I", INCLUDE]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _nccl_flags() -> list[str]:
    """Header and library of the NCCL that ships with the torch wheel (2.28)."""
    try:
        import nvidia.nccl  # type: ignore
        root = os.path.dirname(nvidia.nccl.__file__) if nvidia.nccl.__file__ else list(nvidia.nccl.__path__)[0]
    except Exception:  # pragma: no cover - fall back to the system install
        return ["-lnccl"]
    inc, lib = os.path.join(root, "include"), os.path.join(root, "lib")
    return ["-I", inc, "-L", lib, "-l:libnccl.so.2", "-Xlinker", "-rpath," + lib]


def sources() -> list[str]:
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cu", ".cpp")))


def headers_mtime() -> float:
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    hs += [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE) if f.endswith(".h")]
    return max((os.path.getmtime(h) for h in hs), default=0.0)


def build(verbose: bool = False, force: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    nvcc = _nvcc()
    hmt = headers_mtime()
    nccl = _nccl_flags()
    inc_nccl = [f for i, f in enumerate(nccl) if f == "-I" or (i > 0 and nccl[i - 1] == "-I")]
    objs, jobs = [], []
    for src in sources():
        obj = os.path.join(BUILD, os.path.basename(src) + ".o")
        objs.append(obj)
        if force or not os.path.exists(obj) or os.path.getmtime(obj) < max(os.path.getmtime(src), hmt):
            cmd = [nvcc] + NVCC_FLAGS + inc_nccl + ["-x", "cu" if src.endswith(".cu") else "c++", "-c", src, "-o", obj]
            jobs.append(cmd)

    def run(cmd):
        if verbose:
            print(" ".join(cmd), flush=True)
        p = subprocess.run(cmd, capture_output=True, text=True)
        if p.returncode != 0:
            raise RuntimeError(f"nvcc failed:\n{' '.join(cmd)}\n{p.stdout}\n{p.stderr}")
        return p.stderr

    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        for err in ex.map(run, jobs):
            if verbose and err:
                print(err)
    if jobs or not os.path.exists(LIB) or any(os.path.getmtime(o) > os.path.getmtime(LIB) for o in objs):
        link = [nvcc] + ARCH + ["-shared", "-cudart", "static", "-o", LIB] + objs + nccl + ["-lpthread", "-ldl"]
        run(link)
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, force="-f" in sys.argv))
