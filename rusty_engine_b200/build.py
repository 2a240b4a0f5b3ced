"""Build librmoe.so in-tree: every .cu under csrc/ compiled for sm_100a by nvcc, linked shared.

Run as ``python -m rusty_engine_b200.build`` (or through ``__graft_entry__.build()``).  The
output lands next to this file so it travels with the repository snapshot.
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
OUT = os.path.join(HERE, "librmoe.so")
OBJ = os.path.join(HERE, "_build")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr", "-Xptxas", "-v", "-DRMOE_BUILD",
]


def _nvcc() -> str:
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found")


def _nccl_flags():
    """NCCL headers/lib: prefer the copy torch loads (same soname, one NCCL per process)."""
    try:
        import nvidia.nccl  # type: ignore

        base = os.path.dirname(nvidia.nccl.__file__) if nvidia.nccl.__file__ else list(nvidia.nccl.__path__)[0]
        inc, lib = os.path.join(base, "include"), os.path.join(base, "lib")
        if os.path.exists(os.path.join(inc, "nccl.h")):
            return ["-I" + inc], ["-L" + lib, "-Xlinker", "-rpath=" + lib, "-l:libnccl.so.2"]
    except Exception:
        pass
    return [], ["-lnccl"]


def build(verbose: bool = False, jobs: int = 8) -> str:
    nvcc = _nvcc()
    os.makedirs(OBJ, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    headers = glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(
        os.path.join(HERE, "..", "include", "*.h"))
    newest_h = max(os.path.getmtime(h) for h in headers)
    inc_nccl, link_nccl = _nccl_flags()

    def compile_one(src):
        obj = os.path.join(OBJ, os.path.basename(src) + ".o")
        if os.path.exists(obj) and os.path.getmtime(obj) >= max(os.path.getmtime(src), newest_h):
            return obj, ""
        cmd = [nvcc] + NVCC_FLAGS + inc_nccl + ["-c", src, "-o", obj]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src}:\n{r.stderr}")
        return obj, r.stderr

    with cf.ThreadPoolExecutor(jobs) as ex:
        results = list(ex.map(compile_one, srcs))
    if verbose:
        for obj, log in results:
            if log:
                print(log, file=sys.stderr)
    objs = [o for o, _ in results]
    if not os.path.exists(OUT) or os.path.getmtime(OUT) < max(os.path.getmtime(o) for o in objs):
        cmd = [nvcc] + ARCH + ["-shared", "-o", OUT] + objs + link_nccl
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stderr}")
    return OUT


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
