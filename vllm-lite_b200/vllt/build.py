"""Build libvllt.so in-tree with nvcc for sm_100a (B200).

    python -m vllt.build            (from the vllm-lite_b200 directory)

Each .cu under ../csrc is compiled separately (in parallel) and linked into
vllt/libvllt.so with the CUDA runtime linked statically. The library carries
plain extern "C" entry points (include/vllt.h); Python loads it with ctypes.
"""

from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(ROOT, "csrc")
OBJ = os.path.join(ROOT, "_build")
LIB = os.path.join(PKG, "libvllt.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         "-Xptxas", "-warn-spills"]


# Kernels allowed to spill registers: the fp32 parity GEMM (a few bytes, off
# the bf16 serving path). Any other spill fails the build: a spill in a hot
# kernel is a silent slowdown that only a GPU profile would show.
SPILL_ALLOWED = ("sgemm_kernel",)


def spilled_kernels(ptxas_output: str) -> list[str]:
    """Mangled names of the kernels that ptxas (-warn-spills) reports spilling."""
    out = []
    for line in ptxas_output.splitlines():
        if "Registers are spilled to local memory in function" in line:
            out.append(line.split("'")[1] if "'" in line else line)
    return out


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _stale(src: str, obj: str, deps: list[str]) -> bool:
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    return any(os.path.getmtime(p) > t for p in [src, *deps])


def build(verbose: bool = False, jobs: int | None = None) -> str:
    os.makedirs(OBJ, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    deps = sorted(glob.glob(os.path.join(CSRC, "*.cuh"))) + [
        os.path.join(os.path.dirname(ROOT), "include", "vllt.h")]
    cc = nvcc()

    def compile_one(src: str) -> str:
        obj = os.path.join(OBJ, os.path.basename(src)[:-3] + ".o")
        if _stale(src, obj, deps):
            cmd = [cc, *ARCH, *FLAGS, "-c", src, "-o", obj]
            if verbose:
                print(" ".join(cmd), flush=True)
            r = subprocess.run(cmd, capture_output=True, text=True)
            if r.returncode != 0:
                raise RuntimeError(f"nvcc failed on {src}:\n{r.stdout}\n{r.stderr}")
            if verbose and r.stderr.strip():
                print(r.stderr, file=sys.stderr)
            bad = [k for k in spilled_kernels(r.stdout + r.stderr) if not any(a in k for a in SPILL_ALLOWED)]
            if bad:
                os.remove(obj)
                raise RuntimeError(f"register spills in {os.path.basename(src)}: {', '.join(bad)}")
        return obj

    with cf.ThreadPoolExecutor(max_workers=jobs or os.cpu_count() or 4) as ex:
        objs = list(ex.map(compile_one, srcs))
    if not os.path.exists(LIB) or any(os.path.getmtime(o) > os.path.getmtime(LIB) for o in objs):
        cmd = [cc, *ARCH, "-shared", "-o", LIB, *objs, "-lcuda"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
