"""Build the host-compiled test harnesses (tests/*_host.cpp).

Some kernels keep their per-item arithmetic in CUDA-free headers under
vllm-lite_b200/csrc (prefix_hash.cuh, meta_items.cuh, sampler_row.cuh) so that the same code
compiles for the host, and the SIMT kernels' device code sits in *_kernels.cuh
headers that compile for the host under the fiber emulation of
tests/simt_host.h; a harness wraps them in extern "C" functions that the CPU
tests call through ctypes. Built with g++ into a temporary directory per test
session (nothing is written into the repository).
"""

import ctypes
import os
import shutil
import subprocess

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def build_harness(name: str, out_dir: str):
    """Compile tests/<name>.cpp against the csrc headers; None without g++."""
    gxx = shutil.which("g++")
    if gxx is None:
        return None
    out = os.path.join(out_dir, f"lib{name}.so")
    # no FMA contraction: the device code rounds every product and quotient (__fmul_rn, __fdiv_rn)
    subprocess.run([gxx, "-O2", "-std=c++20", "-ffp-contract=off", "-shared", "-fPIC", "-I",
                    os.path.join(ROOT, "vllm-lite_b200", "csrc"), "-I", os.path.join(ROOT, "tests"),
                    os.path.join(ROOT, "tests", f"{name}.cpp"), "-o", out], check=True)
    return ctypes.CDLL(out)
