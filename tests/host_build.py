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


def tsan_requested() -> bool:
    """VLLT_HOST_TSAN=1: every host build of this process is instrumented for
    ThreadSanitizer (tests/test_race_check_host.py runs host tests that way,
    with the runtime preloaded)."""
    return os.environ.get("VLLT_HOST_TSAN") == "1"


def sanitizer_flags(tsan: bool) -> list:
    """Compiler flags of the instrumented builds: ThreadSanitizer (tsan), and
    UndefinedBehaviorSanitizer when VLLT_HOST_UBSAN=1 (signed overflow,
    shifts, misaligned or null accesses, out-of-range conversions: the
    process stops at the first report)."""
    f = ["-fsanitize=thread", "-g"] if tsan else []
    if os.environ.get("VLLT_HOST_UBSAN") == "1":
        f += ["-fsanitize=undefined", "-fno-sanitize-recover=all", "-g"]
    return f


_BUILT: dict = {}  # (harness, tsan) -> the library built earlier in this process


def build_harness(name: str, out_dir: str, tsan: bool | None = None, load: bool = True):
    """Compile tests/<name>.cpp against the csrc headers; None without g++.
    tsan: instrumented for ThreadSanitizer (default: tsan_requested()).
    load False: only the path. A harness is compiled once per process; later
    calls load the same file."""
    tsan = tsan_requested() if tsan is None else tsan
    gxx = shutil.which("g++")
    if gxx is None:
        return None
    key = (name, tsan, os.environ.get("VLLT_HOST_UBSAN") == "1")
    done = _BUILT.get(key)
    if done is not None and os.path.exists(done):
        return ctypes.CDLL(done) if load else done
    out = os.path.join(out_dir, f"lib{name}.so")
    # no FMA contraction: the device code rounds every product and quotient (__fmul_rn, __fdiv_rn);
    # -march=native: the harness runs where it is built, and fmaf becomes one instruction
    subprocess.run([gxx, "-O2", "-march=native", "-std=c++20", "-ffp-contract=off", "-fno-gnu-unique", "-pthread",
                    "-DVLLT_SIMT_HOST=1", "-shared", "-fPIC", *sanitizer_flags(tsan),
                    "-I", os.path.join(ROOT, "tests", "simt_include"),
                    "-I", os.path.join(ROOT, "vllm-lite_b200", "csrc"), "-I", os.path.join(ROOT, "tests"),
                    os.path.join(ROOT, "tests", f"{name}.cpp"), "-o", out], check=True)
    _BUILT[key] = out
    return ctypes.CDLL(out) if load else out


# libvllt but NCCL: the C ABI, its launchers and their kernels (the tensor-core
# ones on the emulation of tests/simt_include/simt_tc.h)
LIBRARY_SOURCES = ("capi.cu", "norm.cu", "cache_ops.cu", "sampling.cu", "batch_meta.cu", "attention.cu",
                   "attention_static.cu", "prefix_hash.cu", "attention_decode.cu", "forward_bf16.cu", "gemm_bf16.cu",
                   "attention_prefill_tc.cu")


def tsan_runtime():
    """Path of g++'s ThreadSanitizer runtime, or None when it has none."""
    gxx = shutil.which("g++")
    if gxx is None:
        return None
    p = subprocess.run([gxx, "-print-file-name=libtsan.so"], capture_output=True, text=True).stdout.strip()
    return p if os.path.isabs(p) and os.path.exists(p) else None


def build_library_host(out_dir: str, tsan: bool | None = None):
    """libvllt compiled for the host: the library's own sources
    (LIBRARY_SOURCES, unchanged) against the stub CUDA headers of
    tests/simt_include, every launch running on the SIMT emulation of
    tests/simt_host.h, plus tests/simt_stubs.cpp for NCCL and the emulation's
    test hooks. The sources compile in parallel. tsan: instrumented for
    ThreadSanitizer (default: tsan_requested(); the process must preload its
    runtime). Returns the CDLL with the C ABI's signatures set, or None
    without g++."""
    import concurrent.futures as cf

    tsan = tsan_requested() if tsan is None else tsan
    gxx = shutil.which("g++")
    if gxx is None:
        return None
    csrc = os.path.join(ROOT, "vllm-lite_b200", "csrc")
    flags = ["-O2", "-march=native", "-std=c++20", "-ffp-contract=off", "-fno-gnu-unique", "-pthread",
             "-DVLLT_SIMT_HOST=1", "-fPIC", "-I", os.path.join(ROOT, "tests", "simt_include"),
             "-I", os.path.join(ROOT, "tests"), "-I", csrc] + sanitizer_flags(tsan)
    srcs = [os.path.join(csrc, f) for f in LIBRARY_SOURCES] + [os.path.join(ROOT, "tests", "simt_stubs.cpp")]

    def compile_one(src):
        obj = os.path.join(out_dir, os.path.basename(src) + ".o")
        subprocess.run([gxx, *flags, "-x", "c++", "-c", src, "-o", obj], check=True)
        return obj

    with cf.ThreadPoolExecutor(max_workers=min(len(srcs), os.cpu_count() or 4)) as ex:
        objs = list(ex.map(compile_one, srcs))
    out = os.path.join(out_dir, "libvllt_host.so")
    subprocess.run([gxx, "-shared", "-pthread", *sanitizer_flags(tsan), *objs, "-o", out], check=True)
    return load_library_host(out)


def load_library_host(path: str):
    """The host build at `path` (from build_library_host) loaded with the C
    ABI's signatures set: how a spawned test process opens the library its
    parent built."""
    lib = ctypes.CDLL(path)
    from vllt import _lib

    for name, (res, args) in _lib.SIGNATURES.items():
        f = getattr(lib, name, None)
        if f is not None:
            f.restype, f.argtypes = res, args
    return lib
