"""CPU: race checking of the kernels' own code (compute-sanitizer's racecheck
is closed on the GPU pool).

The host build of libvllt and of the test harnesses can be instrumented with
ThreadSanitizer (tests/host_build.py, VLLT_HOST_TSAN=1; the runtime is
preloaded into a child Python). The SIMT emulation (tests/simt_host.h) makes
every emulated GPU thread a sanitizer fiber and states only the orderings the
hardware gives: CTA, warp and cluster barriers, the phases of mbarriers
(arrivals, completed TMA copies, tcgen05.commit), and the start and end of
each CTA. The CTAs of a launch run concurrently on a pool of OS threads and
atomics are real. Any two accesses of the kernels' own code to the same bytes
of shared memory, tensor memory or global memory, one of them a write, that no
such ordering puts one after the other, are reported.

  * the checker itself: kernels with a planted race (a shared-memory read
    of a neighbour's slot with no barrier, a plain read-modify-write of one
    global word from every CTA, a consumer that reads before waiting on the
    producer's mbarrier) are reported at the planted line, and the same
    kernels with the ordering in place are not (tests/race_host.cpp);
  * the library's kernels on a sample of the host tests' cases, every form
    reached: the tcgen05 GEMM forms (persistent, split-K, stream-K with its
    slice reduction, cluster split-K with the distributed shared-memory
    reduction) including a dropped TMA load's error path, the tensor-core
    prefill attention, the TMA decode kernel and its stall injection, the
    generic attention kernel with split-K, and the sampling, metadata, norm
    and cache kernels: no report. The same builds carry
    UndefinedBehaviorSanitizer (VLLT_HOST_UBSAN=1: signed overflow in index
    arithmetic, shifts, misaligned or null accesses, out-of-range
    conversions stop the process); the whole host suite also passes with it.

Found this way: the split-K GEMM's TMA producer read a failure flag that
the MMA issuer could be writing, to decide whether to wait for its copies
in flight before the CTA exits (it now always waits for them, which costs
nothing when nothing failed); the abort flag the roles of the warp-specialized
kernels poll is now read and written through flag_read / flag_write
(volatile on the device, a relaxed atomic here).
"""

import os
import subprocess
import sys

import pytest

from tests.conftest import needs_vllmlite
from tests.host_build import build_harness, tsan_runtime

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
TSAN = tsan_runtime()
pytestmark = pytest.mark.skipif(TSAN is None, reason="g++ has no ThreadSanitizer runtime")


# The two sanitizer runtimes see each other: UBSan's runtime probes memory
# through a pipe when a thread exits, and ThreadSanitizer's pipe interceptor
# reports those probes of two exiting threads as a race.
SUPPRESSIONS = "race:__sanitizer::IsAccessibleMemoryRange\n"


def tsan_env(log_path=None, tmp=None):
    opts = "exitcode=66:history_size=3:report_signal_unsafe=0" + (f":log_path={log_path}" if log_path else "")
    if tmp is not None:
        sup = os.path.join(str(tmp), "tsan.supp")
        with open(sup, "w") as f:
            f.write(SUPPRESSIONS)
        opts += f":suppressions={sup}"
    env = dict(os.environ, LD_PRELOAD=TSAN, VLLT_HOST_TSAN="1", VLLT_HOST_UBSAN="1",
               VLLT_SIMT_THREADS=str(os.cpu_count() or 4),
               # no BLAS worker threads: the builds fork, and the sanitizer's
               # fork handling trips over BLAS's pthread_join at fork
               OPENBLAS_NUM_THREADS="1", OMP_NUM_THREADS="1", MKL_NUM_THREADS="1",
               TSAN_OPTIONS=opts,
               PYTHONPATH=os.pathsep.join([ROOT, os.path.join(ROOT, "vllm-lite_b200"),
                                           os.path.join(ROOT, "baseline", "_ref")]))
    return env


RUN_CASE = """
import ctypes as C, sys
import numpy as np
L = C.CDLL(sys.argv[1])
out = np.zeros(256, np.int32)
rc = getattr(L, "race_" + sys.argv[2])(int(sys.argv[3]), out.ctypes.data_as(C.c_void_p))
sys.exit(0 if rc else 3)
"""


@pytest.mark.parametrize("case,line", [("neighbour", "race_host.cpp:16"), ("count", "race_host.cpp:27"),
                                       ("mbarrier", "race_host.cpp:42")])
def test_planted_races_are_reported_and_ordered_kernels_are_not(tmp_path, case, line):
    lib = build_harness("race_host", str(tmp_path), tsan=True, load=False)
    for ordered in (1, 0):
        r = subprocess.run([sys.executable, "-c", RUN_CASE, lib, case, str(ordered)], env=tsan_env(tmp=tmp_path),
                           capture_output=True, text=True, timeout=300)
        if ordered:
            assert r.returncode == 0 and "ThreadSanitizer" not in r.stderr, r.stderr[-3000:]
        else:
            assert r.returncode == 66 and "data race" in r.stderr, (r.returncode, r.stderr[-3000:])
            assert line in r.stderr.split("SUMMARY:")[1].splitlines()[0], r.stderr[-3000:]


# A sample of the host tests' cases that reaches every kernel form; each is
# the same test as in the regular suite, run in a child process with the
# instrumented builds.
CASES = [
    "tests/test_gemm_bf16_host.py::test_persistent_kernel_matches_float64[300-520-512]",
    "tests/test_gemm_bf16_host.py::test_split_k_kernel_matches_float64_and_is_reusable[64-256-256-3]",
    "tests/test_gemm_bf16_host.py::test_small_m_forms_match_float64[100-1024-1024-cluster]",
    "tests/test_gemm_bf16_host.py::test_small_m_forms_match_float64[37-10240-1024-stream-k]",
    "tests/test_gemm_bf16_host.py::test_a_dropped_tma_load_reports_and_recovers[130-520-1024-4]",
    "tests/test_gemm_bf16_host.py::test_a_dropped_tma_load_reports_and_recovers[100-1024-1024-0]",
    "tests/test_prefill_tc_host.py::test_prefill_kernel_against_float64_and_the_generic_kernel[8-8]",
    "tests/test_prefill_tc_host.py::test_prefill_kernel_dropped_load_reports_and_recovers",
    "tests/test_capi_host.py::test_decode_stall_injection_reports_and_recovers",
    "tests/test_capi_host.py::test_noalloc_entry_is_bit_identical_to_the_workspace_entry",
    "tests/test_kernels_host.py::test_greedy_kernel_on_reference_cases[schedule-default-264-end]",
    "tests/test_kernels_host.py::test_top_p_kernel_on_the_reference_sampler_fixture[schedule-default]",
    "tests/test_kernels_host.py::test_accept_kernel_on_reference_verify_cases[schedule-default]",
    "tests/test_kernels_host.py::test_rmsnorm_kernel_against_the_oracle[schedule-default-64]",
    "tests/test_kernels_host.py::test_embed_and_rope_kernels_against_the_oracle[schedule-default]",
    "tests/test_kernels_host.py::test_bf16_embed_and_fused_add_rmsnorm[schedule-default]",
    "tests/test_kernels_host.py::test_argmax_rows_kernel[schedule-default-264]",
    "tests/test_kernels_host.py::test_reshape_and_cache_and_copy_blocks[schedule-default-1]",
    "tests/test_kernels_host.py::test_generic_attention_kernel_against_float64"
    "[schedule-default-8-4-48-16-qlens0-ctxs0-1-1]",  # decode rows, split-K past 512 keys
    "tests/test_kernels_host.py::test_generic_attention_kernel_against_float64"
    "[schedule-default-8-4-48-16-qlens1-ctxs1-0-1]",  # prefill tiles mixed with decode rows
    "tests/test_kernels_host.py::test_sgemm_store_and_residual[schedule-default-True-40]",  # split-K counters
    "tests/test_kernels_host.py::test_sgemm_qkv_epilogue[schedule-default-8-4-48-16]",
]


@needs_vllmlite
def test_library_kernels_have_no_data_race(tmp_path):
    log = str(tmp_path / "tsan")
    r = subprocess.run([sys.executable, "-m", "pytest", "-q", "-x", "-p", "no:cacheprovider", *CASES],
                       cwd=ROOT, env=tsan_env(log, tmp_path), capture_output=True, text=True, timeout=1800)
    reports = ""
    for f in sorted(os.listdir(tmp_path)):
        if f.startswith("tsan") and not f.endswith(".supp"):
            reports += open(tmp_path / f, errors="replace").read()
    assert r.returncode == 0, (r.stdout[-3000:], r.stderr[-3000:], reports[:6000])
    assert "ThreadSanitizer" not in reports, reports[:6000]
