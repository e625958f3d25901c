"""CPU: libvllt's tcgen05 bf16 GEMM kernels, their own code, on the host emulation.

tests/host_build.py builds gemm_bf16.cu and gemm_bf16_tc.cuh for the host: the
tensor-core, TMA, mbarrier and cluster instructions run on the emulation of
tests/simt_include/simt_tc.h, which decodes and checks the kernels' instruction
and shared-memory descriptors, tensor-memory allocations and lane quarters.
Every form is reached through the C ABI the GPU tests use
(tests/test_gpu_gemm_bf16.py), with the same bars:
  * the persistent kernel (one CTA per SM walking tiles, two TMEM
    accumulators), the split-K kernel (per-tile counters, partials summed in
    slice order), the small-M stream-K kernel with its slice-reduce kernel and
    the cluster split-K kernel (distributed shared-memory reduction);
  * against a float64 product of the same bf16 values: rtol 1e-3,
    atol 1e-3 * sqrt(K);
  * a second call on the same scratch gives the same bits (counters left at 0);
  * a dropped TMA load makes a bounded wait expire: the device error word
    reads 4, every CTA frees its tensor memory, the cluster form runs no
    epilogue for the tile whose CTA gave up, and the next call is clean.
"""

import ctypes as C

import numpy as np
import pytest

torch = pytest.importorskip("torch")


@pytest.fixture
def L(host_library):
    host_library.vllt_host_drop_tma.argtypes = [C.c_int64]
    host_library.vllt_host_schedule_seed.argtypes = [C.c_uint64]
    host_library.vllt_host_mma_count.restype = C.c_int64
    return host_library


def mma_delta(L, fn):
    """fn()'s result and the tcgen05.mma instructions it executed."""
    n0 = L.vllt_host_mma_count()
    r = fn()
    return r, L.vllt_host_mma_count() - n0


def bf16_pair(M, N, K, seed):
    g = torch.Generator().manual_seed(seed)
    A = torch.randn((M, K), generator=g).to(torch.bfloat16)
    W = torch.randn((N, K), generator=g).to(torch.bfloat16)
    return A, W, (A.double() @ W.double().T).numpy()


def run(L, A, W, splits=None, ws=None):
    """vllt_gemm_bf16 (splits None) or vllt_gemm_bf16_splitk; returns (C, flags, ws)."""
    M, K = A.shape
    N = W.shape[0]
    out = torch.full((M, N), float("nan"), dtype=torch.float32)
    flags = torch.zeros(1, dtype=torch.int32)
    if splits is None:
        rc = L.vllt_gemm_bf16(A.data_ptr(), W.data_ptr(), out.data_ptr(), M, N, K, flags.data_ptr(), None)
    else:
        if ws is None:
            ws = torch.zeros(L.vllt_gemm_bf16_splitk_workspace_bytes(M, N, K, splits), dtype=torch.uint8)
        rc = L.vllt_gemm_bf16_splitk(A.data_ptr(), W.data_ptr(), out.data_ptr(), M, N, K, splits, ws.data_ptr(),
                                     ws.numel(), flags.data_ptr(), None)
    assert rc == 0, L.vllt_last_error()
    return out.double().numpy(), int(flags[0]), ws


def close(got, want, K):
    np.testing.assert_allclose(got, want, rtol=1e-3, atol=1e-3 * np.sqrt(K))


# persistent kernel: one tile; one row; ragged edges; more tiles than SMs with
# one k-block per tile (ring phases and both accumulators carried across tiles)
@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (1, 256, 64), (300, 520, 512), (2000, 5120, 64)])
def test_persistent_kernel_matches_float64(L, M, N, K):
    A, W, want = bf16_pair(M, N, K, M * 7 + N + K)
    (got, flags, _), n = mma_delta(L, lambda: run(L, A, W))
    assert flags == 0
    close(got, want, K)
    assert n == -(-M // 128) * -(-N // 256) * (K // 16)  # every 128 x 256 tile, each K step once


@pytest.mark.parametrize("M,N,K,splits", [(64, 256, 256, 3), (130, 520, 1024, 16), (300, 768, 512, 5)])
def test_split_k_kernel_matches_float64_and_is_reusable(L, M, N, K, splits):
    A, W, want = bf16_pair(M, N, K, M + 3 * N + K + splits)
    (got, flags, ws), n = mma_delta(L, lambda: run(L, A, W, splits))
    assert flags == 0
    close(got, want, K)
    assert n == -(-M // 128) * -(-N // 256) * (K // 16)  # the slices cover K once
    again, flags, _ = run(L, A, W, splits, ws)
    assert flags == 0 and np.array_equal(got, again)
    unsplit, _, _ = run(L, A, W, 1)
    np.testing.assert_allclose(got, unsplit, rtol=1e-4, atol=1e-4 * np.sqrt(K))


# splits 0: the forward pass's choice. Few feature tiles: cluster split-K
# (auto_splits -S); many: stream-K over one CTA per SM, spans starting and
# ending inside tiles, reduced by the second kernel; M = 1 and token counts
# around the 32-row chunks
@pytest.mark.parametrize("M,N,K,form", [(100, 1024, 1024, "cluster"), (16, 6144, 4096, "cluster"),
                                        (200, 160, 640, "cluster"), (1, 2048, 2048, "cluster"),
                                        (37, 10240, 1024, "stream-k"), (64, 19968, 512, "stream-k")])
def test_small_m_forms_match_float64(L, M, N, K, form):
    s = L.vllt_gemm_bf16_auto_splits(M, N, K)
    assert (s < 0) if form == "cluster" else (s == 0)
    A, W, want = bf16_pair(M, N, K, M + N + K)
    (got, flags, ws), n = mma_delta(L, lambda: run(L, A, W, 0))
    assert flags == 0
    close(got, want, K)
    assert n == -(-N // 128) * (K // 16)  # every 128-feature tile, each K step once, over all CTAs
    again, flags, _ = run(L, A, W, 0, ws)
    assert flags == 0 and np.array_equal(got, again)


def test_forms_under_the_shuffled_schedule(L):
    """A random runnable thread continues after every barrier and every
    unfinished wait (seeded): the same bits as the default schedule."""
    cases = [((300, 520, 512), None), ((130, 520, 1024), 16), ((100, 1024, 1024), 0), ((37, 10240, 1024), 0)]
    base = []
    for (M, N, K), splits in cases:
        A, W, _ = bf16_pair(M, N, K, 5)
        base.append(run(L, A, W, splits)[0])
    L.vllt_host_schedule_seed(0x5EED)
    try:
        for ((M, N, K), splits), b in zip(cases, base):
            A, W, _ = bf16_pair(M, N, K, 5)
            got, flags, _ = run(L, A, W, splits)
            assert flags == 0 and np.array_equal(got, b)
    finally:
        L.vllt_host_schedule_seed(0)


@pytest.mark.parametrize("M,N,K,splits", [(300, 520, 512, None), (130, 520, 1024, 4), (100, 1024, 1024, 0),
                                          (37, 10240, 1024, 0)])
def test_a_dropped_tma_load_reports_and_recovers(L, M, N, K, splits):
    """The 3rd load of the launch never lands: its stage's wait expires (the
    emulated clock moves 1 us per poll, so the 1 s limit is a million polls),
    the error word reads 4, the CTAs free their tensor memory (the emulation
    fails the launch otherwise) and the next call is clean and correct."""
    A, W, want = bf16_pair(M, N, K, 11)
    L.vllt_host_drop_tma(3)
    try:
        got, flags, ws = run(L, A, W, splits)
    finally:
        L.vllt_host_drop_tma(0)
    assert flags == 4
    if splits == 0 and L.vllt_gemm_bf16_auto_splits(M, N, K) < 0:
        # cluster form: the tile of the CTA that gave up keeps its NaN fill (no
        # CTA of that cluster ran the epilogue), every other tile is right
        bad = np.isnan(got).any(axis=0)
        assert bad.sum() == 128 and not np.isnan(got[:, ~bad]).any()
        close(got[:, ~bad], want[:, ~bad], K)
    got, flags, _ = run(L, A, W, splits, ws)
    assert flags == 0
    close(got, want, K)


# The Llama-3-8B decode projections at the forward's own plan choices (the
# emulated device has a B200's 148 SMs): qkv, o_proj and down (K = 14,336) in
# the cluster form, gate/up (N = 28,672) in stream-K at 64 and 256 tokens, and
# the split-K form past 256 tokens.
@pytest.mark.parametrize("M,N,K,form", [(64, 6144, 4096, "cluster"), (64, 4096, 4096, "cluster"),
                                        (64, 28672, 4096, "stream-k"), (64, 4096, 14336, "cluster"),
                                        (256, 28672, 4096, "stream-k"), (512, 4096, 14336, "split-k")])
def test_llama_decode_projection_shapes(L, M, N, K, form):
    s = L.vllt_gemm_bf16_auto_splits(M, N, K)
    assert {"cluster": s < 0, "stream-k": s == 0, "split-k": s > 1}[form], s
    A, W, want = bf16_pair(M, N, K, N + K)
    (got, flags, ws), n = mma_delta(L, lambda: run(L, A, W, 0))
    assert flags == 0
    close(got, want, K)
    rows = -(-M // 128) if form == "split-k" else 1  # split-K tiles are 128 x 256, the swapped forms 128 features
    assert n == (rows * -(-N // 256) if form == "split-k" else -(-N // 128)) * (K // 16)
