"""CPU: libvllt's tcgen05 prefill attention kernel, its own code, on the host emulation.

Multi-token tiles of bf16 / head_dim 128 / block 16 go to the warp-specialized
tensor-core kernel (csrc/attention_prefill_tc.cu). Built for the host
(tests/host_build.py), its Q (3-D) and K/V (2-D) tensor-map loads, the S = Q K^T
and O += P V MMAs (V as an MN-major operand), the softmax warps' tensor-memory
loads and stores and its mbarriers run on the emulation of
tests/simt_include/simt_tc.h. The cases and bars are the GPU tests'
(tests/test_gpu_kernels.py::test_attention_prefill_tensor_core*), through
vllt_paged_attention_varlen:
  * GQA 1, 2, 4, 8: long prompts (several query and key tiles, diagonal
    masking), chunked prefill over a cached prefix, verify-sized rows and a
    single-token row in one launch, against the float64 oracle and (GQA 1 to
    4) against the generic CUDA-core kernel, which the same call takes
    without a workspace: rtol 2e-2, atol 2e-2;
  * scores that climb or fall by about 10 (log2 units) per 128-key tile, so
    the kernel moves its running max and rescales O in tensor memory;
  * the shuffled schedule; a dropped TMA load (bit 2 of the error word, the
    tensor memory freed, the next call clean and equal to a normal run).
"""

import ctypes as C

import numpy as np
import pytest

from oracle import attention as A
from tests.guarded import guarded, ptr

torch = pytest.importorskip("torch")

D, BS = 128, 16


@pytest.fixture
def L(host_library):
    host_library.vllt_host_drop_tma.argtypes = [C.c_int64]
    host_library.vllt_host_schedule_seed.argtypes = [C.c_uint64]
    host_library.vllt_host_mma_count.restype = C.c_int64
    return host_library


def bf16_bits(x):
    return torch.from_numpy(np.ascontiguousarray(x, np.float32)).bfloat16().view(torch.int16).numpy().view(np.uint16)


def from_bits(b):
    return (b.astype(np.uint32) << 16).view(np.float32)


def attend(L, q, ck, cv, tab, qlens, ctxs, H, KV, workspace=True):
    """vllt_paged_attention_varlen on bf16 inputs; returns (out as float32, error word)."""
    from tests.test_gpu_kernels import to_lib_layout
    from vllt import _lib

    cu = np.concatenate([[0], np.cumsum(qlens)]).astype(np.int32)
    S, T = len(ctxs), int(cu[-1])
    kc, vc = to_lib_layout(ck, BS), to_lib_layout(cv, BS)
    out = guarded(np.zeros((T, H, D), np.uint16))
    ws = None
    if workspace:
        ws = guarded(np.zeros(max(L.vllt_attention_workspace_bytes(S, H, D, max(ctxs)), 256), np.uint8))
    rc = L.vllt_paged_attention_varlen(ptr(guarded(bf16_bits(q))), ptr(guarded(bf16_bits(kc))),
                                       ptr(guarded(bf16_bits(vc))), ptr(guarded(tab)), tab.shape[1], ptr(guarded(cu)),
                                       ptr(guarded(np.asarray(ctxs, np.int32))), S, T, max(qlens), max(ctxs), H, KV, D,
                                       BS, kc.shape[0], 1.0 / np.sqrt(D), _lib.VLLT_BF16, ptr(out),
                                       ptr(ws) if workspace else None, ws.size if workspace else 0, None)
    assert rc == 0, L.vllt_last_error()
    return from_bits(out), (int(ws[:4].view(np.int32)[0]) if workspace else 0)


def check_oracle(got, q, ck, cv, tables, qlens, ctxs, KV):
    cu = np.concatenate([[0], np.cumsum(qlens)])
    for i, c in enumerate(ctxs):
        slots = A.table_slots(tables[i], BS, c)
        want = A.dense_attention(q[cu[i]:cu[i + 1]], ck[slots], cv[slots], KV, 1.0 / np.sqrt(D))
        np.testing.assert_allclose(got[cu[i]:cu[i + 1]], want, rtol=2e-2, atol=2e-2, err_msg=f"seq {i}")


QLENS, CTXS = [300, 64, 5, 1, 129, 9], [300, 1000, 260, 77, 129, 2049]


@pytest.mark.parametrize("H,KV", [(32, 8), (8, 8), (16, 8), (64, 8)])
def test_prefill_kernel_against_float64_and_the_generic_kernel(L, H, KV):
    from tests.test_gpu_kernels import ragged_batch

    rng = np.random.default_rng(H + 7)
    q, ck, cv, tables, tab = ragged_batch(rng, H, KV, D, BS, QLENS, CTXS, "bf16")
    n0 = L.vllt_host_mma_count()
    got, err = attend(L, q, ck, cv, tab, QLENS, CTXS, H, KV)
    assert err == 0 and L.vllt_host_mma_count() > n0  # the tensor-core kernel ran
    check_oracle(got, q, ck, cv, tables, QLENS, CTXS, KV)
    if H <= 32:  # (the generic kernel's 2-position tiles of GQA 8 are slow to emulate)
        generic, _ = attend(L, q, ck, cv, tab, QLENS, CTXS, H, KV, workspace=False)
        np.testing.assert_allclose(got, generic, rtol=2e-2, atol=2e-2)


def test_prefill_kernel_rescales_on_rising_scores(L):
    from tests.test_gpu_kernels import ragged_batch

    rng = np.random.default_rng(11)
    H, KV = 32, 8
    qlens, ctxs = [700, 300, 200], [700, 300, 456]
    q, ck, cv, tables, tab = ragged_batch(rng, H, KV, D, BS, qlens, ctxs, "bf16")
    u = rng.standard_normal((KV, D))
    u *= np.sqrt(D) / np.linalg.norm(u, axis=1, keepdims=True)
    ramps = [lambda t: 0.005 * t, lambda t: 0.005 * (300 - t), lambda t: 0.004 * t]
    for i, c in enumerate(ctxs):
        for t in range(c):
            slot = tables[i][t // BS] * BS + t % BS
            ck[slot] = u * ramps[i](t) + 0.1 * rng.standard_normal((KV, D))
    cu = np.concatenate([[0], np.cumsum(qlens)])
    for i in range(len(qlens)):
        q[cu[i]:cu[i + 1]] = np.repeat(u, H // KV, axis=0)[None] + 0.1 * rng.standard_normal((qlens[i], H, D))
    r = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.float32)).bfloat16().float().numpy()
    q, ck = r(q), r(ck)
    got, err = attend(L, q, ck, cv, tab, qlens, ctxs, H, KV)
    assert err == 0
    check_oracle(got, q, ck, cv, tables, qlens, ctxs, KV)


def test_prefill_kernel_under_the_shuffled_schedule(L):
    from tests.test_gpu_kernels import ragged_batch

    rng = np.random.default_rng(3)
    H, KV, qlens, ctxs = 16, 8, [200, 7, 1], [330, 600, 40]
    q, ck, cv, tables, tab = ragged_batch(rng, H, KV, D, BS, qlens, ctxs, "bf16")
    base, _ = attend(L, q, ck, cv, tab, qlens, ctxs, H, KV)
    L.vllt_host_schedule_seed(0xC0FFEE)
    try:
        got, err = attend(L, q, ck, cv, tab, qlens, ctxs, H, KV)
    finally:
        L.vllt_host_schedule_seed(0)
    assert err == 0
    np.testing.assert_array_equal(got, base)


def test_prefill_kernel_dropped_load_reports_and_recovers(L):
    from tests.test_gpu_kernels import ragged_batch

    rng = np.random.default_rng(4)
    H, KV, qlens, ctxs = 32, 8, [150, 3], [400, 900]
    q, ck, cv, tables, tab = ragged_batch(rng, H, KV, D, BS, qlens, ctxs, "bf16")
    clean, _ = attend(L, q, ck, cv, tab, qlens, ctxs, H, KV)
    L.vllt_host_drop_tma(5)
    try:
        _, err = attend(L, q, ck, cv, tab, qlens, ctxs, H, KV)
    finally:
        L.vllt_host_drop_tma(0)
    assert err & 4
    again, err = attend(L, q, ck, cv, tab, qlens, ctxs, H, KV)
    assert err == 0
    np.testing.assert_array_equal(again, clean)
