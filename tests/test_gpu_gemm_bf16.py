"""GPU: the tcgen05 bf16 GEMM (D = A . W^T, fp32 accumulate) through the C ABI.

Checked against a float64 product of the same bf16 values; the tolerance covers
fp32 accumulation-order differences only (rtol 1e-3, atol 1e-3 * sqrt(K)).
"""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def gemm(A, W):
    from vllt import _lib

    M, K = A.shape
    N = W.shape[0]
    C = torch.full((M, N), float("nan"), dtype=torch.float32, device=A.device)
    flags = torch.zeros(1, dtype=torch.int32, device=A.device)
    _lib.check(_lib.lib().vllt_gemm_bf16(A.data_ptr(), W.data_ptr(), C.data_ptr(), M, N, K, flags.data_ptr(),
                                         _lib.stream_handle()))
    torch.cuda.synchronize()
    assert int(flags.item()) == 0
    return C


# the last three give the persistent kernel several tiles per CTA (both TMEM
# accumulators, ring phases carried across tiles, fewer k-blocks than stages)
@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (1, 256, 64), (300, 520, 1024), (129, 4096, 512),
                                   (512, 768, 4096), (1024, 8192, 256), (4096, 4096, 128), (2000, 6144, 1024)])
def test_gemm_bf16_matches_float64(M, N, K):
    g = torch.Generator(device="cuda").manual_seed(M * 7 + N + K)
    A = torch.randn((M, K), generator=g, device="cuda").to(torch.bfloat16)
    W = torch.randn((N, K), generator=g, device="cuda").to(torch.bfloat16)
    got = gemm(A, W).cpu().double().numpy()
    want = (A.double() @ W.double().T).cpu().numpy()
    np.testing.assert_allclose(got, want, rtol=1e-3, atol=1e-3 * np.sqrt(K))


def test_gemm_bf16_rejects_bad_k():
    from vllt import _lib

    rc = _lib.lib().vllt_gemm_bf16(None, None, None, 4, 4, 100, None, None)
    assert rc == _lib.VLLT_ERR_ARG


def gemm_splitk(A, W, splits, ws=None):
    from vllt import _lib

    L = _lib.lib()
    M, K = A.shape
    N = W.shape[0]
    C = torch.full((M, N), float("nan"), dtype=torch.float32, device=A.device)
    flags = torch.zeros(1, dtype=torch.int32, device=A.device)
    if ws is None:
        ws = torch.zeros(L.vllt_gemm_bf16_splitk_workspace_bytes(M, N, K, splits), dtype=torch.uint8,
                         device=A.device)
    _lib.check(L.vllt_gemm_bf16_splitk(A.data_ptr(), W.data_ptr(), C.data_ptr(), M, N, K, splits, ws.data_ptr(),
                                       ws.numel(), flags.data_ptr(), _lib.stream_handle()))
    torch.cuda.synchronize()
    assert int(flags.item()) == 0
    return C, ws


@pytest.mark.parametrize("M,N,K,splits", [(1, 4096, 4096, 8), (37, 6144, 4096, 6), (256, 4096, 14336, 4),
                                          (130, 520, 1024, 16), (64, 256, 256, 3)])
def test_gemm_bf16_split_k_matches_float64_and_is_reusable(M, N, K, splits):
    g = torch.Generator(device="cuda").manual_seed(M + N * 3 + K + splits)
    A = torch.randn((M, K), generator=g, device="cuda").to(torch.bfloat16)
    W = torch.randn((N, K), generator=g, device="cuda").to(torch.bfloat16)
    want = (A.double() @ W.double().T).cpu().numpy()
    got, ws = gemm_splitk(A, W, splits)
    np.testing.assert_allclose(got.cpu().double().numpy(), want, rtol=1e-3, atol=1e-3 * np.sqrt(K))
    # counters left at zero: a second call on the same scratch gives the same bits
    again, _ = gemm_splitk(A, W, splits, ws)
    assert torch.equal(got, again)
    # close to the unsplit kernel (only the fp32 summation order differs)
    np.testing.assert_allclose(got.cpu().numpy(), gemm(A, W).cpu().numpy(), rtol=1e-4, atol=1e-4 * np.sqrt(K))


# the small-M forms (splits 0): cluster split-K when the feature tiles are few
# (auto_splits < 0), stream-K otherwise (auto_splits == 0); spans that start
# and end inside tiles, several tiles per CTA, token counts around the 32-row
# chunks, M = 1
@pytest.mark.parametrize("M,N,K", [(1, 4096, 4096), (16, 6144, 4096), (37, 4096, 14336), (64, 28672, 4096),
                                   (100, 1024, 1024), (256, 4096, 4096), (200, 160, 640), (129, 128256, 4096)])
def test_gemm_bf16_small_m_forms_match_float64(M, N, K):
    from vllt import _lib

    assert _lib.lib().vllt_gemm_bf16_auto_splits(M, N, K) <= 0
    test_gemm_bf16_split_k_matches_float64_and_is_reusable(M, N, K, 0)


def test_gemm_bf16_forward_form_choice():
    from vllt import _lib

    L = _lib.lib()
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    # decode projections with few feature tiles: cluster split-K (-S CTAs per tile,
    # all clusters resident at once); qkv's 48 tiles may fall back to stream-K
    for M, N, K in [(64, 4096, 14336), (256, 4096, 4096), (16, 6144, 4096)]:
        s = L.vllt_gemm_bf16_auto_splits(M, N, K)
        assert s <= 0 and -s * (N // 128) <= sms and -s <= 8
        assert s < 0 or N == 6144
    # many feature tiles: stream-K; 512-row batches with few tiles split K; prefill does neither
    assert L.vllt_gemm_bf16_auto_splits(64, 28672, 4096) == 0
    assert L.vllt_gemm_bf16_auto_splits(256, 128256, 4096) == 0
    assert L.vllt_gemm_bf16_auto_splits(512, 4096, 4096) > 1
    assert L.vllt_gemm_bf16_auto_splits(8192, 4096, 4096) == 1
    for M, N, K in [(512, 6144, 4096), (512, 4096, 14336)]:
        s = L.vllt_gemm_bf16_auto_splits(M, N, K)
        tiles = -(-N // 256) * -(-M // 128)
        assert s * tiles <= sms and s <= K // 64 // 4


def test_gemm_bf16_split_k_rejects_more_slices_than_k_blocks():
    from vllt import _lib

    rc = _lib.lib().vllt_gemm_bf16_splitk(None, None, None, 4, 256, 128, 3, None, 0, None, None)
    assert rc == _lib.VLLT_ERR_ARG
