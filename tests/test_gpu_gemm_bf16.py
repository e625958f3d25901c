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


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (1, 256, 64), (300, 520, 1024), (129, 4096, 512),
                                   (512, 768, 4096)])
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
