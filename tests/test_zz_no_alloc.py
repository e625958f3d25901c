"""GPU: the allocation-free attention entry point.

`vllt_paged_attention_varlen_noalloc` serves callers that cannot allocate
device memory (a framework allocator owns the GPU, a hard memory cap, or a hot
loop where cudaMalloc's device synchronization is not acceptable). It keeps
its split-K scratch in a static device array inside the library. Here it is
called through the C ABI, twice in a row on different inputs (the array keeps
the previous call's contents), and each output must equal, bit for bit, the
workspace-taking entry point `vllt_paged_attention_varlen` on the same inputs
(both run the same kernels with the same split-K decisions): the TMA decode
kernel's splits, the generic kernel's single-query splits and a mixed batch of
prefill tiles. An empty batch must still clear the caller's flag word. The file sorts last so a run that
stops at the first failure has already run every other test; it also passes
alone in a fresh process (the first call sets the scratch address up).
"""

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _case(rng, H, KV, D, bs, qlens, ctxs, dtype):
    nb_need = [(c + bs - 1) // bs for c in ctxs]
    total = sum(nb_need) + 5
    perm = rng.permutation(total)
    W = max(nb_need)
    tab = np.zeros((len(ctxs), W), np.int32)
    o = 0
    for i, n in enumerate(nb_need):
        tab[i, :n] = perm[o:o + n]
        o += n
    dev = torch.device("cuda", 0)
    kc = torch.randn((total, KV, bs, D), device=dev).to(dtype)
    vc = torch.randn((total, KV, bs, D), device=dev).to(dtype)
    q = torch.randn((sum(qlens), H, D), device=dev).to(dtype)
    cu = torch.tensor(np.concatenate([[0], np.cumsum(qlens)]), dtype=torch.int32, device=dev)
    return dict(q=q, kc=kc, vc=vc, tab=torch.from_numpy(tab).to(dev), W=W, cu=cu,
                ctx=torch.tensor(ctxs, dtype=torch.int32, device=dev), S=len(ctxs), T=sum(qlens),
                max_q=max(qlens), max_ctx=max(ctxs), H=H, KV=KV, D=D, bs=bs, nb=total,
                code=0 if dtype == torch.float32 else 1)


def _with_workspace(L, c):
    from vllt import _lib

    n = L.vllt_attention_workspace_bytes(c["S"], c["H"], c["D"], c["max_ctx"])
    ws = torch.zeros(max(n, 256), dtype=torch.uint8, device=c["q"].device)
    out = torch.empty_like(c["q"])
    _lib.check(L.vllt_paged_attention_varlen(
        c["q"].data_ptr(), c["kc"].data_ptr(), c["vc"].data_ptr(), c["tab"].data_ptr(), c["W"], c["cu"].data_ptr(),
        c["ctx"].data_ptr(), c["S"], c["T"], c["max_q"], c["max_ctx"], c["H"], c["KV"], c["D"], c["bs"], c["nb"],
        float(1 / np.sqrt(c["D"])), c["code"], out.data_ptr(), ws.data_ptr(), ws.numel(), _lib.stream_handle()))
    return out


def _no_alloc(L, c, flags):
    from vllt import _lib

    out = torch.empty_like(c["q"])
    _lib.check(L.vllt_paged_attention_varlen_noalloc(
        c["q"].data_ptr(), c["kc"].data_ptr(), c["vc"].data_ptr(), c["tab"].data_ptr(), c["W"], c["cu"].data_ptr(),
        c["ctx"].data_ptr(), c["S"], c["T"], c["max_q"], c["max_ctx"], c["H"], c["KV"], c["D"], c["bs"], c["nb"],
        float(1 / np.sqrt(c["D"])), c["code"], out.data_ptr(), flags.data_ptr(), _lib.stream_handle()))
    return out


@pytest.mark.parametrize("kind", ["bf16-decode", "f32-decode", "f32-mixed"])
def test_no_alloc_entry_matches_workspace_entry(kind):
    """Both entry points run the same kernels with the same split decisions
    (the static scratch and the caller's workspace both hold every split's
    partials), so the outputs must be bit-identical, call after call."""
    from vllt import _lib

    assert torch.cuda.is_available(), "needs a CUDA device"
    torch.cuda.set_device(0)
    L = _lib.lib()
    rng = np.random.default_rng(21)
    flags = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    for call in range(2):  # two calls in a row: the shared scratch must not leak between them
        if kind == "bf16-decode":  # TMA decode kernel, its split-K partials in the scratch
            c = _case(rng, 32, 8, 128, 16, [1] * 6, [4096, 1, 17, 1500 + call, 2048, 333], torch.bfloat16)
        elif kind == "f32-decode":  # generic kernel, single-query rows: 512-key split-K partials and merge
            c = _case(rng, 8, 4, 48, 16, [1] * 5, [1300, 600, 2048 + call, 1, 513], torch.float32)
        else:  # generic kernel, mixed query lengths (max_qlen 20): prefill tiles, no split
            c = _case(rng, 8, 4, 48, 16, [1, 7, 1, 20], [1300, 40, 900 + call, 20], torch.float32)
        want = _with_workspace(L, c)
        got = _no_alloc(L, c, flags)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(got.float().cpu().numpy(), want.float().cpu().numpy())
        assert int(flags.item()) == 0


def test_no_alloc_entry_clears_the_flag_word_of_an_empty_batch():
    from vllt import _lib

    L = _lib.lib()
    flags = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    _lib.check(L.vllt_paged_attention_varlen_noalloc(None, None, None, None, 1, None, None, 0, 0, 0, 0,
                                                     8, 4, 48, 16, 4, 0.1, 0, None, flags.data_ptr(),
                                                     _lib.stream_handle()))
    torch.cuda.synchronize()
    assert int(flags.item()) == 0


def test_no_alloc_entry_rejects_batches_beyond_its_scratch():
    from vllt import _lib

    L = _lib.lib()
    # 4096 single-query sequences of 32 heads at 4096 context need far more than 16 MiB
    rc = L.vllt_paged_attention_varlen_noalloc(None, None, None, None, 256, None, None, 4096, 4096, 1, 4096,
                                               32, 8, 128, 16, 100000, 0.088, 1, None, None, None)
    assert rc == _lib.VLLT_ERR_ARG
    assert b"static scratch" in L.vllt_last_error()
