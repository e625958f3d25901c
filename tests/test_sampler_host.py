"""CPU: the device sampler's algorithm against the reference's sample().

top_p_kernel (csrc/sampling.cu) runs sampler_row.cuh with a CTA's reductions;
tests/sampler_host.cpp runs the same header on 256 host fibers that reduce
in the kernel's order (so the float32 sums are the kernel's). On the
96 rows of sampling_full.npz (written by the reference's sample(): EOS masks,
repetition penalties, temperatures, top-k from 0 to beyond the vocabulary,
top-p from 0.2 to 1) the host-compiled sampler must keep the reference's keep
set and, given the uniform the reference's generator handed numpy's choice(),
pick the reference's token, except where u lies within 1e-5 of a CDF
boundary (float32 sums in another order). Beyond the fixture, rows of the
Llama-3 vocabulary (128256) with top-k of 1, 50 and vocab - 1, a nucleus of
one token and a row with every token but one at -inf are checked against the
oracle's restatement (oracle.sampling.sample_with_uniform): the top-k
bisection over the full 32-bit key range must end and keep exactly k tokens.
"""

import ctypes

import numpy as np
import pytest

from oracle import sampling as SP
from tests.test_oracle_golden import full_sampling_rows


@pytest.fixture(scope="module")
def sampler(tmp_path_factory):
    from tests.host_build import build_harness

    lib = build_harness("sampler_host", str(tmp_path_factory.mktemp("sampler")))
    if lib is None:
        pytest.skip("g++ is not available")
    f = lib.sample_row_host
    f.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_void_p,
                  ctypes.c_float, ctypes.c_int, ctypes.c_float, ctypes.c_double, ctypes.c_void_p]
    return f


def run(sampler, x, temperature, top_k, top_p, u, mask_eos=0, eos_id=0, penalty=1.0, bits=None):
    x = np.ascontiguousarray(x, np.float32)
    keep = np.zeros(x.size, np.uint8)
    tok = sampler(x.ctypes.data, x.size, mask_eos, eos_id, penalty, bits.ctypes.data if bits is not None else None,
                  temperature, top_k, top_p, u, keep.ctypes.data)
    assert tok >= 0  # -2: the CTA's threads disagreed; -3: they met different barriers
    return tok, keep.astype(bool)


def test_kernel_sampler_matches_reference_sample(sampler):
    from vllt.engine import seen_bitmaps

    exact = keep_equal = n = 0
    for i, row, kw, pick, keep, probs in full_sampling_rows():
        x = np.ascontiguousarray(row, np.float32)
        bits = seen_bitmaps([type("S", (), {"token_ids": list(kw["seen"])})()], x.size)[0]
        mask = int(kw["num_generated"] < kw["min_tokens"])
        got_keep = np.zeros(x.size, np.uint8)
        tok = sampler(x.ctypes.data, x.size, mask, kw["eos_id"], kw["penalty"], bits.ctypes.data,
                      kw["temperature"], kw["top_k"], kw["top_p"], kw["u"], got_keep.ctypes.data)
        assert tok >= 0 and keep[tok], (i, tok)
        keep_equal += bool((got_keep.astype(bool) == keep).all())
        cdf = np.cumsum(probs.astype(np.float64))
        cdf /= cdf[-1]
        if np.abs(cdf - kw["u"]).min() > 1e-5:
            assert tok == pick, (i, tok, pick)
            exact += 1
        n += 1
    assert n == 96 and exact >= n - 2 and keep_equal == n


@pytest.mark.parametrize("top_k,top_p", [(1, 1.0), (50, 1.0), (128255, 1.0), (0, 0.9), (50, 0.8), (0, 1e-6)])
def test_kernel_sampler_llama3_vocabulary(sampler, top_k, top_p):
    rng = np.random.default_rng(top_k + int(top_p * 100))
    x = (rng.standard_normal(128256) * 3).astype(np.float32)
    for u in (0.0, 0.37, 0.999999):
        tok, keep = run(sampler, x, 0.8, top_k, top_p, u)
        want, want_keep, _ = SP.sample_with_uniform(x, 0.8, top_k, top_p, u)
        np.testing.assert_array_equal(keep, want_keep)
        assert tok == want
        if 0 < top_k and top_p == 1.0:
            assert keep.sum() == top_k  # distinct values: exactly k kept
        if top_p == 1e-6:
            assert keep.sum() == 1 and keep[np.argmax(x)]


def test_kernel_sampler_single_finite_token(sampler):
    x = np.full(4096, -np.inf, np.float32)
    x[1234] = -5.0
    for k, p in ((0, 1.0), (1, 1.0), (7, 0.5)):
        tok, keep = run(sampler, x, 1.3, k, p, 0.999)
        assert tok == 1234 and keep.tolist() == (np.arange(4096) == 1234).tolist()
