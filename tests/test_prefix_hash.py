"""CPU: the device prefix-cache hash.

csrc/prefix_hash.cuh holds the hashing code of the vllt_prefix_hash_chains
kernel as __host__ __device__ functions; tests/prefix_hash_host.cpp compiles
the same header for the host (g++), so these tests run the exact functions the
kernel runs:
  * every digest equals the reference's hash_block (vllmlite/block.py:34-40)
    for chained blocks of 1 to 64 tokens, token ids up to int32's range, with
    and without a previous block (messages of one and several BLAKE2b blocks);
  * chains packed by vllt.prefix_hash.pack_chains come back in order;
  * GpuLLMEngine with device_prefix_hash=True gives the reference engine's
    token streams and prefix-cache hits on a shared-prefix workload (with and
    without speculation). Its hashes come from vllt_prefix_hash_chains itself
    (the library's entry point and kernel, built for the host on the SIMT
    emulation, tests/host_build.py), and every hash the BlockManager asks
    for is planned ahead (no on-the-spot launches).
"""

import ctypes

import numpy as np
import pytest

from tests.conftest import needs_vllmlite

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def host_hash(tmp_path_factory):
    from tests.host_build import build_harness

    lib = build_harness("prefix_hash_host", str(tmp_path_factory.mktemp("ph")))
    if lib is None:
        pytest.skip("g++ is not available")
    lib.hash_chain_host.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    return lib


def chain_host(lib, prev, toks, bs):
    toks = np.ascontiguousarray(toks, np.int32)
    n = toks.size // bs
    out = ctypes.create_string_buffer(32 * max(n, 1))
    pv = ctypes.create_string_buffer(prev.encode(), 32) if prev else None
    lib.hash_chain_host(ctypes.cast(pv, ctypes.c_void_p) if pv else None, toks.ctypes.data, n, bs, out)
    return [out.raw[32 * b:32 * b + 32].decode() for b in range(n)]


@needs_vllmlite
@pytest.mark.parametrize("bs", [1, 4, 16, 64])
def test_host_compiled_kernel_code_matches_hash_block(host_hash, bs):
    from vllmlite.block import hash_block

    rng = np.random.default_rng(bs)
    for trial in range(20):
        hi = (261, 128256, 2**31 - 1)[trial % 3]
        toks = rng.integers(0, hi, size=bs * 6).astype(np.int32)
        prev = None if trial % 2 else hash_block(None, (1, 2, 3))
        got = chain_host(host_hash, prev, toks, bs)
        want, p = [], prev
        for b in range(6):
            p = hash_block(p, tuple(int(t) for t in toks[b * bs:(b + 1) * bs]))
            want.append(p)
        assert got == want


def test_pack_chains_layout():
    from vllt.prefix_hash import pack_chains, unpack_digests

    chains = [(None, [1, 2, 3, 4]), ("a" * 32, [5, 6]), (None, [])]
    tokens, tok_off, nblk, out_off, prev, total = pack_chains(chains, 2)
    assert tokens.tolist() == [1, 2, 3, 4, 5, 6] and tok_off.tolist() == [0, 4, 6]
    assert nblk.tolist() == [2, 1, 0] and out_off.tolist() == [0, 2, 3] and total == 3
    assert not prev[0].any() and bytes(prev[1]) == b"a" * 32
    raw = np.frombuffer(b"".join(bytes([48 + i]) * 32 for i in range(3)), np.uint8)
    assert unpack_digests(raw, nblk) == [["0" * 32, "1" * 32], ["2" * 32], []]
    with pytest.raises(ValueError):
        pack_chains([(None, [1, 2, 3])], 2)  # a partial block


@needs_vllmlite
@pytest.mark.parametrize("spec_k", [0, 4])
def test_engine_with_device_prefix_hash_matches_reference(host_library, spec_k, monkeypatch):
    from vllmlite.engine import LLMEngine
    from vllmlite.sequence import SamplingParams

    import vllt._lib as _lib
    from tests import fixtures as F
    from tests.test_engine_host import OracleLib, ReferenceLogitsRunner, run
    from vllt.engine import GpuLLMEngine, cuda_engine
    from vllt.prefix_hash import DevicePrefixHasher
    from vllt.workloads import mixed_lengths

    monkeypatch.setattr(_lib, "stream_handle", lambda stream=None: 0)

    class Lib(OracleLib):
        def vllt_prefix_hash_chains(self, *args):  # the library's own entry point, built for the host
            return host_library.vllt_prefix_hash_chains(*args)

    from vllmlite.config import CacheConfig, EngineConfig, ModelConfig, SchedulerConfig

    def cfg():
        return EngineConfig(model=ModelConfig(vocab_size=261, **dict(F.TINY, max_seq_len=768)),
                            cache=CacheConfig(block_size=4, num_blocks=2048, enable_prefix_caching=True),
                            scheduler=SchedulerConfig(max_seqs=8, max_batched_tokens=128))

    p = SamplingParams(max_tokens=12, temperature=0.0, ignore_eos=True)
    reqs = [(f"r{i}", ids[:90], p) for i, (ids, _) in enumerate(mixed_lengths(12, 1, shared_prefix=40))]
    want_eng = LLMEngine(cfg(), None, spec_k)
    want = run(want_eng, reqs)
    lib = Lib()
    eng = cuda_engine(cfg(), speculative_tokens=spec_k, engine_cls=GpuLLMEngine.resolve(),
                      runner_cls=ReferenceLogitsRunner, lib=lib)
    eng.prefix_hasher = DevicePrefixHasher(eng, lib=lib)
    got = run(eng, reqs)
    assert got == want
    a, b = eng.scheduler.blocks.allocator, want_eng.scheduler.blocks.allocator
    assert (a.hits, a.misses) == (b.hits, b.misses) and a.hits > 0
    h = eng.prefix_hasher
    assert h.lookups > 100 and h.planned >= h.lookups / 2 and h.misses == 0
