"""Test infrastructure: a pytest plugin that puts libvllt's runner behind the
reference's own engine tests (tests/test_reference_suite_host.py loads it into
a pytest run over the reference's test files).

At configure time it builds libvllt for the host (host_build.py) and makes
`vllmlite.engine.NumpyRunner`, the runner `LLMEngine.__init__` constructs
(vllmlite/engine.py:46), build a HostRunner (host_runner.py): CudaRunner's
packer, descriptor and flag checks over the library's compiled forward. That
is the one-line backend switch a maintainer would add, so every LLMEngine the
reference's tests build runs its passes through libvllt's code. With
VLLT_REFSUITE_ENGINE=gpu (or gpu-run-ahead) `vllmlite.engine.LLMEngine`
itself becomes the product's GpuLLMEngine (device token picks; run-ahead on or
off), which the tests then construct in its place. The reference's
hash_block (vllmlite/block.py:34), which the BlockManager's prefix cache and
the block tests call, becomes the device prefix hash's own code
(csrc/prefix_hash.cuh, the function vllt_prefix_hash_chains runs per block)
compiled for the host. And the reference's paged_attention
(vllmlite/attention.py:59), which its attention tests call, becomes
vllt.ops.paged_attention, the NumPy-signature drop-in, over the host build's
C ABI. Requests without a seed draw from a generator seeded with a fixed
value instead of fresh entropy (LLMEngine.add_request, engine.py:81): the HTTP
tests sample at temperature 1.0 without a seed and count the tokens they get
back, so with entropy a sampled EOS would end one early now and then, whatever
the runner. Imported as a
top-level module (this directory on sys.path), since the reference's tests
own the package name `tests`.
"""

import os
import tempfile

_STATE = {}


def pytest_configure(config):
    import host_build
    import host_runner

    prebuilt = os.environ.get("VLLT_REFSUITE_LIB")  # a host build made by the calling test session
    lib = (host_build.load_library_host(prebuilt) if prebuilt else
           host_build.build_library_host(os.environ.get("VLLT_REFSUITE_BUILD") or tempfile.mkdtemp()))
    if lib is None:
        raise RuntimeError("g++ is not available")
    host_runner.HostRunner.lib = lib
    import vllt._lib as _lib
    import vllmlite.engine as E
    from types import SimpleNamespace

    _lib.stream_handle = lambda stream=None: 0  # the host build has no streams
    # LLMEngine passes only the model and cache configs (engine.py:46); the
    # capacities cover the reference tests' scheduler settings
    sched = SimpleNamespace(max_seqs=64, max_batched_tokens=4096)

    def runner(model_cfg, cache_cfg):
        r = host_runner.HostRunner(model_cfg, cache_cfg, sched)
        _STATE["passes"] = _STATE.get("passes", 0)
        _STATE.setdefault("runners", []).append(r)
        return r

    _STATE["orig"] = E.NumpyRunner
    E.NumpyRunner = runner
    _patch_hash_block(host_build)
    _patch_paged_attention(lib)
    _seed_unseeded_requests(E)
    mode = os.environ.get("VLLT_REFSUITE_ENGINE", "reference")
    if mode != "reference":  # the product's engine in LLMEngine's place: device picks
        from vllt.engine import GpuLLMEngine

        cls = GpuLLMEngine.resolve()
        cls.run_ahead = mode == "gpu-run-ahead"
        E.LLMEngine = cls


def _patch_hash_block(host_build):
    import ctypes

    import vllmlite.block as B
    import vllmlite.block_manager as BM
    import numpy as np

    lib = host_build.build_harness("prefix_hash_host", os.environ.get("VLLT_REFSUITE_BUILD") or tempfile.mkdtemp())
    lib.hash_chain_host.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]

    def hash_block(prev_hash, token_ids):
        toks = np.ascontiguousarray(np.asarray(token_ids, np.int64).astype(np.int32))
        out = ctypes.create_string_buffer(32)
        prev = ctypes.create_string_buffer(prev_hash.encode(), 32) if prev_hash else None
        lib.hash_chain_host(ctypes.cast(prev, ctypes.c_void_p) if prev else None, toks.ctypes.data if toks.size else None,
                            1, int(toks.size), out)
        _STATE["hashes"] = _STATE.get("hashes", 0) + 1
        return out.raw.decode()

    B.hash_block = BM.hash_block = hash_block


def _patch_paged_attention(lib):
    import vllmlite.attention as A
    import vllt._lib as _lib
    import vllt.ops as ops

    _lib._lib = lib  # vllt's ops load the host build of the library
    ops.stream_handle = lambda stream=None: 0

    def paged_attention(q, cache_k, cache_v, read_slots, n_kv_heads, scale):
        _STATE["attention_calls"] = _STATE.get("attention_calls", 0) + 1
        return ops.paged_attention(q, cache_k, cache_v, read_slots, n_kv_heads, scale, device="cpu")

    A.paged_attention = paged_attention


UNSEEDED = 20240601


def _seed_unseeded_requests(E):
    import numpy as np

    class _Random:
        def __getattr__(self, name):
            return getattr(np.random, name)

        def default_rng(self, seed=None, *args):
            return np.random.default_rng(UNSEEDED if seed is None else seed, *args)

    class _NumPy:  # vllmlite.engine's numpy, but for default_rng's unseeded case
        random = _Random()

        def __getattr__(self, name):
            return getattr(np, name)

    E.np = _NumPy()


def pytest_terminal_summary(terminalreporter):
    runners = _STATE.get("runners", [])
    passes = sum(r.passes for r in runners)
    terminalreporter.write_line(f"VLLT_REFSUITE runners={len(runners)} forward_passes={passes} "
                                f"block_hashes={_STATE.get('hashes', 0)} "
                                f"attention_calls={_STATE.get('attention_calls', 0)}")
