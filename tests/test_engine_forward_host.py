"""CPU: the whole device path of GpuLLMEngine, its own compiled code, against
the reference engine's token streams.

HostRunner gives GpuLLMEngine libvllt's fp32 path built for the host
(tests/host_build.py build_library_host). It keeps CudaRunner's state in
host memory and uses the runner's own pieces: packer, descriptor, bucketed
bounds, pick buffer and error check. So every pass goes through the same
code as on the GPU:
  * the engine's scheduling and bookkeeping, including run-ahead;
  * the pooled step record with stand-in tokens;
  * vllt_forward with the compiled metadata builder (which resolves the
    stand-ins), RMSNorm, SGEMM epilogues and attention;
  * vllt_sample_greedy's compiled kernel, the pick buffer and the error word.

The benchmarks' requests must give the token streams the reference engine
gave (tests/golden/streams_*.npz): C1 (mixed lengths), C2 (a 256-token shared
prefix with the prefix cache, so copy-on-write runs through the compiled
copy kernel) and C5 (periodic prompts with speculative k = 4, verified by
the compiled accept kernel against the k = 0 streams). Greedy streams do not
depend on which requests share a batch, so a subset of each is run.
"""

import ctypes as C

import numpy as np
import pytest

from tests import fixtures as F
from tests.conftest import needs_vllmlite

torch = pytest.importorskip("torch")
pytestmark = needs_vllmlite


@pytest.fixture
def host_lib(host_library):
    return host_library


@pytest.fixture(autouse=True)
def _no_stream(monkeypatch):
    import vllt._lib as _lib

    monkeypatch.setattr(_lib, "stream_handle", lambda stream=None: 0)


class HostRunner:
    """CudaRunner's state and launch in host memory, over the host library."""

    tp_size = 1
    lib = None

    def __init__(self, model_cfg, cache_cfg, sched_cfg=None, device=None):
        from types import SimpleNamespace

        from vllt import _lib
        from vllt.model import DeviceWeights, initial_weights
        from vllt.runner import CudaRunner, StepPacker

        L = self.L = self.lib
        self.model_cfg, self.dev = model_cfg, torch.device("cpu")
        self.block_size, self.num_blocks = cache_cfg.block_size, cache_cfg.num_blocks
        self.check_step_flags = CudaRunner.check_step_flags.__get__(self)
        self.pick_buffer = CudaRunner.pick_buffer.__get__(self)
        self.bucket = CudaRunner.bucket.__get__(self)
        self.w = DeviceWeights(model_cfg, initial_weights(model_cfg), device="cpu")
        self.head_dim = model_cfg.d_model // model_cfg.n_heads
        shape = (model_cfg.n_layers, self.num_blocks, model_cfg.n_kv_heads, self.block_size, self.head_dim)
        self.cache_k = torch.zeros(shape, dtype=torch.float32)
        self.cache_v = torch.zeros(shape, dtype=torch.float32)
        me = SimpleNamespace(model_cfg=model_cfg, w=self.w, _ptrs=self.w.pointer_arrays(), block_size=self.block_size,
                             num_blocks=self.num_blocks, head_dim=self.head_dim, cache_k=self.cache_k,
                             cache_v=self.cache_v)
        self._ptrs = me._ptrs
        self.desc = CudaRunner._make_desc(me)
        self.qp = L.vllt_query_tile_positions(C.byref(self.desc))
        seqs, toks = sched_cfg.max_seqs, sched_cfg.max_batched_tokens
        self.caps = _lib.Caps(seqs, toks, min(toks, 4 * seqs), -(-model_cfg.max_seq_len // self.block_size))
        self.meta = torch.zeros(L.vllt_meta_bytes(C.byref(self.caps)) // 4, dtype=torch.int32)
        self.ws = torch.zeros(L.vllt_forward_workspace_bytes(C.byref(self.desc), C.byref(self.caps)), dtype=torch.uint8)
        self.logits_dev = torch.zeros((self.caps.max_rows, self.w.vocab_padded), dtype=torch.float32)
        self.picks_dev = torch.zeros(2 * (self.caps.max_rows + self.caps.max_seqs) + 1, dtype=torch.int32)
        self.desc.token_source, self.desc.token_source_len = self.picks_dev.data_ptr(), self.picks_dev.numel()
        slots = 2 * seqs
        self.table_pool = torch.full((slots, self.caps.max_table_width), -1, dtype=torch.int32)
        self.desc.table_pool, self.desc.table_pool_slots = self.table_pool.data_ptr(), slots
        self.packer = StepPacker(self.block_size, self.num_blocks, model_cfg.vocab_size, self.w.rope_len, self.qp,
                                 pool_slots=slots, pool_width=self.caps.max_table_width,
                                 token_refs=self.picks_dev.numel())
        self.passes = self.stand_ins = 0

    @property
    def vocab_size(self):
        return self.model_cfg.vocab_size

    def launch(self, out):
        from vllt import _lib

        if out.cow:
            pairs = np.ascontiguousarray(np.asarray(out.cow, np.int32).reshape(-1, 2))
            cfg = self.model_cfg
            assert self.L.vllt_copy_blocks(self.cache_k.data_ptr(), self.cache_v.data_ptr(), pairs.ctypes.data,
                                           len(pairs), cfg.n_layers, self.num_blocks, cfg.n_kv_heads,
                                           self.block_size, self.head_dim, _lib.VLLT_F32, None) == 0
        rec, bounds, rows, (S, T, R, W) = self.packer.pack(out)
        self.stand_ins += int((rec[5 + 3 * S:5 + 3 * S + T] < 0).sum())
        rec = np.ascontiguousarray(rec, np.int32)
        gb = self.bucket(bounds)  # the bounds of the CUDA graph that would serve this pass
        rc = self.L.vllt_forward(C.byref(self.desc), rec.ctypes.data, C.byref(self.caps), C.byref(gb),
                                 self.meta.data_ptr(), self.ws.data_ptr(), self.ws.numel(), self.logits_dev.data_ptr(),
                                 None)
        assert rc == 0, self.L.vllt_last_error()
        self.passes += 1
        return rows, R


def fixture_streams(name):
    z = F.load(name)
    out, o = [], 0
    for n in z["lens"]:
        out.append(z["tokens"][o:o + int(n)].tolist())
        o += int(n)
    return out


@pytest.mark.parametrize("workload,pick,maxlen,nb,prefix,spec,seqs,budget", [
    ("mixed", [1, 9, 30, 46], 512, 512, False, 0, 16, 1024),           # C1, run-ahead
    ("shared", [0, 7, 15, 33], 768, 768, True, 0, 16, 384),            # C2: prefix cache hits, run-ahead
    ("periodic", [0, 5], 1024, 4096, False, 4, 64, 2048),             # C5: speculative k = 4
])
def test_engine_streams_through_the_compiled_device_path(host_lib, workload, pick, maxlen, nb, prefix, spec, seqs,
                                                          budget):
    from vllmlite.config import CacheConfig, EngineConfig, ModelConfig, SchedulerConfig

    from vllt.engine import GpuLLMEngine, cuda_engine
    from vllt.workloads import mixed_workload, periodic_workload

    if workload == "periodic":
        reqs, want_all = periodic_workload(128, seed=0), fixture_streams("streams_periodic.npz")
    else:
        reqs = mixed_workload(48, 0, 256 if workload == "shared" else 0)
        want_all = fixture_streams(f"streams_{workload}.npz")
    HostRunner.lib = host_lib
    shape = {k: v for k, v in F.BENCH.items() if k != "max_seq_len"}
    cfg = EngineConfig(model=ModelConfig(vocab_size=261, max_seq_len=maxlen, **shape),
                       cache=CacheConfig(block_size=16, num_blocks=nb, enable_prefix_caching=prefix),
                       scheduler=SchedulerConfig(max_seqs=seqs, max_batched_tokens=budget))
    eng = cuda_engine(cfg, speculative_tokens=spec, engine_cls=GpuLLMEngine.resolve(), runner_cls=HostRunner)
    ids = [eng.add_request(params=reqs[i][2], request_id=reqs[i][0], prompt_token_ids=reqs[i][1]) for i in pick]
    while eng.has_work:
        eng.step()
    got = [eng.seqs[i].output_token_ids for i in ids]
    assert got == [want_all[i] for i in pick]
    if spec:  # proposals read the new tokens: no pass runs ahead; drafts were verified on the device
        assert eng.passes_ahead == 0 and eng.spec.accepted > 0
    else:
        assert eng.passes_ahead >= eng.total_steps // 2 and eng.runner.stand_ins > 0
    if prefix:
        assert eng.scheduler.blocks.allocator.hits > 0
