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

The benchmark's requests (C1: 6 layers, d 384, greedy with ignore_eos,
budget 1024, block 16) must give the streams the reference engine gave
(tests/golden/streams_mixed.npz). Greedy streams do not depend on which
requests share a batch, so a subset of the 48 requests is run.
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


def test_engine_streams_through_the_compiled_device_path(host_lib):
    from vllmlite.config import CacheConfig, EngineConfig, ModelConfig, SchedulerConfig

    from vllt.engine import GpuLLMEngine, cuda_engine
    from vllt.workloads import mixed_workload

    z = F.load("streams_mixed.npz")
    lens, toks = z["lens"], z["tokens"]
    want_all, o = [], 0
    for n in lens:
        want_all.append(toks[o:o + int(n)].tolist())
        o += int(n)
    reqs = mixed_workload(48, 0, 0)
    pick = [1, 4, 9, 17, 23, 30, 38, 46]  # a subset of the 48 requests
    HostRunner.lib = host_lib
    cfg = EngineConfig(model=ModelConfig(vocab_size=261, max_seq_len=512, **{k: v for k, v in F.BENCH.items()
                                                                           if k != "max_seq_len"}),
                       cache=CacheConfig(block_size=16, num_blocks=512),
                       scheduler=SchedulerConfig(max_seqs=16, max_batched_tokens=1024))
    eng = cuda_engine(cfg, engine_cls=GpuLLMEngine.resolve(), runner_cls=HostRunner)
    ids = [eng.add_request(params=reqs[i][2], request_id=reqs[i][0], prompt_token_ids=reqs[i][1]) for i in pick]
    while eng.has_work:
        eng.step()
    got = [eng.seqs[i].output_token_ids for i in ids]
    assert got == [want_all[i] for i in pick]
    assert eng.passes_ahead >= eng.total_steps // 2 and eng.runner.stand_ins > 0
