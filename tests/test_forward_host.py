"""CPU: libvllt's fp32 forward, its own compiled code, on the reference's replays.

tests/host_build.py builds the library's fp32 path for the host:
  * the C ABI and the forward's orchestration (capi.cu's vllt_forward);
  * the launchers of the metadata builder, RMSNorm, embedding, SGEMM with its
    fused epilogues, generic attention and sampling.

The sources are built unchanged, against stub CUDA headers. Every launch
runs its kernel on the SIMT emulation of tests/simt_host.h. The test drives
vllt_forward the way CudaRunner does: the runner's own packer, descriptor and
weight layout (on the CPU), a zeroed workspace, exact step bounds and the
CUDA graphs' bucketed bounds, classic and pooled step records. It compares
every pass's logits with the reference's own logits in the replay fixtures
(vllmlite/runner.py:62-100 run by tests/golden/make_golden.py): the
benchmark model with chunked prefill (block 16), and speculative verify with
the prefix cache (block 4). These are the bars of the GPU test of the same
replays (tests/test_gpu_engine.py::test_runner_replay_logits): relative error
below 1e-4, identical argmax. The metadata builder's error word is 0 on every
pass.
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


class HostForward:
    """What CudaRunner keeps between passes, in host memory."""

    def __init__(self, lib, model_cfg, bs, nb, pooled, bucketed):
        from types import SimpleNamespace

        from vllt import _lib
        from vllt.model import DeviceWeights, initial_weights
        from vllt.runner import CudaRunner, StepPacker

        self.L, self.cfg, self.bs, self.nb, self.bucketed = lib, model_cfg, bs, nb, bucketed
        w = DeviceWeights(model_cfg, initial_weights(model_cfg), device="cpu")
        hd = model_cfg.d_model // model_cfg.n_heads
        shape = (model_cfg.n_layers, nb, model_cfg.n_kv_heads, bs, hd)
        self.cache_k = torch.zeros(shape, dtype=torch.float32)
        self.cache_v = torch.zeros(shape, dtype=torch.float32)
        me = SimpleNamespace(model_cfg=model_cfg, w=w, _ptrs=w.pointer_arrays(), block_size=bs, num_blocks=nb,
                             head_dim=hd, cache_k=self.cache_k, cache_v=self.cache_v)
        self.desc = CudaRunner._make_desc(me)  # the runner's own descriptor
        self.keep = (w, me._ptrs)
        self.w = w
        self.qp = lib.vllt_query_tile_positions(C.byref(self.desc))
        self.caps = _lib.Caps(16, 1024, 64, -(-model_cfg.max_seq_len // bs))
        self.meta = np.zeros(lib.vllt_meta_bytes(C.byref(self.caps)) // 4, np.int32)
        self.ws = np.zeros(lib.vllt_forward_workspace_bytes(C.byref(self.desc), C.byref(self.caps)), np.uint8)
        self.logits = np.zeros((self.caps.max_rows, w.vocab_padded), np.float32)
        self.picks = np.zeros(2 * (self.caps.max_rows + self.caps.max_seqs) + 1, np.int32)
        self.desc.token_source, self.desc.token_source_len = self.picks.ctypes.data, self.picks.size
        slots = 2 * self.caps.max_seqs if pooled else 0
        if pooled:
            self.pool = np.full((slots, self.caps.max_table_width), -1, np.int32)
            self.desc.table_pool, self.desc.table_pool_slots = self.pool.ctypes.data, slots
        self.packer = StepPacker(bs, nb, model_cfg.vocab_size, w.rope_len, self.qp, pool_slots=slots,
                                 pool_width=self.caps.max_table_width, token_refs=self.picks.size)

    def execute(self, out):
        from vllt.runner import CudaRunner

        assert not out.cow
        rec, bounds, rows, (S, T, R, W) = self.packer.pack(out)
        if self.bucketed:  # the bounds a CUDA graph of this pass's bucket was captured with
            bounds = CudaRunner.bucket(self, bounds)
        rec = np.ascontiguousarray(rec, np.int32)
        rc = self.L.vllt_forward(C.byref(self.desc), rec.ctypes.data, C.byref(self.caps), C.byref(bounds),
                                 self.meta.ctypes.data, self.ws.ctypes.data, self.ws.size, self.logits.ctypes.data,
                                 None)
        assert rc == 0, self.L.vllt_last_error()
        assert self.meta[7] == 0  # the metadata builder's error word
        return self.logits[:R, :self.cfg.vocab_size].copy(), rows


@pytest.mark.parametrize("name,bs,pooled,bucketed,seed", [("replay_bench.npz", 16, True, False, 0),
                                                          ("replay_spec.npz", 4, False, True, 0),
                                                          ("replay_bench.npz", 16, False, False, 0xC0FFEE)])
def test_host_forward_reproduces_the_reference_logits(host_lib, name, bs, pooled, bucketed, seed):
    """seed != 0: every kernel of the forward runs under the emulation's
    shuffled schedule (a random thread continues after each barrier)."""
    from vllmlite.config import ModelConfig

    host_lib.vllt_host_schedule_seed.argtypes = [C.c_uint64]
    host_lib.vllt_host_schedule_seed(seed)
    run = HostForward(host_lib, ModelConfig(vocab_size=261, **F.BENCH), bs, 512, pooled, bucketed)
    worst, n = 0.0, 0
    for seqs, cow, want in F.replay_steps(name):
        out = F.as_scheduler_output(seqs, cow)
        for item, s in zip(out.scheduled, seqs):
            item.seq.request_id = f"b{s['block_ids'][0]}"
        got, rows = run.execute(out)
        assert got.shape == want.shape
        rel = float(np.abs(got - want).max() / np.abs(want).max())
        worst = max(worst, rel)
        assert (got.argmax(1) == want.argmax(1)).all(), n
        n += 1
    host_lib.vllt_host_schedule_seed(0)
    assert n > 10 and worst < 1e-4, worst
