"""Test infrastructure: CudaRunner's state and launch in host memory, over
the host build of libvllt (tests/host_build.py).

HostRunner keeps the runner's device buffers as CPU tensors and uses
CudaRunner's own pieces: packer, descriptor, graph-bucket bounds, pick buffer
and error check. Every pass then goes through the library's compiled code on
the SIMT emulation. Set `HostRunner.lib` to the host library before building
an engine with it. This module imports nothing from the tests package, so a
pytest plugin that runs the reference's own test files can load it by path.
"""

import ctypes as C

import numpy as np
import torch


class HostRunner:
    """CudaRunner's state and launch in host memory, over the host library;
    with `bf16` (HostLlamaRunner) LlamaRunner's: the Llama-shaped model's bf16
    weights and caches and its descriptor, so the forward takes the bf16
    path (tcgen05 GEMMs, TMA decode, tensor-core prefill)."""

    tp_size = 1
    tp_rank = 0
    tp_comm = None
    bf16 = False
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
        self.copy_blocks_on_device = CudaRunner.copy_blocks_on_device.__get__(self)
        self.torch = torch
        self.head_dim = model_cfg.d_model // model_cfg.n_heads
        shape = (model_cfg.n_layers, self.num_blocks, model_cfg.n_kv_heads // self.tp_size, self.block_size,
                 self.head_dim)
        dt = torch.bfloat16 if self.bf16 else torch.float32
        self.cache_k = torch.zeros(shape, dtype=dt)
        self.cache_v = torch.zeros(shape, dtype=dt)
        if self.bf16:
            from vllt.llama import LlamaRunner, LlamaWeights

            self.w = LlamaWeights(model_cfg, "cpu", self.tp_rank, self.tp_size)
            self._ptrs = self.w.pointer_arrays()
            self.desc = LlamaRunner._make_desc(self)
        else:
            self.w = DeviceWeights(model_cfg, initial_weights(model_cfg), device="cpu")
            me = SimpleNamespace(model_cfg=model_cfg, w=self.w, _ptrs=self.w.pointer_arrays(),
                                 block_size=self.block_size, num_blocks=self.num_blocks, head_dim=self.head_dim,
                                 cache_k=self.cache_k, cache_v=self.cache_v)
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
            self.copy_blocks_on_device(pairs.ctypes.data, len(pairs))
            self._cow_pairs = pairs
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

    def execute(self, out):
        """(logits float32 [n_rows, vocab], rows), as CudaRunner.execute returns
        them to an unmodified LLMEngine (vllmlite/runner.py:62-100)."""
        rows, R = self.launch(out)
        self.check_step_flags(int(self.meta[7]))
        return self.logits_dev[:R, :self.model_cfg.vocab_size].numpy().copy(), rows

    @property
    def cache_bytes(self) -> int:
        return 2 * self.cache_k.numel() * self.cache_k.element_size()


class HostLlamaRunner(HostRunner):
    """LlamaRunner (the bf16 path, one rank) over the host library."""

    bf16 = True


class HostTPRunner(HostLlamaRunner):
    """TPLlamaRunner over the host library, its ranks gloo processes: the
    shard's weights and KV heads, and TPLlamaRunner's own protocol code
    (launch with its copy-on-write message, record broadcast, vocab-parallel
    greedy, row gathers, stop) on CPU tensors. The forward's all-reduce goes
    to the host collective the process registered (vllt_host_set_allreduce).
    Set `group` (rank, world) and `lib` before building one."""

    group = None
    COMM = 0x7C  # the opaque communicator handle the host collective checks

    def __init__(self, model_cfg, cache_cfg, sched_cfg=None, device=None):
        from vllt.tp import CTRL_WORDS, ControlPlane

        self.tp_rank, self.tp_size, self.tp_comm = self.group.rank, self.group.world, self.COMM
        super().__init__(model_cfg, cache_cfg, sched_cfg, device)
        c = self.caps
        words = 5 + 4 * c.max_seqs + c.max_tokens + 3 * c.max_seqs * c.max_table_width
        self.rec_dev = torch.zeros(words + CTRL_WORDS, dtype=torch.int32)
        self.rec_host = self.rec_dev
        self.plane = ControlPlane(self.rec_dev)
        self._val = torch.empty(c.max_rows, dtype=torch.float32)
        self._idx = torch.empty(c.max_rows, dtype=torch.int32)
        self._vals = torch.empty(self.tp_size * c.max_rows, dtype=torch.float32)
        self._idxs = torch.empty(self.tp_size * c.max_rows, dtype=torch.int32)
        self._pending_rows = self.steps = self.h2d_bytes = self.cows = 0
        self.pooled_tables, self.use_graphs, self.bucket_bounds, self._fixed = True, False, True, True

    from vllt.runner import CudaRunner as _C
    from vllt.tp import TPLlamaRunner as _T

    launch, _broadcast, greedy_picks, gather_rows, _gather, stop_workers, _reserve = (
        _T.launch, _T._broadcast, _T.greedy_picks, _T.gather_rows, _T._gather, _T.stop_workers, _T._reserve)
    pack, _timed_forward, _dispatch, _forward = _C.pack, _C._timed_forward, _C._dispatch, _C._forward
    del _C, _T

    def copy_on_write(self, pairs) -> None:  # CudaRunner's, without the pinned staging copy
        a = np.ascontiguousarray(np.asarray(pairs, np.int32).reshape(-1, 2))
        self.copy_blocks_on_device(a.ctypes.data, len(a))
        self.cows += len(a)

    def execute(self, out):
        """Rank 0 for an unmodified LLMEngine: the full-vocabulary logits of
        the pass, gathered from every rank's slice (TPLlamaRunner.gather_rows)."""
        rows, R = self.launch(out)
        self.check_step_flags(int(self.meta[7]))
        self.greedy_picks(R)  # launch's greedy flag: every worker takes this all-gather after the forward
        return self.gather_rows(list(range(R))).numpy().copy(), rows

    def worker_loop(self):
        """TPLlamaRunner.worker_loop without the device synchronizations (the
        host build runs each launch to completion)."""
        from vllt.tp import serve

        def forward(bounds, greedy):
            self._dispatch(bounds)
            if greedy:
                self.picks_dev[:bounds.rows].copy_(self.greedy_picks(bounds.rows))

        def cow(n):
            self.copy_blocks_on_device(self.rec_dev.data_ptr(), n // 2)
            self.cows += n // 2

        return serve(self.plane, forward, lambda tag: None, self._gather, cow)
