"""CPU: libvllt's bf16 forward (the Llama-3-8B-shaped path) built for the host.

tests/host_build.py builds forward_bf16.cu for the host with the rest of the
library, so the whole pass is the library's own code: its orchestration, the
RMSNorm and embedding kernels, the tcgen05 GEMMs (the small-M cluster and
stream-K forms a decode-sized pass takes, with their fused epilogues: QKV with
RoPE and the bf16 KV-cache write, SwiGLU, fp32 residual, stores) and the
attention kernels (TMA decode for decode rows, the tcgen05 prefill kernel for
multi-token tiles), with the tensor-core, TMA and cluster instructions on the
emulation of tests/simt_include/simt_tc.h.

As the GPU test does (tests/test_gpu_llama.py), the bf16 logits are compared
with the fp32 parity forward (also built for the host) running the same
weights widened to fp32, over the same three-pass schedule (chunked prefill,
decode, a verify row set). The bar is the GPU test's: 2e-2 for both the max
relative error and the per-row relative norm (three times the error that the
CPU model of the bf16 rounding points measures). Every row whose fp32 top-1 /
top-2 gap exceeds twice the pass's error picks the same token.
"""

import ctypes as C

import numpy as np
import pytest

from tests import fixtures as F
from tests.conftest import needs_vllmlite

torch = pytest.importorskip("torch")
pytestmark = needs_vllmlite

BAR = 2e-2


@pytest.fixture
def L(host_library):
    host_library.vllt_host_mma_count.restype = C.c_int64
    return host_library


class Forward:
    """A runner's descriptor, caches and buffers in host memory. bf16 with
    tp_size > 1: shard tp_rank of the model (vllt.llama.LlamaWeights), this
    rank's KV heads in the caches, `tp_comm` passed through the descriptor as
    TPLlamaRunner passes its NCCL communicator; the logits are this rank's
    vocabulary slice."""

    def __init__(self, L, shape, bf16, num_blocks=64, bs=16, tp_rank=0, tp_size=1, tp_comm=None, max_tokens=256,
                 max_seqs=8):
        from types import SimpleNamespace

        from vllt import _lib
        from vllt.llama import LlamaRunner, LlamaWeights, fp32_reference_weights
        from vllt.model import DeviceWeights
        from vllt.runner import CudaRunner, StepPacker

        self.L, self.shape = L, shape
        D = shape.head_dim
        dt = torch.bfloat16 if bf16 else torch.float32
        kv = (shape.n_layers, num_blocks, shape.n_kv_heads // tp_size, bs, D)
        self.cache_k, self.cache_v = torch.zeros(kv, dtype=dt), torch.zeros(kv, dtype=dt)
        self.vocab = shape.vocab_size
        if bf16:
            w = LlamaWeights(shape, "cpu", tp_rank, tp_size)
            me = SimpleNamespace(model_cfg=shape, w=w, _ptrs=w.pointer_arrays(), tp_size=tp_size, head_dim=D,
                                 block_size=bs, num_blocks=num_blocks, tp_comm=tp_comm, cache_k=self.cache_k,
                                 cache_v=self.cache_v)
            self.desc = LlamaRunner._make_desc(me)
            self.vocab = w.vocab_local
        else:
            w = DeviceWeights(shape, fp32_reference_weights(shape, "cpu"), device="cpu")
            me = SimpleNamespace(model_cfg=shape, w=w, _ptrs=w.pointer_arrays(), block_size=bs,
                                 num_blocks=num_blocks, head_dim=D, cache_k=self.cache_k, cache_v=self.cache_v)
            self.desc = CudaRunner._make_desc(me)
        self.keep = (w, me)
        self.vocab_padded = w.vocab_padded
        self.qp = L.vllt_query_tile_positions(C.byref(self.desc))
        self.caps = _lib.Caps(max_seqs, max_tokens, 32, -(-shape.max_seq_len // bs))
        self.meta = np.zeros(L.vllt_meta_bytes(C.byref(self.caps)) // 4, np.int32)
        self.ws = np.zeros(L.vllt_forward_workspace_bytes(C.byref(self.desc), C.byref(self.caps)), np.uint8)
        self.logits = np.zeros((self.caps.max_rows, w.vocab_padded), np.float32)
        self.packer = StepPacker(bs, num_blocks, shape.vocab_size, w.rope_len, self.qp)

    def execute(self, out):
        if out.cow:  # the runner's copy-on-write before the forward (vllmlite/runner.py:63-64)
            from vllt import _lib

            pairs = np.ascontiguousarray(np.asarray(out.cow, np.int32).reshape(-1, 2))
            L_, nb, n_kv, bs, D = self.cache_k.shape
            dt = _lib.VLLT_BF16 if self.cache_k.dtype == torch.bfloat16 else _lib.VLLT_F32
            rc = self.L.vllt_copy_blocks(self.cache_k.data_ptr(), self.cache_v.data_ptr(), pairs.ctypes.data,
                                         len(pairs), L_, nb, n_kv, bs, D, dt, None)
            assert rc == 0, self.L.vllt_last_error()
        rec, bounds, rows, (S, T, R, W) = self.packer.pack(out)
        self.last_bounds = bounds
        rec = np.ascontiguousarray(rec, np.int32)
        rc = self.L.vllt_forward(C.byref(self.desc), rec.ctypes.data, C.byref(self.caps), C.byref(bounds),
                                 self.meta.ctypes.data, self.ws.ctypes.data, self.ws.size, self.logits.ctypes.data,
                                 None)
        assert rc == 0, self.L.vllt_last_error()
        assert self.meta[7] == 0
        return self.logits[:R, :self.vocab].copy()


def test_bf16_forward_matches_the_fp32_forward_on_the_same_weights(L):
    from vllt.llama import LlamaShape

    from tests.test_gpu_llama import schedule

    shape = LlamaShape(n_layers=2, n_heads=8, n_kv_heads=2, d_model=1024, d_ff=2048, vocab_size=1000,
                       max_seq_len=2048, seed=1)
    bf, ref = Forward(L, shape, True), Forward(L, shape, False)
    mma0 = L.vllt_host_mma_count()
    worst = worst_row = 0.0
    decided = 0
    for seqs in schedule(shape.vocab_size, np.random.default_rng(3)):
        out = F.as_scheduler_output(seqs)
        a, b = bf.execute(out), ref.execute(out)
        assert a.shape == b.shape and np.isfinite(a).all()
        err = np.abs(a - b).max()
        worst = max(worst, float(err / np.abs(b).max()))
        worst_row = max(worst_row, float((np.linalg.norm(a - b, axis=1) / np.linalg.norm(b, axis=1)).max()))
        top2 = np.sort(b, axis=1)[:, -2:]
        clear = (top2[:, 1] - top2[:, 0]) > 2 * err
        assert (a.argmax(1) == b.argmax(1))[clear].all()
        decided += int(clear.sum())
    assert worst <= BAR and worst_row <= BAR, (worst, worst_row)
    assert decided > 0
    assert L.vllt_host_mma_count() > mma0  # the tensor-core kernels ran


def oracle_weights(w, shape):
    """The product's unsharded bf16 weights (vllt.llama.LlamaWeights) in the
    oracle's naming (oracle/llama_bf16.py), as float32 values: wqkv split into
    wq / wk / wv, the interleaved gate/up rows taken apart."""
    D, H, KV = shape.head_dim, shape.n_heads, shape.n_kv_heads
    out = {"tok_emb": w.tok_emb.float(), "lm_head": w.lm_head.float()}
    for i, l in enumerate(w.layers):
        qkv = l["wqkv"].float()
        out[f"{i}.wq"], out[f"{i}.wk"], out[f"{i}.wv"] = qkv[:H * D], qkv[H * D:(H + KV) * D], qkv[(H + KV) * D:]
        out[f"{i}.wo"], out[f"{i}.w_down"] = l["wo"].float(), l["w_down"].float()
        out[f"{i}.w_gate"], out[f"{i}.w_up"] = l["w_gu"][0::2].float(), l["w_gu"][1::2].float()
    return out


# Three times the worst error of the host build against the oracle measured on
# this schedule (the two follow the same bf16 rounding points and differ only in
# the order of fp32 accumulation, the prefill kernel's lazily moved running max
# and exp2 against exp).
LONG_BAR = 1e-2


def test_bf16_forward_long_contexts_over_cached_prefixes(L):
    """The GPU test's long-context schedule (tests/test_gpu_llama.py
    long_schedule: prefill chunks of 2,400 and 4,100 tokens over cached
    prefixes of 2,100 and 4,000, then a decode row at 4,501 keys and four
    verify rows at 8,101-8,104, block tables from a shuffled pool of 800
    blocks, the RoPE table at the C4 max_seq_len of 9216) on a narrow model of
    the head size the kernels are built for. Reference: the bf16 forward's
    rounding points restated on the CPU (oracle/llama_bf16.py) over the same
    weights, each sequence whole with its chunking."""
    from oracle.llama_bf16 import forward_sequence, schedule_sequences
    from vllt.llama import LlamaShape

    from tests.test_gpu_llama import long_schedule

    shape = LlamaShape(n_layers=1, n_heads=2, n_kv_heads=1, d_model=256, d_ff=512, vocab_size=300,
                       max_seq_len=9216, seed=4)
    passes = long_schedule(shape.vocab_size, np.random.default_rng(8))
    fw = Forward(L, shape, True, num_blocks=800, max_tokens=8192, max_seqs=2)
    w = oracle_weights(fw.keep[0], shape)
    seqs, rows = schedule_sequences(passes)
    with torch.no_grad():
        want = {k: forward_sequence(shape, w, toks, chunks, bf16=True).numpy() for k, (toks, chunks) in seqs.items()}
    worst = 0.0
    mma0 = L.vllt_host_mma_count()
    for step, pass_rows in zip(passes, rows):
        got = fw.execute(F.as_scheduler_output(step))
        ref = np.concatenate([want[k][pos] for k, pos in pass_rows])
        assert got.shape == ref.shape and np.isfinite(got).all()
        worst = max(worst, float(np.abs(got - ref).max() / np.abs(ref).max()))
        assert (got.argmax(1) == ref.argmax(1)).all()
    print(f"long contexts: worst {worst:.3e} of max |logit|")
    assert worst <= LONG_BAR
    assert L.vllt_host_mma_count() > mma0
