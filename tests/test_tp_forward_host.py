"""CPU, gloo ranks: libvllt's tensor-parallel bf16 forward, its own code.

Each rank opens the host build of libvllt (tests/host_build.py; every kernel,
the tcgen05 GEMMs and the tensor-core prefill attention included, runs as
compiled on the emulation of tests/simt_host.h and tests/simt_include/simt_tc.h)
and runs its shard of the Llama-shaped model as TPLlamaRunner sets it up:
vllt.llama.LlamaWeights(tp_rank, tp_size) (column-parallel QKV and gate/up,
row-parallel o_proj and down_proj, vocab-parallel lm_head), this rank's KV
heads in its caches, the descriptor built by LlamaRunner._make_desc. The
forward's two all-reduces per layer (ncclAllReduce of the bf16 partial in
csrc/tp.cu on the GPU) are reached through the same call in forward_bf16.cu
and run as a gloo all-reduce of the same bf16 buffer. Greedy picks are
vocab-parallel as in TPLlamaRunner.greedy_picks: vllt_argmax_rows over this
rank's slice, the (max, index) pairs all-gathered, vllt.tp.merge_argmax.

On the GPU test's schedule (tests/tp_parity.py: chunked prefill, decode, a
verify row set, then a pass that forks a partly filled block by copy-on-write
and continues a sequence from the copy), at 2 ranks (8 heads / 2 KV heads: 4 / 1 per rank) and 4 ranks
(8 / 4: 2 / 1 per rank), against a 1-rank bf16 forward of the same weights:
  * the gathered logits (vllt.tp.gather_vocab_rows over every rank's slice)
    within TP_BAR of the largest |logit|, the bar of the GPU test
    (three times the error of two bf16 ranks against one that
    oracle/llama_bf16.py measures at the full-width shape); measured here
    7.0e-3 at 2 ranks and 9.2e-3 at 4;
  * the merged picks equal np.argmax of the gathered rows on every row
    (vllt_argmax_rows plus the merge keep np.argmax's first-index rule), and
    equal the 1-rank picks on all rows but at most one near-tie;
  * every rank ran exactly 2 * n_layers all-reduces per pass, each of the
    pass's token bound times d_model values.
"""

import datetime
import json
import os
import socket
import sys

import numpy as np
import pytest

from tests.conftest import needs_vllmlite

torch = pytest.importorskip("torch")
pytestmark = needs_vllmlite

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
TP_BAR = 3e-2
COMM = 0x7C  # the opaque communicator handle: any non-null value reaches the host collective


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, lib_path, shape_kw, result_dir):
    sys.path[:0] = [ROOT, os.path.join(ROOT, "vllm-lite_b200"), os.path.join(ROOT, "baseline", "_ref")]
    import ctypes as C

    import torch.distributed as dist

    from tests import fixtures as F
    from tests.host_build import load_library_host
    from tests.test_forward_bf16_host import Forward
    from tests.test_gpu_llama import schedule
    from vllt.llama import LlamaShape
    from vllt.tp import gather_vocab_rows, merge_argmax

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=300))
    try:
        L = load_library_host(lib_path)
        sizes = []
        AllReduce = C.CFUNCTYPE(C.c_int, C.c_void_p, C.c_int64, C.c_void_p)

        def allreduce(buf, count, comm):
            if comm != COMM:
                return 1
            t = torch.frombuffer((C.c_uint16 * count).from_address(buf), dtype=torch.bfloat16)
            dist.all_reduce(t)
            sizes.append(int(count))
            return 0

        hook = AllReduce(allreduce)
        L.vllt_host_set_allreduce.argtypes = [AllReduce]
        L.vllt_host_set_allreduce(hook)

        shape = LlamaShape(**shape_kw)
        shard = Forward(L, shape, True, tp_rank=rank, tp_size=world, tp_comm=COMM)
        vl, off = shard.keep[0].vocab_local, shard.keep[0].vocab_offset
        one = Forward(L, shape, True) if rank == 0 else None
        worst, agree, rows, exact, want_sizes = 0.0, 0, 0, True, []
        # the GPU test's passes (tests/tp_parity.py), the fork through copy-on-write last
        fork = [dict(start=46, n=1, count=1, tokens=[7], block_ids=[0, 1, 14], drafts=[])]
        passes = [(p, ()) for p in schedule(shape.vocab_size, np.random.default_rng(3))] + [(fork, [(2, 14)])]
        for seqs, cow in passes:
            out = F.as_scheduler_output(seqs, cow)
            local = shard.execute(out)
            want_sizes += [shard.last_bounds.tokens * shape.d_model] * (2 * shape.n_layers)
            R = local.shape[0]
            val, idx = np.zeros(R, np.float32), np.zeros(R, np.int32)
            rc = L.vllt_argmax_rows(shard.logits.ctypes.data, R, vl, shard.vocab_padded, off, val.ctypes.data,
                                    idx.ctypes.data, None)
            assert rc == 0, L.vllt_last_error()
            vals, idxs = torch.empty(world * R, dtype=torch.float32), torch.empty(world * R, dtype=torch.int32)
            dist.all_gather_into_tensor(vals, torch.from_numpy(val))
            dist.all_gather_into_tensor(idxs, torch.from_numpy(idx))
            picks = merge_argmax(vals.view(world, R), idxs.view(world, R)).numpy()
            full = gather_vocab_rows(torch.from_numpy(local), world).numpy()
            exact &= bool(np.array_equal(picks, full.argmax(1)) and np.array_equal(full[:, off:off + vl], local))
            if one is not None:
                want = one.execute(out)
                worst = max(worst, float(np.abs(full - want).max() / np.abs(want).max()))
                agree += int((picks == want.argmax(1)).sum())
                rows += R
        L.vllt_host_set_allreduce(AllReduce())
        res = dict(sizes=sizes, want_sizes=want_sizes, exact=exact, worst=worst, agree=agree, rows=rows)
        with open(os.path.join(result_dir, f"rank{rank}.json"), "w") as f:
            json.dump(res, f)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,shape_kw", [
    (2, dict(n_layers=2, n_heads=8, n_kv_heads=2, d_model=1024, d_ff=2048, vocab_size=1000, max_seq_len=2048,
             seed=1)),
    (4, dict(n_layers=2, n_heads=8, n_kv_heads=4, d_model=1024, d_ff=2048, vocab_size=1000, max_seq_len=2048,
             seed=2)),
])
def test_tensor_parallel_forward_matches_one_rank(host_library, tmp_path, world, shape_kw):
    import torch.multiprocessing as mp

    mp.start_processes(_rank, args=(world, _free_port(), host_library._name, shape_kw, str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    res = [json.load(open(tmp_path / f"rank{r}.json")) for r in range(world)]
    for r in res:
        assert r["exact"]
        assert r["sizes"] == r["want_sizes"]
    r0 = res[0]
    print(f"tensor parallel {world}: worst {r0['worst']:.3e} of max |logit|, picks {r0['agree']}/{r0['rows']}")
    assert r0["worst"] < TP_BAR
    assert r0["agree"] >= r0["rows"] - 1 and r0["rows"] == 13
