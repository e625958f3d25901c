"""CPU: host-side logic of the product (no device work).

  * the C ABI library loads and exports every symbol include/vllt.h declares;
  * the step record packed by the runner describes the same flatten as the
    reference's ModelRunner.execute (oracle.runner.flatten);
  * the seeded workloads and weights of the product equal the reference's.
"""

import hashlib
import os
import re

import numpy as np
import pytest

from oracle import model as OM
from oracle import runner as OR
from tests import fixtures as F
from tests.conftest import ROOT, needs_vllmlite


def header_functions():
    src = open(os.path.join(ROOT, "include", "vllt.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(vllt_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    import ctypes

    from vllt import _lib

    lib = ctypes.CDLL(_lib.LIB_PATH)
    names = header_functions()
    assert len(names) >= 18
    for n in names:
        assert hasattr(lib, n), f"libvllt.so does not export {n}"
    # and the Python binding declares a signature for each of them
    assert set(names) == set(_lib.SIGNATURES), set(names) ^ set(_lib.SIGNATURES)


def test_library_calls_reject_bad_arguments_without_a_gpu():
    import ctypes

    from vllt import _lib

    L = _lib.lib()
    assert L.vllt_version() >= 100
    # argument validation happens on the host before any launch
    rc = L.vllt_reshape_and_cache(None, None, None, None, None, 3, 0, 8, 16, 4, 0, None)
    assert rc == _lib.VLLT_ERR_ARG
    assert b"bad sizes" in L.vllt_last_error()
    assert L.vllt_sgemm(None, None, None, 4, 4, 4, None) == _lib.VLLT_ERR_ARG
    # the decode wait injection is bounded: a positive index and at most 1 s
    assert L.vllt_test_decode_stall(-1, 1000) == _lib.VLLT_ERR_ARG
    assert L.vllt_test_decode_stall(3, 0) == _lib.VLLT_ERR_ARG
    assert L.vllt_test_decode_stall(3, 2_000_000_000) == _lib.VLLT_ERR_ARG
    # the pooled metadata builder refuses a missing pool before any launch
    caps = _lib.Caps(16, 1024, 1024, 32)
    assert L.vllt_build_batch_meta_pooled(None, ctypes.byref(caps), 16, 64, 2, None, 0, None, None) == _lib.VLLT_ERR_ARG
    assert L.vllt_meta_bytes(ctypes.byref(caps)) > 0
    assert L.vllt_meta_bytes(ctypes.byref(_lib.Caps(0, 1, 1, 1))) == -1


def test_gemm_form_choice_is_host_logic():
    """The bf16 GEMM picks its form on the host from (M, N, K) alone, so eager
    runs and graph replays of one shape agree. Without a device the SM count
    falls back to 148 and the cluster occupancy query to "none", which leaves
    stream-K for every small-M shape; on a GPU (tests/test_gpu_gemm_bf16.py)
    few-tile shapes may take the cluster form (negative values) instead."""
    from vllt import _lib

    L = _lib.lib()
    # decode batches (<= 256 tokens): weights-on-M forms
    for M, N, K in [(1, 4096, 4096), (64, 28672, 4096), (256, 6144, 4096), (37, 4096, 14336)]:
        assert L.vllt_gemm_bf16_auto_splits(M, N, K) <= 0
    # prefill batches: the persistent kernel
    assert L.vllt_gemm_bf16_auto_splits(8192, 4096, 4096) == 1
    assert L.vllt_gemm_bf16_auto_splits(8192, 28672, 4096) == 1
    # 257-512 tokens: split-K while the tile grid covers under half the SMs, within the
    # SM count and with >= 4 k-blocks per slice; otherwise unsplit
    for M, N, K in [(512, 4096, 4096), (300, 4096, 14336), (512, 6144, 4096)]:
        s = L.vllt_gemm_bf16_auto_splits(M, N, K)
        tiles = -(-N // 256) * -(-M // 128)
        assert s >= 1 and s * tiles <= max(148, tiles) and s <= max(1, K // 64 // 4)
        assert (s > 1) == (2 * tiles <= 148)
    # same inputs, same answer
    assert L.vllt_gemm_bf16_auto_splits(512, 4096, 4096) == L.vllt_gemm_bf16_auto_splits(512, 4096, 4096)
    # workspace sizes: the forward's scratch for the automatic form, exact tiles for a forced split
    assert L.vllt_gemm_bf16_splitk_workspace_bytes(64, 4096, 4096, 0) >= 2 * 148 * 64 * 128 * 4
    assert L.vllt_gemm_bf16_splitk_workspace_bytes(512, 4096, 4096, 2) >= 2 * 64 * 128 * 256 * 4
    # splits beyond K/64 are refused before any launch
    assert L.vllt_gemm_bf16_splitk(None, None, None, 4, 256, 128, 3, None, 0, None, None) == _lib.VLLT_ERR_ARG


def _record_to_flatten(rec):
    S, T, R, W = (int(x) for x in rec[:4])
    o = 4
    starts, qlens, counts = rec[o:o + S], rec[o + S:o + 2 * S], rec[o + 2 * S:o + 3 * S]
    o += 3 * S
    toks = rec[o:o + T]
    tabs = rec[o + T:o + T + S * W].reshape(S, W)
    return S, T, R, W, starts, qlens, counts, toks, tabs


@pytest.mark.parametrize("name,bs", [("replay_bench.npz", 16), ("replay_spec.npz", 4)])
def test_packed_record_matches_reference_flatten(name, bs):
    from vllt.runner import pack_step, tile_positions

    for seqs, cow, want in F.replay_steps(name):
        out = F.as_scheduler_output(seqs, cow)
        rec, bounds, rows, (S, T, R, W) = pack_step(out, bs, 512, 261, 512, tile_positions(2))
        tok, pos, meta, last, orows = OR.flatten(seqs, bs)
        S2, T2, R2, W2, starts, qlens, counts, toks, tabs = _record_to_flatten(rec)
        assert (S2, T2, R2) == (len(seqs), len(tok), len(last)) == (S, T, R)
        assert rows == orows
        assert toks.tolist() == tok.tolist()
        # positions and slots the device derives from the record
        for i, (off, n, wslots, rslots) in enumerate(meta):
            p = np.arange(starts[i], starts[i] + qlens[i])
            assert p.tolist() == pos[off:off + n].tolist()
            slots = tabs[i][p // bs] * bs + p % bs
            assert slots.tolist() == wslots.tolist()
        assert want.shape[0] == R
        assert bounds.tokens == T and bounds.rows == R
        assert bounds.decode_seqs == int((qlens == 1).sum())


def test_pack_rejects_what_the_reference_cannot_index():
    from vllt.runner import pack_step

    good = dict(start=0, n=3, count=1, tokens=[256, 1, 2], block_ids=[5], drafts=[])
    with pytest.raises(IndexError):
        pack_step(F.as_scheduler_output([dict(good, block_ids=[9999])]), 16, 512, 261, 512, 8)
    with pytest.raises(IndexError):
        pack_step(F.as_scheduler_output([dict(good, tokens=[256, 1, 999])]), 16, 512, 261, 512, 8)
    with pytest.raises(IndexError):
        pack_step(F.as_scheduler_output([dict(good, n=20, tokens=list(range(20)))]), 16, 512, 261, 512, 8)
    with pytest.raises(IndexError):
        pack_step(F.as_scheduler_output([dict(good, start=510, tokens=[0] * 3)]), 16, 512, 261, 512, 8)


def test_product_seeded_weights_equal_reference():
    from vllt.model import seeded_weights

    for name in ("tiny", "bench"):
        man = F.weights_manifest()[name]
        cfg = OM.Shape(vocab_size=261, **man["shape"])
        w = seeded_weights(cfg)
        got = {k: hashlib.sha256(np.ascontiguousarray(v).tobytes()).hexdigest() for k, v in w.items()}
        assert got == man["sha256"]


def test_product_rope_tables_equal_reference():
    from vllt.model import rope_tables

    z = F.load("rope.npz")
    for key in z.files:
        if key.startswith("cos_"):
            _, D, P = key.split("_")
            c, s = rope_tables(int(D), int(P))
            np.testing.assert_array_equal(c, z[key])
            np.testing.assert_array_equal(s, z[f"sin_{D}_{P}"])


@needs_vllmlite
def test_workloads_equal_reference_generator():
    from vllt.workloads import mixed_workload

    z = F.load("workload.npz")
    for name, prefix in (("mixed", 0), ("shared", 256)):
        reqs = mixed_workload(48, 0, prefix)
        lens = [len(r[1]) for r in reqs]
        assert lens == z[f"{name}_lens"].tolist()
        assert [t for r in reqs for t in r[1]] == z[f"{name}_tokens"].tolist()
        assert [r[2].max_tokens for r in reqs] == z[f"{name}_max_tokens"].tolist()


def test_pick_inputs_follow_the_reference_row_rules():
    """Host inputs of the device token picks (vllt.engine.pick_inputs): verify
    rows (sequences with drafts) take plain argmax and contribute their drafts;
    temperature rows are sampled; EOS is masked while min_tokens is not reached
    (sampling.py:51-52, only with an EOS id); the repetition penalty lands on
    the sequence's last row (sampling.py:54); a chunk that leaves tokens of its
    sequence uncomputed is neither masked, penalised nor sampled, since the
    reference only samples once every token has KV (engine.py:131-149)."""
    from types import SimpleNamespace as NS

    from vllt.engine import pick_inputs

    def item(drafts=(), greedy=True, min_tokens=0, out=0, pen=1.0, final=True):
        p = NS(greedy=greedy, min_tokens=min_tokens, repetition_penalty=pen)
        seq = NS(draft_token_ids=list(drafts), params=p, output_token_ids=[7] * out, num_tokens=10)
        return NS(seq=seq, start_pos=10 - 1 - (0 if final else 3), num_tokens=1)

    sched = [item(), item(drafts=(11, 12, 13)), item(greedy=False), item(min_tokens=5, out=2),
             item(min_tokens=5, out=5, pen=1.3), item(greedy=False, final=False),
             item(min_tokens=5, out=1, pen=1.5, final=False)]
    rows = [(0, 1), (1, 4), (5, 1), (6, 1), (7, 1), (8, 1), (9, 1)]
    cu, doff, drafts, mask, pen, sampled = pick_inputs(sched, rows, 10, eos=257)
    assert cu.tolist() == [0, 1, 5, 6, 7, 8, 9, 10] and cu.dtype == np.int32
    assert doff.tolist() == [0, 0, 3, 3, 3, 3, 3]
    assert drafts == [11, 12, 13]
    assert sampled == [(2, 5)]  # the non-final temperature chunk draws nothing
    assert mask.tolist() == [0, 0, 0, 0, 0, 0, 1, 0, 0, 0]
    assert pen.dtype == np.float32 and pen[7] == np.float32(1.3)
    assert (np.delete(pen, 7) == 1).all()  # nothing on the non-final chunk's row 9
    # no EOS id: min_tokens cannot mask anything
    assert not pick_inputs(sched, rows, 10, eos=None)[3].any()


def test_seen_bitmaps_mark_each_distinct_token_once():
    from types import SimpleNamespace as NS

    from vllt.engine import seen_bitmaps

    b = seen_bitmaps([NS(token_ids=[0, 31, 32, 260, 31]), None, NS(token_ids=[])], 261)
    assert b.shape == (3, 9) and b.dtype == np.uint32
    assert b[0, 0] == (1 | (1 << 31)) and b[0, 1] == 1 and b[0, 8] == 1 << (260 - 256)
    assert not b[1].any() and not b[2].any()


def test_graph_bucket_bounds_cover_every_step_of_the_bucket():
    """A captured forward serves every step whose token count fits its bucket:
    tokens round up to the next rung (multiples of 16 to 64, then four rungs
    per doubling, capped at the capacity) and the other bounds are derived
    from that alone, so they hold for any step of the bucket."""
    from types import SimpleNamespace as NS

    from vllt._lib import Caps, StepBounds
    from vllt.runner import CudaRunner, token_bucket

    fake = NS(caps=Caps(64, 1024, 1024, 32), qp=4, w=NS(rope_len=2048))
    for T in (1, 15, 16, 17, 65, 100, 257, 512, 513, 1000, 1024):
        b = CudaRunner.bucket(fake, StepBounds(T, min(T, 64), min(T, 64), 1, 2048))
        assert b.tokens >= max(T, 16) and b.tokens <= 1024
        assert b.rows >= min(T, 64) and b.decode_seqs >= min(T, 64)
        assert b.tiles >= (T + 3) // 4 and b.max_ctx == 2048
        # every smaller step in the same bucket maps to the same bounds
        same = CudaRunner.bucket(fake, StepBounds(b.tokens, 1, 1, 1, 1))
        assert (same.tokens, same.rows, same.decode_seqs, same.tiles) == (b.tokens, b.rows, b.decode_seqs, b.tiles)
    rungs = sorted({token_bucket(t) for t in range(1, 8193)})
    assert rungs[:8] == [16, 32, 48, 64, 80, 96, 112, 128] and rungs[-1] == 8192
    assert len(rungs) <= 4 + 4 * 7  # at most four graphs per doubling
    for t in range(1, 8193):  # at most 15 padded tokens up to 64, at most 25 % above
        assert t <= token_bucket(t) <= (t + 15 if t <= 64 else t * 1.25)
        assert token_bucket(token_bucket(t)) == token_bucket(t)


def test_llama_workload_has_the_benchmark_shape():
    """C4 requests: lognormal prompts of mean ~1024 clipped to [32, 8192] and
    outputs of mean ~256 clipped to [16, 1024], tokens over the vocabulary,
    deterministic per seed."""
    from vllt.workloads import llama_lengths

    a = llama_lengths(512, seed=0)
    assert a == llama_lengths(512, seed=0)
    plen = np.array([len(p) for p, _ in a])
    olen = np.array([m for _, m in a])
    assert plen.min() >= 32 and plen.max() <= 8192 and olen.min() >= 16 and olen.max() <= 1024
    assert 900 < plen.mean() < 1150 and 220 < olen.mean() < 290
    assert max(max(p) for p, _ in a) < 128256 and min(min(p) for p, _ in a) >= 0


def test_sources_hold_no_peer_memory_access():
    """No kernel or host file of the product maps or dereferences another
    GPU's memory: a fused all-reduce over CUDA IPC mappings faulted a GPU on
    this pool with a cause that reading did not find, so cross-GPU data moves
    through NCCL only. Every source that travels with the package is checked
    for the calls and instructions such code needs."""
    import glob

    banned = ("cudaIpcOpenMemHandle", "cudaIpcGetMemHandle", "cuMemImportFromShareableHandle",
              "multimem.", ".multicast::cluster", "ld.acquire.sys", "st.release.sys",
              "cudaDeviceEnablePeerAccess", "cuMulticast")
    files = (glob.glob(os.path.join(ROOT, "vllm-lite_b200", "csrc", "*")) +
             glob.glob(os.path.join(ROOT, "vllm-lite_b200", "vllt", "*.py")) +
             [os.path.join(ROOT, "include", "vllt.h"), os.path.join(ROOT, "bench.py")])
    assert len(files) > 20
    for f in files:
        src = open(f, errors="replace").read()
        for b in banned:
            assert b not in src, f"{os.path.relpath(f, ROOT)} names {b}"


def _fake_desc(dtype=0, tp_size=1, head_dim=48):
    """A model descriptor whose pointers are placeholders: every check below
    fails on the host, before any of them would be dereferenced."""
    import ctypes as C

    from vllt import _lib

    d = _lib.ModelDesc()
    d.n_layers, d.n_heads, d.n_kv_heads, d.head_dim = 2, 8, 4, head_dim
    d.d_model, d.d_ff, d.vocab, d.vocab_padded = 384, 1024, 261, 264
    d.max_seq_len, d.block_size, d.num_blocks, d.rms_eps = 512, 16, 64, 1e-5
    d.dtype, d.tp_size, d.embed_rows = dtype, tp_size, 261
    fake = 4096
    for k in ("tok_emb", "final_norm", "lm_head", "rope_cos", "rope_sin", "k_cache", "v_cache"):
        setattr(d, k, fake)
    arr = (C.c_void_p * 2)(fake, fake)
    for k in ("attn_norm", "wqkv", "wo", "ffn_norm", "w_gu", "w_down"):
        setattr(d, k, C.cast(arr, C.POINTER(C.c_void_p)))
    d._keep = arr
    return d


def test_c_abi_rejects_inconsistent_calls_before_any_launch():
    """Inconsistent calls come back as VLLT_ERR_ARG with a message, decided
    on the host from the arguments alone (no device is present here)."""
    import ctypes as C

    from vllt import _lib

    L = _lib.lib()
    caps = _lib.Caps(8, 64, 16, 32)
    bounds = _lib.StepBounds(64, 16, 8, 8, 512)
    fake = 4096

    def forward(desc, ws_bytes=16):
        return L.vllt_forward(C.byref(desc) if desc is not None else None, fake, C.byref(caps), C.byref(bounds),
                              fake, fake, ws_bytes, fake, None)

    assert forward(None) == _lib.VLLT_ERR_ARG and b"NULL" in L.vllt_last_error()
    assert forward(_fake_desc(dtype=7)) == _lib.VLLT_ERR_ARG and b"dtype" in L.vllt_last_error()
    assert forward(_fake_desc(tp_size=2)) == _lib.VLLT_ERR_ARG and b"tensor parallelism" in L.vllt_last_error()
    d = _fake_desc()
    d.table_pool, d.table_pool_slots = fake, 0
    assert forward(d) == _lib.VLLT_ERR_ARG and b"table_pool" in L.vllt_last_error()
    for hd in (6, 24, 256):  # a head size the attention kernels are not built for fails before any launch
        assert forward(_fake_desc(head_dim=hd)) == _lib.VLLT_ERR_ARG and b"head_dim" in L.vllt_last_error()
    assert forward(_fake_desc()) == _lib.VLLT_ERR_ARG and b"workspace too small" in L.vllt_last_error()
    need = L.vllt_forward_workspace_bytes(C.byref(_fake_desc()), C.byref(caps))
    assert need > 16
    # sampling: more rows than the logits buffer holds, and no row index to pick them
    assert L.vllt_sample_top_p(fake, 5, 261, 264, 4, None, None, 257, None, None, fake, None, None, fake, fake,
                               None) == _lib.VLLT_ERR_ARG
    # prefix hash: no chains is a no-op, a zero block size is refused
    assert L.vllt_prefix_hash_chains(None, None, None, None, None, 0, 16, None, None) == _lib.VLLT_OK
    assert L.vllt_prefix_hash_chains(fake, fake, fake, fake, None, 3, 0, fake, None) == _lib.VLLT_ERR_ARG
    # the allocation-free attention: unknown dtype
    assert L.vllt_paged_attention_varlen_noalloc(fake, fake, fake, fake, 4, fake, fake, 1, 1, 1, 16, 8, 4, 48, 16, 64,
                                                 0.1, 9, fake, None, None) == _lib.VLLT_ERR_ARG


def test_allreduce_share_counts_two_bucket_reductions_per_layer():
    """bench.py's estimate of the tensor-parallel collectives per pass: two
    all-reduces per layer of the pass's graph bucket of rows."""
    import bench

    ar_us = {16: 10.0, 32: 12.0, 512: 40.0, 640: 50.0}
    log = [(1, 1, None, None), (20, 20, None, None), (512, 512, None, None), (513, 10, None, None)]
    got = bench.allreduce_share(log, ar_us, n_layers=32, max_tokens=8192)
    assert abs(got - 2 * 32 * (10 + 12 + 40 + 50) / 1e6) < 1e-12


def test_latency_summary_uses_the_reference_percentiles():
    """bench.py reports p50 / p99 of TTFT, TPOT and request latency as the
    reference bench does (numpy percentiles of per-request seconds, in ms)."""
    import numpy as np

    import bench

    lat = bench.merge_latency([{"ttft": [0.1, 0.2], "tpot": [0.01], "e2e": [1.0, 2.0]},
                               {"ttft": [0.3], "tpot": [], "e2e": [3.0]}])
    got = bench.latency_summary(lat)
    assert got["ttft_p50_ms"] == 200.0 and got["ttft_p99_ms"] == round(1e3 * np.percentile([0.1, 0.2, 0.3], 99), 2)
    assert got["tpot_p50_ms"] == 10.0 and got["e2e_p99_ms"] == round(1e3 * np.percentile([1, 2, 3], 99), 2)
    assert bench.latency_summary({"ttft": [], "tpot": [], "e2e": []})["ttft_p50_ms"] is None


def test_build_fails_on_register_spills_outside_the_parity_gemm():
    """vllt/build.py compiles with ptxas -warn-spills and refuses a spill in
    any kernel but the fp32 parity GEMM: a spill in the decode, GEMM or
    attention kernels costs time that only a GPU profile would show."""
    from vllt import build as B

    out = ("ptxas warning : Registers are spilled to local memory in function "
           "'_ZN4vllt2dk13decode_kernelILi8EEEv14CUtensorMap_stS2_NS0_12DecodeParamsE', 8 bytes spill stores\n"
           "ptxas warning : Registers are spilled to local memory in function "
           "'_ZN4vllt12sgemm_kernelILi64ELi64ELi16ELi4ELi4ELi256ENS_8EpiStoreEEEvPKfiS3_iiPKiiiiPfPiT5_', 12 bytes\n"
           "ptxas info    : Used 165 registers, used 1 barriers\n")
    spilled = B.spilled_kernels(out)
    assert len(spilled) == 2
    bad = [k for k in spilled if not any(a in k for a in B.SPILL_ALLOWED)]
    assert bad == ["_ZN4vllt2dk13decode_kernelILi8EEEv14CUtensorMap_stS2_NS0_12DecodeParamsE"]
    assert "-warn-spills" in B.FLAGS


def test_device_helpers_do_not_call_themselves():
    """Helpers with a host alternative under the SIMT emulation have a device
    body that the host build never compiles; none of them may call itself (a
    refactor once turned an inline-PTX fence into a self-call)."""
    import glob

    n = 0
    for f in glob.glob(os.path.join(ROOT, "vllm-lite_b200", "csrc", "*.cu*")):
        src = open(f).read()
        for m in re.finditer(r"__device__ __forceinline__ [\w:<>]+ (\w+)\([^)]*\) \{", src):
            name, depth, i = m.group(1), 1, m.end()
            while depth:  # the body, to its matching brace
                depth += {"{": 1, "}": -1}.get(src[i], 0)
                i += 1
            body = src[m.end():i - 1]
            n += 1
            assert not re.search(r"\b%s\(" % name, body), f"{os.path.basename(f)}: {name} calls itself"
    assert n > 30


# The PTX instructions the library's inline assembly uses. The host build runs
# each helper's host branch, so the device branches' bodies are checked only
# on a GPU; this list holds what ran on the B200 (plus ld.shared::cluster.s32,
# the cluster's abort-flag read), and a new instruction has to be added here
# on purpose.
PTX_VOCABULARY = {
    "barrier.cluster.arrive.release.aligned", "barrier.cluster.wait.acquire.aligned",
    "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes",
    "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes",
    "cp.async.cg.shared.global", "cp.async.commit_group", "cp.async.wait_group", "ex2.approx.ftz.f32",
    "fence.mbarrier_init.release.cluster", "fence.proxy.async.shared::cta", "griddepcontrol.launch_dependents",
    "griddepcontrol.wait", "ld.shared::cluster.s32", "ld.shared::cluster.v4.f32", "mapa.shared::cluster.u32",
    "mbarrier.arrive.expect_tx.shared::cta.b64", "mbarrier.arrive.shared::cta.b64", "mbarrier.init.shared::cta.b64",
    "mbarrier.try_wait.parity.shared::cta.b64", "mov.u32", "mov.u64", "selp.u32", "setp.ne.b32",
    "tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32",
    "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64",
    "tcgen05.dealloc.cta_group::1.sync.aligned.b32", "tcgen05.fence::after_thread_sync",
    "tcgen05.fence::before_thread_sync", "tcgen05.ld.sync.aligned.32x32b.x32.b32", "tcgen05.mma.cta_group::1.kind::f16",
    "tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned", "tcgen05.st.sync.aligned.32x32b.x32.b32",
    "tcgen05.wait::ld.sync.aligned", "tcgen05.wait::st.sync.aligned",
}


def _asm_templates(src):
    """The instruction templates of every asm statement: the string literals
    before the statement's first operand colon."""
    import re

    out = []
    for m in re.finditer(r"\basm\s*(?:volatile)?\s*\(", src):
        i, depth, in_str, tpl = m.end(), 1, False, []
        while depth:
            c = src[i]
            if in_str:
                if c == "\\":
                    tpl.append(src[i:i + 2])
                    i += 1
                elif c == '"':
                    in_str = False
                else:
                    tpl.append(c)
            elif c == '"':
                in_str = True
            elif c == "(":
                depth += 1
            elif c == ")":
                depth -= 1
            elif c == ":":
                break
            i += 1
        out.append("".join(tpl))
    return out


def test_inline_ptx_uses_only_the_instructions_that_ran_on_the_b200():
    import glob
    import re

    used = set()
    for f in glob.glob(os.path.join(ROOT, "vllm-lite_b200", "csrc", "*")):
        for tpl in _asm_templates(open(f).read()):
            for stmt in re.split(r";|\\n", tpl):  # statements; a "{ ... }" scope opens one
                stmt = stmt.strip().lstrip("{").strip()
                if stmt and stmt != "}" and not stmt.startswith("."):  # .reg declarations
                    used.add(stmt.split()[0])
    assert used, "no inline assembly found"
    assert used <= PTX_VOCABULARY, sorted(used - PTX_VOCABULARY)
