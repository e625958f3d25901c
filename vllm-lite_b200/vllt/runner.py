"""CudaRunner: the B200 forward pass behind vllm-lite's ModelRunner interface.

Drop-in for `vllmlite.runner.NumpyRunner` (vllmlite/runner.py:35-100): same
constructor arguments (ModelConfig, CacheConfig), same
`execute(SchedulerOutput) -> (logits float32 [n_rows, V], rows)` contract,
`vocab_size` and `cache_bytes`. It
  * applies `out.cow` before any KV write (runner.py:63-64) with one copy kernel;
  * packs the step (per-sequence start / qlen / logit count, the pushed token
    ids and the block-table entries that changed since the last pass; the
    tables themselves stay in a persistent device pool) into one int32 record,
    uploads it with one host-to-device copy, and lets the device build
    positions, slots and rows (runner.py:66-90);
  * runs the whole TinyLlama forward (model.py:80-120) in libvllt with one call;
  * downloads only the logit rows.

There is no CPU fallback: without a CUDA device or without libvllt.so the
constructor raises.
"""

from __future__ import annotations

import ctypes as C
import math

import numpy as np

from . import _lib
from ._lib import Caps, ModelDesc, StepBounds, check, lib
from .model import DeviceWeights, initial_weights

try:  # the plug-in ABC of the host engine, when vllm-lite is importable
    from vllmlite.runner import ModelRunner as _Base
except Exception:  # pragma: no cover - standalone use of the runner
    from abc import ABC as _Base

EOS_ID = 257  # ByteTokenizer.eos_id (vllmlite/tokenizer.py:10)


def tile_positions(n_rep: int) -> int:
    """Query positions per attention tile (16 (position, head) rows)."""
    return 1 if n_rep >= 16 else 16 // n_rep


def _tokens(seq, start: int, n: int) -> list:
    """seq.token_ids[start:start+n] (prompt + output + drafts, vllmlite/sequence.py:70)
    without building the whole concatenation."""
    p = getattr(seq, "prompt_token_ids", None)
    if p is None:  # a duck-typed sequence that only carries token_ids
        return seq.token_ids[start:start + n]
    if n == 1 and start >= 0:  # a decode row: one token
        if start < len(p):
            return [p[start]]
        j = start - len(p)
        o = seq.output_token_ids
        if j < len(o):
            return [o[j]]
        d = seq.draft_token_ids
        return [d[j - len(o)]] if j - len(o) < len(d) else []
    end, out = start + n, []
    for part in (p, seq.output_token_ids, seq.draft_token_ids):
        ln = len(part)
        if start < ln and end > 0:
            out += part[max(start, 0):min(end, ln)]
        start -= ln
        end -= ln
        if end <= 0:
            break
    return out


def record_fields(rec, pooled: bool) -> dict:
    """Named views of a packed step record (layouts in include/vllt.h)."""
    S, T, R, W = (int(x) for x in rec[:4])
    U = int(rec[4]) if pooled else 0
    o = 5 if pooled else 4
    f = dict(S=S, T=T, R=R, W=W, U=U, start=rec[o:o + S], qlen=rec[o + S:o + 2 * S],
             count=rec[o + 2 * S:o + 3 * S], tokens=rec[o + 3 * S:o + 3 * S + T])
    o += 3 * S + T
    if pooled:
        f["slot"] = rec[o:o + S]
        f["updates"] = rec[o + S:o + S + 3 * U].reshape(U, 3)
    else:
        f["tables"] = rec[o:o + S * W].reshape(S, W)
    return f


class StepPacker:
    """Host side of the batch flatten: SchedulerOutput -> (record int32 words,
    StepBounds, rows, (S, T, R, W)).

    Reads exactly what vllmlite/runner.py:72-90 reads: item.start_pos,
    item.num_tokens, seq.token_ids (via _tokens), seq.draft_token_ids,
    seq.table.block_ids. The record layouts are documented in include/vllt.h.
    Metadata the reference would fail on (NumPy IndexError) raises here, before
    anything reaches the device.

    Only entries from the block being written onward can change between two
    passes of a sequence whose BlockTable object stays the same: blocks are
    appended, or the block at num_filled // block_size (= start_pos //
    block_size) is replaced by copy-on-write (block_manager.py:65-93); a table
    replaced after preemption or retirement is a new object.

    Classic record (pool_slots == 0): block tables are cached per sequence
    between passes, only the changed suffix is copied and validated, and the
    whole S x W table goes into the record.

    Pooled record (pool_slots > 0): the tables stay on the device in a
    persistent pool of pool_slots rows of pool_width ids. Each live sequence
    holds a row (keyed by request id; the least recently scheduled sequence
    gives its row up when none is free). The packer keeps a mirror of every
    row as the device holds it (-1 where unknown, the pool's initial value)
    and emits (row, index, block id) only for entries whose value differs:
    per decode pass that is the new or copied-on-write block, if any."""

    def __init__(self, block_size: int, num_blocks: int, vocab: int, max_pos: int, qp: int,
                 pool_slots: int = 0, pool_width: int = 0, token_refs: int = 0):
        self.bs, self.nb, self.vocab, self.max_pos, self.qp = block_size, num_blocks, vocab, max_pos, qp
        # token ids t in [-token_refs, -1] are references to entry -t - 1 of
        # the forward's token source (a token picked on the device, not yet read)
        self.token_refs = token_refs
        self.cache = {}
        self.pool_slots, self.pool_width = pool_slots, pool_width
        if pool_slots:
            if pool_width < 1:
                raise ValueError("a table pool needs a positive width")
            self.slot_of = {}  # sequence key -> pool row
            self.owner = [None] * pool_slots  # pool row -> [key, BlockTable, entries in use]
            self.mirror = np.full((pool_slots, pool_width), -1, np.int32)  # the device rows
            self.free = list(range(pool_slots - 1, -1, -1))
            self.last_used = np.full(pool_slots, -1, np.int64)
            self.passes = 0

    def _table(self, key, seq, start: int, new_cache):
        """(int32 buffer, length) of the sequence's block table, validated."""
        tbl = seq.table
        ids = tbl.block_ids
        n = len(ids)
        nb = self.nb
        ent = self.cache.get(key)
        if ent is None or ent[0] is not tbl or ent[2] > n:
            full = np.asarray(ids, dtype=np.int64) if n else np.zeros(0, np.int64)
            if n and (int(full.min()) < 0 or int(full.max()) >= nb):
                raise IndexError("block id out of range")
            arr = full.astype(np.int32)
        else:
            arr, first = ent[1], min(ent[2], start // self.bs)
            if arr.size < n:
                grown = np.empty(max(n, 2 * arr.size), np.int32)
                grown[:arr.size] = arr
                arr = grown
            if n - first <= 8:  # a decode step touches one or two entries: plain Python is cheaper
                for j in range(first, n):
                    v = ids[j]
                    if v < 0 or v >= nb:
                        raise IndexError("block id out of range")
                    arr[j] = v
            else:
                seg = np.asarray(ids[first:n], dtype=np.int64)
                if int(seg.min()) < 0 or int(seg.max()) >= nb:
                    raise IndexError("block id out of range")
                arr[first:n] = seg
        new_cache[key] = (tbl, arr, n)
        return arr, n

    def _take_row(self, in_step: set) -> int:
        if self.free:
            return self.free.pop()
        best = -1
        for r in range(self.pool_slots):  # least recently scheduled row not in this pass
            if self.owner[r][0] not in in_step and (best < 0 or self.last_used[r] < self.last_used[best]):
                best = r
        if best < 0:
            raise ValueError(f"more sequences in one pass than table pool rows ({self.pool_slots})")
        del self.slot_of[self.owner[best][0]]
        return best

    def _pool_row(self, key, seq, start: int, in_step: set, updates: list) -> tuple:
        """(pool row, table length) of the sequence; appends the (row, index,
        block) entries the device row lacks to `updates`."""
        tbl = seq.table
        ids = tbl.block_ids
        n = len(ids)
        if n > self.pool_width:
            raise ValueError(f"block table of {n} entries exceeds the pool width {self.pool_width}")
        r = self.slot_of.get(key)
        if r is None:
            r = self._take_row(in_step)
            self.slot_of[key] = r
            self.owner[r] = [key, None, 0]
        own = self.owner[r]
        # entries before the written block keep their values while the table object is the same
        first = min(own[2], start // self.bs) if own[1] is tbl and own[2] <= n else 0
        row, nb = self.mirror[r], self.nb
        if n - first <= 16:  # a decode pass: one or two entries, plain Python is cheaper
            for j in range(first, n):
                v = ids[j]
                if v < 0 or v >= nb:
                    raise IndexError("block id out of range")
                if v != row[j]:
                    row[j] = v
                    updates += (r, j, v)
        elif n > first:
            seg = np.asarray(ids[first:n], dtype=np.int64)
            if int(seg.min()) < 0 or int(seg.max()) >= nb:
                raise IndexError("block id out of range")
            diff = np.flatnonzero(seg != row[first:n]) + first
            row[first:n] = seg
            if diff.size:
                trip = np.empty((diff.size, 3), np.int64)
                trip[:, 0], trip[:, 1], trip[:, 2] = r, diff, row[diff]
                updates += trip.ravel().tolist()
        own[1], own[2] = tbl, n
        self.last_used[r] = self.passes
        in_step.add(key)
        return r, n

    def pack(self, out):
        items = out.scheduled
        S = len(items)
        pooled = self.pool_slots > 0
        starts, qlens, counts = [0] * S, [0] * S, [0] * S
        tabs, tab_n = [None] * S, [0] * S
        toks = []
        new_cache = {}
        in_step, updates = set(), []
        bs, max_pos = self.bs, self.max_pos
        W, max_ctx = 1, 1
        if pooled:
            self.passes += 1
        for i, item in enumerate(items):
            seq = item.seq
            start, n = item.start_pos, item.num_tokens
            if n < 1:
                raise ValueError("a scheduled sequence has no tokens")
            ctx = start + n
            if ctx > max_pos:
                raise IndexError(f"position {ctx - 1} beyond max_seq_len {max_pos}")
            key = getattr(seq, "request_id", None) or id(seq)
            if pooled:
                if key in in_step:
                    raise ValueError("a sequence is scheduled twice in one pass")
                arr, tn = self._pool_row(key, seq, start, in_step, updates)
            else:
                arr, tn = self._table(key, seq, start, new_cache)
            if tn * bs < ctx:
                raise IndexError(f"block table of sequence {i} too short for {ctx} positions")
            starts[i] = start
            qlens[i] = n
            d = len(seq.draft_token_ids) + 1
            counts[i] = d if d < n else n
            toks += _tokens(seq, start, n)
            tabs[i] = arr
            tab_n[i] = tn
            if tn > W:
                W = tn
            if ctx > max_ctx:
                max_ctx = ctx
        if not pooled:
            self.cache = new_cache
        T = len(toks)
        R = sum(counts)
        tok = np.asarray(toks, dtype=np.int64)
        if T and (int(tok.min()) < -self.token_refs or int(tok.max()) >= self.vocab):
            raise IndexError("token id out of the vocabulary")
        if pooled:
            U = len(updates) // 3
            hdr = 5 + 3 * S
            rec = np.empty(hdr + T + S + 3 * U, np.int32)
            rec[0], rec[1], rec[2], rec[3], rec[4] = S, T, R, W, U
            o = 5
        else:
            hdr = 4 + 3 * S
            rec = np.zeros(hdr + T + S * W, np.int32)
            rec[0], rec[1], rec[2], rec[3] = S, T, R, W
            o = 4
        rec[o:o + S] = starts
        rec[o + S:o + 2 * S] = qlens
        rec[o + 2 * S:hdr] = counts
        rec[hdr:hdr + T] = tok
        if pooled:
            rec[hdr + T:hdr + T + S] = tabs
            rec[hdr + T + S:] = updates
        else:
            table = rec[hdr + T:].reshape(S, W)
            for i in range(S):
                tn = tab_n[i]
                table[i, :tn] = tabs[i][:tn]
        n_dec = qlens.count(1)
        qp = self.qp
        tiles = sum((q + qp - 1) // qp for q in qlens if q > 1)
        bounds = StepBounds(T, R, n_dec, tiles, max_ctx)
        rows, r0 = [], 0
        for c in counts:
            rows.append((r0, c))
            r0 += c
        return rec, bounds, rows, (S, T, R, W)

    def fields(self, rec) -> dict:
        return record_fields(rec, self.pool_slots > 0)


def pack_step(out, block_size: int, num_blocks: int, vocab: int, max_pos: int, qp: int):
    """One-off packing (no table cache); see StepPacker."""
    return StepPacker(block_size, num_blocks, vocab, max_pos, qp).pack(out)


def token_bucket(tokens: int) -> int:
    """The token capacity of the CUDA graph that serves a pass of `tokens`
    tokens: multiples of 16 up to 64, then four rungs per doubling
    (80, 96, 112, 128, 160, ...). The forward's GEMMs, attention grids and
    the tensor-parallel all-reduces (`rows x d_model` words) work on the
    bucket's rows, so a pass of more than 64 tokens pays at most 25 % over
    its tokens (at most 15 tokens below) instead of the up to 2x of
    power-of-two buckets, with at most 4 graphs per doubling."""
    if tokens <= 64:
        return max(16, -(-tokens // 16) * 16)
    top = 64
    while top < tokens:
        top *= 2
    step = top // 8  # the rungs of (top/2, top]: top/2 + j * top/8
    return -(-tokens // step) * step


def step_needs(out):
    """(S, T, R, W) of a SchedulerOutput without packing it: sequences, tokens,
    logit rows (runner.py:88) and the widest block table."""
    S = len(out.scheduled)
    T = R = 0
    W = 1
    for item in out.scheduled:
        n = item.num_tokens
        T += n
        d = len(item.seq.draft_token_ids) + 1
        R += d if d < n else n
        w = len(item.seq.table.block_ids)
        if w > W:
            W = w
    return S, T, R, W


class CudaRunner(_Base):
    """fp32 parity-mode forward pass on one GPU."""

    def __init__(self, model_cfg, cache_cfg, sched_cfg=None, *, weights=None, device=None,
                 max_seqs: int | None = None, max_tokens: int | None = None, use_graphs: bool = True,
                 bucket_bounds: bool = False, pooled_tables: bool = True):
        import torch

        self.pooled_tables = pooled_tables  # block tables resident on the device (pooled records)
        if not torch.cuda.is_available():
            raise RuntimeError("CudaRunner needs a CUDA device; there is no CPU fallback")
        self.torch = torch
        self.L = lib()
        self.model_cfg = model_cfg
        self.block_size = cache_cfg.block_size
        self.num_blocks = cache_cfg.num_blocks
        self.dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.head_dim = model_cfg.d_model // model_cfg.n_heads
        self.n_rep = model_cfg.n_heads // model_cfg.n_kv_heads
        self.qp = tile_positions(self.n_rep)
        with torch.cuda.device(self.dev):
            self._init_model(weights)
        self._ptrs = self.w.pointer_arrays()
        self.desc = self._make_desc()
        self.qp = self.L.vllt_query_tile_positions(C.byref(self.desc))  # tile height the forward uses
        self.caps = Caps(0, 0, 0, 0)
        self.use_graphs = use_graphs
        self.bucket_bounds = bucket_bounds  # eager runs with the graphs' bounds (tests)
        self.graphs = {}  # token bucket -> (CUDAGraph, StepBounds, kernels in the graph)
        self.replayed_kernels = 0  # kernels launched by graph replays
        self.captured_kernels = 0  # launch-site calls made while capturing (not executed)
        seqs = max_seqs or (sched_cfg.max_seqs if sched_cfg is not None else 64)
        toks = max_tokens or (sched_cfg.max_batched_tokens if sched_cfg is not None else 2048)
        # logit rows: one per sequence plus drafts; grown on demand (_reserve)
        self._reserve(seqs, toks, min(toks, 4 * seqs), self._table_width_for(model_cfg.max_seq_len))
        self.steps = 0
        self.h2d_bytes = 0  # host->device bytes copied by execute()/launch()
        self.d2h_bytes = 0  # device->host bytes copied by execute()

    def _init_model(self, weights) -> None:
        """fp32 parity weights in libvllt's layout and the fp32 paged KV cache."""
        torch, cfg = self.torch, self.model_cfg
        w = weights if weights is not None else initial_weights(cfg)
        self.w = DeviceWeights(cfg, w, self.dev)
        shape = (cfg.n_layers, self.num_blocks, cfg.n_kv_heads, self.block_size, self.head_dim)
        self.cache_k = torch.zeros(shape, dtype=torch.float32, device=self.dev)
        self.cache_v = torch.zeros(shape, dtype=torch.float32, device=self.dev)

    # ---- ModelRunner properties ------------------------------------------------
    @property
    def vocab_size(self) -> int:
        return self.model_cfg.vocab_size

    @property
    def cache_bytes(self) -> int:
        return self.cache_k.numel() * self.cache_k.element_size() * 2

    # ---- buffers -----------------------------------------------------------------
    def _table_width_for(self, ctx: int) -> int:
        return max(1, math.ceil(ctx / self.block_size))

    def _make_desc(self) -> ModelDesc:
        cfg, w, p = self.model_cfg, self.w, self._ptrs
        d = ModelDesc()
        d.n_layers, d.n_heads, d.n_kv_heads = cfg.n_layers, cfg.n_heads, cfg.n_kv_heads
        d.head_dim, d.d_model, d.d_ff = self.head_dim, cfg.d_model, cfg.d_ff
        d.vocab, d.vocab_padded = cfg.vocab_size, w.vocab_padded
        d.max_seq_len, d.block_size, d.num_blocks = w.rope_len, self.block_size, self.num_blocks
        d.rms_eps, d.dtype = 1e-5, _lib.VLLT_F32
        d.tp_size, d.embed_rows, d.tp_comm = 1, cfg.vocab_size, None
        d.tok_emb, d.final_norm, d.lm_head = w.tok_emb.data_ptr(), w.final_norm.data_ptr(), w.lm_head.data_ptr()
        d.rope_cos, d.rope_sin = w.rope_cos.data_ptr(), w.rope_sin.data_ptr()
        for k in ("attn_norm", "wqkv", "wo", "ffn_norm", "w_gu", "w_down"):
            setattr(d, k, C.cast(p[k], C.POINTER(C.c_void_p)))
        d.k_cache, d.v_cache = self.cache_k.data_ptr(), self.cache_v.data_ptr()
        return d

    def _reserve(self, S: int, T: int, R: int, W: int) -> None:
        """Grow the step buffers to at least (S, T, R, W); never shrinks."""
        torch = self.torch
        c = self.caps
        if S <= c.max_seqs and T <= c.max_tokens and R <= c.max_rows and W <= c.max_table_width:
            return
        torch.cuda.current_stream(self.dev).synchronize()
        caps = Caps(max(S, c.max_seqs), max(T, c.max_tokens), max(R, c.max_rows), max(W, c.max_table_width))
        # words of the largest record: the classic one, or a pooled one whose every entry is new
        rec_words = 5 + 4 * caps.max_seqs + caps.max_tokens + 3 * caps.max_seqs * caps.max_table_width
        meta_bytes = self.L.vllt_meta_bytes(C.byref(caps))
        ws_bytes = self.L.vllt_forward_workspace_bytes(C.byref(self.desc), C.byref(caps))
        if meta_bytes < 0 or ws_bytes < 0:
            raise ValueError("bad runner capacities")
        kw = dict(device=self.dev)
        # two pinned staging buffers for the record, used in turn: with the
        # engine running ahead, the previous record's copy may still be queued
        # behind a running pass when the next record is packed
        self._rec_bufs = [torch.empty(rec_words, dtype=torch.int32, pin_memory=True) for _ in range(2)]
        self._rec_copied = [None, None]  # event after the copy that last read each buffer
        self._rec_i = 0
        self.rec_host = self._rec_bufs[0]
        self.rec_dev = torch.empty(rec_words, dtype=torch.int32, **kw)
        self.meta = torch.empty((meta_bytes + 3) // 4, dtype=torch.int32, **kw)
        self.ws = torch.zeros(max(ws_bytes, 16), dtype=torch.uint8, **kw)  # split-K counters start at 0
        self.logits_dev = torch.empty((caps.max_rows, self.w.vocab_padded), dtype=torch.float32, **kw)
        self.logits_host = None  # pinned, allocated by the first execute()
        if self.pooled_tables:
            # the persistent block tables: one row per live sequence, twice the
            # sequences of a pass so that finished sequences rarely have to be
            # evicted before their rows are reused; -1 = unknown, as the packer's mirror
            slots = 2 * caps.max_seqs
            self.table_pool = torch.full((slots, caps.max_table_width), -1, dtype=torch.int32, **kw)
            self.desc.table_pool, self.desc.table_pool_slots = self.table_pool.data_ptr(), slots
        # the pick buffer of the engine's token picks (row picks, flag word,
        # accepted drafts, masked / sampled picks: 2 (R + S) + 1 words at most);
        # the forward reads tokens it has not handed to the host yet from it
        # (record ids < 0), so it keeps its contents when it grows
        words = 2 * (caps.max_rows + caps.max_seqs) + 1
        old = getattr(self, "picks_dev", None)
        self.picks_dev = torch.zeros(words, dtype=torch.int32, **kw)
        if old is not None:
            self.picks_dev[:old.numel()].copy_(old)
        self.desc.token_source, self.desc.token_source_len = self.picks_dev.data_ptr(), words
        self.packer = None  # its mirror describes the old pool
        self._on_reserve(caps)
        self.counters_host = torch.empty(16, dtype=torch.int32, pin_memory=True)
        self.caps = caps
        self.graphs = {}  # captured pointers are stale now

    # ---- the step ------------------------------------------------------------------
    def pack(self, out):
        """Reserve capacity for the step, then pack it (a grown table pool
        starts a new packer, whose first record reloads every table)."""
        self._reserve(*step_needs(out))
        if getattr(self, "packer", None) is None or self.packer.qp != self.qp:
            pool = self.desc.table_pool_slots if self.pooled_tables else 0
            self.packer = StepPacker(self.block_size, self.num_blocks, self.model_cfg.vocab_size,
                                     self.w.rope_len, self.qp, pool_slots=pool,
                                     pool_width=self.caps.max_table_width, token_refs=self.picks_dev.numel())
        return self.packer.pack(out)

    def pick_buffer(self, n: int):
        """The first n words of the pick buffer (device int32), where the
        engine's pick kernels write and the next forward resolves record
        token ids < 0 from."""
        if n > self.picks_dev.numel():
            raise ValueError("pick buffer smaller than the step's picks")
        return self.picks_dev[:n]

    def copy_on_write(self, pairs) -> None:
        """Apply (src_block, dst_block) copies in every layer (runner.py:54-60)."""
        if not pairs:
            return
        torch = self.torch
        a = np.asarray(pairs, np.int64).reshape(-1, 2)
        if int(a.min()) < 0 or int(a.max()) >= self.num_blocks:  # checked on the host: no device read
            raise IndexError("copy-on-write block id out of range")
        p = torch.from_numpy(a.astype(np.int32)).pin_memory().to(self.dev, non_blocking=True)  # no wait on the stream
        self._cow_pairs = p  # referenced until the copy kernel has been enqueued
        self.copy_blocks_on_device(p.data_ptr(), len(pairs))

    def copy_blocks_on_device(self, pairs_ptr: int, n_pairs: int) -> None:
        """Enqueue the block copies of n_pairs (src, dst) int32 pairs at a
        device address, in this runner's caches: every layer, this rank's KV
        heads ([L][blocks][n_kv][block][D]), the caches' element type."""
        L, nb, n_kv, bs, D = self.cache_k.shape
        dtype = _lib.VLLT_BF16 if self.cache_k.dtype == self.torch.bfloat16 else _lib.VLLT_F32
        check(self.L.vllt_copy_blocks(self.cache_k.data_ptr(), self.cache_v.data_ptr(), pairs_ptr, n_pairs, L, nb,
                                      n_kv, bs, D, dtype, _lib.stream_handle()))

    def _on_reserve(self, caps) -> None:
        """Hook for subclasses that size extra buffers by the capacities."""

    def check_step_flags(self, err: int) -> None:
        """Raise if the device's metadata builder flagged the last pass (bit 0
        capacity, bit 1 block table / range). Its pool updates may not all
        have landed, so the packer is dropped: the next pass uploads every
        table it needs whole."""
        if err:
            self.packer = None
            raise RuntimeError(f"libvllt rejected the step metadata on the device (flags {err})")

    def launch(self, out):
        """Enqueue CoW + H2D + forward for one SchedulerOutput; returns (rows, R)."""
        torch = self.torch
        self.copy_on_write(out.cow)
        rec, bounds, rows, (S, T, R, W) = self.pack(out)
        n = rec.size
        self._last_n = n
        self._last_rec = rec
        i = self._rec_i
        if self._rec_copied[i] is not None:
            self._rec_copied[i].synchronize()  # the copy that last read this buffer has run
        buf = self._rec_bufs[i]
        buf[:n].numpy()[:] = rec
        self.rec_dev[:n].copy_(buf[:n], non_blocking=True)
        ev = self._rec_copied[i] = torch.cuda.Event()
        ev.record()
        self._rec_i = i ^ 1
        self.rec_host = buf
        self.h2d_bytes += 4 * n + 8 * len(out.cow)
        self._timed_forward(bounds)
        self.steps += 1
        return rows, R

    def _timed_forward(self, bounds) -> None:
        """Enqueue the forward (graph or eager); with `pass_log` set (a list),
        bracket it with CUDA events and log (tokens, decode_seqs, e0, e1)."""
        log = getattr(self, "pass_log", None)
        if log is not None:
            e0 = self.torch.cuda.Event(enable_timing=True)
            e1 = self.torch.cuda.Event(enable_timing=True)
            e0.record()
        self._dispatch(bounds)
        if log is not None:
            e1.record()
            log.append((bounds.tokens, bounds.decode_seqs, e0, e1))

    def _dispatch(self, bounds) -> None:
        if self.use_graphs:
            self._forward_graph(bounds)
        else:
            self._forward(self.bucket(bounds) if self.bucket_bounds else bounds)

    def pass_summary(self) -> dict:
        """GPU seconds of the logged passes, split into passes with prompt
        tokens (tokens > decode sequences) and decode-only passes."""
        log = getattr(self, "pass_log", None) or []
        if log:
            log[-1][3].synchronize()
        pre = dec = 0.0
        n_pre = n_dec = 0
        for tokens, dec_seqs, e0, e1 in log:
            t = e0.elapsed_time(e1) / 1e3
            if tokens > dec_seqs:
                pre, n_pre = pre + t, n_pre + 1
            else:
                dec, n_dec = dec + t, n_dec + 1
        return {"passes": len(log), "gpu_s": round(pre + dec, 4), "prefill_passes": n_pre,
                "prefill_pass_gpu_s": round(pre, 4), "decode_passes": n_dec, "decode_pass_gpu_s": round(dec, 4)}

    def _forward(self, bounds) -> None:
        check(self.L.vllt_forward(C.byref(self.desc), self.rec_dev.data_ptr(), C.byref(self.caps),
                                  C.byref(bounds), self.meta.data_ptr(), self.ws.data_ptr(),
                                  self.ws.numel(), self.logits_dev.data_ptr(), _lib.stream_handle()))

    def bucket(self, b) -> StepBounds:
        """Bounds of the graph that serves a step: tokens rounded up to the
        next rung of token_bucket's ladder; everything else derived from that,
        so the graph is valid for every step whose token count fits."""
        c = self.caps
        T = min(token_bucket(b.tokens), c.max_tokens)
        return StepBounds(T, min(T, c.max_rows), min(T, c.max_seqs), T // self.qp + c.max_seqs, self.w.rope_len)

    def _forward_graph(self, bounds) -> None:
        """Replay the captured forward of this step's bucket; the first step of
        a bucket runs eagerly (that run is the step's result) and is captured."""
        torch = self.torch
        gb = self.bucket(bounds)
        hit = self.graphs.get(gb.tokens)
        if hit is not None:
            hit[0].replay()
            self.replayed_kernels += hit[2]
            return
        self._forward(gb)  # eager: this step's result, and first-use setup of every kernel
        g = torch.cuda.CUDAGraph()
        n0 = self.L.vllt_kernel_launches()
        with torch.cuda.graph(g):
            self._forward(gb)  # captured only; replays recompute a step idempotently
        n = self.L.vllt_kernel_launches() - n0
        self.captured_kernels += n
        self.graphs[gb.tokens] = (g, gb, n)

    def execute(self, out):
        """(logits float32 [n_rows, vocab], rows), as vllmlite/runner.py:62-100."""
        torch = self.torch
        with torch.cuda.device(self.dev):
            rows, R = self.launch(out)
            if self.logits_host is None or self.logits_host.shape[0] < self.logits_dev.shape[0]:
                self.logits_host = torch.empty(self.logits_dev.shape, dtype=torch.float32, pin_memory=True)
            self.logits_host[:R].copy_(self.logits_dev[:R], non_blocking=True)
            self.counters_host.copy_(self.meta[:16], non_blocking=True)
            self.d2h_bytes += R * self.w.vocab_padded * 4 + 64
            torch.cuda.current_stream(self.dev).synchronize()
        self.check_step_flags(int(self.counters_host[7]))
        logits = self.logits_host[:R, :self.model_cfg.vocab_size].numpy().copy()
        return logits, rows
