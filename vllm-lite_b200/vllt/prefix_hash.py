"""Prefix-cache block hashes on the device (vllt_prefix_hash_chains).

vllm-lite's BlockManager names every full KV block by a chained content hash,
`hash_block(prev_hex, token_ids)` (vllmlite/block.py:34-40), computed on the
host one block at a time when a prompt is admitted (reuse_prefix,
vllmlite/block_manager.py:33-62) and when a pass fills blocks (commit,
:98-120). `hash_chains` computes whole chains of such hashes in one launch,
bit-identical to the reference's digests.

`DevicePrefixHasher` plugs the device hashes into an engine without changing
the BlockManager: before each pass it hashes the prompts the scheduler may
admit (sequences in `waiting` without blocks), and right after the forward is
enqueued it enqueues the chains that the pass's commits can complete
(per scheduled sequence, the blocks from num_filled // block_size up to its
pushed tokens, capped at the tokens present once drafts are cleared); their
digests come back with the token picks. While the pass runs, the
BlockManager's `hash_block` is a lookup in those digests; a key that was not
planned is hashed on the device on the spot (one launch) and counted in
`misses`. Measured with the reference scheduler on the shared-prefix benchmark
the host hashes are ~1.5 % of the engine's host time, so the engine leaves
this off unless asked (`gpu_engine(..., device_prefix_hash=True)`).
"""

from __future__ import annotations

import contextlib

import numpy as np

from . import _lib
from ._lib import check


def pack_chains(chains, block_size: int):
    """Host arrays of vllt_prefix_hash_chains for chains [(prev_hex or None,
    tokens)], len(tokens) a multiple of block_size: (tokens int32,
    token_offsets int64, n_blocks int32, out_offsets int64, prev_hex uint8
    [n][32] with zero rows for None, total blocks)."""
    n = len(chains)
    nblk = np.empty(n, np.int32)
    tok_off = np.empty(n, np.int64)
    out_off = np.empty(n, np.int64)
    prev = np.zeros((n, 32), np.uint8)
    parts = []
    t = o = 0
    for c, (p, toks) in enumerate(chains):
        if len(toks) % block_size:
            raise ValueError("a hash chain holds whole blocks only")
        if p:
            raw = p.encode()
            if len(raw) != 32:
                raise ValueError("a previous block hash is 32 hex characters")
            prev[c] = np.frombuffer(raw, np.uint8)
        nb = len(toks) // block_size
        nblk[c], tok_off[c], out_off[c] = nb, t, o
        parts.append(np.asarray(toks, np.int32))
        t += len(toks)
        o += nb
    tokens = np.concatenate(parts) if parts else np.zeros(0, np.int32)
    return tokens, tok_off, nblk, out_off, prev, int(o)


def unpack_digests(out: np.ndarray, nblk) -> list:
    """uint8 [total * 32] -> per chain, the list of hex digests."""
    res, o = [], 0
    raw = out.tobytes()
    for nb in nblk:
        res.append([raw[32 * (o + b):32 * (o + b + 1)].decode() for b in range(int(nb))])
        o += int(nb)
    return res


class PendingHashes:
    """Digests of one launch, readable once the stream has passed it."""

    def __init__(self, chains, out, nblk, keep):
        self.chains, self.out, self.nblk, self.keep = chains, out, nblk, keep

    def result(self) -> list:
        return unpack_digests(self.out.cpu().numpy(), self.nblk)


def launch_chains(chains, block_size: int, device, lib=None) -> PendingHashes:
    """Enqueue one vllt_prefix_hash_chains launch on the current stream."""
    import torch

    L = lib or _lib.lib()
    tokens, tok_off, nblk, out_off, prev, total = pack_chains(chains, block_size)

    def up(a):
        return torch.from_numpy(np.ascontiguousarray(a)).to(device, non_blocking=True)

    d = [up(a) for a in (tokens if tokens.size else np.zeros(1, np.int32), tok_off, nblk, out_off, prev)]
    out = torch.empty(max(total, 1) * 32, dtype=torch.uint8, device=device)
    check(L.vllt_prefix_hash_chains(d[0].data_ptr(), d[1].data_ptr(), d[2].data_ptr(), d[3].data_ptr(),
                                    d[4].data_ptr(), len(chains), block_size, out.data_ptr(),
                                    _lib.stream_handle()))
    return PendingHashes(chains, out[:total * 32], nblk, d)


def hash_chains(chains, block_size: int, device=None, lib=None) -> list:
    """Per chain (prev_hex or None, tokens), the hex digest of every block, as
    the reference's hash_block chains them. Runs on the device; returns after
    the digests are on the host."""
    import torch

    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    return launch_chains(chains, block_size, dev, lib).result()


class DevicePrefixHasher:
    """Device-computed block hashes behind an engine's unchanged BlockManager."""

    def __init__(self, engine, lib=None):
        import vllmlite.block_manager as bm

        self.eng = engine
        self.bm = bm
        self.blocks = engine.scheduler.blocks
        self.bs = self.blocks.block_size
        self.lib = lib
        self.prompt_memo = {}  # (prev, tokens) -> digest of the waiting prompts' chains
        self.prompt_refs = {}  # key -> waiting requests whose chain holds it (shared prefixes)
        self.prompt_keys = {}  # request id -> (prompt length, its keys) while it waits
        self.step_memo = {}  # digests of the current pass's commits
        self.pending = None
        self.misses = self.planned = self.lookups = 0

    @contextlib.contextmanager
    def active(self):
        """The BlockManager's hash_block reads the device digests meanwhile."""
        orig = self.bm.hash_block
        self.bm.hash_block = self.lookup
        try:
            yield self
        finally:
            self.bm.hash_block = orig

    def _dev(self):
        return self.eng.runner.dev

    def _digests(self, chains, digests, into):
        keys = []
        for (prev, toks), hs in zip(chains, digests):
            for b, h in enumerate(hs):
                key = (prev or None, tuple(toks[b * self.bs:(b + 1) * self.bs]))
                into[key] = h
                keys.append(key)
                prev = h
            self.planned += len(hs)
        return keys

    def lookup(self, prev_hash, token_ids):
        self.lookups += 1
        key = (prev_hash or None, tuple(token_ids))
        h = self.step_memo.get(key)
        if h is None:
            h = self.prompt_memo.get(key)
        if h is None:  # not planned: hash it now, still on the device
            self.misses += 1
            h = hash_chains([(prev_hash, list(token_ids))], len(token_ids), self._dev(), self.lib)[0][0]
            self.step_memo[key] = h
        return h

    def _drop_prompt(self, rid):
        for key in self.prompt_keys.pop(rid)[1]:
            n = self.prompt_refs[key] - 1
            if n:
                self.prompt_refs[key] = n
            else:
                del self.prompt_refs[key]
                del self.prompt_memo[key]

    def prepare_prompts(self):
        """Before schedule(): the prompt chains reuse_prefix may ask for
        (block_manager.py:43-55: the first (len - 1) // block_size blocks of
        each waiting sequence that holds no blocks), hashed in one launch;
        a request's chain is kept while it waits and dropped once admitted."""
        if not self.blocks.prefix_caching:
            return
        chains, rids, waiting = [], [], set()
        for seq in self.eng.scheduler.waiting:
            if seq.num_computed or seq.table.block_ids:
                continue
            toks = seq.prompt_token_ids
            n = (len(toks) - 1) // self.bs
            if n <= 0:
                continue
            waiting.add(seq.request_id)
            have = self.prompt_keys.get(seq.request_id)
            if have is not None and have[0] == len(toks):
                continue
            if have is not None:  # the prompt changed (a preempted sequence): re-hash it
                self._drop_prompt(seq.request_id)
            chains.append((None, list(toks[:n * self.bs])))
            rids.append((seq.request_id, len(toks)))
        for rid in [r for r in self.prompt_keys if r not in waiting]:
            self._drop_prompt(rid)
        if chains:
            for chain, hs, (rid, n) in zip(chains, hash_chains(chains, self.bs, self._dev(), self.lib), rids):
                keys = self._digests([chain], [hs], self.prompt_memo)
                for key in keys:
                    self.prompt_refs[key] = self.prompt_refs.get(key, 0) + 1
                self.prompt_keys[rid] = (n, keys)

    def prepare_commits(self, sched):
        """After the forward is enqueued: the chains this pass's commits can
        complete (block_manager.py:98-120), enqueued on the same stream."""
        self.step_memo = {}
        if not self.blocks.prefix_caching:
            return
        chains, allocator = [], self.blocks.allocator
        for item in sched.scheduled:
            seq = item.seq
            tbl = seq.table
            before = tbl.num_filled
            # commit hashes seq.token_ids after the drafts are cleared (engine.py:119-129)
            n_tok = len(seq.prompt_token_ids) + len(seq.output_token_ids)
            first, last = before // self.bs, min(before + item.num_tokens, n_tok) // self.bs
            if last <= first:
                continue
            prev = allocator.blocks[tbl.block_ids[first - 1]].content_hash if first > 0 else None
            toks = (seq.prompt_token_ids + seq.output_token_ids)[first * self.bs:last * self.bs]
            chains.append((prev, toks))
        self.pending = launch_chains(chains, self.bs, self._dev(), self.lib) if chains else None

    def collect(self):
        """After the pass's token picks are on the host: install the digests."""
        if self.pending is not None:
            self._digests(self.pending.chains, self.pending.result(), self.step_memo)
            self.pending = None
