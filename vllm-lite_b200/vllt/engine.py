"""Engine entry points: vllm-lite's LLMEngine driving the CUDA runner.

`cuda_engine(cfg, ...)` returns an unmodified `vllmlite.engine.LLMEngine`
whose runner is `CudaRunner` instead of the hard-coded NumpyRunner
(vllmlite/engine.py:46): Scheduler, BlockManager, prefix hashing,
preemption, sampling and the n-gram proposer are the reference's own code.
Logits come back to the host every step, exactly as the reference expects.

`GpuLLMEngine` keeps all of that but replaces the sampling half of
LLMEngine.step (engine.py:113-148) by device kernels: one launch picks the
argmax of every logit row (with the min_tokens EOS mask and the repetition
penalty, sampling.py:41-57) and one applies the speculative accept/reject rule
(speculative.py:86-100); temperature rows go through the device sampler
(mask, penalty, temperature, top-k, top-p, sampling.py:41-64) with the
request's own generator supplying the uniform numpy's choice() would draw.
Only the picked token ids cross back to the host; no row is sampled on the
CPU.

Run-ahead: the reference's step is strictly serial (schedule, forward, read
the tokens, bookkeeping, schedule again), so the GPU idles during the host's
bookkeeping and the host idles during the forward. When no sequence that
completes a pass can stop on the value of its new token (stops_on_length),
the scheduler's next decisions do not depend on those values: the step
commits the pass, appends a stand-in for each new token (a reference to
where the token lands in the device pick buffer, resolved by the next
forward's metadata builder on the device), runs the length stop checks,
schedules and launches the next pass, and only then waits for this pass's
tokens and writes them over the stand-ins. The schedule, the token streams,
the per-call outputs and the step count are the reference's.
"""

from __future__ import annotations

import time

import numpy as np

from .runner import CudaRunner


def cuda_engine(cfg=None, tokenizer=None, speculative_tokens: int = 0, weights=None, device=None,
                engine_cls=None, runner_cls=None, **runner_kw):
    """Build an LLMEngine (or `engine_cls`) with a CudaRunner (or `runner_cls`,
    e.g. vllt.llama.LlamaRunner / vllt.tp.TPLlamaRunner) behind it."""
    import vllmlite.engine as E
    from vllmlite.config import EngineConfig

    cfg = cfg or EngineConfig()
    orig = E.NumpyRunner
    cls_r = runner_cls or CudaRunner
    if weights is not None:
        runner_kw["weights"] = weights

    def factory(model_cfg, cache_cfg):
        return cls_r(model_cfg, cache_cfg, cfg.scheduler, device=device, **runner_kw)

    E.NumpyRunner = factory
    try:
        cls = engine_cls or E.LLMEngine
        return cls(cfg, tokenizer, speculative_tokens)
    finally:
        E.NumpyRunner = orig


def completes(item) -> bool:
    """Whether this pass computes the last token of the item's sequence: the
    reference engine only picks a token for such sequences; chunked-prefill
    and post-preemption chunks that leave tokens uncomputed pick nothing and
    draw nothing from the request's generator (vllmlite/engine.py:131-149).
    Evaluated before commit: the sequence then has num_computed == start_pos."""
    return item.start_pos + item.num_tokens >= item.seq.num_tokens


def pick_inputs(scheduled, rows, R: int, eos):
    """Host inputs of the device token picks for one step, following the
    reference's per-row rules (vllmlite/engine.py:106-149, sampling.py:41-64):
    cu_rows[S+1] and draft offsets[S] (int32), the flat draft tokens, eos_mask[R]
    (min_tokens not reached, greedy rows), penalty[R] (repetition penalty of a
    greedy row), and the (sequence index, row) pairs that sample with
    temperature. Rows of sequences that verify drafts take plain argmax
    (speculative.py:92). Only the last row of a sequence that completes this
    pass is masked, penalised or sampled: that is the only row the reference
    hands to sample()."""
    S = len(scheduled)
    cu, doff, drafts = [0] * (S + 1), [0] * S, []
    mask_rows, pen_rows, pen_vals, sampled = [], [], [], []
    for i, item in enumerate(scheduled):
        seq = item.seq
        r0, cnt = rows[i]
        cu[i + 1] = r0 + cnt
        doff[i] = len(drafts)
        d = seq.draft_token_ids
        if d:
            drafts += d[:cnt - 1]
            continue
        if not completes(item):
            continue
        p = seq.params
        last = r0 + cnt - 1
        if not p.greedy:
            sampled.append((i, last))
            continue
        if eos is not None and p.min_tokens and len(seq.output_token_ids) < p.min_tokens:
            mask_rows.append(last)
        if p.repetition_penalty != 1.0:
            pen_rows.append(last)
            pen_vals.append(p.repetition_penalty)
    eos_mask = np.zeros(R, np.uint8)
    if mask_rows:
        eos_mask[mask_rows] = 1
    penalty = np.ones(R, np.float32)
    if pen_rows:
        penalty[pen_rows] = pen_vals
    return np.asarray(cu, np.int32), np.asarray(doff, np.int32), drafts, eos_mask, penalty, sampled


def stops_on_length(params, eos) -> bool:
    """Whether the reference's stop checks for a new token of a request with
    these SamplingParams depend only on lengths (vllmlite/engine.py:218-234):
    EOS and stop_token_ids are ignored (ignore_eos, or no EOS id and no stop
    ids) and there are no stop strings; max_tokens and max_seq_len remain."""
    return not params.stop and (params.ignore_eos or (eos is None and not params.stop_token_ids))


class PendingPicks:
    """One pass's device picks on their way to the host: the layout of the
    pick buffer (R rows, S sequences, tail, special rows, sampled (seq, row)
    pairs, whether drafts were verified), token_at {seq index: buffer entry
    of the sequence's new token}, the host copy and the event after it."""

    __slots__ = ("R", "S", "tail", "special", "sampled", "drafts", "token_at", "host", "event")

    def __init__(self, R, S, tail, special, sampled, drafts, token_at, host, event):
        self.R, self.S, self.tail, self.special, self.sampled = R, S, tail, special, sampled
        self.drafts, self.token_at, self.host, self.event = drafts, token_at, host, event


def seen_bitmaps(seqs, vocab: int) -> np.ndarray:
    """uint32 [len(seqs)][ceil(vocab/32)]: bit t of row j is set when token t
    occurs in seqs[j].token_ids (the `seen_tokens` of sampling.py:54, which
    penalises each distinct seen token once, :11)."""
    b = np.zeros((len(seqs), (vocab + 31) // 32), np.uint32)
    for j, seq in enumerate(seqs):
        if seq is None:
            continue
        seen = np.unique(np.asarray(seq.token_ids, np.int64))
        if seen.size:
            np.bitwise_or.at(b[j], seen >> 5, np.uint32(1) << (seen & 31).astype(np.uint32))
    return b


def sample_inputs(seqs, eos, rngs):
    """Per-row arrays of the device sampler for temperature rows, one row per
    sequence: temperature, top_k, top_p, the float64 uniform numpy's choice()
    would draw from the request's generator (one rng.random() per pick,
    sampling.py:64), the min_tokens EOS mask and the repetition penalty."""
    n = len(seqs)
    temp = np.empty(n, np.float32)
    top_k = np.empty(n, np.int32)
    top_p = np.empty(n, np.float32)
    u = np.empty(n, np.float64)
    mask = np.zeros(n, np.uint8)
    pen = np.ones(n, np.float32)
    for j, seq in enumerate(seqs):
        p = seq.params
        temp[j], top_k[j], top_p[j] = p.temperature, p.top_k, p.top_p
        u[j] = rngs[seq.request_id].random()
        if eos is not None and p.min_tokens and len(seq.output_token_ids) < p.min_tokens:
            mask[j] = 1
        pen[j] = p.repetition_penalty
    return temp, top_k, top_p, u, mask, pen


def _engine_base():
    from vllmlite.engine import LLMEngine

    return LLMEngine


class _Lazy(type):
    """Create GpuLLMEngine as a real LLMEngine subclass on first use, so this
    module imports without vllm-lite installed."""

    _cls = None

    def __call__(cls, *a, **k):
        return cls.resolve()(*a, **k)

    def resolve(cls):
        if cls._cls is None:
            cls._cls = _make_gpu_engine(_engine_base())
        return cls._cls


class GpuLLMEngine(metaclass=_Lazy):
    """Use `gpu_engine(cfg, ...)`; instances are LLMEngine subclasses."""


def gpu_engine(cfg=None, tokenizer=None, speculative_tokens: int = 0, weights=None, device=None,
               runner_cls=None, device_prefix_hash: bool = False, run_ahead: bool = True, **runner_kw):
    """A GpuLLMEngine (device token picks). device_prefix_hash: the prefix
    cache's block hashes are computed on the device (vllt.prefix_hash).
    run_ahead: schedule and launch the next pass while the current one runs
    when its tokens cannot stop a sequence (GpuLLMEngine.can_run_ahead); a
    request added or aborted between two step() calls then takes effect one
    pass later than in the reference engine."""
    eng = cuda_engine(cfg, tokenizer, speculative_tokens, weights, device,
                      engine_cls=GpuLLMEngine.resolve(), runner_cls=runner_cls, **runner_kw)
    eng.run_ahead = run_ahead
    if device_prefix_hash:
        from .prefix_hash import DevicePrefixHasher

        eng.prefix_hasher = DevicePrefixHasher(eng, lib=runner_kw.get("lib"))
    return eng


def _make_gpu_engine(Base):
    import torch
    from vllmlite.sequence import RequestOutput

    from . import _lib
    from ._lib import check

    class _GpuLLMEngine(Base):
        run_ahead = True  # see gpu_engine
        passes_ahead = 0  # passes launched before the previous pass's tokens were on the host
        _next = None  # (SchedulerOutput, dropped reports, (rows, R, launch time) or None) for the next call

        def _h2d(self, a):
            """Upload through a pinned staging block: a copy from pageable
            memory may wait for the stream, which would stall the host behind
            a pass that is still running."""
            t = torch.from_numpy(np.ascontiguousarray(a))
            if self.runner.dev.type == "cuda":
                t = t.pin_memory()
            return t.to(self.runner.dev, non_blocking=True)

        def _greedy(self, logits, n_rows, ld, vocab, mask, pen, seqs, out, keep):
            """Greedy kernel over logits rows [0, n_rows) with the EOS mask and
            penalty arrays of those rows (seqs[j]: the sequence of a penalised
            row j, else None)."""
            L, eos = self.runner.L, self.tokenizer.eos_id
            d_mask = self._h2d(mask) if mask.any() else None
            d_pen = bits = None
            if (pen != 1.0).any():
                d_pen = self._h2d(pen)
                bits = self._h2d(seen_bitmaps([s if pen[j] != 1.0 else None for j, s in enumerate(seqs)], vocab))
            keep += [d_mask, d_pen, bits]
            check(L.vllt_sample_greedy(logits.data_ptr(), n_rows, vocab, ld, _lib.ptr(d_mask),
                                       eos if eos is not None else -1, _lib.ptr(d_pen), _lib.ptr(bits),
                                       out.data_ptr(), _lib.stream_handle()))

        def _sample(self, logits, n_logit_rows, ld, vocab, row_index, seqs, out, keep):
            """Device sampler (vllt_sample_top_p) for temperature rows: row j
            reads logits[row_index[j]] and belongs to seqs[j]."""
            L, eos = self.runner.L, self.tokenizer.eos_id
            temp, top_k, top_p, u, mask, pen = sample_inputs(seqs, eos, self.rngs)
            d = [self._h2d(a) for a in (np.asarray(row_index, np.int32), temp, top_k, top_p, u)]
            d_mask = self._h2d(mask) if mask.any() else None
            d_pen = bits = None
            if (pen != 1.0).any():
                d_pen = self._h2d(pen)
                bits = self._h2d(seen_bitmaps(seqs, vocab))
            keep += d + [d_mask, d_pen, bits]
            check(L.vllt_sample_top_p(logits.data_ptr(), len(seqs), vocab, ld, n_logit_rows, d[0].data_ptr(),
                                      _lib.ptr(d_mask), eos if eos is not None else -1, _lib.ptr(d_pen),
                                      _lib.ptr(bits), d[1].data_ptr(), d[2].data_ptr(), d[3].data_ptr(),
                                      d[4].data_ptr(), out.data_ptr(), _lib.stream_handle()))

        def _enqueue_picks(self, sched, rows, R):
            """Enqueue the device picks of one pass and their copy to the
            host; returns a PendingPicks (read it with _collect_picks).

            One GPU: the greedy kernel over all R rows (EOS mask / penalty on
            the rows that need them), the sampler over the temperature rows
            (read in place through a row index), the accept rule over the
            verify rows. Tensor parallel: the vocab-parallel argmax over all
            rows; rows that need a mask, a penalty or a draw have their
            full-vocabulary logits gathered from every rank first and go
            through the same two kernels. Every result lands in one device
            buffer (the runner's pick buffer, which the next forward can read
            tokens from), copied back with one copy per pass:
              [0, R) row picks | R: the metadata builder's error word |
              [R+1, R+1+S) accepted drafts | then the sampled / masked picks."""
            run = self.runner
            S = len(sched.scheduled)
            V = run.model_cfg.vocab_size
            eos = self.tokenizer.eos_id
            tp = getattr(run, "tp_size", 1) > 1
            cu, doff, drafts, eos_mask, penalty, sampled = pick_inputs(sched.scheduled, rows, R, eos)
            keep = []  # device temporaries stay referenced until their kernels are enqueued:
            # a tensor freed earlier could be handed to the next copy by the
            # caching allocator and overwritten before the kernel reads it
            seq_of_row = {}
            for i, item in enumerate(sched.scheduled):
                seq_of_row[rows[i][0] + rows[i][1] - 1] = item.seq
            special = [int(r) for r in np.flatnonzero(eos_mask | (penalty != 1.0))] if tp else []
            tail = R + 1 + S  # first word of the sampled / masked picks
            n = tail + len(special) + len(sampled)
            buf = getattr(run, "pick_buffer", None)
            res = buf(n) if buf is not None else torch.empty(n, dtype=torch.int32, device=run.dev)
            if tp:
                res[:R] = run.greedy_picks(R)
            else:
                self._greedy(run.logits_dev, R, run.w.vocab_padded, V, eos_mask, penalty,
                             [seq_of_row.get(r) for r in range(R)], res, keep)
            res[R:R + 1] = run.meta[7:8]
            if drafts:  # cu_rows[S+1] | draft offsets[S] | drafts, one upload
                d = self._h2d(np.concatenate([cu, doff, np.asarray(drafts, np.int32)]))
                keep.append(d)
                check(run.L.vllt_spec_accept(d.data_ptr(), d[2 * S + 1:].data_ptr(), d[S + 1:].data_ptr(), S,
                                             res.data_ptr(), res[R + 1:].data_ptr(), _lib.stream_handle()))
            seqs = [sched.scheduled[i].seq for i, _ in sampled]
            if tp and (special or sampled):
                full = run.gather_rows(special + [r for _, r in sampled])  # [n, V] fp32 on every rank
                if special:
                    self._greedy(full, len(special), V, V, eos_mask[special], penalty[special],
                                 [seq_of_row[r] for r in special], res[tail:], keep)
                if sampled:
                    self._sample(full, full.shape[0], V, V, [len(special) + j for j in range(len(sampled))], seqs,
                                 res[tail + len(special):], keep)
            elif sampled:
                self._sample(run.logits_dev, R, run.w.vocab_padded, V, [r for _, r in sampled], seqs, res[tail:], keep)
            # where the token of each completing sequence without drafts lands
            token_at = {}
            sampled_at = {i: tail + len(special) + j for j, (i, _) in enumerate(sampled)}
            special_at = {r: tail + j for j, r in enumerate(special)}
            for i, item in enumerate(sched.scheduled):
                if item.seq.draft_token_ids or not completes(item):
                    continue
                last = rows[i][0] + rows[i][1] - 1
                token_at[i] = sampled_at.get(i, special_at.get(last, last))
            host = torch.empty(n, dtype=torch.int32, pin_memory=res.is_cuda)
            host.copy_(res, non_blocking=True)
            ev = None
            if res.is_cuda:
                ev = torch.cuda.Event()
                ev.record()
            return PendingPicks(R, S, tail, special, sampled, bool(drafts), token_at, host, ev)

        def _collect_picks(self, pend):
            """Wait for a pass's picks; (picks[R], n_accepted[S], {seq index:
            sampled token}, the whole host copy)."""
            if pend.event is not None:
                pend.event.synchronize()
            res_h = pend.host.numpy()
            R, S, tail, special = pend.R, pend.S, pend.tail, pend.special
            self.runner.check_step_flags(int(res_h[R]))
            picks_h = res_h[:R].copy()
            if special:
                picks_h[special] = res_h[tail:tail + len(special)]
            sampled_tok = {i: int(res_h[tail + len(special) + j]) for j, (i, _) in enumerate(pend.sampled)}
            acc_h = res_h[R + 1:R + 1 + S].copy() if pend.drafts else np.zeros(S, np.int32)
            return picks_h, acc_h, sampled_tok, res_h

        def _device_picks(self, sched, rows, R):
            """Picks of one pass, waited for: (picks[R], n_accepted[S],
            {seq index: sampled token})."""
            return self._collect_picks(self._enqueue_picks(sched, rows, R))[:3]

        @property
        def has_work(self) -> bool:
            """The reference's answer (vllmlite/engine.py:96), plus a pass
            launched ahead that still has a live sequence or undelivered
            reports: one whose sequences were all aborted since is no work,
            so an abort of the last request leaves the engine idle at once,
            as in the reference (the next step() still collects that pass)."""
            if self.scheduler.has_work:
                return True
            if self._next is None:
                return False
            sched, dropped, _ = self._next
            return bool(dropped) or any(not item.seq.status.finished for item in sched.scheduled)

        def can_run_ahead(self, sched, pend) -> bool:
            """Whether the pass after `sched` can be scheduled before this
            pass's tokens (enqueued as `pend`) reach the host: no speculation,
            no device prefix hashes, and every sequence that completes this
            pass stops only on its length (see stops_on_length). Under tensor
            parallelism their tokens must also be plain greedy picks (entries
            below R of the pick buffer, which every rank holds); masked,
            penalised and sampled rows are picked on rank 0 only."""
            if not self.run_ahead or self.proposer is not None:
                return False
            run = self.runner
            if getattr(self, "prefix_hasher", None) is not None or getattr(run, "pick_buffer", None) is None:
                return False
            tp = getattr(run, "tp_size", 1) > 1
            eos = self.tokenizer.eos_id
            for i, item in enumerate(sched.scheduled):
                if item.seq.draft_token_ids:
                    return False
                if completes(item):
                    if not stops_on_length(item.seq.params, eos):
                        return False
                    if tp and pend.token_at[i] >= pend.R:
                        return False
            return True

        def _mark_busy(self, t_launch):
            """busy_time as the reference counts it (time spent in forward
            passes), without counting the overlap of two passes twice."""
            now = time.perf_counter()
            self.busy_time += now - max(t_launch, getattr(self, "_busy_until", 0.0))
            self._busy_until = now

        def step(self):
            """engine.py:99-181 with device-side token picks (and, with a
            prefix_hasher, device-side prefix-cache hashes). With run_ahead,
            the next pass is scheduled and launched while this one runs
            whenever this pass's tokens cannot stop a sequence (can_run_ahead):
            every call still returns its own pass's outputs, and the
            scheduler sees the state the reference's would."""
            hasher = getattr(self, "prefix_hasher", None)
            if hasher is None:
                return self._step(None)
            with hasher.active():
                return self._step(hasher)

        def _step(self, hasher):
            nxt, self._next = self._next, None
            if nxt is None:
                if hasher is not None:
                    hasher.prepare_prompts()
                sched = self.scheduler.schedule()
                dropped = self.scheduler.drain_reports()
                launched = None
            else:  # scheduled (and launched) by the previous call
                sched, dropped, launched = nxt
            results = [self._retired_output(s) for s in dropped]
            if sched.is_empty:
                return results
            if launched is None:
                t0 = time.perf_counter()
                rows, R = self.runner.launch(sched)
            else:
                rows, R, t0 = launched
            if hasher is not None:
                hasher.prepare_commits(sched)
            pend = self._enqueue_picks(sched, rows, R)
            if self.can_run_ahead(sched, pend):
                waiting = self._commit_ahead(sched, pend)
                sched2 = self.scheduler.schedule()
                dropped2 = self.scheduler.drain_reports()
                if not sched2.is_empty:
                    t2 = time.perf_counter()
                    self._next = (sched2, dropped2, (*self.runner.launch(sched2), t2))
                    self.passes_ahead += 1
                elif dropped2:
                    self._next = (sched2, dropped2, None)
                res_h = self._collect_picks(pend)[3]
                self._mark_busy(t0)
                self.total_steps += 1
                return results + self._patch_ahead(waiting, res_h)
            picks, accepted, sampled_tok, _ = self._collect_picks(pend)
            if hasher is not None:
                hasher.collect()
            self._mark_busy(t0)
            self.total_steps += 1
            eos = self.tokenizer.eos_id
            for i, item in enumerate(sched.scheduled):
                seq = item.seq
                if seq.status.finished:  # aborted while its pass was in flight
                    continue
                row0, count = rows[i]
                drafts = list(seq.draft_token_ids)
                if drafts:
                    acc = int(accepted[i])
                    new_tokens = [int(t) for t in picks[row0:row0 + acc + 1]]
                    seq.draft_token_ids.clear()
                    self.spec.proposed += len(drafts)
                    self.spec.accepted += acc
                    keep = acc + 1
                else:
                    new_tokens, keep = None, item.num_tokens
                self.scheduler.blocks.commit(seq, keep)
                seq.num_computed += keep
                if seq.num_computed < seq.num_tokens:
                    continue
                if new_tokens is None:
                    if i in sampled_tok:
                        new_tokens = [sampled_tok[i]]
                    else:
                        new_tokens = [int(picks[row0 + count - 1])]
                emitted = []
                for tok in new_tokens:
                    seq.append_token(tok)
                    self.total_output_tokens += 1
                    emitted.append(tok)
                    self._check_stop(seq, tok, eos)
                    if seq.status.finished:
                        break
                results.append(self._output(seq, emitted))
            if self.proposer is not None:
                self.spec.rounds += 1
                self._make_proposals()
            return results

        def _output(self, seq, emitted):
            delta = self._advance_detok(seq)
            if seq.status.finished:
                self.scheduler.finish(seq)
            return RequestOutput(
                request_id=seq.request_id, token_ids=list(seq.output_token_ids),
                new_token_ids=emitted, text_delta=delta, finished=seq.status.finished,
                finish_reason=self._reason(seq), num_prompt_tokens=seq.num_prompt_tokens,
                num_output_tokens=len(seq.output_token_ids),
                cached_prefix_tokens=seq.cached_prefix_tokens)

        def _commit_ahead(self, sched, pend):
            """engine.py:113-160 for a pass whose tokens are still on the
            device: commit and num_computed as the reference, then each
            completing sequence takes a stand-in token -1 - j (j: where its
            token lands in the pick buffer, which the next forward resolves on
            the device), the length stop checks run (can_run_ahead guarantees
            no other check applies) and finished sequences free their blocks.
            Returns what _patch_ahead needs."""
            eos = self.tokenizer.eos_id
            waiting = []
            for i, item in enumerate(sched.scheduled):
                seq = item.seq
                if seq.status.finished:  # aborted while its pass was in flight
                    continue
                self.scheduler.blocks.commit(seq, item.num_tokens)
                seq.num_computed += item.num_tokens
                if seq.num_computed < seq.num_tokens:
                    continue
                j = pend.token_at[i]
                first = seq.first_token_at is None
                seq.append_token(-1 - j)
                self.total_output_tokens += 1
                self._check_stop(seq, -1 - j, eos)
                if seq.status.finished:
                    self.scheduler.finish(seq)
                waiting.append((seq, len(seq.output_token_ids) - 1, j, first))
            return waiting

        def _patch_ahead(self, waiting, res_h):
            """The picked tokens replace the stand-ins; first-token and finish
            times are taken now (when the token is on the host, as the
            reference's); detokenise and report in the reference's order."""
            now = time.perf_counter()
            out = []
            for seq, k, j, first in waiting:
                tok = int(res_h[j])
                seq.output_token_ids[k] = tok
                if first:
                    seq.first_token_at = now
                if seq.status.finished:
                    seq.finished_at = now
                delta = self._advance_detok(seq)
                out.append(RequestOutput(
                    request_id=seq.request_id, token_ids=list(seq.output_token_ids),
                    new_token_ids=[tok], text_delta=delta, finished=seq.status.finished,
                    finish_reason=self._reason(seq), num_prompt_tokens=seq.num_prompt_tokens,
                    num_output_tokens=len(seq.output_token_ids),
                    cached_prefix_tokens=seq.cached_prefix_tokens))
            return out

    return _GpuLLMEngine
