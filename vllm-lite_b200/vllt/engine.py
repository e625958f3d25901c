"""Engine entry points: vllm-lite's LLMEngine driving the CUDA runner.

`cuda_engine(cfg, ...)` returns an unmodified `vllmlite.engine.LLMEngine`
whose runner is `CudaRunner` instead of the hard-coded NumpyRunner
(vllmlite/engine.py:46): Scheduler, BlockManager, prefix hashing,
preemption, sampling and the n-gram proposer are the reference's own code.
Logits come back to the host every step, exactly as the reference expects.

`GpuLLMEngine` keeps all of that but replaces the sampling half of
LLMEngine.step (engine.py:113-148) by device kernels: one launch picks the
argmax of every logit row and applies the speculative accept/reject rule
(speculative.py:86-100); non-greedy rows draw on the device with the
request's own generator supplying the uniform (sampling.py:59-64). Only the
picked token ids cross back to the host.
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


def pick_inputs(scheduled, rows, R: int, eos):
    """Host inputs of the device token picks for one step, following the
    reference's per-row rules (vllmlite/engine.py:106-130, sampling.py:41-64):
    cu_rows[S+1] and draft offsets[S] (int32), the flat draft tokens, eos_mask[R]
    (min_tokens not reached), penalty[R] (repetition penalty of the row), and the
    (sequence index, row) pairs that sample with temperature. Rows of sequences
    that verify drafts take plain argmax (speculative.py:92)."""
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
               runner_cls=None, **runner_kw):
    return cuda_engine(cfg, tokenizer, speculative_tokens, weights, device,
                       engine_cls=GpuLLMEngine.resolve(), runner_cls=runner_cls, **runner_kw)


def _make_gpu_engine(Base):
    import torch
    from vllmlite.sampling import sample
    from vllmlite.sequence import RequestOutput

    from . import _lib
    from ._lib import check

    class _GpuLLMEngine(Base):
        def _device_picks(self, sched, rows, R):
            """Pick every row's token on the device; return host arrays
            (picks[R], n_accepted[S], {seq index: sampled token})."""
            run = self.runner
            dev = run.dev
            S = len(sched.scheduled)
            V = run.model_cfg.vocab_size
            ld = run.w.vocab_padded
            eos = self.tokenizer.eos_id
            cu, doff, drafts, eos_mask, penalty, sampled = pick_inputs(sched.scheduled, rows, R, eos)
            st = _lib.stream_handle()

            def h2d(a):
                return torch.from_numpy(np.ascontiguousarray(a)).to(dev, non_blocking=True)

            acc = torch.empty(max(S, 1), dtype=torch.int32, device=dev)
            L = run.L
            if getattr(run, "tp_size", 1) > 1:
                # vocab-parallel greedy; rows needing masks or sampling are not supported across shards
                if eos_mask.any() or (penalty != 1.0).any() or sampled:
                    raise NotImplementedError("tensor-parallel engine: greedy rows without min_tokens / "
                                              "repetition penalty only")
                picks = run.greedy_picks(R)
                if drafts:
                    d_cu, d_dr, d_doff = h2d(cu), h2d(np.asarray(drafts, np.int32)), h2d(doff)
                    check(L.vllt_spec_accept(d_cu.data_ptr(), d_dr.data_ptr(), d_doff.data_ptr(), S,
                                             picks.data_ptr(), acc.data_ptr(), st))
                acc_h = acc[:S].cpu().numpy() if drafts else np.zeros(S, np.int32)
                return picks[:R].cpu().numpy(), acc_h, {}
            picks = torch.empty(max(R, 1), dtype=torch.int32, device=dev)
            d_mask = h2d(eos_mask) if eos_mask.any() else None
            d_pen = bits = None
            if (penalty != 1.0).any():
                d_pen = h2d(penalty)
                words = (V + 31) // 32
                b = np.zeros((R, words), np.uint32)
                for i, item in enumerate(sched.scheduled):
                    last = rows[i][0] + rows[i][1] - 1
                    if penalty[last] != 1.0:
                        seen = np.unique(np.asarray(item.seq.token_ids, np.int64))
                        np.bitwise_or.at(b[last], seen >> 5, (np.uint32(1) << (seen & 31).astype(np.uint32)))
                bits = h2d(b)
            check(L.vllt_sample_greedy(run.logits_dev.data_ptr(), R, V, ld, _lib.ptr(d_mask),
                                       eos if eos is not None else -1, _lib.ptr(d_pen), _lib.ptr(bits),
                                       picks.data_ptr(), st))
            # device temporaries stay referenced until their kernels are enqueued:
            # a tensor freed earlier could be handed to the next copy by the
            # caching allocator and overwritten before the kernel reads it
            if drafts:
                d_cu, d_dr, d_doff = h2d(cu), h2d(np.asarray(drafts, np.int32)), h2d(doff)
                check(L.vllt_spec_accept(d_cu.data_ptr(), d_dr.data_ptr(), d_doff.data_ptr(), S,
                                         picks.data_ptr(), acc.data_ptr(), st))
            sampled_tok = {}
            plain = [(i, r) for i, r in sampled
                     if sched.scheduled[i].seq.params.repetition_penalty == 1.0
                     and len(sched.scheduled[i].seq.output_token_ids) >= sched.scheduled[i].seq.params.min_tokens]
            other = [x for x in sampled if x not in plain]
            if plain:
                prm = [sched.scheduled[i].seq.params for i, _ in plain]
                # the request's generator supplies the uniform numpy's choice() would draw
                u = np.asarray([self.rngs[sched.scheduled[i].seq.request_id].random() for i, _ in plain], np.float32)
                sel = h2d(np.asarray([r for _, r in plain], np.int64))
                sub = run.logits_dev.index_select(0, sel).contiguous()
                out = torch.empty(len(plain), dtype=torch.int32, device=dev)
                d_t = h2d(np.asarray([q.temperature for q in prm], np.float32))
                d_k = h2d(np.asarray([q.top_k for q in prm], np.int32))
                d_p = h2d(np.asarray([q.top_p for q in prm], np.float32))
                d_u = h2d(u)
                check(L.vllt_sample_top_p(sub.data_ptr(), len(plain), V, ld, d_t.data_ptr(), d_k.data_ptr(),
                                          d_p.data_ptr(), d_u.data_ptr(), out.data_ptr(), st))
                for (i, _), t in zip(plain, out.cpu().numpy()):
                    sampled_tok[i] = int(t)
            for i, r in other:  # temperature with penalty / min_tokens: the reference sampler on that row
                seq = sched.scheduled[i].seq
                row = run.logits_dev[r, :V].cpu().numpy()
                sampled_tok[i] = sample(row, seq.params, seq.token_ids, self.rngs[seq.request_id],
                                        len(seq.output_token_ids), eos)
            picks_h = picks[:R].cpu().numpy()
            acc_h = acc[:S].cpu().numpy() if drafts else np.zeros(S, np.int32)
            return picks_h, acc_h, sampled_tok

        def step(self):
            """engine.py:99-181 with device-side token picks."""
            sched = self.scheduler.schedule()
            dropped = [self._retired_output(s) for s in self.scheduler.drain_reports()]
            if sched.is_empty:
                return dropped
            t0 = time.perf_counter()
            rows, R = self.runner.launch(sched)
            picks, accepted, sampled_tok = self._device_picks(sched, rows, R)
            self.busy_time += time.perf_counter() - t0
            self.total_steps += 1
            results = list(dropped)
            eos = self.tokenizer.eos_id
            for i, item in enumerate(sched.scheduled):
                seq = item.seq
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
                delta = self._advance_detok(seq)
                if seq.status.finished:
                    self.scheduler.finish(seq)
                results.append(RequestOutput(
                    request_id=seq.request_id, token_ids=list(seq.output_token_ids),
                    new_token_ids=emitted, text_delta=delta, finished=seq.status.finished,
                    finish_reason=self._reason(seq), num_prompt_tokens=seq.num_prompt_tokens,
                    num_output_tokens=len(seq.output_token_ids),
                    cached_prefix_tokens=seq.cached_prefix_tokens))
            if self.proposer is not None:
                self.spec.rounds += 1
                self._make_proposals()
            return results

    return _GpuLLMEngine
