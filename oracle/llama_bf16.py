"""Oracle: the bf16 Llama-shaped forward's rounding points (test infrastructure only).

The reference has no bf16 path; the product's bf16 forward (the Llama-3-8B-shaped
model) is checked against an fp32 re-run of the same weights on the GPU with a
stated tolerance. This module restates the forward of vllmlite/model.py:80-120
with the bf16 forward's rounding points, on the CPU with torch, so the size of
the bf16 error -- and from it the tolerance of the GPU tests -- is measured
rather than guessed:

  x = embedding row (bf16 table, fp32 residual stream)
  per layer:
    h = bf16(rmsnorm(x))                       rmsnorm_bf16
    q, k = RoPE(h . Wq^T, h . Wk^T) in fp32, then bf16; v = bf16(h . Wv^T)
                                               EpiQKVBF16 (fp32 accumulate)
    a = bf16(attention(q, k, v))               fp32 scores and softmax; the
        probabilities of multi-token chunks are rounded to bf16 before P.V
        (the tensor-core prefill kernel stages P in shared memory as bf16),
        single-query rows keep them fp32 (the decode kernel)
    x += a . Wo^T                              tp = 1: fp32 epilogue add;
        tp > 1: each rank's partial rounded to bf16, the bf16 sum of the
        partials (NCCL all-reduce) rounded to bf16, added by the next norm
    h = bf16(rmsnorm(x)); act = bf16(silu(h . Wg^T) * (h . Wu^T))
    x += act . Wd^T                            as o_proj
  logits = bf16(rmsnorm(x)) . lm_head^T        fp32

`bf16=False` runs the same arithmetic in fp32 with no rounding (the fp32
re-run). Weights are N(0, std) drawn on the CPU and rounded to bf16, so both
runs see the same bf16 values; their distribution is the product's (its
device generator gives other values of the same law). Sequences are computed
whole: with causal attention the logits at a position do not depend on how the
prompt was chunked, except for where P is rounded, which follows `chunks`.
"""

from __future__ import annotations

import numpy as np

from .attention import rope_tables


def _bf(t, on: bool):
    import torch

    return t.to(torch.bfloat16).to(torch.float32) if on else t


def llama_weights(shape, seed: int = 0, std: float = 0.02) -> dict:
    """Unsharded weights [out][in] (the product's layout), bf16 values in fp32."""
    import torch

    g = torch.Generator().manual_seed(seed)
    D, H, KV, d, f, V = shape.head_dim, shape.n_heads, shape.n_kv_heads, shape.d_model, shape.d_ff, shape.vocab_size

    def nrm(*s):
        return (torch.randn(s, generator=g) * std).to(torch.bfloat16).to(torch.float32)

    w = {"tok_emb": nrm(V, d), "lm_head": nrm(V, d)}
    for i in range(shape.n_layers):
        w[f"{i}.wq"], w[f"{i}.wk"], w[f"{i}.wv"] = nrm(H * D, d), nrm(KV * D, d), nrm(KV * D, d)
        w[f"{i}.wo"], w[f"{i}.w_gate"], w[f"{i}.w_up"] = nrm(d, H * D), nrm(f, d), nrm(f, d)
        w[f"{i}.w_down"] = nrm(d, f)
    return w


def _rmsnorm(x, eps=1e-5):
    import torch

    return x * torch.rsqrt((x * x).mean(-1, keepdim=True) + eps)


def _rope(x, pos, cos, sin):
    c, s = cos[pos][:, None, :], sin[pos][:, None, :]
    e, o = x[..., 0::2], x[..., 1::2]
    y = x.clone()
    y[..., 0::2] = e * c - o * s
    y[..., 1::2] = e * s + o * c
    return y


def forward_sequence(shape, w: dict, tokens, chunks, bf16: bool = True, tp: int = 1, drop_head=None,
                     wide: bool = False):
    """fp32 logits [len(tokens), V] of one sequence at every position.

    chunks: list of (start, n) in which the sequence's prompt went through the
    forward (a query row of a chunk with n > 1 gets bf16-rounded attention
    probabilities when bf16). tp: tensor-parallel ranks whose row-parallel
    partials are rounded and summed in bf16. drop_head: a query head whose
    attention output is zeroed in every layer (a planted kernel mistake, to
    show what the tolerances catch). wide: every contraction (projections,
    scores, P.V) accumulates in float64 before it is rounded to fp32, to
    measure how much the order of fp32 accumulation alone moves the result
    (the GPU accumulates in another order than the CPU)."""
    import torch

    def mm(a, b):
        return (a.double() @ b.double()).float() if wide else a @ b

    def es(eq, a, b):
        return torch.einsum(eq, a.double(), b.double()).float() if wide else torch.einsum(eq, a, b)

    D, H, KV = shape.head_dim, shape.n_heads, shape.n_kv_heads
    T = len(tokens)
    cos, sin = (torch.from_numpy(a) for a in rope_tables(D, max(shape.max_seq_len, T)))
    pos = torch.arange(T)
    multi = torch.zeros(T, dtype=torch.bool)
    for start, n in chunks:
        if n > 1:
            multi[start:start + n] = True
    causal = torch.ones(T, T, dtype=torch.bool).tril()  # [query, key]
    rep = H // KV

    def rowpar(a, wm, parts):
        """a . wm^T, in `parts` column slices of `a` (rows of wm^T) when bf16 TP."""
        if not bf16 or parts == 1:
            return mm(a, wm.T)
        k = a.shape[1] // parts
        acc = None
        for r in range(parts):
            p = _bf(mm(a[:, r * k:(r + 1) * k], wm[:, r * k:(r + 1) * k].T), True)
            acc = p if acc is None else _bf(acc + p, True)
        return acc

    x = w["tok_emb"][torch.as_tensor(tokens)]
    for i in range(shape.n_layers):
        h = _bf(_rmsnorm(x), bf16)
        q = _bf(_rope(mm(h, w[f"{i}.wq"].T).view(T, H, D), pos, cos, sin), bf16)
        k = _bf(_rope(mm(h, w[f"{i}.wk"].T).view(T, KV, D), pos, cos, sin), bf16)
        v = _bf(mm(h, w[f"{i}.wv"].T).view(T, KV, D), bf16)
        kk = k.repeat_interleave(rep, dim=1)
        vv = v.repeat_interleave(rep, dim=1)
        o = torch.empty(T, H, D)
        for q0 in range(0, T, 512):  # query blocks: bounded memory at long contexts
            q1 = min(T, q0 + 512)
            s = es("thd,shd->hts", q[q0:q1], kk[:q1]) / np.float32(np.sqrt(D))
            s = s.masked_fill(~causal[None, q0:q1, :q1], float("-inf"))
            m = s.max(-1, keepdim=True).values
            p = torch.exp(s - m)
            l = p.sum(-1, keepdim=True)
            if bf16:
                p = torch.where(multi[None, q0:q1, None], _bf(p, True), p)
            o[q0:q1] = es("hts,shd->thd", p, vv[:q1]) / l.permute(1, 0, 2)
        if drop_head is not None:
            o[:, drop_head] = 0
        a = _bf(o.reshape(T, H * D), bf16)
        x = x + rowpar(a, w[f"{i}.wo"], tp)
        h = _bf(_rmsnorm(x), bf16)
        g, u = mm(h, w[f"{i}.w_gate"].T), mm(h, w[f"{i}.w_up"].T)
        act = _bf(g / (1 + torch.exp(-g)) * u, bf16)
        x = x + rowpar(act, w[f"{i}.w_down"], tp)
    return mm(_bf(_rmsnorm(x), bf16), w["lm_head"].T)


def schedule_sequences(passes):
    """Whole sequences and logit rows of a pass schedule in the step-record
    form of the GPU tests (dicts with start, n, count, tokens, block_ids):
    sequences are told apart by their first block id. Returns
    {key: (tokens, chunks)} and per pass the list of (key, positions) whose
    logits the pass returns."""
    seqs, rows = {}, []
    for step in passes:
        out = []
        for s in step:
            key = s["block_ids"][0]
            toks, chunks = seqs.setdefault(key, ([], []))
            assert len(toks) == s["start"], "a pass must continue its sequence"
            toks += list(s["tokens"])
            chunks.append((s["start"], s["n"]))
            end = s["start"] + s["n"]
            out.append((key, list(range(end - s["count"], end))))
        rows.append(out)
    return seqs, rows


def _errors(got, ref):
    """(max |got - ref| / max |ref|, max over rows of ||got - ref|| / ||ref||)."""
    mx = float((got - ref).abs().max() / ref.abs().max())
    rms = float(((got - ref).norm(dim=1) / ref.norm(dim=1)).max())
    return mx, rms


def schedule_error(shape, passes, seed: int = 0, tp: int = 1, drop_head=None, order: bool = False):
    """The errors the GPU tests bound, worst over the passes of a schedule:
    {"bf16": (max-rel, row-rel) of bf16 against fp32, "tp": the same of bf16
    with `tp` ranks against bf16 on one rank (when tp > 1), "dropped": bf16
    with `drop_head` zeroed against fp32 (when given), "order": bf16 with
    float64 accumulation against bf16 with fp32 accumulation (when order)}.
    max-rel is max |a - b| / max |b| over a pass's rows; row-rel is the
    largest ||a_r - b_r|| / ||b_r|| of a row."""
    import torch

    w = llama_weights(shape, seed)
    seqs, rows = schedule_sequences(passes)
    out = {}
    with torch.no_grad():
        for key, (toks, chunks) in seqs.items():
            r = {"fp32": forward_sequence(shape, w, toks, chunks, bf16=False),
                 "bf16": forward_sequence(shape, w, toks, chunks, bf16=True)}
            if tp > 1:
                r["tp"] = forward_sequence(shape, w, toks, chunks, bf16=True, tp=tp)
            if drop_head is not None:
                r["dropped"] = forward_sequence(shape, w, toks, chunks, bf16=True, drop_head=drop_head)
            if order:
                r["wide"] = forward_sequence(shape, w, toks, chunks, bf16=True, wide=True)
            out[key] = r
    worst = {}
    for step in rows:
        pick = lambda name: torch.cat([out[k][name][p] for k, p in step])
        pairs = {"bf16": ("bf16", "fp32")}
        if tp > 1:
            pairs["tp"] = ("tp", "bf16")
        if drop_head is not None:
            pairs["dropped"] = ("dropped", "fp32")
        if order:
            pairs["order"] = ("wide", "bf16")
        for name, (a, b) in pairs.items():
            e = _errors(pick(a), pick(b))
            old = worst.get(name, (0.0, 0.0))
            worst[name] = (max(old[0], e[0]), max(old[1], e[1]))
    return worst
