"""Python mirrors of the reference's hot-path functions, backed by libvllt.

Device-tensor functions (torch CUDA tensors in, results in place or returned):
  write_kv        vllmlite/attention.py:47-49   -> vllt_reshape_and_cache
  copy_blocks     vllmlite/runner.py:54-60      -> vllt_copy_blocks
  paged_attention_varlen  attention.py:59-98 over a ragged batch
  rms_norm        vllmlite/model.py:17-19       -> vllt_rmsnorm
  apply_rope      vllmlite/attention.py:28-37   -> vllt_rope
  matmul          the fp32 projections          -> vllt_sgemm
  greedy / sample_top_p / verify   sampling.py:41-64, speculative.py:86-100

`paged_attention(q, cache_k, cache_v, read_slots, n_kv_heads, scale)` keeps
the reference's NumPy signature exactly (attention.py:59): it uploads the
arrays, runs the CUDA kernel and returns a NumPy array. The reference cache
[slots, n_kv, D] is the library's paged layout with block_size 1, so the
slot list is used directly as the block table.

Cache tensors use the library layout [num_blocks, n_kv, block_size, D].
"""

from __future__ import annotations

import numpy as np

from . import _lib
from ._lib import check, lib, ptr, stream_handle


def _dtype_code(t) -> int:
    import torch

    if t.dtype == torch.float32:
        return _lib.VLLT_F32
    if t.dtype == torch.bfloat16:
        return _lib.VLLT_BF16
    raise ValueError(f"unsupported dtype {t.dtype}")


def _i32(x, device):
    import torch

    if isinstance(x, torch.Tensor):
        return x.to(device=device, dtype=torch.int32).contiguous()
    return torch.as_tensor(np.asarray(x, np.int32), device=device)


def write_kv(cache_k, cache_v, k, v, slots) -> None:
    """cache[slot[t]] = k[t], v[t]; caches [NB, n_kv, bs, D], k/v [T, n_kv, D]."""
    nb, n_kv, bs, D = cache_k.shape
    sl = _i32(slots, cache_k.device)
    k, v = k.contiguous(), v.contiguous()  # keep temporaries alive past the launch
    check(lib().vllt_reshape_and_cache(ptr(k), ptr(v), ptr(cache_k),
                                       ptr(cache_v), ptr(sl), k.shape[0], n_kv, D, bs, nb,
                                       _dtype_code(cache_k), stream_handle()))


def copy_blocks(cache_k, cache_v, pairs) -> None:
    """Copy blocks src->dst in every layer; caches [L, NB, n_kv, bs, D]."""
    L, nb, n_kv, bs, D = cache_k.shape
    if len(pairs) == 0:
        return
    p = _i32(np.asarray(pairs, np.int32).reshape(-1, 2), cache_k.device)
    check(lib().vllt_copy_blocks(ptr(cache_k), ptr(cache_v), ptr(p), p.shape[0], L, nb, n_kv, bs, D,
                                 _dtype_code(cache_k), stream_handle()))


def paged_attention_varlen(q, cache_k, cache_v, block_tables, cu_seqlens_q, ctx_lens, scale,
                           max_qlen=None, max_ctx=None, workspace=None):
    """Ragged-batch causal GQA attention; q [T, H, D] -> out [T, H, D]."""
    import torch

    T, H, D = q.shape
    nb, n_kv, bs, _ = cache_k.shape
    bt = _i32(block_tables, q.device)
    cu = _i32(cu_seqlens_q, q.device)
    cl = _i32(ctx_lens, q.device)
    S = cl.shape[0]
    if max_qlen is None:
        max_qlen = int((cu[1:] - cu[:-1]).max()) if S else 0
    if max_ctx is None:
        max_ctx = int(cl.max()) if S else 0
    q = q.contiguous()
    out = torch.empty_like(q)
    if workspace is None:
        nbytes = lib().vllt_attention_workspace_bytes(S, H, D, max_ctx)
        workspace = torch.zeros(max(nbytes, 256), dtype=torch.uint8, device=q.device)
    check(lib().vllt_paged_attention_varlen(
        ptr(q), ptr(cache_k), ptr(cache_v), ptr(bt), bt.shape[1], ptr(cu), ptr(cl), S, T,
        max_qlen, max_ctx, H, n_kv, D, bs, nb, float(scale), _dtype_code(q), ptr(out), ptr(workspace),
        workspace.numel() if workspace is not None else 0, stream_handle()))
    if workspace is not None:
        paged_attention_varlen.last_workspace = workspace  # flags readable by callers
    return out


def attention_flags(workspace) -> int:
    """Device error flags from an attention workspace header (syncs)."""
    return int(workspace[:4].view(__import__("torch").int32).item())


def paged_attention(q, cache_k, cache_v, read_slots, n_kv_heads, scale, *, device=None):
    """NumPy drop-in for vllmlite.attention.paged_attention (one sequence).

    q [q_len, H, D]; cache_* [slots, n_kv, D]; read_slots [ctx]. Runs on
    `device` (default: the current CUDA device) and returns float32
    [q_len, H, D].
    """
    import torch

    q = np.asarray(q, np.float32)
    q_len, H, D = q.shape
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    ck = torch.from_numpy(np.ascontiguousarray(cache_k, np.float32)).to(dev)
    cv = torch.from_numpy(np.ascontiguousarray(cache_v, np.float32)).to(dev)
    slots_n, n_kv, _ = ck.shape
    if n_kv != n_kv_heads:
        raise ValueError("cache heads do not match n_kv_heads")
    ck = ck.view(slots_n, n_kv, 1, D)
    cv = cv.view(slots_n, n_kv, 1, D)
    rs = np.asarray(read_slots, np.int64)
    if rs.size and (rs.min() < 0 or rs.max() >= slots_n):
        raise IndexError("read slot out of range")
    out = paged_attention_varlen(torch.from_numpy(q).to(dev), ck, cv, rs.reshape(1, -1), [0, q_len],
                                 [rs.size], scale, max_qlen=q_len, max_ctx=rs.size)
    return out.cpu().numpy()


def rms_norm(x, w, eps=1e-5, idx=None):
    import torch

    rows = idx.shape[0] if idx is not None else x.shape[0]
    out = torch.empty((rows, x.shape[1]), dtype=torch.float32, device=x.device)
    ix = _i32(idx, x.device) if idx is not None else None
    x = x.contiguous()
    check(lib().vllt_rmsnorm(ptr(x), ptr(ix), ptr(w), ptr(out), rows, x.shape[1], float(eps),
                             stream_handle()))
    return out


def apply_rope(x, positions, cos, sin):
    """In place on a float32 CUDA tensor x [T, heads, D]; returns x."""
    T, heads, D = x.shape
    pos = _i32(positions, x.device)
    check(lib().vllt_rope(ptr(x), ptr(pos), ptr(cos), ptr(sin), T, heads, D, cos.shape[0], stream_handle()))
    return x


def matmul(a, b):
    """fp32 A[M,K] @ B[K,N] on CUDA cores (no TF32)."""
    import torch

    M, K = a.shape
    N = b.shape[1]
    c = torch.empty((M, N), dtype=torch.float32, device=a.device)
    a, b = a.contiguous(), b.contiguous()
    check(lib().vllt_sgemm(ptr(a), ptr(b), ptr(c), M, N, K, stream_handle()))
    return c


def greedy(logits, eos_mask=None, eos_id=257, penalty=None, seen_bits=None, vocab=None):
    """Greedy tokens per row with min_tokens EOS masking and repetition penalty."""
    import torch

    rows, ld = logits.shape
    vocab = vocab or ld
    out = torch.empty(rows, dtype=torch.int32, device=logits.device)
    em = eos_mask.to(torch.uint8).contiguous() if eos_mask is not None else None
    check(lib().vllt_sample_greedy(ptr(logits), rows, vocab, ld, ptr(em), eos_id, ptr(penalty),
                                   ptr(seen_bits), ptr(out), stream_handle()))
    return out


def sample_top_p(logits, temperature, top_k, top_p, u, vocab=None, row_index=None, eos_mask=None, eos_id=257,
                 penalty=None, seen_bits=None):
    """Temperature rows of vllmlite.sampling.sample (sampling.py:41-64) on the
    device: EOS mask, repetition penalty, temperature, top-k, top-p, then the
    inverse-CDF draw of the float64 uniform u[r] (what the request's generator
    hands numpy's choice()). Row r reads logits[row_index[r]] (row r when
    row_index is None). Returns int32 tokens [rows]."""
    import torch

    n_logit_rows, ld = logits.shape
    vocab = vocab or ld
    rows = row_index.shape[0] if row_index is not None else n_logit_rows
    out = torch.empty(rows, dtype=torch.int32, device=logits.device)
    ri = _i32(row_index, logits.device) if row_index is not None else None
    em = eos_mask.to(torch.uint8).contiguous() if eos_mask is not None else None
    u = u.to(torch.float64).contiguous()
    check(lib().vllt_sample_top_p(ptr(logits), rows, vocab, ld, n_logit_rows, ptr(ri), ptr(em), eos_id,
                                  ptr(penalty), ptr(seen_bits), ptr(temperature), ptr(top_k), ptr(top_p),
                                  ptr(u), ptr(out), stream_handle()))
    return out


def verify(logits, cu_rows, drafts, draft_offsets, vocab=None):
    """Batched speculative accept/reject; returns (tokens per row, n_accepted)."""
    import torch

    rows, ld = logits.shape
    vocab = vocab or ld
    cu = _i32(cu_rows, logits.device)
    S = cu.shape[0] - 1
    dr = _i32(drafts if len(drafts) else [0], logits.device)
    do = _i32(draft_offsets, logits.device)
    toks = torch.empty(rows, dtype=torch.int32, device=logits.device)
    acc = torch.empty(S, dtype=torch.int32, device=logits.device)
    check(lib().vllt_spec_verify(ptr(logits), ld, vocab, ptr(cu), rows, ptr(dr), ptr(do), S, ptr(toks),
                                 ptr(acc), stream_handle()))
    return toks, acc
