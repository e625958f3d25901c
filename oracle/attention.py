"""Oracle: paged attention, RoPE and slot arithmetic (test infrastructure only).

Restates vllmlite/attention.py of the reference in plain NumPy. Every function
names the reference lines it follows. The arithmetic order that matters for
fp32 agreement (scale applied after the dot product, max-subtracted softmax,
RoPE on interleaved even/odd pairs) is kept; loop structure is our own.
"""

from __future__ import annotations

import numpy as np


def rope_tables(head_dim: int, max_pos: int, theta: float = 10000.0):
    """cos/sin tables [max_pos, head_dim/2] in fp32.

    Follows vllmlite/attention.py:21-25: inverse frequencies
    1/theta**(2i/D) computed in fp32, angle = pos * inv_freq in fp32, then
    cos/sin of the fp32 angle rounded to fp32.
    """
    exps = np.arange(0, head_dim, 2, dtype=np.float32) / np.float32(head_dim)
    inv_freq = np.float32(1.0) / (np.float32(theta) ** exps)
    pos = np.arange(max_pos, dtype=np.float32)
    ang = pos[:, None] * inv_freq[None, :]
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


def rotate(x: np.ndarray, positions: np.ndarray, cos: np.ndarray, sin: np.ndarray) -> np.ndarray:
    """Rotate interleaved pairs (x[2i], x[2i+1]) of every head by its position.

    x is [T, heads, D]. Follows vllmlite/attention.py:28-37 (interleaved, not
    half-split: pair i is elements 2i and 2i+1).
    """
    c = cos[positions][:, None, :]
    s = sin[positions][:, None, :]
    even = x[..., 0::2]
    odd = x[..., 1::2]
    y = np.empty_like(x)
    y[..., 0::2] = even * c - odd * s
    y[..., 1::2] = even * s + odd * c
    return y


def table_slots(block_ids, block_size: int, count: int) -> np.ndarray:
    """Flat cache slots of positions 0..count-1: block_ids[p//bs]*bs + p%bs.

    Follows vllmlite/attention.py:40-44 and vllmlite/block.py:154-156.
    """
    pos = np.arange(count, dtype=np.int64)
    bids = np.asarray(block_ids, dtype=np.int64)
    return bids[pos // block_size] * block_size + pos % block_size


def scatter_kv(cache_k, cache_v, k, v, slots) -> None:
    """cache[slot[t]] = k[t] / v[t]. Follows vllmlite/attention.py:47-49."""
    cache_k[slots] = k
    cache_v[slots] = v


def paged_attention(q, cache_k, cache_v, read_slots, n_kv_heads: int, scale: float) -> np.ndarray:
    """Causal GQA attention of one sequence over its gathered context.

    q [q_len, H, D]; cache_* [slots, n_kv, D]; read_slots [ctx] in position
    order. Query j sits at absolute position ctx - q_len + j and sees keys
    0..that position. Query head h reads KV head h // (H // n_kv).
    Follows vllmlite/attention.py:59-98 (scores scaled after the dot product,
    softmax by max subtraction, then P @ V), in fp32 like the reference.
    """
    q_len, n_heads, d = q.shape
    ctx = len(read_slots)
    group = n_heads // n_kv_heads
    keys = cache_k[read_slots]  # [ctx, n_kv, D]
    vals = cache_v[read_slots]
    qpos = np.arange(ctx - q_len, ctx)
    allowed = np.arange(ctx)[None, :] <= qpos[:, None]  # [q_len, ctx]
    out = np.empty_like(q)
    for g in range(n_kv_heads):
        heads = slice(g * group, (g + 1) * group)
        # [group, q_len, D] x [D, ctx] -> [group, q_len, ctx]
        s = np.einsum("jhd,cd->hjc", q[:, heads, :], keys[:, g, :]).astype(np.float32)
        s *= np.float32(scale)
        s = np.where(allowed[None], s, np.float32(-np.inf)).astype(np.float32)
        s -= s.max(axis=-1, keepdims=True)
        p = np.exp(s)
        p /= p.sum(axis=-1, keepdims=True)
        out[:, heads, :] = np.einsum("hjc,cd->jhd", p, vals[:, g, :])
    return out


def dense_attention(q, k, v, n_kv_heads: int, scale: float) -> np.ndarray:
    """Contiguous causal GQA attention in float64 (the tighter checker).

    Same semantics as the reference's test oracle
    tests/test_attention.py:13-30: KV heads repeated per group, query row i
    masked past position ctx - q_len + i.
    """
    q = q.astype(np.float64)
    k = k.astype(np.float64)
    v = v.astype(np.float64)
    q_len, n_heads, _ = q.shape
    ctx = k.shape[0]
    group = n_heads // n_kv_heads
    out = np.zeros_like(q)
    qpos = np.arange(ctx - q_len, ctx)
    for h in range(n_heads):
        s = q[:, h] @ k[:, h // group].T * scale
        s[np.arange(ctx)[None, :] > qpos[:, None]] = -np.inf
        s = np.exp(s - s.max(axis=-1, keepdims=True))
        out[:, h] = (s / s.sum(axis=-1, keepdims=True)) @ v[:, h // group]
    return out
