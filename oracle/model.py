"""Oracle: seeded TinyLlama weights and the batched forward pass (test infrastructure only).

Restates vllmlite/model.py of the reference in NumPy. `forward` can run in
float32 (the reference's own precision) or float64 (the tighter checker used
for the 1e-3 relative logit bound).
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from .attention import paged_attention, rope_tables, rotate, scatter_kv

LAYER_KEYS = ("attn_norm", "wq", "wk", "wv", "wo", "ffn_norm", "w_gate", "w_up", "w_down")


@dataclass
class Shape:
    """Model dimensions; field meaning follows vllmlite/config.py:5-25."""

    n_layers: int = 6
    n_heads: int = 8
    n_kv_heads: int = 8
    d_model: int = 512
    d_ff: int = 2048
    vocab_size: int = 261
    max_seq_len: int = 2048
    seed: int = 1337

    @property
    def head_dim(self) -> int:
        return self.d_model // self.n_heads


def seeded_weights(cfg: Shape) -> dict[str, np.ndarray]:
    """The reference's random init, draw for draw.

    Follows vllmlite/model.py:29-43 and :47-55: one numpy Generator seeded with
    cfg.seed; tok_emb first, then per layer wq, wk, wv, wo, w_gate, w_up scaled by
    1/sqrt(d_model) and w_down divided by sqrt(d_ff) (float64 draws, cast to
    float32); norms are ones and lm_head is a copy of tok_emb transposed.
    """
    rng = np.random.default_rng(cfg.seed)
    d, hd = cfg.d_model, cfg.head_dim
    s = 1.0 / np.sqrt(d)
    w: dict[str, np.ndarray] = {}
    w["tok_emb"] = (rng.standard_normal((cfg.vocab_size, d)) * s).astype(np.float32)
    for i in range(cfg.n_layers):
        p = f"layers.{i}."
        w[p + "attn_norm"] = np.ones(d, np.float32)
        w[p + "wq"] = (rng.standard_normal((d, cfg.n_heads * hd)) * s).astype(np.float32)
        w[p + "wk"] = (rng.standard_normal((d, cfg.n_kv_heads * hd)) * s).astype(np.float32)
        w[p + "wv"] = (rng.standard_normal((d, cfg.n_kv_heads * hd)) * s).astype(np.float32)
        w[p + "wo"] = (rng.standard_normal((cfg.n_heads * hd, d)) * s).astype(np.float32)
        w[p + "ffn_norm"] = np.ones(d, np.float32)
        w[p + "w_gate"] = (rng.standard_normal((d, cfg.d_ff)) * s).astype(np.float32)
        w[p + "w_up"] = (rng.standard_normal((d, cfg.d_ff)) * s).astype(np.float32)
        w[p + "w_down"] = (rng.standard_normal((cfg.d_ff, d)) / np.sqrt(cfg.d_ff)).astype(np.float32)
    w["final_norm"] = np.ones(d, np.float32)
    w["lm_head"] = w["tok_emb"].T.copy()
    return w


def rms_norm(x, w, eps=1e-5):
    """x / sqrt(mean(x^2) + eps) * w. Follows vllmlite/model.py:17-19."""
    ms = np.mean(x * x, axis=-1, keepdims=True)
    return (x / np.sqrt(ms + x.dtype.type(eps))) * w


def silu(x):
    """x / (1 + exp(-x)). Follows vllmlite/model.py:22-23."""
    return x / (x.dtype.type(1.0) + np.exp(-x))


def forward(cfg: Shape, w, token_ids, positions, cache_k, cache_v, seq_meta, last_idx,
            dtype=np.float32):
    """One batched forward pass; returns logits [len(last_idx), V].

    Follows vllmlite/model.py:80-120. seq_meta is a list of
    (offset, q_len, write_slots, read_slots); cache_* are
    [L, slots, n_kv, D] arrays of `dtype` updated in place. Within each layer
    every sequence writes its K/V before it attends, so a chunk sees itself
    causally (model.py:105-112).
    """
    hd, H, KV = cfg.head_dim, cfg.n_heads, cfg.n_kv_heads
    cos, sin = rope_tables(hd, cfg.max_seq_len)
    cos, sin = cos.astype(dtype), sin.astype(dtype)
    scale = 1.0 / np.sqrt(hd)
    W = {k: v.astype(dtype) for k, v in w.items()}
    x = W["tok_emb"][np.asarray(token_ids)]
    for li in range(cfg.n_layers):
        p = f"layers.{li}."
        h = rms_norm(x, W[p + "attn_norm"])
        q = rotate((h @ W[p + "wq"]).reshape(-1, H, hd), positions, cos, sin)
        k = rotate((h @ W[p + "wk"]).reshape(-1, KV, hd), positions, cos, sin)
        v = (h @ W[p + "wv"]).reshape(-1, KV, hd)
        attn = np.empty_like(q)
        for off, n, wslots, rslots in seq_meta:
            scatter_kv(cache_k[li], cache_v[li], k[off:off + n], v[off:off + n], wslots)
            attn[off:off + n] = paged_attention(q[off:off + n], cache_k[li], cache_v[li],
                                                rslots, KV, scale)
        x = x + attn.reshape(-1, H * hd) @ W[p + "wo"]
        h = rms_norm(x, W[p + "ffn_norm"])
        x = x + (silu(h @ W[p + "w_gate"]) * (h @ W[p + "w_up"])) @ W[p + "w_down"]
    tail = rms_norm(x[np.asarray(last_idx)], W["final_norm"])
    return tail @ W["lm_head"]
