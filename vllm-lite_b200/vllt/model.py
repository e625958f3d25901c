"""TinyLlama weights for the CUDA forward pass: creation, loading and device layout.

Three sources, all in the reference's naming (vllmlite/model.py:26-71):
  * `seeded_weights(cfg)` - the reference's random init, draw for draw
    (vllmlite/model.py:29-43, :47-55), so the same seed gives bit-identical
    arrays (pinned by tests/golden/weights.json);
  * `load_npz(path, cfg)`  - the reference's .npz checkpoint keys
    (vllmlite/model.py:64-71), used when cfg.weights_path is set, as the
    reference's constructor does (`initial_weights`);
  * `from_reference_model(m)` - the arrays of a live vllmlite TinyLlama.

`DeviceWeights` lays them out for libvllt: [wq|wk|wv] fused per layer,
w_gate/w_up interleaved column by column (the SwiGLU epilogue pairs them), the
lm_head padded to a multiple of 4 columns, and the RoPE tables.
"""

from __future__ import annotations

import numpy as np

LAYER_KEYS = ("attn_norm", "wq", "wk", "wv", "wo", "ffn_norm", "w_gate", "w_up", "w_down")


def _dims(cfg):
    head_dim = cfg.d_model // cfg.n_heads
    return cfg.d_model, head_dim, cfg.n_heads, cfg.n_kv_heads, cfg.d_ff, cfg.vocab_size


def seeded_weights(cfg) -> dict[str, np.ndarray]:
    """Random init identical to vllmlite.model.TinyLlama(cfg) for cfg.seed."""
    d, hd, H, KV, dff, V = _dims(cfg)
    rng = np.random.default_rng(cfg.seed)
    scale = 1.0 / np.sqrt(d)

    def draw(*shape):
        return (rng.standard_normal(shape) * scale).astype(np.float32)

    out = {"tok_emb": draw(V, d)}
    for i in range(cfg.n_layers):
        p = f"layers.{i}."
        out[p + "attn_norm"] = np.ones(d, np.float32)
        out[p + "wq"] = draw(d, H * hd)
        out[p + "wk"] = draw(d, KV * hd)
        out[p + "wv"] = draw(d, KV * hd)
        out[p + "wo"] = draw(H * hd, d)
        out[p + "ffn_norm"] = np.ones(d, np.float32)
        out[p + "w_gate"] = draw(d, dff)
        out[p + "w_up"] = draw(d, dff)
        out[p + "w_down"] = (rng.standard_normal((dff, d)) / np.sqrt(dff)).astype(np.float32)
    out["final_norm"] = np.ones(d, np.float32)
    out["lm_head"] = out["tok_emb"].T.copy()  # tied
    return out


def load_npz(path: str, cfg) -> dict[str, np.ndarray]:
    """Weights from a reference-format .npz (lm_head optional, then tied)."""
    z = np.load(path)
    out = {"tok_emb": z["tok_emb"].astype(np.float32), "final_norm": z["final_norm"].astype(np.float32)}
    out["lm_head"] = z["lm_head"].astype(np.float32) if "lm_head" in z else out["tok_emb"].T.copy()
    for i in range(cfg.n_layers):
        for k in LAYER_KEYS:
            out[f"layers.{i}.{k}"] = z[f"layers.{i}.{k}"].astype(np.float32)
    return out


def initial_weights(cfg) -> dict[str, np.ndarray]:
    """The weights TinyLlama(cfg) ends up with: the seeded init, replaced by
    the checkpoint at cfg.weights_path when one is set (vllmlite/model.py:61-62)."""
    path = getattr(cfg, "weights_path", None)
    return load_npz(path, cfg) if path else seeded_weights(cfg)


def from_reference_model(model) -> dict[str, np.ndarray]:
    """Copy the arrays of a vllmlite.model.TinyLlama instance."""
    out = {"tok_emb": model.tok_emb, "final_norm": model.final_norm, "lm_head": model.lm_head}
    for i, layer in enumerate(model.layers):
        for k in LAYER_KEYS:
            out[f"layers.{i}.{k}"] = getattr(layer, k)
    return {k: np.ascontiguousarray(v, dtype=np.float32) for k, v in out.items()}


def rope_tables(head_dim: int, max_pos: int, theta: float = 10000.0):
    """fp32 cos/sin [max_pos, head_dim/2] exactly as vllmlite/attention.py:21-25
    computes them (fp32 inverse frequencies and angles)."""
    inv = np.float32(1.0) / (np.float32(theta) ** (np.arange(0, head_dim, 2, dtype=np.float32)
                                                  / np.float32(head_dim)))
    ang = np.arange(max_pos, dtype=np.float32)[:, None] * inv[None, :]
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


class DeviceWeights:
    """fp32 device copies in libvllt's layout; keeps the tensors alive."""

    def __init__(self, cfg, weights: dict, device="cuda", rope_len: int | None = None):
        """weights: NumPy arrays or torch tensors (any device) in the reference's
        naming and [in][out] orientation."""
        import torch

        d, hd, H, KV, dff, V = _dims(cfg)
        self.vocab_padded = (V + 3) // 4 * 4
        dev = torch.device(device)

        def up(a):
            if isinstance(a, torch.Tensor):
                return a.to(device=dev, dtype=torch.float32).contiguous()
            return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(dev)

        self.tok_emb = up(weights["tok_emb"])
        self.final_norm = up(weights["final_norm"])
        self.lm_head = torch.zeros((d, self.vocab_padded), dtype=torch.float32, device=dev)
        self.lm_head[:, :V] = up(weights["lm_head"])
        cos, sin = rope_tables(hd, rope_len or cfg.max_seq_len)
        self.rope_cos, self.rope_sin = up(cos), up(sin)
        self.rope_len = cos.shape[0]
        self.layers = []
        for i in range(cfg.n_layers):
            p = f"layers.{i}."
            gu = torch.empty((d, 2 * dff), dtype=torch.float32, device=dev)
            gu[:, 0::2] = up(weights[p + "w_gate"])
            gu[:, 1::2] = up(weights[p + "w_up"])
            self.layers.append(dict(
                attn_norm=up(weights[p + "attn_norm"]),
                wqkv=torch.cat([up(weights[p + "wq"]), up(weights[p + "wk"]), up(weights[p + "wv"])], 1).contiguous(),
                wo=up(weights[p + "wo"]),
                ffn_norm=up(weights[p + "ffn_norm"]),
                w_gu=gu,
                w_down=up(weights[p + "w_down"]),
            ))

    def pointer_arrays(self):
        import ctypes as C

        names = ("attn_norm", "wqkv", "wo", "ffn_norm", "w_gu", "w_down")
        n = len(self.layers)
        arrs = {k: (C.c_void_p * n)(*[l[k].data_ptr() for l in self.layers]) for k in names}
        return arrs
