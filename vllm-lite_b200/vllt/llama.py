"""The Llama-3-8B-shaped bf16 model behind the same runner interface.

Shape (the north star's large config): 32 layers, d_model 4096, 32 query / 8 KV
heads of 128, SwiGLU FFN 14336, vocabulary 128256, RoPE theta 10000 as in
vllmlite/attention.py:21, bf16 weights drawn N(0, 0.02) from a seed. There is no
reference checkpoint at this shape; by default every weight matrix is
generated on the device from (seed, layer, name), so its values do not depend
on the tensor-parallel split and a TP run computes the same model as a 1-GPU
run. A checkpoint in the reference's .npz naming (bf16 as uint16 bits, or any
float type) loads instead (`load_llama_npz`, `LlamaRunner(weights=path)` or
`ModelConfig.weights_path`).

Layout for the tcgen05 GEMM (K-major, [out][in]); per rank r of N:
  wqkv   rows [q heads of r | k heads of r | v heads of r]      [(H+2KV)/N*128][4096]
  wo     columns of r's heads                                   [4096][H/N*128]
  w_gu   rows of r's FFN columns, gate/up interleaved           [2*14336/N][4096]
  w_down columns of r's FFN rows                                [4096][14336/N]
  lm_head rows of r's vocabulary slice                          [128256/N][4096]
  tok_emb, norms: replicated.
"""

from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from . import _lib
from .model import rope_tables
from .runner import CudaRunner

NAMES = ("wq", "wk", "wv", "wo", "w_gate", "w_up", "w_down", "tok_emb", "lm_head")


@dataclass
class LlamaShape:
    """Field names follow vllmlite/config.py:5-25 so it can stand in for ModelConfig."""

    n_layers: int = 32
    n_heads: int = 32
    n_kv_heads: int = 8
    d_model: int = 4096
    d_ff: int = 14336
    vocab_size: int = 128256
    max_seq_len: int = 9216
    seed: int = 0

    @property
    def head_dim(self) -> int:
        return self.d_model // self.n_heads


def _normal(shape, key: int, std: float, device):
    import torch

    g = torch.Generator(device=device)
    g.manual_seed(int(key) & 0x7FFFFFFFFFFFFFFF)
    return (torch.randn(shape, generator=g, device=device, dtype=torch.float32) * std).to(torch.bfloat16)


def full_matrix(cfg, layer: int, name: str, device, std: float = 0.02):
    """One unsharded weight in its natural [out][in] orientation."""
    D, H, KV, d, f, V = cfg.head_dim, cfg.n_heads, cfg.n_kv_heads, cfg.d_model, cfg.d_ff, cfg.vocab_size
    shape = {"wq": (H * D, d), "wk": (KV * D, d), "wv": (KV * D, d), "wo": (d, H * D), "w_gate": (f, d),
             "w_up": (f, d), "w_down": (d, f), "tok_emb": (V, d), "lm_head": (V, d)}[name]
    key = (cfg.seed * 1000003 + (layer + 1) * 7919 + NAMES.index(name) * 104729) * 2654435761
    return _normal(shape, key, std, device)


def checkpoint_tensor(a, device, dtype):
    """A checkpoint array as a torch tensor of `dtype` on `device`: floating
    arrays (float16 / float32 / float64) are rounded to dtype; uint16 arrays
    are bf16 bit patterns (NumPy has no bfloat16: that is how a bf16
    checkpoint is stored in an .npz)."""
    import torch

    a = np.asarray(a)
    if a.dtype == np.uint16:
        t = torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16)
    elif a.dtype.kind == "f":
        t = torch.from_numpy(np.ascontiguousarray(a))
    else:
        raise ValueError(f"checkpoint array of dtype {a.dtype}: expected float or uint16 (bf16 bits)")
    return t.to(device=device, dtype=dtype)


def load_llama_npz(path: str):
    """A Llama-shaped checkpoint in the reference's .npz naming and
    orientation (vllmlite/model.py:64-71): tok_emb [V][d], final_norm [d],
    lm_head [d][V] (optional: tied to tok_emb), layers.{i}.{attn_norm, wq
    [d][H*D], wk, wv [d][KV*D], wo [H*D][d], ffn_norm, w_gate, w_up [d][f],
    w_down [f][d]}. Arrays are read when used."""
    return np.load(path)


class LlamaWeights:
    """This rank's bf16 shard on the device, in libvllt's layout: drawn from
    the seed (`source` None), or taken from a checkpoint mapping in the
    reference's naming and [in][out] orientation (see load_llama_npz), each
    array transposed to [out][in], rounded to bf16 and sliced to this rank."""

    def __init__(self, cfg, device, tp_rank: int = 0, tp_size: int = 1, source=None):
        import torch

        D, H, KV, f, V = cfg.head_dim, cfg.n_heads, cfg.n_kv_heads, cfg.d_ff, cfg.vocab_size
        if H % tp_size or KV % tp_size or f % tp_size or V % tp_size:
            raise ValueError(f"heads, KV heads, d_ff and vocab must divide by tp_size={tp_size}")
        hl, kl, fl, vl = H // tp_size, KV // tp_size, f // tp_size, V // tp_size
        r = tp_rank
        bf = torch.bfloat16

        def mat(layer, name):  # [out][in] bf16
            if source is None:
                return full_matrix(cfg, layer, name, device)
            key = name if layer < 0 else f"layers.{layer}.{name}"
            if name == "lm_head" and key not in source:
                return checkpoint_tensor(source["tok_emb"], device, bf)  # tied: lm_head = tok_emb.T
            t = checkpoint_tensor(source[key], device, bf)
            return t if name == "tok_emb" else t.T

        def norm(key):
            if source is None:
                return torch.ones(cfg.d_model, dtype=torch.float32, device=device)
            return checkpoint_tensor(source[key], device, torch.float32).contiguous()

        self.vocab_local, self.vocab_offset = vl, r * vl
        self.vocab_padded = (vl + 3) // 4 * 4
        self.layers = []
        for i in range(cfg.n_layers):
            wq = mat(i, "wq")[r * hl * D:(r + 1) * hl * D]
            wk = mat(i, "wk")[r * kl * D:(r + 1) * kl * D]
            wv = mat(i, "wv")[r * kl * D:(r + 1) * kl * D]
            wo = mat(i, "wo")[:, r * hl * D:(r + 1) * hl * D]
            g = mat(i, "w_gate")[r * fl:(r + 1) * fl]
            u = mat(i, "w_up")[r * fl:(r + 1) * fl]
            gu = torch.empty((2 * fl, cfg.d_model), dtype=bf, device=device)
            gu[0::2], gu[1::2] = g, u
            wd = mat(i, "w_down")[:, r * fl:(r + 1) * fl]
            self.layers.append(dict(
                attn_norm=norm(f"layers.{i}.attn_norm"),
                wqkv=torch.cat([wq, wk, wv], 0).contiguous(), wo=wo.contiguous(),
                ffn_norm=norm(f"layers.{i}.ffn_norm"),
                w_gu=gu, w_down=wd.contiguous()))
            del wq, wk, wv, g, u
        self.tok_emb = mat(-1, "tok_emb").contiguous()
        self.lm_head = mat(-1, "lm_head")[r * vl:(r + 1) * vl].contiguous()
        self.final_norm = norm("final_norm")
        cos, sin = rope_tables(D, cfg.max_seq_len)
        self.rope_cos = torch.from_numpy(cos).to(device)
        self.rope_sin = torch.from_numpy(sin).to(device)
        self.rope_len = cos.shape[0]

    def pointer_arrays(self):
        names = ("attn_norm", "wqkv", "wo", "ffn_norm", "w_gu", "w_down")
        n = len(self.layers)
        return {k: (C.c_void_p * n)(*[l[k].data_ptr() for l in self.layers]) for k in names}


def fp32_reference_weights(cfg, device) -> dict:
    """The same (unsharded) model in the fp32 parity path's reference layout
    ([in][out], vllmlite/model.py:34-43), values = the bf16 weights exactly.
    Used to validate the bf16 path against an fp32 GPU re-run."""
    out = {"tok_emb": full_matrix(cfg, -1, "tok_emb", device).float(),
           "lm_head": full_matrix(cfg, -1, "lm_head", device).float().T.contiguous()}
    import torch

    out["final_norm"] = torch.ones(cfg.d_model, dtype=torch.float32, device=device)
    for i in range(cfg.n_layers):
        p = f"layers.{i}."
        for n in ("wq", "wk", "wv", "wo", "w_gate", "w_up", "w_down"):
            out[p + n] = full_matrix(cfg, i, n, device).float().T.contiguous()
        out[p + "attn_norm"] = torch.ones(cfg.d_model, dtype=torch.float32, device=device)
        out[p + "ffn_norm"] = torch.ones(cfg.d_model, dtype=torch.float32, device=device)
    return out


class LlamaRunner(CudaRunner):
    """bf16 forward of the Llama-shaped model (tcgen05 GEMMs), optionally one
    tensor-parallel shard. Same ModelRunner contract as CudaRunner."""

    def __init__(self, model_cfg, cache_cfg, sched_cfg=None, *, tp_rank: int = 0, tp_size: int = 1,
                 tp_comm=None, **kw):
        self.tp_rank, self.tp_size, self.tp_comm = tp_rank, tp_size, tp_comm
        if tp_size > 1 and not tp_comm:
            raise ValueError("tp_size > 1 needs a communicator (vllt.tp.TPGroup)")
        kw.setdefault("max_seqs", sched_cfg.max_seqs if sched_cfg is not None else 256)
        super().__init__(model_cfg, cache_cfg, sched_cfg, **kw)

    def _init_model(self, weights) -> None:
        """weights: None (seeded, or cfg.weights_path when set), a checkpoint
        path, or a mapping in the reference's naming (see load_llama_npz)."""
        torch, cfg = self.torch, self.model_cfg
        if weights is None and getattr(cfg, "weights_path", None):
            weights = cfg.weights_path
        if isinstance(weights, str):
            weights = load_llama_npz(weights)
        self.w = LlamaWeights(cfg, self.dev, self.tp_rank, self.tp_size, source=weights)
        kv_local = cfg.n_kv_heads // self.tp_size
        shape = (cfg.n_layers, self.num_blocks, kv_local, self.block_size, self.head_dim)
        self.cache_k = torch.zeros(shape, dtype=torch.bfloat16, device=self.dev)
        self.cache_v = torch.zeros(shape, dtype=torch.bfloat16, device=self.dev)

    @property
    def vocab_size(self) -> int:
        return self.model_cfg.vocab_size

    def _make_desc(self):
        cfg, w, p, n = self.model_cfg, self.w, self._ptrs, self.tp_size
        d = _lib.ModelDesc()
        d.n_layers, d.n_heads, d.n_kv_heads = cfg.n_layers, cfg.n_heads // n, cfg.n_kv_heads // n
        d.head_dim, d.d_model, d.d_ff = self.head_dim, cfg.d_model, cfg.d_ff // n
        d.vocab, d.vocab_padded = w.vocab_local, w.vocab_padded
        d.max_seq_len, d.block_size, d.num_blocks = w.rope_len, self.block_size, self.num_blocks
        d.rms_eps, d.dtype = 1e-5, _lib.VLLT_BF16
        d.tp_size, d.embed_rows, d.tp_comm = n, cfg.vocab_size, self.tp_comm
        d.tok_emb, d.final_norm, d.lm_head = w.tok_emb.data_ptr(), w.final_norm.data_ptr(), w.lm_head.data_ptr()
        d.rope_cos, d.rope_sin = w.rope_cos.data_ptr(), w.rope_sin.data_ptr()
        for k in ("attn_norm", "wqkv", "wo", "ffn_norm", "w_gu", "w_down"):
            setattr(d, k, C.cast(p[k], C.POINTER(C.c_void_p)))
        d.k_cache, d.v_cache = self.cache_k.data_ptr(), self.cache_v.data_ptr()
        return d

    # ---- per-step roofline (for the benchmark) -----------------------------------
    def step_roofline(self, rec, bounds, hbm_gbs: float, tflops: float) -> float:
        """Lower bound on one forward pass's time on this rank: the larger of
        (weights + KV read/written) / HBM bandwidth and (GEMM + attention
        FLOPs) / tensor peak. Attention FLOPs count the causal pairs only."""
        cfg, n = self.model_cfg, self.tp_size
        f = self.packer.fields(rec)
        T, R = f["T"], f["R"]
        starts = f["start"].astype(np.int64)
        qlens = f["qlen"].astype(np.int64)
        ctx = starts + qlens
        d, f, D = cfg.d_model, cfg.d_ff, self.head_dim
        layer_params = d * (cfg.n_heads + 2 * cfg.n_kv_heads) * D + d * cfg.n_heads * D + 3 * d * f
        w_bytes = 2 * (cfg.n_layers * layer_params + cfg.vocab_size * d) / n
        kv_token = 2 * cfg.n_layers * cfg.n_kv_heads * D * 2 / n
        kv_bytes = kv_token * (float(ctx.sum()) + T)
        # causal (query, key) pairs: query j of a chunk sees start + j + 1 keys
        pairs = float(np.sum(qlens * starts + qlens * (qlens + 1) // 2))
        flops = (2 * T * cfg.n_layers * layer_params + 2 * R * cfg.vocab_size * d
                 + 4 * cfg.n_layers * cfg.n_heads * D * pairs) / n
        return max((w_bytes + kv_bytes) / (hbm_gbs * 1e9), flops / (tflops * 1e12))

    def launch(self, out):
        rows, R = super().launch(out)
        if getattr(self, "roofline_peaks", None):
            self.roofline_s += self.step_roofline(self._last_rec, None, *self.roofline_peaks)
        return rows, R

    def execute(self, out):
        if self.tp_size > 1:
            raise NotImplementedError("host logits are not gathered across vocabulary shards; use gpu_engine")
        return super().execute(out)
