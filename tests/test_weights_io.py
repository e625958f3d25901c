"""CPU: loading weights from checkpoints.

  * load_npz (fp32 model) reads the reference's checkpoint format exactly as
    the reference's TinyLlama.load does (vllmlite/model.py:64-71): the same
    .npz, loaded by both, gives bit-identical arrays, with and without an
    lm_head (tied when absent) and from float64 arrays;
  * initial_weights follows the reference constructor: the seeded init, or the
    checkpoint when ModelConfig.weights_path is set;
  * LlamaWeights (bf16 model) takes a checkpoint in the same naming and
    orientation, bf16 given as uint16 bit patterns or as floats rounded to
    bf16, and lays out each tensor-parallel rank's shard: [q|k|v] rows of its
    heads, gate/up rows interleaved, wo / w_down columns, lm_head rows of its
    vocabulary slice (tok_emb when the checkpoint has no lm_head).
"""

import numpy as np
import pytest

from tests import fixtures as F
from tests.conftest import needs_vllmlite

torch = pytest.importorskip("torch")


def reference_checkpoint(path, cfg, seed, lm_head=True, dtype=np.float32):
    from vllmlite.model import Layer, TinyLlama

    m = TinyLlama(cfg)
    rng = np.random.default_rng(seed)
    arrays = {"tok_emb": m.tok_emb, "final_norm": m.final_norm + rng.standard_normal(m.final_norm.shape)}
    if lm_head:
        arrays["lm_head"] = rng.standard_normal(m.lm_head.shape)
    for i, layer in enumerate(m.layers):
        for k in Layer.__slots__:
            arrays[f"layers.{i}.{k}"] = getattr(layer, k) + 0.01 * rng.standard_normal(getattr(layer, k).shape)
    np.savez(path, **{k: np.asarray(v, dtype) for k, v in arrays.items()})


@needs_vllmlite
@pytest.mark.parametrize("lm_head,dtype", [(True, np.float32), (False, np.float32), (True, np.float64)])
def test_load_npz_matches_the_reference_loader(tmp_path, lm_head, dtype):
    from vllmlite.config import ModelConfig
    from vllmlite.model import Layer, TinyLlama

    from vllt.model import initial_weights, load_npz

    path = str(tmp_path / "ckpt.npz")
    cfg = ModelConfig(vocab_size=261, **F.TINY)
    reference_checkpoint(path, cfg, 5, lm_head, dtype)
    cfg_w = ModelConfig(vocab_size=261, weights_path=path, **F.TINY)
    ref = TinyLlama(cfg_w)  # the reference constructor loads weights_path
    for got in (load_npz(path, cfg), initial_weights(cfg_w)):
        np.testing.assert_array_equal(got["tok_emb"], ref.tok_emb)
        np.testing.assert_array_equal(got["lm_head"], ref.lm_head)
        np.testing.assert_array_equal(got["final_norm"], ref.final_norm)
        for i, layer in enumerate(ref.layers):
            for k in Layer.__slots__:
                a = got[f"layers.{i}.{k}"]
                assert a.dtype == np.float32
                np.testing.assert_array_equal(a, getattr(layer, k))
    # without weights_path: the reference's seeded init
    seeded = initial_weights(cfg)
    np.testing.assert_array_equal(seeded["tok_emb"], TinyLlama(cfg).tok_emb)


def _llama_checkpoint(shape, seed, as_bits, lm_head):
    rng = np.random.default_rng(seed)
    D, H, KV, d, f, V = shape.head_dim, shape.n_heads, shape.n_kv_heads, shape.d_model, shape.d_ff, shape.vocab_size
    dims = {"wq": (d, H * D), "wk": (d, KV * D), "wv": (d, KV * D), "wo": (H * D, d), "w_gate": (d, f),
            "w_up": (d, f), "w_down": (f, d)}
    arrays = {"tok_emb": rng.standard_normal((V, d)) * 0.02, "final_norm": 1 + 0.1 * rng.standard_normal(d)}
    if lm_head:
        arrays["lm_head"] = rng.standard_normal((d, V)) * 0.02
    for i in range(shape.n_layers):
        for k, s in dims.items():
            arrays[f"layers.{i}.{k}"] = rng.standard_normal(s) * 0.02
        arrays[f"layers.{i}.attn_norm"] = 1 + 0.1 * rng.standard_normal(d)
        arrays[f"layers.{i}.ffn_norm"] = 1 + 0.1 * rng.standard_normal(d)
    bf = {k: torch.from_numpy(v.astype(np.float32)).to(torch.bfloat16) for k, v in arrays.items()}
    if as_bits:
        stored = {k: (t.view(torch.int16).numpy().view(np.uint16) if "norm" not in k else arrays[k].astype(np.float32))
                  for k, t in bf.items()}
    else:
        stored = {k: v.astype(np.float32) for k, v in arrays.items()}
    return stored, {k: t.float() for k, t in bf.items()}, {k: torch.from_numpy(v.astype(np.float32))
                                                           for k, v in arrays.items()}


@pytest.mark.parametrize("as_bits", [True, False])
@pytest.mark.parametrize("lm_head", [True, False])
def test_llama_checkpoint_shards(tmp_path, as_bits, lm_head):
    from vllt.llama import LlamaShape, LlamaWeights, load_llama_npz

    shape = LlamaShape(n_layers=2, n_heads=4, n_kv_heads=2, d_model=64, d_ff=96, vocab_size=100, max_seq_len=64)
    D, H, KV, f, V = shape.head_dim, shape.n_heads, shape.n_kv_heads, shape.d_ff, shape.vocab_size
    stored, want_bf, want32 = _llama_checkpoint(shape, 7, as_bits, lm_head)
    path = str(tmp_path / "llama.npz")
    np.savez(path, **stored)
    src = load_llama_npz(path)
    for n in (1, 2):
        for r in range(n):
            w = LlamaWeights(shape, "cpu", r, n, source=src)
            hl, kl, fl, vl = H // n, KV // n, f // n, V // n
            for i, lay in enumerate(w.layers):
                p = f"layers.{i}."
                wqkv = torch.cat([want_bf[p + "wq"].T[r * hl * D:(r + 1) * hl * D],
                                  want_bf[p + "wk"].T[r * kl * D:(r + 1) * kl * D],
                                  want_bf[p + "wv"].T[r * kl * D:(r + 1) * kl * D]])
                assert lay["wqkv"].dtype == torch.bfloat16 and lay["wqkv"].is_contiguous()
                assert torch.equal(lay["wqkv"].float(), wqkv)
                assert torch.equal(lay["wo"].float(), want_bf[p + "wo"].T[:, r * hl * D:(r + 1) * hl * D])
                assert torch.equal(lay["w_gu"][0::2].float(), want_bf[p + "w_gate"].T[r * fl:(r + 1) * fl])
                assert torch.equal(lay["w_gu"][1::2].float(), want_bf[p + "w_up"].T[r * fl:(r + 1) * fl])
                assert torch.equal(lay["w_down"].float(), want_bf[p + "w_down"].T[:, r * fl:(r + 1) * fl])
                assert lay["attn_norm"].dtype == torch.float32
                assert torch.equal(lay["attn_norm"], want32[p + "attn_norm"])
            assert torch.equal(w.tok_emb.float(), want_bf["tok_emb"])
            head = want_bf["lm_head"].T if lm_head else want_bf["tok_emb"]  # tied when absent
            assert torch.equal(w.lm_head.float(), head[r * vl:(r + 1) * vl])
            assert (w.vocab_local, w.vocab_offset) == (vl, r * vl)


def test_llama_checkpoint_rejects_integer_arrays():
    from vllt.llama import checkpoint_tensor

    with pytest.raises(ValueError):
        checkpoint_tensor(np.zeros(4, np.int32), "cpu", torch.bfloat16)
    bits = np.asarray([0x3F80, 0xBF00], np.uint16)  # bf16 1.0 and -0.5
    assert checkpoint_tensor(bits, "cpu", torch.float32).tolist() == [1.0, -0.5]
