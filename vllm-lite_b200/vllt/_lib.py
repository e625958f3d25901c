"""ctypes binding of libvllt.so (the C ABI in include/vllt.h).

The product path has no fallback: if the library is missing or the process
has no CUDA device, the calls raise instead of computing anything on the CPU.
"""

from __future__ import annotations

import ctypes as C
import os

VLLT_OK, VLLT_ERR_ARG, VLLT_ERR_CUDA, VLLT_ERR_TIMEOUT, VLLT_ERR_UNSUPPORTED, VLLT_ERR_DATA = range(6)
VLLT_F32, VLLT_BF16 = 0, 1

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libvllt.so")

i32, i64, f32, vp = C.c_int32, C.c_int64, C.c_float, C.c_void_p
P_i32 = C.POINTER(C.c_int32)


class Caps(C.Structure):
    _fields_ = [("max_seqs", i32), ("max_tokens", i32), ("max_rows", i32), ("max_table_width", i32)]


class StepBounds(C.Structure):
    _fields_ = [("tokens", i32), ("rows", i32), ("decode_seqs", i32), ("tiles", i32), ("max_ctx", i32)]


PP = C.POINTER(vp)


class ModelDesc(C.Structure):
    _fields_ = [
        ("n_layers", i32), ("n_heads", i32), ("n_kv_heads", i32), ("head_dim", i32),
        ("d_model", i32), ("d_ff", i32), ("vocab", i32), ("vocab_padded", i32),
        ("max_seq_len", i32), ("block_size", i32), ("num_blocks", i32),
        ("rms_eps", f32), ("dtype", i32), ("tp_size", i32), ("embed_rows", i32), ("tp_comm", vp),
        ("tok_emb", vp), ("final_norm", vp), ("lm_head", vp), ("rope_cos", vp), ("rope_sin", vp),
        ("attn_norm", PP), ("wqkv", PP), ("wo", PP), ("ffn_norm", PP), ("w_gu", PP), ("w_down", PP),
        ("k_cache", vp), ("v_cache", vp), ("table_pool", vp), ("table_pool_slots", i32),
        ("token_source", vp), ("token_source_len", i32),
    ]


# name -> (restype, argtypes); mirrors include/vllt.h
SIGNATURES = {
    "vllt_last_error": (C.c_char_p, []),
    "vllt_version": (C.c_int, []),
    "vllt_kernel_launches": (i64, []),
    "vllt_reshape_and_cache": (C.c_int, [vp, vp, vp, vp, vp, i32, i32, i32, i32, i32, i32, vp]),
    "vllt_copy_blocks": (C.c_int, [vp, vp, vp, i32, i32, i32, i32, i32, i32, i32, vp]),
    "vllt_meta_bytes": (i64, [C.POINTER(Caps)]),
    "vllt_build_batch_meta": (C.c_int, [vp, C.POINTER(Caps), i32, i32, i32, vp, vp]),
    "vllt_build_batch_meta_pooled": (C.c_int, [vp, C.POINTER(Caps), i32, i32, i32, vp, i32, vp, vp]),
    "vllt_meta_field": (vp, [vp, C.POINTER(Caps), i32]),
    "vllt_attention_workspace_bytes": (i64, [i32, i32, i32, i32]),
    "vllt_paged_attention_varlen": (C.c_int, [vp, vp, vp, vp, i32, vp, vp, i32, i32, i32, i32, i32,
                                              i32, i32, i32, i32, f32, i32, vp, vp, i64, vp]),
    "vllt_paged_attention_varlen_noalloc": (C.c_int, [vp, vp, vp, vp, i32, vp, vp, i32, i32, i32, i32, i32,
                                                      i32, i32, i32, i32, f32, i32, vp, vp, vp]),
    "vllt_test_decode_stall": (C.c_int, [i32, i64]),
    "vllt_rmsnorm": (C.c_int, [vp, vp, vp, vp, i32, i32, f32, vp]),
    "vllt_rope": (C.c_int, [vp, vp, vp, vp, i32, i32, i32, i32, vp]),
    "vllt_sgemm": (C.c_int, [vp, vp, vp, i32, i32, i32, vp]),
    "vllt_gemm_bf16": (C.c_int, [vp, vp, vp, i32, i32, i32, vp, vp]),
    "vllt_gemm_bf16_splitk_workspace_bytes": (i64, [i32, i32, i32, i32]),
    "vllt_gemm_bf16_auto_splits": (i32, [i32, i32, i32]),
    "vllt_gemm_bf16_splitk": (C.c_int, [vp, vp, vp, i32, i32, i32, i32, vp, i64, vp, vp]),
    "vllt_sample_greedy": (C.c_int, [vp, i32, i32, i32, vp, i32, vp, vp, vp, vp]),
    "vllt_sample_top_p": (C.c_int, [vp, i32, i32, i32, i32, vp, vp, i32, vp, vp, vp, vp, vp, vp, vp, vp]),
    "vllt_spec_verify": (C.c_int, [vp, i32, i32, vp, i32, vp, vp, i32, vp, vp, vp]),
    "vllt_spec_accept": (C.c_int, [vp, vp, vp, i32, vp, vp, vp]),
    "vllt_prefix_hash_chains": (C.c_int, [vp, vp, vp, vp, vp, i32, i32, vp, vp]),
    "vllt_tp_unique_id": (C.c_int, [vp]),
    "vllt_tp_init": (C.c_int, [vp, i32, i32, C.POINTER(vp)]),
    "vllt_tp_destroy": (C.c_int, [vp]),
    "vllt_tp_allreduce_bf16": (C.c_int, [vp, i64, vp, vp]),
    "vllt_argmax_rows": (C.c_int, [vp, i32, i32, i32, i32, vp, vp, vp]),
    "vllt_query_tile_positions": (i32, [C.POINTER(ModelDesc)]),
    "vllt_forward_workspace_bytes": (i64, [C.POINTER(ModelDesc), C.POINTER(Caps)]),
    "vllt_forward": (C.c_int, [C.POINTER(ModelDesc), vp, C.POINTER(Caps), C.POINTER(StepBounds),
                               vp, vp, i64, vp, vp]),
}

_lib = None


def lib() -> C.CDLL:
    """Load libvllt.so once (built in-tree by `python -m vllt.build`)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build it with `python -m vllt.build`")
        handle = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


class VlltError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"vllt error {code}: {msg}")
        self.code = code


def check(rc: int) -> None:
    """Raise like the reference does (Python exceptions): bad arguments become
    ValueError, everything else VlltError."""
    if rc == VLLT_OK:
        return
    msg = (lib().vllt_last_error() or b"").decode(errors="replace")
    if rc == VLLT_ERR_ARG:
        raise ValueError(msg)
    raise VlltError(rc, msg)


def ptr(t) -> int | None:
    """Device address of a torch tensor (None for None)."""
    return None if t is None else t.data_ptr()


def stream_handle(stream=None) -> int:
    import torch

    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream
