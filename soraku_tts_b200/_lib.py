"""ctypes binding of libsoraku_b200.so (the C ABI in include/soraku_b200.h).

The product has no CPU fallback: if the library is missing or a call fails,
this module raises.  Status codes map to the exception types the reference
raises: SKB_ERR_ARG -> ValueError, everything else -> RuntimeError.
"""

from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libsoraku_b200.so")

SKB_OK, SKB_ERR_ARG, SKB_ERR_STATE, SKB_ERR_CUDA, SKB_ERR_CAPACITY, SKB_ERR_NOMEM = range(6)
SKB_LAYER_PTRS = 11

c_int, c_float, c_void_p, c_int64, c_uint64 = (ctypes.c_int, ctypes.c_float, ctypes.c_void_p,
                                               ctypes.c_int64, ctypes.c_uint64)

# Every exported symbol and its signature (restype, argtypes).
SIGNATURES = {
    "skb_last_error": (ctypes.c_char_p, []),
    "skb_abi_version": (c_int, []),
    "skb_add_rmsnorm": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_float, c_void_p]),
    "skb_rmsnorm": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_float, c_void_p]),
    "skb_swiglu_gemv": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p]),
    "skb_down_residual_gemv": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p]),
    "skb_classifier_gemv": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p]),
    "skb_frame_embed": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_float, c_void_p]),
    "skb_prefix_add": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_float, c_void_p]),
    "skb_sampling_prep": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_void_p]),
    "skb_cfg_sample": (c_int, [c_void_p, c_int, c_int, c_int, c_void_p, c_int, c_int, c_int, c_void_p,
                               c_void_p, c_void_p]),
    "skb_decode_attention": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_void_p, c_float, c_void_p,
                                     c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int,
                                     c_void_p, c_void_p, c_void_p, c_void_p]),
    "skb_decode_attention_noalloc": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_void_p, c_float,
                                             c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_int, c_int,
                                             c_int, c_int, c_void_p, c_void_p]),
    "skb_test_exp": (c_int, [c_void_p, c_void_p, c_int, c_void_p]),
    "skb_test_philox": (c_int, [c_void_p, c_void_p, c_int, c_void_p]),
    "skb_test_wait_timeout": (c_int, [c_void_p, c_int, c_void_p]),
    "skb_test_gemm": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_void_p]),
    "skb_engine_create": (c_int, [c_void_p, c_void_p, c_void_p]),
    "skb_engine_destroy": (c_int, [c_void_p]),
    "skb_engine_set_rng_stream": (c_int, [c_void_p, c_int, ctypes.c_uint32]),
    "skb_engine_status": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_void_p]),
    "skb_engine_move_request": (c_int, [c_void_p, c_int, c_int, c_void_p]),
    "skb_engine_map_pages": (c_int, [c_void_p, c_int, c_int, c_int, c_void_p]),
    "skb_engine_prefill_many": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                        c_void_p, c_void_p, c_void_p]),
    "skb_engine_prefill": (c_int, [c_void_p, c_int, c_void_p, c_int, c_void_p, c_int, c_void_p, c_int,
                                   c_void_p, c_void_p]),
    "skb_engine_set_sampling": (c_int, [c_void_p, c_int, c_float, c_float, c_float, c_int, c_float, c_int,
                                        c_float, c_uint64, c_int, c_int]),
    "skb_engine_capture": (c_int, [c_void_p, c_int, c_int, c_void_p]),
    "skb_engine_step": (c_int, [c_void_p, c_int, c_void_p]),
    "skb_engine_step_eager": (c_int, [c_void_p, c_int, c_int, c_void_p]),
    "skb_engine_read_codes": (c_int, [c_void_p, c_int, c_int, c_int, c_void_p, c_void_p]),
    "skb_engine_frames": (c_int, [c_void_p, c_int]),
    "skb_engine_view": (c_int, [c_void_p, c_int, ctypes.POINTER(c_void_p), ctypes.POINTER(c_int64)]),
    "skb_engine_set_debug": (c_int, [c_void_p, c_int]),
    "skb_engine_kernels_per_frame": (c_int, [c_void_p]),
    "skb_engine_launches_per_step": (c_int, [c_void_p]),
}


class skb_sample_params(ctypes.Structure):
    _fields_ = [("cfg_scale", c_float), ("temperature", c_float), ("top_k", c_int), ("top_p", c_float),
                ("mask_eos", c_int), ("request", ctypes.c_uint32), ("frame", ctypes.c_uint32),
                ("q", ctypes.c_uint32), ("seed", c_uint64)]


class skb_model_desc(ctypes.Structure):
    _fields_ = [
        ("n_layers", c_int), ("d_model", c_int), ("n_heads", c_int), ("n_kv_heads", c_int),
        ("head_dim", c_int), ("ffn_dim", c_int), ("text_vocab", c_int), ("n_codebooks", c_int),
        ("audio_vocab", c_int), ("depth_inner", c_int), ("speaker_dim", c_int),
        ("rms_eps", c_float), ("depth_eps", c_float), ("frame_scale", c_float),
        ("bos_id", c_int), ("eos_id", c_int), ("pad_id", c_int), ("n_lang", c_int),
        ("lang_ids", c_int * 4),
        ("embed_tokens", c_void_p), ("lang_embed", c_void_p), ("final_norm", c_void_p),
        ("table", c_void_p), ("depth_bias", c_void_p), ("depth_norm_in", c_void_p),
        ("depth_norm_out", c_void_p), ("depth_gate", c_void_p), ("depth_up", c_void_p),
        ("depth_down", c_void_p), ("speaker_proj", c_void_p), ("speaker_slot", c_void_p),
        ("speaker_slot_mode", c_int), ("rope_inv_freq", c_void_p), ("layers", c_void_p),
    ]


class skb_engine_opts(ctypes.Structure):
    _fields_ = [("max_requests", c_int), ("rows_per_request", c_int), ("max_len", c_int),
                ("max_frames", c_int), ("max_prefill", c_int), ("page_size", c_int),
                ("attn_splits", c_int), ("use_pdl", c_int), ("l2_prefetch", c_int), ("gemm_min_rows", c_int),
                ("prefill_batch", c_int), ("kv_pages", c_int),
                ("split_depth_head", c_int)]


_lib = None


def lib() -> ctypes.CDLL:
    """Load the library (once).  Raises if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python -c 'import __graft_entry__ as g; g.build()'` "
                "(there is no CPU fallback)")
        handle = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def last_error() -> str:
    msg = lib().skb_last_error()
    return msg.decode() if msg else ""


def check(status: int, what: str = "") -> None:
    if status == SKB_OK:
        return
    msg = f"{what}: {last_error()}" if what else last_error()
    if status == SKB_ERR_ARG:
        raise ValueError(msg)
    raise RuntimeError(msg)


def call(name: str, *args) -> None:
    check(getattr(lib(), name)(*args), name)


def stream_ptr(stream=None) -> int:
    """Raw cudaStream_t of a torch stream (default: the current stream)."""
    import torch

    s = torch.cuda.current_stream() if stream is None else stream
    return int(s.cuda_stream)
