"""Drop-in op surface for soraku_inference/acceleration/tilelang_kernels.py.

Same eight factory names, same static parameters, same call signatures and
output allocation (the last argument of each TileLang kernel is the output,
``out_idx=[-1]``): ``factory(*static_shape)`` returns a callable that takes
the input tensors and returns a new output tensor.  The work runs on the
current CUDA stream through libsoraku_b200.so; inputs must be contiguous
CUDA tensors (float32, codes int64), as the reference's packed ABI requires
(fast_generate.py:94-97).  There is no CPU path.

    from soraku_tts_b200 import kernels as TLK
    k1 = TLK.add_rmsnorm(B, d, eps)
    a = k1(hidden, prefix, weight)
"""

from __future__ import annotations

import torch

from . import _lib

NEG_INF = -1e30  # tilelang_kernels.py:31


def _check(t: torch.Tensor, name: str, shape, dtype=torch.float32):
    if not isinstance(t, torch.Tensor):
        raise ValueError(f"{name}: expected a tensor")
    if t.device.type != "cuda":
        raise ValueError(f"{name}: must be a CUDA tensor (no CPU path)")
    if t.dtype != dtype:
        raise ValueError(f"{name}: expected {dtype}, got {t.dtype}")
    if tuple(t.shape) != tuple(shape):
        raise ValueError(f"{name}: expected shape {tuple(shape)}, got {tuple(t.shape)}")
    if not t.is_contiguous():
        raise ValueError(f"{name}: must be contiguous")


def _stream() -> int:
    return _lib.stream_ptr()


def add_rmsnorm(B: int, D: int, eps: float):
    """tilelang_kernels.py:34-55: out = rmsnorm(hidden + prefix) * weight."""

    def kernel(hidden, prefix, weight):
        _check(hidden, "hidden", (B, D))
        _check(prefix, "prefix", (B, D))
        _check(weight, "weight", (D,))
        out = torch.empty((B, D), dtype=torch.float32, device=hidden.device)
        _lib.call("skb_add_rmsnorm", hidden.data_ptr(), prefix.data_ptr(), weight.data_ptr(),
                  out.data_ptr(), B, D, float(eps), _stream())
        return out

    return kernel


def rmsnorm(B: int, D: int, eps: float):
    """tilelang_kernels.py:58-78: out = rmsnorm(x) * weight."""

    def kernel(x, weight):
        _check(x, "x", (B, D))
        _check(weight, "weight", (D,))
        out = torch.empty((B, D), dtype=torch.float32, device=x.device)
        _lib.call("skb_rmsnorm", x.data_ptr(), weight.data_ptr(), out.data_ptr(), B, D, float(eps),
                  _stream())
        return out

    return kernel


def swiglu_gemv(B: int, I: int, D: int, block_I: int = 128):  # noqa: E741 - reference name
    """tilelang_kernels.py:81-112: act = silu(x @ wg^T) * (x @ wu^T).

    ``block_I`` is accepted for signature compatibility; the sm_100a kernel
    chooses its own tiling."""

    def kernel(x, wg, wu):
        _check(x, "x", (B, D))
        _check(wg, "wg", (I, D))
        _check(wu, "wu", (I, D))
        out = torch.empty((B, I), dtype=torch.float32, device=x.device)
        _lib.call("skb_swiglu_gemv", x.data_ptr(), wg.data_ptr(), wu.data_ptr(), out.data_ptr(),
                  B, I, D, _stream())
        return out

    return kernel


def down_residual_gemv(B: int, D: int, I: int, block_D: int = 128):  # noqa: E741
    """tilelang_kernels.py:115-143: y = act @ wd^T + residual."""

    def kernel(act, wd, residual):
        _check(act, "act", (B, I))
        _check(wd, "wd", (D, I))
        _check(residual, "residual", (B, D))
        out = torch.empty((B, D), dtype=torch.float32, device=act.device)
        _lib.call("skb_down_residual_gemv", act.data_ptr(), wd.data_ptr(), residual.data_ptr(),
                  out.data_ptr(), B, D, I, _stream())
        return out

    return kernel


def classifier_gemv(B: int, V: int, D: int, block_V: int = 128):
    """tilelang_kernels.py:146-173: logits = body @ wq^T + bias."""

    def kernel(body, wq, bias):
        _check(body, "body", (B, D))
        _check(wq, "wq", (V, D))
        _check(bias, "bias", (V,))
        out = torch.empty((B, V), dtype=torch.float32, device=body.device)
        _lib.call("skb_classifier_gemv", body.data_ptr(), wq.data_ptr(), bias.data_ptr(),
                  out.data_ptr(), B, V, D, _stream())
        return out

    return kernel


def frame_embed(R: int, Q: int, V: int, D: int, scale: float, block_D: int = 256):
    """tilelang_kernels.py:176-196: out[r] = scale * sum_q table[q, codes[r, q]]."""

    def kernel(codes, table):
        _check(codes, "codes", (R, Q), torch.int64)
        _check(table, "table", (Q, V, D))
        out = torch.empty((R, D), dtype=torch.float32, device=table.device)
        _lib.call("skb_frame_embed", codes.data_ptr(), table.data_ptr(), out.data_ptr(), R, Q, V, D,
                  float(scale), _stream())
        return out

    return kernel


def prefix_add(B: int, V: int, D: int, scale: float, block_D: int = 256):
    """tilelang_kernels.py:199-216: out = prefix + table_q[code] * scale."""

    def kernel(prefix, table_q, codes):
        _check(prefix, "prefix", (B, D))
        _check(table_q, "table_q", (V, D))
        _check(codes, "codes", (1,), torch.int64)
        out = torch.empty((B, D), dtype=torch.float32, device=prefix.device)
        _lib.call("skb_prefix_add", prefix.data_ptr(), table_q.data_ptr(), codes.data_ptr(),
                  out.data_ptr(), B, V, D, float(scale), _stream())
        return out

    return kernel


def sampling_prep(V: int, bos_id: int, pad_id: int, eos_id: int, block_V: int = 256):
    """tilelang_kernels.py:219-254: logits / temperature with BOS/PAD (and EOS
    when mask_eos > 0) set to -1e30."""

    def kernel(logits, temperature, mask_eos):
        _check(logits, "logits", (V,))
        _check(temperature, "temperature", (1,))
        _check(mask_eos, "mask_eos", (1,), torch.int32)
        out = torch.empty((V,), dtype=torch.float32, device=logits.device)
        _lib.call("skb_sampling_prep", logits.data_ptr(), temperature.data_ptr(), mask_eos.data_ptr(),
                  out.data_ptr(), V, bos_id, pad_id, eos_id, _stream())
        return out

    return kernel


# ---------------------------------------------------------------- extensions
def pack_sample_params(rows) -> torch.Tensor:
    """Device array of skb_sample_params from dicts with keys cfg_scale,
    temperature, top_k, top_p, mask_eos, request, frame, q, seed."""
    arr = (_lib.skb_sample_params * len(rows))()
    for i, r in enumerate(rows):
        V = r.get("V", 1 << 30)
        k = r.get("top_k")
        p = r.get("top_p")
        arr[i] = _lib.skb_sample_params(
            float(r.get("cfg_scale", 1.0)), float(r["temperature"]),
            int(k) if k is not None and 0 < int(k) < V else 0,
            float(p) if p is not None and 0.0 < float(p) < 1.0 else -1.0,
            1 if r.get("mask_eos") else 0, int(r.get("request", 0)), int(r.get("frame", 0)),
            int(r.get("q", 0)), int(r.get("seed", 0)) & 0xFFFFFFFFFFFFFFFF)
    raw = bytes(memoryview(arr).cast("B"))
    host = torch.frombuffer(bytearray(raw), dtype=torch.uint8)
    return host.cuda()


def cfg_sample(logits: torch.Tensor, params: torch.Tensor, *, rows_per_req: int, bos_id: int,
               pad_id: int, eos_id: int, return_uniform: bool = False):
    """Fused CFG + masks + temperature + top-k + top-p + Philox draw (one CTA per
    request).  logits [n_req * rows_per_req, V]; params from pack_sample_params."""
    if logits.dim() != 2 or logits.dtype != torch.float32 or not logits.is_cuda or not logits.is_contiguous():
        raise ValueError("logits must be a contiguous CUDA float32 [rows, V] tensor")
    n_req = logits.shape[0] // rows_per_req
    if n_req * rows_per_req != logits.shape[0]:
        raise ValueError("rows not a multiple of rows_per_req")
    if params.numel() != n_req * _ctypes_size():
        raise ValueError("params do not match the number of requests")
    codes = torch.empty(n_req, dtype=torch.int64, device=logits.device)
    uni = torch.empty(n_req, dtype=torch.float32, device=logits.device)
    _lib.call("skb_cfg_sample", logits.data_ptr(), rows_per_req, n_req, logits.shape[1], params.data_ptr(),
              bos_id, pad_id, eos_id, codes.data_ptr(), uni.data_ptr(), _stream())
    return (codes, uni) if return_uniform else codes


def _ctypes_size() -> int:
    import ctypes

    return ctypes.sizeof(_lib.skb_sample_params)


def decode_attention(qkv: torch.Tensor, *, n_heads: int, n_kv_heads: int, q_norm: torch.Tensor,
                     k_norm: torch.Tensor, eps: float, rope_cos: torch.Tensor, rope_sin: torch.Tensor,
                     pos: torch.Tensor, kv_pool: torch.Tensor, page_table: torch.Tensor, page_size: int,
                     splits: int) -> torch.Tensor:
    """One Qwen3 decode-attention step over a paged FP32 KV cache (updated in
    place at ``pos``); see skb_decode_attention in include/soraku_b200.h."""
    rows = qkv.shape[0]
    hd = 128
    n_rep = n_heads // n_kv_heads
    for name, t in (("qkv", qkv), ("q_norm", q_norm), ("k_norm", k_norm), ("rope_cos", rope_cos),
                    ("rope_sin", rope_sin), ("kv_pool", kv_pool)):
        _check(t, name, tuple(t.shape))
    _check(pos, "pos", (rows,), torch.int32)
    _check(page_table, "page_table", tuple(page_table.shape), torch.int32)
    part = torch.empty(rows * n_kv_heads * splits * n_rep * (hd + 2), dtype=torch.float32, device=qkv.device)
    tickets = torch.zeros(rows * n_kv_heads, dtype=torch.int32, device=qkv.device)
    out = torch.empty((rows, n_heads * hd), dtype=torch.float32, device=qkv.device)
    n_pages = kv_pool.numel() // (2 * n_kv_heads * page_size * hd)
    _lib.call("skb_decode_attention", qkv.data_ptr(), rows, n_heads, n_kv_heads, hd, q_norm.data_ptr(),
              k_norm.data_ptr(), float(eps), rope_cos.data_ptr(), rope_sin.data_ptr(), rope_cos.shape[0],
              pos.data_ptr(), kv_pool.data_ptr(), page_table.data_ptr(), page_table.shape[1], page_size, n_pages,
              splits, part.data_ptr(), tickets.data_ptr(), out.data_ptr(), _stream())
    return out
