"""skb_decode_attention_noalloc against skb_decode_attention.

The no-alloc entry point serves callers that cannot allocate device memory
while decoding: a streaming or audio thread that cannot take the device-wide
stall an allocation may cause, or a host application that owns all device
memory through its own allocator.  It keeps its scratch in a library-owned
device array instead of caller buffers.  This test calls both entry points
through the C ABI on identical inputs, twice in a row (the second call
continues decoding on the caches the first one updated), and requires the
same attention output and the same cache updates within the tolerance the
other attention tests use (rel/abs 1e-4).  It passes alone in a fresh process
as well as after the rest of the suite."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
H, KVH, HD, P = 16, 8, 128, 64
TOL = dict(rtol=1e-4, atol=1e-4)


def _case(seed):
    g = np.random.default_rng(seed)
    rows, max_len = 2, 512
    max_pages = max_len // P
    n_pages = rows * max_pages
    table = g.permutation(n_pages).reshape(rows, max_pages).astype(np.int32)
    pool = g.standard_normal((n_pages, 2, KVH, P, HD)).astype(np.float32)
    qn = (1 + 0.1 * g.standard_normal(HD)).astype(np.float32)
    kn = (1 + 0.1 * g.standard_normal(HD)).astype(np.float32)
    inv = (1.0 / (1e6 ** (np.arange(0, HD, 2, dtype=np.int64).astype(np.float32) / HD))).astype(np.float32)
    ang = (np.arange(max_len, dtype=np.float32)[:, None] * inv[None, :]).astype(np.float32)
    cos = np.cos(ang.astype(np.float64)).astype(np.float32)
    sin = np.sin(ang.astype(np.float64)).astype(np.float32)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    return dict(rows=rows, max_len=max_len, max_pages=max_pages, n_pages=n_pages, table=t(table), pool=t(pool),
                qn=t(qn), kn=t(kn), cos=t(cos), sin=t(sin), g=g)


def _call(lib, name, c, qkv, pos, pool, splits, out, scratch=None):
    stream = torch.cuda.current_stream().cuda_stream
    head = [qkv.data_ptr(), c["rows"], H, KVH, HD, c["qn"].data_ptr(), c["kn"].data_ptr(), ctypes.c_float(1e-6),
            c["cos"].data_ptr(), c["sin"].data_ptr(), c["max_len"], pos.data_ptr(), pool.data_ptr(),
            c["table"].data_ptr(), c["max_pages"], P, c["n_pages"], splits]
    if scratch is None:
        status = getattr(lib.lib(), name)(*head, out.data_ptr(), stream)
    else:
        part, tickets = scratch
        status = getattr(lib.lib(), name)(*head, part.data_ptr(), tickets.data_ptr(), out.data_ptr(), stream)
    lib.check(status, name)


def test_noalloc_matches_allocating_entry_point_twice():
    from soraku_tts_b200 import _lib

    c = _case(11)
    splits = 18
    part = torch.empty(c["rows"] * KVH * splits * (H // KVH) * (HD + 2), dtype=torch.float32, device="cuda")
    tickets = torch.zeros(c["rows"] * KVH, dtype=torch.int32, device="cuda")
    pool_a = c["pool"].clone()
    pool_b = c["pool"].clone()
    pos = torch.tensor([200, 73], dtype=torch.int32, device="cuda")
    for call in range(2):
        qkv = torch.from_numpy(c["g"].standard_normal((c["rows"], (H + 2 * KVH) * HD)).astype(np.float32)).cuda()
        out_a = torch.empty((c["rows"], H * HD), device="cuda")
        out_b = torch.full((c["rows"], H * HD), float("nan"), device="cuda")
        _call(_lib, "skb_decode_attention", c, qkv, pos, pool_a, splits, out_a, scratch=(part, tickets))
        _call(_lib, "skb_decode_attention_noalloc", c, qkv, pos, pool_b, splits, out_b)
        torch.cuda.synchronize()
        np.testing.assert_allclose(out_b.cpu().numpy(), out_a.cpu().numpy(), err_msg=f"call {call}", **TOL)
        np.testing.assert_allclose(pool_b.cpu().numpy(), pool_a.cpu().numpy(), err_msg=f"call {call}", **TOL)
        pos += 1


def test_noalloc_rejects_sizes_beyond_its_scratch():
    from soraku_tts_b200 import _lib

    st = _lib.lib().skb_decode_attention_noalloc(1, 64, H, KVH, HD, 1, 1, ctypes.c_float(1e-6), 1, 1, 512, 1, 1, 1,
                                                 8, P, 16, 64, 1, None)
    assert st == _lib.SKB_ERR_ARG
    assert "scratch" in _lib.last_error()


def test_noalloc_at_its_exact_partials_limit():
    """2 rows x 8 kv heads x 2 heads per group x 130 floats: 126 splits need
    2,096,640 bytes of partials (the largest count within the 2 MiB array) and
    must match the allocating entry point; 127 splits (2,113,280 bytes) must be
    refused."""
    from soraku_tts_b200 import _lib

    c = _case(12)
    pos = torch.tensor([300, 129], dtype=torch.int32, device="cuda")
    qkv = torch.from_numpy(c["g"].standard_normal((c["rows"], (H + 2 * KVH) * HD)).astype(np.float32)).cuda()
    splits = 126
    assert c["rows"] * KVH * splits * (H // KVH) * (HD + 2) * 4 <= 2 * 1024 * 1024
    part = torch.empty(c["rows"] * KVH * splits * (H // KVH) * (HD + 2), dtype=torch.float32, device="cuda")
    tickets = torch.zeros(c["rows"] * KVH, dtype=torch.int32, device="cuda")
    pool_a, pool_b = c["pool"].clone(), c["pool"].clone()
    out_a = torch.empty((c["rows"], H * HD), device="cuda")
    out_b = torch.full((c["rows"], H * HD), float("nan"), device="cuda")
    _call(_lib, "skb_decode_attention", c, qkv, pos, pool_a, splits, out_a, scratch=(part, tickets))
    _call(_lib, "skb_decode_attention_noalloc", c, qkv, pos, pool_b, splits, out_b)
    torch.cuda.synchronize()
    np.testing.assert_allclose(out_b.cpu().numpy(), out_a.cpu().numpy(), **TOL)
    np.testing.assert_allclose(pool_b.cpu().numpy(), pool_a.cpu().numpy(), **TOL)
    with pytest.raises(ValueError, match="scratch"):  # SKB_ERR_ARG
        _call(_lib, "skb_decode_attention_noalloc", c, qkv, pos, pool_b, splits + 1, out_b)
