"""The decode-attention op (skb_decode_attention) against the oracle's numpy
restatement of the Qwen3 attention step: q/k RMSNorm, neox RoPE, KV append at
the row's position, GQA softmax attention -- within rel/abs 1e-4, on a paged
cache whose page table is a permutation, for several split counts (including
more splits than positions), with 2 rows and with 10 ragged rows, on pages of
16 positions, and on 300 ragged rows."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle.model_np import apply_rope, rmsnorm, rope_tables

pytestmark = pytest.mark.gpu
H, KVH, HD, P = 16, 8, 128, 64


def make_case(lengths, max_len=512, seed=0, page=P):
    g = np.random.default_rng(seed)
    rows = len(lengths)
    max_pages = max_len // page
    n_pages = rows * max_pages + 3
    perm = g.permutation(n_pages)[: rows * max_pages].reshape(rows, max_pages).astype(np.int32)
    pool = g.standard_normal((n_pages, 2, KVH, page, HD)).astype(np.float32)
    qkv = g.standard_normal((rows, (H + 2 * KVH) * HD)).astype(np.float32)
    qn = (1 + 0.1 * g.standard_normal(HD)).astype(np.float32)
    kn = (1 + 0.1 * g.standard_normal(HD)).astype(np.float32)
    inv = (1.0 / (1e6 ** (np.arange(0, HD, 2, dtype=np.int64).astype(np.float32) / HD))).astype(np.float32)
    cos, sin = rope_tables(inv, np.arange(max_len))
    return dict(rows=rows, pos=np.array(lengths, np.int32), perm=perm, pool=pool, qkv=qkv, qn=qn, kn=kn,
                cos=np.ascontiguousarray(cos[:, : HD // 2]), sin=np.ascontiguousarray(sin[:, : HD // 2]),
                cos_full=cos, sin_full=sin, max_len=max_len, P=page)


def oracle(c):
    P = c["P"]
    outs, newk, newv = [], [], []
    for r in range(c["rows"]):
        p = int(c["pos"][r])
        q = rmsnorm(c["qkv"][r, : H * HD].reshape(H, 1, HD), c["qn"], 1e-6)
        k = rmsnorm(c["qkv"][r, H * HD:(H + KVH) * HD].reshape(KVH, 1, HD), c["kn"], 1e-6)
        v = c["qkv"][r, (H + KVH) * HD:].reshape(KVH, 1, HD)
        cs, sn = c["cos_full"][p:p + 1], c["sin_full"][p:p + 1]
        q, k = apply_rope(q, cs, sn), apply_rope(k, cs, sn)
        K = np.stack([c["pool"][c["perm"][r, t // P], 0, :, t % P] for t in range(p)], 1) if p else np.zeros((KVH, 0, HD), np.float32)
        V = np.stack([c["pool"][c["perm"][r, t // P], 1, :, t % P] for t in range(p)], 1) if p else np.zeros((KVH, 0, HD), np.float32)
        K = np.concatenate([K, k], 1).astype(np.float64)
        V = np.concatenate([V, v], 1).astype(np.float64)
        o = []
        for h in range(H):
            s = (q[h, 0].astype(np.float64) @ K[h // (H // KVH)].T) / np.sqrt(HD)
            w = np.exp(s - s.max())
            o.append((w / w.sum()) @ V[h // (H // KVH)])
        outs.append(np.concatenate(o))
        newk.append(k[:, 0])
        newv.append(v[:, 0])
    return np.stack(outs), np.stack(newk), np.stack(newv)


def run(c, splits):
    from soraku_tts_b200 import kernels

    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    pool = t(c["pool"])
    out = kernels.decode_attention(t(c["qkv"]), n_heads=H, n_kv_heads=KVH, q_norm=t(c["qn"]), k_norm=t(c["kn"]),
                                   eps=1e-6, rope_cos=t(c["cos"]), rope_sin=t(c["sin"]), pos=t(c["pos"]),
                                   kv_pool=pool, page_table=t(c["perm"]), page_size=c["P"], splits=splits)
    return out.cpu().numpy(), pool.cpu().numpy()


@pytest.mark.parametrize("lengths", [[37, 300], [0, 5], [511, 63]])
@pytest.mark.parametrize("splits", [1, 3, 8, 9, 40])
def test_decode_attention_matches_oracle(lengths, splits):
    c = make_case(lengths, seed=sum(lengths) + splits)
    got, pool = run(c, splits)
    want, k_new, v_new = oracle(c)
    np.testing.assert_allclose(got, want, rtol=1e-4, atol=1e-4)
    for r, p in enumerate(c["pos"]):
        page = c["perm"][r, p // P]
        np.testing.assert_allclose(pool[page, 0, :, p % P], k_new[r], rtol=1e-5, atol=1e-6)
        np.testing.assert_allclose(pool[page, 1, :, p % P], v_new[r], rtol=0, atol=0)


# More than 4 rows (> 32 (row, kv head) groups) take the double-buffered
# variant (rounds of 48 positions): lengths around the round edges, a row
# with no cached position, and rows long enough for several rounds per CTA.
@pytest.mark.parametrize("splits", [1, 2, 8])
def test_decode_attention_many_rows_double_buffered(splits):
    lengths = [0, 1, 47, 48, 49, 96, 97, 300, 511, 144]
    c = make_case(lengths, seed=11 + splits)
    got, pool = run(c, splits)
    want, k_new, v_new = oracle(c)
    np.testing.assert_allclose(got, want, rtol=1e-4, atol=1e-4)
    for r, p in enumerate(c["pos"]):
        page = c["perm"][r, p // P]
        np.testing.assert_allclose(pool[page, 1, :, p % P], v_new[r], rtol=0, atol=0)


def _check(c, got, pool):
    want, k_new, v_new = oracle(c)
    np.testing.assert_allclose(got, want, rtol=1e-4, atol=1e-4)
    P = c["P"]
    for r, p in enumerate(c["pos"]):
        page = c["perm"][r, p // P]
        np.testing.assert_allclose(pool[page, 0, :, p % P], k_new[r], rtol=1e-5, atol=1e-6)
        np.testing.assert_allclose(pool[page, 1, :, p % P], v_new[r], rtol=0, atol=0)


# Pages of 16 positions (several copies of K and of V per round), lengths on
# and around the page and round edges, single- and double-buffered variants.
@pytest.mark.parametrize("splits", [1, 2, 9])
def test_decode_attention_small_pages(splits):
    lengths = [0, 1, 15, 16, 17, 47, 48, 49, 63, 64, 65, 111, 112, 113, 255, 400, 511]
    c = make_case(lengths, seed=5 + splits, page=16)
    _check(c, *run(c, splits))
    c = make_case(lengths[:4], seed=6 + splits, page=16)
    _check(c, *run(c, splits))


# 300 ragged rows: 2400 (row, kv head) groups, several waves of clusters.
@pytest.mark.parametrize("splits", [1, 2])
def test_decode_attention_many_ragged_rows(splits):
    g = np.random.default_rng(77)
    lengths = [int(x) for x in g.integers(0, 512, 300)]
    c = make_case(lengths, seed=78 + splits)
    _check(c, *run(c, splits))


def test_decode_attention_rejects_bad_shapes():
    from soraku_tts_b200 import _lib

    with pytest.raises(ValueError):
        _lib.call("skb_decode_attention", 1, 1, 16, 8, 64, 1, 1, 1e-6, 1, 1, 8, 1, 1, 1, 1, 64, 1, 1, 1, 1, 1, None)


# The kernels read qkv, the norm weights, the RoPE tables and the cache with
# 16-byte loads and bulk copies: a pointer off a 16-byte boundary is refused
# before anything is launched.
def test_decode_attention_rejects_misaligned_pointers():
    from soraku_tts_b200 import _lib

    c = make_case([5, 9], seed=3)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    qkv, qn, kn, cs, sn, pos, pt, pool = (t(c[k]) for k in ("qkv", "qn", "kn", "cos", "sin", "pos", "perm", "pool"))
    part = torch.empty(2 * KVH * 2 * (HD + 2), device="cuda")
    tickets = torch.zeros(2 * KVH, dtype=torch.int32, device="cuda")
    out = torch.empty((2, H * HD), device="cuda")
    ptrs = dict(qkv=qkv.data_ptr(), qn=qn.data_ptr(), kn=kn.data_ptr(), cos=cs.data_ptr(), sin=sn.data_ptr(),
                pool=pool.data_ptr())
    for name in ptrs:
        p = dict(ptrs)
        p[name] += 4
        st = _lib.lib().skb_decode_attention(p["qkv"], 2, H, KVH, HD, p["qn"], p["kn"], 1e-6, p["cos"], p["sin"],
                                             c["max_len"], pos.data_ptr(), p["pool"], pt.data_ptr(),
                                             c["perm"].shape[1], P, pool.shape[0], 1, part.data_ptr(),
                                             tickets.data_ptr(), out.data_ptr(), None)
        assert st == _lib.SKB_ERR_ARG, name
        assert "aligned" in _lib.last_error(), name
