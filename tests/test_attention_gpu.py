"""The decode-attention op (skb_decode_attention) against the oracle's numpy
restatement of the Qwen3 attention step: q/k RMSNorm, neox RoPE, KV append at
the row's position, GQA softmax attention -- within rel/abs 1e-4, on a paged
cache whose page table is a permutation, for several split counts (including
more splits than positions), with 2 rows and with 10 ragged rows."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle.model_np import apply_rope, rmsnorm, rope_tables

pytestmark = pytest.mark.gpu
H, KVH, HD, P = 16, 8, 128, 64


def make_case(lengths, max_len=512, seed=0):
    g = np.random.default_rng(seed)
    rows = len(lengths)
    max_pages = max_len // P
    n_pages = rows * max_pages + 3
    perm = g.permutation(n_pages)[: rows * max_pages].reshape(rows, max_pages).astype(np.int32)
    pool = g.standard_normal((n_pages, 2, KVH, P, HD)).astype(np.float32)
    qkv = g.standard_normal((rows, (H + 2 * KVH) * HD)).astype(np.float32)
    qn = (1 + 0.1 * g.standard_normal(HD)).astype(np.float32)
    kn = (1 + 0.1 * g.standard_normal(HD)).astype(np.float32)
    inv = (1.0 / (1e6 ** (np.arange(0, HD, 2, dtype=np.int64).astype(np.float32) / HD))).astype(np.float32)
    cos, sin = rope_tables(inv, np.arange(max_len))
    return dict(rows=rows, pos=np.array(lengths, np.int32), perm=perm, pool=pool, qkv=qkv, qn=qn, kn=kn,
                cos=np.ascontiguousarray(cos[:, : HD // 2]), sin=np.ascontiguousarray(sin[:, : HD // 2]),
                cos_full=cos, sin_full=sin, max_len=max_len)


def oracle(c):
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
                                   kv_pool=pool, page_table=t(c["perm"]), page_size=P, splits=splits)
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


def test_decode_attention_rejects_bad_shapes():
    from soraku_tts_b200 import _lib

    with pytest.raises(ValueError):
        _lib.call("skb_decode_attention", 1, 1, 16, 8, 64, 1, 1, 1e-6, 1, 1, 8, 1, 1, 1, 1, 64, 1, 1, 1, 1, 1, None)
