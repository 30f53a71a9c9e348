"""The fused sampler on the GPU against the C restatement in the oracle:
identical code for identical logits and uniforms (bit-exact), Philox and exp
identical to the oracle's."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import sampler as osamp
from tests._util import load_golden

pytestmark = pytest.mark.gpu
V, BOS, EOS, PAD = 2051, 2048, 2049, 2050


@pytest.fixture(scope="module")
def lib():
    from soraku_tts_b200 import _lib

    return _lib


def test_exp_bit_exact_with_oracle(lib):
    xs = np.concatenate([np.linspace(-110, 0, 50001, dtype=np.float32),
                         -np.abs(np.random.default_rng(1).standard_normal(20000).astype(np.float32)) * 30,
                         np.array([0.0, -0.0, -np.inf, -1e-30, -87.33655, -103.9, -104.0], dtype=np.float32)])
    x = torch.from_numpy(xs).cuda()
    y = torch.empty_like(x)
    lib.call("skb_test_exp", x.data_ptr(), y.data_ptr(), x.numel(), lib.stream_ptr())
    got = y.cpu().numpy()
    want = np.array([osamp.exp(float(v)) for v in xs], dtype=np.float32)
    np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))
    # and within 2 ulp of CUDA's own expf where the result is normal
    ref = torch.exp(x).cpu().numpy()
    normal = ref > 1.2e-38
    ulp = np.abs(got[normal].view(np.int32).astype(np.int64) - ref[normal].view(np.int32).astype(np.int64))
    assert ulp.max() <= 2


def test_philox_known_answers_on_device(lib):
    ck = np.array([[0, 0, 0, 0, 0, 0],
                   [0xFFFFFFFF] * 6,
                   [0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344, 0xA4093822, 0x299F31D0]], dtype=np.uint32)
    inp = torch.from_numpy(ck.view(np.int32)).cuda()
    out = torch.empty((3, 4), dtype=torch.int32, device="cuda")
    lib.call("skb_test_philox", inp.data_ptr(), out.data_ptr(), 3, lib.stream_ptr())
    got = out.cpu().numpy().view(np.uint32).tolist()
    assert got == [[0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8],
                   [0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD],
                   [0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1]]


def _run_cases(cases):
    """cases: list of dict(cond, uncond|None, cfg, temperature, top_k, top_p, mask_eos, seed, request,
    frame, q).  Returns (gpu codes, gpu uniforms)."""
    from soraku_tts_b200 import kernels

    out_codes, out_u = [], []
    for rows_per_req in (1, 2):
        group = [c for c in cases if (c["uncond"] is not None) == (rows_per_req == 2)]
        if not group:
            continue
        logits = []
        for c in group:
            logits.append(c["cond"])
            if rows_per_req == 2:
                logits.append(c["uncond"])
        lg = torch.from_numpy(np.stack(logits).astype(np.float32)).cuda()
        params = kernels.pack_sample_params([dict(c, cfg_scale=c["cfg"], V=V) for c in group])
        codes, uni = kernels.cfg_sample(lg, params, rows_per_req=rows_per_req, bos_id=BOS, pad_id=PAD,
                                        eos_id=EOS, return_uniform=True)
        for c, code, u in zip(group, codes.cpu().tolist(), uni.cpu().tolist()):
            c["gpu_code"], c["gpu_u"] = code, u
    for c in cases:
        out_codes.append(c["gpu_code"])
        out_u.append(c["gpu_u"])
    return out_codes, out_u


def _oracle(c, u):
    return osamp.sample(c["cond"], c["uncond"], cfg=c["cfg"], temperature=c["temperature"], top_k=c["top_k"],
                        top_p=c["top_p"], mask_eos=c["mask_eos"], bos=BOS, pad=PAD, eos=EOS, u=u)


def _random_cases(n, seed):
    g = np.random.default_rng(seed)
    cases = []
    for i in range(n):
        sigma = [0.3, 1.0, 3.0, 8.0][i % 4]
        cond = (g.standard_normal(V) * sigma).astype(np.float32)
        un = (cond * 0.6 + g.standard_normal(V) * sigma * 0.5).astype(np.float32)
        if i % 7 == 0:
            cond = np.round(cond * 2) / 2  # ties
            un = np.round(un * 2) / 2
        cases.append(dict(
            cond=cond.astype(np.float32), uncond=None if i % 5 == 4 else un.astype(np.float32),
            cfg=[1.5, 2.0, 0.7][i % 3], temperature=[0.9, 0.5, 1.3, 0.0, 2.0][(i // 3) % 5],
            top_k=[50, 1, None, 2051, 7, 3000][(i // 2) % 6], top_p=[0.95, 0.5, None, 1.0, 0.99][(i // 4) % 5],
            mask_eos=bool(i % 2), seed=1000 + i, request=i % 3, frame=i, q=i % 16))
    return cases


def test_fused_sampler_bit_exact_random(lib):
    cases = _random_cases(240, 99)
    codes, us = _run_cases(cases)
    for i, (c, code, u) in enumerate(zip(cases, codes, us)):
        u_ref = osamp.uniform(c["seed"], c["request"], c["frame"], c["q"])
        assert np.float32(u).view(np.uint32) == np.float32(u_ref).view(np.uint32), f"case {i}: uniform"
        assert code == _oracle(c, u_ref), f"case {i}: code {code} != oracle"


def test_fused_sampler_edge_uniforms(lib):
    """Seeds chosen so that the Philox uniform lands near 0 and near 1."""
    g = np.random.default_rng(5)
    cases = []
    lo = hi = None
    for seed in range(20000):
        u = osamp.uniform(seed, 0, 0, 0)
        if lo is None or u < lo[1]:
            lo = (seed, u)
        if hi is None or u > hi[1]:
            hi = (seed, u)
    for seed, _ in (lo, hi):
        for top_k, top_p in ((50, 0.95), (None, None), (1, None), (2051, 0.3)):
            cond = (g.standard_normal(V) * 2).astype(np.float32)
            cases.append(dict(cond=cond, uncond=None, cfg=1.0, temperature=0.9, top_k=top_k, top_p=top_p,
                              mask_eos=True, seed=seed, request=0, frame=0, q=0))
    codes, _ = _run_cases(cases)
    for c, code in zip(cases, codes):
        assert code == _oracle(c, osamp.uniform(c["seed"], 0, 0, 0))


def test_fused_sampler_on_reference_cases(lib):
    """The golden cases' logits (produced by the reference's CFG/mask lines)."""
    data, meta = load_golden("sampler_cases")
    cases = []
    for i in range(data["cond"].shape[0]):
        cfg = float(data["cfg"][i])
        cases.append(dict(cond=data["cond"][i], uncond=None if cfg == 1.0 else data["uncond"][i], cfg=cfg,
                          temperature=float(data["temp"][i]),
                          top_k=None if data["top_k"][i] < 0 else int(data["top_k"][i]),
                          top_p=None if data["top_p"][i] < 0 else float(data["top_p"][i]),
                          mask_eos=bool(data["mask_eos"][i]), seed=7 + i, request=0, frame=i, q=0))
    codes, _ = _run_cases(cases)
    for i, (c, code) in enumerate(zip(cases, codes)):
        assert code == _oracle(c, osamp.uniform(c["seed"], 0, c["frame"], 0)), f"case {i}"
        if c["temperature"] <= 0:
            assert code == int(data["code"][i])  # the reference's own argmax
        else:
            assert data["probs"][i][code] > 0  # drawn from the reference's support


def test_fused_sampler_rejects_bad_arguments(lib):
    from soraku_tts_b200 import kernels

    lg = torch.zeros((3, V), device="cuda")
    params = kernels.pack_sample_params([dict(temperature=1.0)])
    with pytest.raises(ValueError):
        kernels.cfg_sample(lg, params, rows_per_req=2, bos_id=BOS, pad_id=PAD, eos_id=EOS)


def _bin_edge_tie_case():
    """top-k whose k-th largest logit sits on a lower edge of the sampler's
    histogram bins (1.0) with ten logits one float below it: at this
    temperature those ten divide to the same f as the cutoff, so the top-k
    set (ties kept) holds 15 entries, 10 of them from the bin below."""
    t = np.float32(0.30051)
    edge = np.float32(1.0)
    below = np.nextafter(edge, np.float32(0))
    assert np.float32(edge / t) == np.float32(below / t)
    g = np.random.default_rng(11)
    cond = (g.standard_normal(V) * 0.2 - 3.0).astype(np.float32)
    idx = g.permutation(np.arange(10, V - 10))[:15]
    cond[idx[:4]] = np.array([1.2, 1.15, 1.1, 1.05], np.float32)
    cond[idx[4]] = edge
    cond[idx[5:]] = below
    return cond, float(t)


def test_topk_tie_at_histogram_bin_edge():
    cond, t = _bin_edge_tie_case()
    _, info = osamp.sample(cond, None, cfg=1.0, temperature=t, top_k=5, top_p=None, mask_eos=True, bos=BOS,
                           pad=PAD, eos=EOS, u=0.5, return_info=True)
    assert info["n_kept"] == 15  # the oracle keeps the ties below the bin edge
    cases = [dict(cond=cond, uncond=None, cfg=1.0, temperature=t, top_k=5, top_p=None, mask_eos=True, seed=s,
                  request=0, frame=0, q=0) for s in range(48)]
    codes, _ = _run_cases(cases)
    picked_below = 0
    for c, code in zip(cases, codes):
        want = _oracle(c, osamp.uniform(c["seed"], 0, 0, 0))
        assert code == want
        picked_below += cond[code] < 1.0
    assert picked_below > 0  # the draw reached the tied entries
