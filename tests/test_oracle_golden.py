"""Pin the CPU oracle against fixtures produced by the reference itself
(tests/golden/make_golden.py).  No GPU needed."""

from __future__ import annotations

import numpy as np
import pytest

from oracle import sampler as osamp
from tests._util import assert_close, load_golden, oracle_from_meta

TOL = dict(rtol=1e-4, atol=1e-4)  # logits and hidden states within rel/abs 1e-4


def _teacher(name):
    data, meta = load_golden(name)
    orc, dims, _ = oracle_from_meta(meta)
    speaker = data.get("speaker")
    out = orc.teacher_forced(input_ids=data["input_ids"][0], uncond_input_ids=data["uncond_input_ids"][0],
                             prompt_codes=data["prompt_codes"], codes=data["codes"],
                             cfg_scale=meta["cfg_scale"], record_q=data["record_q"].tolist(),
                             speaker=None if speaker is None else speaker[0])
    return data, meta, orc, out


@pytest.mark.parametrize("name", ["model_small", "model_route_d", "model_bos"])
def test_oracle_teacher_forced_small(name):
    data, meta, _, out = _teacher(name)
    assert_close(out["hidden"], data["hidden"], what=f"{name} hidden", **TOL)
    assert_close(out["logits"], data["logits"], what=f"{name} logits", **TOL)
    assert_close(out["hidden_after"], data["hidden_after"], what=f"{name} hidden_after", **TOL)


@pytest.mark.slow
def test_oracle_teacher_forced_full_model():
    """28 layers, text vocab 151936, config-1 prompt shape."""
    data, meta, _, out = _teacher("model_full")
    assert_close(out["hidden"], data["hidden"], what="full hidden", **TOL)
    assert_close(out["logits"], data["logits"], what="full logits", **TOL)


@pytest.mark.slow
def test_oracle_teacher_forced_full_route_d():
    """28 layers, route D (config 3): language ID, slot-mode speaker vector,
    text and reference lengths drawn from U[16, 96] and U[24, 144]."""
    data, meta, _, out = _teacher("model_route_d_full")
    assert_close(out["hidden"], data["hidden"], what="route-D full hidden", **TOL)
    assert_close(out["logits"], data["logits"], what="route-D full logits", **TOL)
    assert_close(out["hidden_after"], data["hidden_after"], what="route-D full hidden_after", **TOL)


def test_oracle_greedy_generate_matches_reference():
    data, meta = load_golden("model_small")
    orc, dims, _ = oracle_from_meta(meta)
    n = data["greedy_codes"].shape[0]
    codes, info = orc.generate(input_ids=data["input_ids"][0], prompt_codes=data["prompt_codes"],
                               max_new_frames=n, min_new_frames=n, temperature=0.0,
                               cfg_scale=meta["cfg_scale"], uncond_input_ids=data["uncond_input_ids"][0])
    np.testing.assert_array_equal(codes, data["greedy_codes"])
    assert info["stop_reason"] == "max_frames"


def _cases():
    data, meta = load_golden("sampler_cases")
    n = data["cond"].shape[0]
    return data, meta, n


def test_sampler_restatement_matches_reference_distribution():
    """The restatement's final distribution equals the reference's
    (``torch.multinomial``'s input) within FP32 rounding; greedy cases return
    the reference's argmax.  Where the logits hold ties at the top-p boundary
    (every 11th case), torch.sort orders equal values arbitrarily, so there the
    sorted probability multiset is compared instead of per-index values."""
    data, meta, n = _cases()
    V, bos, eos, pad = meta["V"], meta["bos"], meta["eos"], meta["pad"]
    checked = 0
    for i in range(n):
        cfg = float(data["cfg"][i])
        un = None if cfg == 1.0 else data["uncond"][i]
        kw = dict(cfg=cfg, temperature=float(data["temp"][i]),
                  top_k=None if data["top_k"][i] < 0 else int(data["top_k"][i]),
                  top_p=None if data["top_p"][i] < 0 else float(data["top_p"][i]),
                  mask_eos=bool(data["mask_eos"][i]), bos=bos, pad=pad, eos=eos)
        if kw["temperature"] <= 0:
            assert osamp.sample(data["cond"][i], un, u=0.5, **kw) == int(data["code"][i])
            continue
        keep, p = osamp.kept_set(data["cond"][i], un, **kw)
        mine = np.zeros(V)
        mine[keep] = p
        ref = data["probs"][i].astype(np.float64)
        if i % 11 == 0:
            np.testing.assert_allclose(np.sort(mine)[::-1], np.sort(ref)[::-1], rtol=2e-6, atol=1e-7,
                                       err_msg=f"case {i}")
        else:
            np.testing.assert_allclose(mine, ref, rtol=2e-6, atol=1e-7, err_msg=f"case {i}")
            big = ref > 1e-6
            assert set(np.nonzero(big)[0]) <= set(keep), f"case {i}"
        checked += 1
    assert checked > 30


def test_sampler_draw_follows_inverse_cdf():
    """Draws over a grid of uniforms land on kept codes with the expected frequencies."""
    data, meta, n = _cases()
    i = 0
    cfg = float(data["cfg"][i])
    kw = dict(cfg=cfg, temperature=float(data["temp"][i]), top_k=int(data["top_k"][i]),
              top_p=float(data["top_p"][i]), mask_eos=True, bos=meta["bos"], pad=meta["pad"],
              eos=meta["eos"])
    un = None if cfg == 1.0 else data["uncond"][i]
    keep, p = osamp.kept_set(data["cond"][i], un, **kw)
    grid = (np.arange(4096) + 0.5) / 4096
    draws = [osamp.sample(data["cond"][i], un, u=float(u), **kw) for u in grid]
    freq = np.array([draws.count(k) for k in keep]) / len(grid)
    assert set(draws) <= set(keep)
    np.testing.assert_allclose(freq, p, atol=2.0 / 4096 + 1e-9)


def test_philox_known_answers():
    """Random123 philox4x32-10 known-answer vectors."""
    assert osamp.philox4x32_10([0, 0, 0, 0], [0, 0]) == [0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8]
    assert osamp.philox4x32_10([0xFFFFFFFF] * 4, [0xFFFFFFFF] * 2) == [
        0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD]
    assert osamp.philox4x32_10([0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344],
                               [0xA4093822, 0x299F31D0]) == [0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1]


def test_exp_accuracy():
    import math

    xs = np.linspace(-87.0, 0.0, 20001, dtype=np.float32)
    worst = 0.0
    for x in xs:
        ref = math.exp(float(x))
        worst = max(worst, abs(osamp.exp(float(x)) - ref) / ref)
    assert worst < 2.0 ** -22
    assert osamp.exp(float("-inf")) == 0.0
    assert osamp.exp(-200.0) == 0.0
    assert osamp.exp(0.0) == 1.0
