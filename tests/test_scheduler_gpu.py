"""Continuous batching on the GPU: 7 ragged requests (different prompt
lengths, frame budgets, seeds, EOS allowed for some) through 3 slots with
2 frames per graph replay -- requests join as slots free up, finished slots
are compacted by moving a running request's state (codes, residual stream,
positions, KV pages by page-table exchange) -- must give every request
exactly the codes it gets in a static batch of all 7 requests decoded
together (bit-exact: one random stream per request, the tensor-core GEMM
path and one attention variant at every batch width)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import sampler as osamp
from tests._util import load_golden, oracle_from_meta

pytestmark = pytest.mark.gpu
EOS = 2049


@pytest.fixture(scope="module")
def small():
    from soraku_tts_b200.model import SorakuModel

    data, meta = load_golden("model_small")
    orc, dims, sd = oracle_from_meta(meta)
    return data, SorakuModel(dims, sd, "cuda"), orc


def _requests(data):
    ids, unc, pc = data["input_ids"][0], data["uncond_input_ids"][0], data["prompt_codes"]
    budgets = [5, 9, 2, 7, 1, 4, 8]
    mins = [10 ** 6, 0, 10 ** 6, 2, 10 ** 6, 0, 10 ** 6]
    reqs = []
    for i, (m, mn) in enumerate(zip(budgets, mins)):
        L = max(2, ids.shape[-1] - 3 * i)
        R = max(1, pc.shape[0] - 2 * i)
        reqs.append(dict(rid=i, input_ids=np.asarray(ids).reshape(1, -1)[:, :L], uncond_ids=np.asarray(unc).reshape(1, -1),
                         prompt_codes=np.asarray(pc)[:R], max_new_frames=m, min_new_frames=mn, seed=300 + i))
    return reqs


def _static(model, reqs):
    from soraku_tts_b200.graph_frame import NativeEngine

    n = len(reqs)
    frames = max(r["max_new_frames"] for r in reqs)
    eng = NativeEngine(model, max_requests=n, rows_per_request=2, max_len=512, max_frames=64, max_prefill=512,
                       gemm_min_rows=1, attn_splits=1)
    for j, r in enumerate(reqs):
        eng.set_sampling(j, cfg=1.5, temperature=0.9, temperature_q0=0.9, top_k=50, top_p=0.95, top_k_q0=50,
                         top_p_q0=0.95, seed=r["seed"], min_new_frames=r["min_new_frames"], eos_rule=1)
        eng.set_rng_stream(j, 0)
        eng.prefill(j, r["input_ids"], r["uncond_ids"], r["prompt_codes"])
    eng.capture(n, 1)
    for _ in range(frames):
        eng.step(True)
    out = {}
    for j, r in enumerate(reqs):
        c = eng.read_codes(j, 0, frames).clone().numpy()
        end = r["max_new_frames"]
        for f in range(end):
            if f >= r["min_new_frames"] and int(c[f, 0]) == EOS:
                end = f
                break
        out[r["rid"]] = c[:end]
    err = eng.view(6, torch.int32).cpu().numpy()
    assert (err == 0).all(), f"device error flags raised: {err}"
    eng.close()
    return out


@pytest.mark.parametrize("kv_pages", [None, 9])
def test_continuous_batching_equals_static_batch(small, kv_pages):
    """kv_pages 9: a shared KV pool of 9 pages of 16 positions (a request
    needs 3-4), so admission also waits for free pages."""
    from soraku_tts_b200.scheduler import ContinuousBatcher, DecodeRequest

    data, model, _ = small
    reqs = _requests(data)
    want = _static(model, reqs)
    streamed = {}
    b = ContinuousBatcher(model, slots=3, max_len=512, max_frames=64, frames_per_graph=2, kv_pages=kv_pages,
                          page_size=16 if kv_pages else 64)
    for r in reqs:
        b.submit(DecodeRequest(**r, on_frame=lambda rid, c: streamed.setdefault(rid, []).append(c)))
    got = b.run()
    err = b.engine.view(6, torch.int32).cpu().numpy()
    assert (err == 0).all(), f"device error flags raised: {err}"
    assert b.stats["moves"] > 0 and b.stats["admitted"] == len(reqs)
    for r in reqs:
        np.testing.assert_array_equal(got[r["rid"]], want[r["rid"]], err_msg=f"request {r['rid']}")
        if len(want[r["rid"]]):
            np.testing.assert_array_equal(np.stack(streamed[r["rid"]]), want[r["rid"]])
    if kv_pages:
        assert b.pool.available() == kv_pages
    b.close()


def test_continuous_batching_matches_oracle(small):
    """Every request of a continuous run (joins, leaves, slot moves) against the
    oracle teacher-forced on that request's own codes: each emitted code is the
    oracle sampler's draw from the oracle's logits with the request's Philox
    uniform (stream 0, its own seed); a code may differ only where the oracle's
    draw flips under a shift of the uniform by 1e-4 (logits agree within
    rel/abs 1e-4, so a draw that close to a CDF boundary may go either way), and
    no more than 1 % of draws may sit that close.  A request that stopped on EOS
    must be one whose next q0 draw is EOS in the oracle."""
    from soraku_tts_b200.scheduler import ContinuousBatcher, DecodeRequest

    data, model, orc = small
    reqs = _requests(data)
    b = ContinuousBatcher(model, slots=3, max_len=512, max_frames=64, frames_per_graph=2)
    for r in reqs:
        b.submit(DecodeRequest(**r))
    got = b.run()
    assert b.stats["moves"] > 0
    near = total = 0
    for r in reqs:
        codes = got[r["rid"]]
        stopped_eos = b.stop_reason[r["rid"]] == "eos"
        n = codes.shape[0]
        check = np.concatenate([codes, np.zeros((1, 16), np.int64)]) if stopped_eos else codes
        if check.shape[0] == 0:
            continue
        tf = orc.teacher_forced(input_ids=r["input_ids"][0], uncond_input_ids=r["uncond_ids"][0],
                                prompt_codes=r["prompt_codes"], codes=check, cfg_scale=1.5)
        for f in range(check.shape[0]):
            for q in range(16 if f < n else 1):
                c, u = tf["logits"][f, q, 0], tf["logits"][f, q, 1]
                kw = dict(cfg=1.5, temperature=0.9, top_k=50, top_p=0.95,
                          mask_eos=(q != 0 or f < r["min_new_frames"]), bos=2048, pad=2050, eos=EOS)
                uni = osamp.uniform(r["seed"], 0, f, q)
                want = osamp.sample(c, u, u=uni, **kw)
                have = EOS if f == n else int(codes[f, q])
                total += 1
                if have != want:
                    alt = {osamp.sample(c, u, u=min(max(uni + d, 0.0), 1.0 - 2 ** -24), **kw) for d in (-1e-4, 1e-4)}
                    assert have in alt, f"request {r['rid']} frame {f} q {q}: {have} vs oracle {want}"
                    near += 1
    b.close()
    assert total > 100 and near <= 0.01 * total, f"{near} near-boundary draws of {total}"
