"""Batched decode (more rows than the ring GEMV's 4: the row-norm + tiled
GEMM path) against the oracle: 4 CFG requests (8 rows) decoded together,
each checked like a single request -- per-(frame, q) logits within rel/abs
1e-4 of the oracle teacher-forced on that request's own codes, and every
code bit-exact with the oracle's sampler fed the engine's logits and the
request's own Philox uniform (counter = (q, frame, request))."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import sampler as osamp
from tests._util import assert_close, load_golden, oracle_from_meta

pytestmark = pytest.mark.gpu
TOL = dict(rtol=1e-4, atol=1e-4)


@pytest.fixture(scope="module")
def small():
    from soraku_tts_b200.model import SorakuModel

    data, meta = load_golden("model_small")
    orc, dims, sd = oracle_from_meta(meta)
    return data, meta, orc, SorakuModel(dims, sd, "cuda")


def _run(model, data, nreq, frames, graph=True):
    from soraku_tts_b200.graph_frame import NativeEngine

    Q, V = model.config.num_codebooks, model.config.audio_vocab_size
    eng = NativeEngine(model, max_requests=nreq, rows_per_request=2, max_len=512, max_frames=64, max_prefill=512)
    eng.set_debug(True)
    for r in range(nreq):
        eng.set_sampling(r, cfg=1.5, temperature=0.9, temperature_q0=0.9, top_k=50, top_p=0.95, top_k_q0=50,
                         top_p_q0=0.95, seed=1000 + r, min_new_frames=10 ** 6, eos_rule=1)
        eng.prefill(r, data["input_ids"][0], data["uncond_input_ids"][0], data["prompt_codes"])
    if graph:
        eng.capture(nreq, 1)
    logits = []
    for _ in range(frames):
        if graph:
            eng.step(True)
        else:
            eng.step_eager(nreq, True)
        torch.cuda.synchronize()
        logits.append(eng.view(4).view(Q, 2 * nreq, V).cpu().numpy().copy())
    codes = [eng.read_codes(r, 0, frames).clone().numpy() for r in range(nreq)]
    err = eng.view(6, torch.int32).cpu().numpy()
    assert (err == 0).all(), f"device error flags raised: {err}"
    eng.close()
    return codes, np.stack(logits)


def test_batched_requests_match_oracle_per_request(small):
    data, meta, orc, model = small
    nreq, frames = 4, 3
    codes, logits = _run(model, data, nreq, frames)
    for r in range(nreq):
        tf = orc.teacher_forced(input_ids=data["input_ids"][0], uncond_input_ids=data["uncond_input_ids"][0],
                                prompt_codes=data["prompt_codes"], codes=codes[r], cfg_scale=1.5)
        lr = logits[:, :, 2 * r:2 * r + 2, :]
        assert_close(lr, tf["logits"], what=f"request {r} logits", **TOL)
        for f in range(frames):
            for q in range(codes[r].shape[1]):
                u = osamp.uniform(1000 + r, r, f, q)
                want = osamp.sample(lr[f, q, 0], lr[f, q, 1], cfg=1.5, temperature=0.9, top_k=50, top_p=0.95,
                                    mask_eos=True, bos=2048, pad=2050, eos=2049, u=u)
                assert int(codes[r][f, q]) == want, f"request {r} frame {f} q {q}"
    # different seeds, different streams
    assert not all(np.array_equal(codes[0], codes[r]) for r in range(1, nreq))


def test_batched_graph_equals_eager(small):
    data, meta, orc, model = small
    a, la = _run(model, data, 3, 2, graph=True)
    b, lb = _run(model, data, 3, 2, graph=False)
    for x, y in zip(a, b):
        np.testing.assert_array_equal(x, y)
    np.testing.assert_array_equal(la, lb)
