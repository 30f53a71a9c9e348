"""Several prompts in one prefill pass (skb_engine_prefill_many) against one
prefill per request: every request's residual stream, KV cache and first
decoded frames' logits agree (rel/abs 1e-5 / 1e-4), request 0's final hidden
state matches the reference golden (1e-4), and bad calls are refused."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from tests._util import assert_close, load_golden, oracle_from_meta

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def small():
    from soraku_tts_b200.model import SorakuModel

    data, meta = load_golden("model_small")
    orc, dims, sd = oracle_from_meta(meta)
    return data, SorakuModel(dims, sd, "cuda")


def _prompts(data, n):
    ids, unc, pc = np.asarray(data["input_ids"]).reshape(1, -1), np.asarray(data["uncond_input_ids"]).reshape(1, -1), \
        np.asarray(data["prompt_codes"])
    out = []
    for i in range(n):
        L = max(2, ids.shape[1] - 4 * i)
        R = max(0, pc.shape[0] - 2 * i)
        out.append((ids[:, :L], unc, pc[:R]))
    return out


def _engine(model, n, batch):
    from soraku_tts_b200.graph_frame import NativeEngine

    eng = NativeEngine(model, max_requests=n, rows_per_request=2, max_len=256, max_frames=8, max_prefill=128,
                       prefill_batch=batch)
    for r in range(n):
        eng.set_sampling(r, cfg=1.5, temperature=0.9, temperature_q0=0.9, top_k=50, top_p=0.95, top_k_q0=50,
                         top_p_q0=0.95, seed=50 + r, min_new_frames=10 ** 6, eos_rule=1)
    return eng


def _decode(eng, n, frames=2):
    eng.set_debug(True)
    eng.capture(n, 1)
    logits = []
    for _ in range(frames):
        eng.step(True)
        torch.cuda.synchronize()
        logits.append(eng.view(4).cpu().numpy().copy())
    return np.stack(logits)


def _final_norm(x, model):
    w = model.params["trunk.norm.weight"]
    eps = model.dims.trunk.rms_norm_eps
    return (x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w)


def test_prefill_many_equals_one_prefill_per_request(small):
    data, model = small
    n = 3
    ps = _prompts(data, n)
    a = _engine(model, n, batch=n)
    a.prefill_many(list(range(n)), [p[0] for p in ps], [p[1] for p in ps], [p[2] for p in ps])
    b = _engine(model, n, batch=1)
    for r, p in enumerate(ps):
        b.prefill(r, *p)
    xa, xb = a.view(0).view(2 * n, -1).cpu().numpy(), b.view(0).view(2 * n, -1).cpu().numpy()
    np.testing.assert_allclose(xa, xb, rtol=1e-5, atol=1e-5)
    np.testing.assert_array_equal(a.view(3, torch.int32).cpu().numpy(), b.view(3, torch.int32).cpu().numpy())
    h0 = _final_norm(a.view(0).view(2 * n, -1)[:2], model).cpu().numpy()
    assert_close(h0, data["hidden"][0], what="prefill_many request 0 hidden (vs reference golden)", rtol=1e-4,
                 atol=1e-4)
    la, lb = _decode(a, n), _decode(b, n)
    assert_close(la, lb, what="logits after prefill_many vs single prefills", rtol=1e-4, atol=1e-4)
    for e in (a, b):
        assert (e.view(6, torch.int32).cpu().numpy() == 0).all()
    a.close()
    b.close()


def test_prefill_many_refuses_bad_calls(small):
    data, model = small
    ps = _prompts(data, 2)
    eng = _engine(model, 3, batch=2)
    with pytest.raises(ValueError):  # more requests than one pass holds
        eng.prefill_many([0, 1, 2], [ps[0][0]] * 3, [ps[0][1]] * 3, [ps[0][2]] * 3)
    with pytest.raises(ValueError):  # the same request twice
        eng.prefill_many([1, 1], [p[0] for p in ps], [p[1] for p in ps], [p[2] for p in ps])
    eng.prefill_many([2, 0], [p[0] for p in ps], [p[1] for p in ps], [p[2] for p in ps])
    eng.close()
