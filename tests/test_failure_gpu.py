"""Failure detection on the GPU without a GPU fault.

* A device wait that runs out: a one-thread kernel waits, with a 1 ms limit,
  on an mbarrier phase that nothing completes (no copy is in flight), through
  the bounded wait every decode kernel uses.  The wait gives up, sets the
  caller's error flag and returns; the C ABI reports SKB_ERR_CUDA, the Python
  layer raises, and the CUDA context keeps working.
* An engine error flag (a weight copy that did not arrive in time, flag 2)
  raised on the device surfaces as an exception from a later
  ``NativeEngine.step`` and at once from ``NativeEngine.status``, as the
  reference's engine raises RuntimeError when it cannot go on
  (graph_frame.py:155-156, 301-302)."""

from __future__ import annotations

import pytest
import torch

from tests._util import load_golden, oracle_from_meta

pytestmark = pytest.mark.gpu


def test_bounded_wait_gives_up_and_reports():
    from soraku_tts_b200 import _lib

    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    with pytest.raises(RuntimeError, match="gave up"):
        _lib.call("skb_test_wait_timeout", flag.data_ptr(), 1000, stream)
    assert int(flag.item()) == 1
    # the context is still usable: torch work and another library call
    x = torch.arange(1024, device="cuda", dtype=torch.float32)
    assert float(x.sum()) == 1023 * 1024 / 2
    y = torch.empty_like(x)
    _lib.call("skb_test_exp", x.data_ptr(), y.data_ptr(), 1, stream)
    torch.cuda.synchronize()
    assert float(y[0]) == 1.0


def test_engine_error_flag_surfaces_on_step_and_status():
    from soraku_tts_b200.graph_frame import NativeEngine
    from soraku_tts_b200.model import SorakuModel

    data, meta = load_golden("model_small")
    orc, dims, sd = oracle_from_meta(meta)
    model = SorakuModel(dims, sd, "cuda")
    eng = NativeEngine(model, max_requests=1, rows_per_request=2, max_len=256, max_frames=16, max_prefill=256)
    eng.set_sampling(0, cfg=1.5, temperature=0.9, temperature_q0=0.9, top_k=50, top_p=0.95, top_k_q0=50,
                     top_p_q0=0.95, seed=1, min_new_frames=10 ** 6, eos_rule=1)
    eng.prefill(0, data["input_ids"][0], data["uncond_input_ids"][0], data["prompt_codes"])
    eng.capture(1, 1)
    eng.step(True)
    torch.cuda.synchronize()
    eng.status(1)  # no flag raised: no exception
    eng.view(6, torch.int32)[2] = 1  # as a GEMV whose weight copy timed out would
    torch.cuda.synchronize()
    raised = False
    for _ in range(3):
        try:
            eng.step(True)
        except RuntimeError as exc:
            assert "flag 2" in str(exc)
            raised = True
            break
        torch.cuda.synchronize()
    assert raised, "the raised flag did not surface from step()"
    with pytest.raises(RuntimeError, match="flag 2"):  # sticky
        eng.step(True)
    eng.close()


def test_engine_error_flag_surfaces_on_status():
    from soraku_tts_b200.graph_frame import NativeEngine
    from soraku_tts_b200.model import SorakuModel

    data, meta = load_golden("model_small")
    orc, dims, sd = oracle_from_meta(meta)
    model = SorakuModel(dims, sd, "cuda")
    eng = NativeEngine(model, max_requests=1, rows_per_request=2, max_len=256, max_frames=16, max_prefill=256)
    eng.prefill(0, data["input_ids"][0], data["uncond_input_ids"][0], data["prompt_codes"])
    eng.status(1)
    eng.view(6, torch.int32)[0] = 1  # a position out of range
    with pytest.raises(RuntimeError, match="flag 0"):
        eng.status(1)
    eng.close()
