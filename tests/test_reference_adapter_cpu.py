"""The adapter runtime.py:129-140 would hit with the reference's own model.

Builds the reference's ``SorakuTTSv2`` (soraku_inference/model.py:177) on a
2-layer transformers Qwen3 trunk from the reference checkout (skipped where the
checkout is absent, e.g. on the GPU box) and checks that
``dims_from_reference`` recovers the dimensions, that every weight the engine
consumes is present under the name and shape the engine reads, that
``as_soraku_model`` borrows the reference's FP32 parameters without copying
them, and that the engine's model descriptor is filled from them."""

from __future__ import annotations

import os
import sys

import pytest
import torch

REF = "/root/reference"
pytestmark = pytest.mark.skipif(not os.path.isdir(os.path.join(REF, "soraku_inference")),
                                reason="reference checkout not present")


def _build(dims):
    if REF not in sys.path:
        sys.path.insert(0, REF)
    from tests.golden.make_golden import build_reference
    from soraku_tts_b200.weights import random_state_dict

    return build_reference(dims, random_state_dict(dims, 3))


@pytest.mark.parametrize("route", ["plain", "slot", "bos"])
def test_reference_model_through_the_adapter(route):
    from soraku_tts_b200.config import ModelDims, SorakuV2Config, TrunkConfig
    from soraku_tts_b200.model import LAYER_KEYS, as_soraku_model, dims_from_reference
    from soraku_tts_b200.weights import random_state_dict

    s = SorakuV2Config()
    if route != "plain":
        s = SorakuV2Config(speaker_conditioning=True, speaker_condition_mode=route,
                           language_token_ids=(4091, 4092, 4093, 4094) if route == "slot" else ())
    dims = ModelDims(s, TrunkConfig(num_hidden_layers=2, vocab_size=4096))
    ref = _build(dims)
    got = dims_from_reference(ref)
    assert got.soraku == dims.soraku
    assert got.trunk == dims.trunk

    sd = ref.state_dict()
    want = random_state_dict(dims, 3)
    assert set(want) <= set(sd), f"missing: {sorted(set(want) - set(sd))[:5]}"
    for k, v in want.items():
        assert tuple(sd[k].shape) == tuple(v.shape), k
    for i in range(dims.trunk.num_hidden_layers):
        for key in LAYER_KEYS:
            assert f"trunk.layers.{i}.{key}" in sd

    m = as_soraku_model(ref, device="cpu")
    for k in want:
        assert m.params[k].data_ptr() == sd[k].data_ptr(), f"{k} was copied"
    desc = m.model_desc()
    assert desc.n_layers == 2 and desc.d_model == 1024 and desc.audio_vocab == 2051
    assert desc.speaker_dim == (192 if route != "plain" else 0)
    assert desc.speaker_slot_mode == (1 if route == "slot" else 0)
    assert desc.n_lang == (4 if route == "slot" else 0)
    assert desc.table == sd["audio_codebooks.table"].data_ptr()
    torch.testing.assert_close(m.params["depth_head.bias"], sd["depth_head.bias"])
