"""Shared helpers for the tests (fixture loading, model construction)."""

from __future__ import annotations

import json
import os

import numpy as np

from soraku_tts_b200.config import ModelDims, SorakuV2Config, TrunkConfig
from soraku_tts_b200.weights import random_state_dict, rope_inv_freq

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load_golden(name: str):
    z = np.load(os.path.join(GOLDEN, f"{name}.npz"))
    data = {k: z[k] for k in z.files}
    meta = json.loads(str(data.pop("meta")))
    return data, meta


def dims_from_meta(meta) -> ModelDims:
    s = dict(meta["soraku"])
    s["language_token_ids"] = tuple(s.get("language_token_ids", ()))
    return ModelDims(SorakuV2Config(**s), TrunkConfig(**meta["trunk"]))


def weights_from_meta(meta):
    dims = dims_from_meta(meta)
    sd = random_state_dict(dims, meta["seed"], random_norms=meta["random_norms"],
                           random_bias=meta["random_bias"])
    return dims, sd


def oracle_from_meta(meta):
    from oracle.model_np import OracleModel

    dims, sd = weights_from_meta(meta)
    return OracleModel(sd, dims, rope_inv_freq(dims).numpy()), dims, sd


def assert_close(actual, expected, rtol=1e-4, atol=1e-4, what=""):
    actual = np.asarray(actual, dtype=np.float64)
    expected = np.asarray(expected, dtype=np.float64)
    err = np.abs(actual - expected)
    tol = atol + rtol * np.abs(expected)
    bad = err > tol
    if bad.any():
        i = np.unravel_index(np.argmax(err - tol), err.shape)
        raise AssertionError(
            f"{what}: {int(bad.sum())}/{bad.size} outside rtol={rtol} atol={atol}; worst at {i}: "
            f"actual={actual[i]!r} expected={expected[i]!r} max_abs_err={err.max():.3e}")
