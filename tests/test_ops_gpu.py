"""Op-surface parity: the eight TileLang-mirror ops on the GPU against the
oracle's numpy FP32 restatement, on seeded inputs at config 5's shapes
(M = 1, 2, 8, 64; more than 4 rows run the 3xTF32 tensor-core GEMM).
Tolerance: rel/abs 1e-4 on logits and activations."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle.model_np import DEPTH_NORM_EPS, rmsnorm, silu
from tests._util import assert_close

pytestmark = pytest.mark.gpu
TOL = dict(rtol=1e-4, atol=1e-4)


@pytest.fixture(scope="module")
def K():
    from soraku_tts_b200 import kernels

    return kernels


def _rand(gen, *shape, std=0.02):
    return (gen.standard_normal(shape) * std).astype(np.float32)


def _cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("B", [1, 2, 8, 64])
@pytest.mark.parametrize("eps", [1e-6, DEPTH_NORM_EPS])
def test_add_rmsnorm_and_rmsnorm(K, B, eps):
    g = np.random.default_rng(3)
    D = 1024
    h, p = _rand(g, B, D, std=1.0), _rand(g, B, D, std=0.5)
    w = (1 + _rand(g, D, std=0.1)).astype(np.float32)
    out = K.add_rmsnorm(B, D, eps)(_cuda(h), _cuda(p), _cuda(w)).cpu().numpy()
    assert_close(out, rmsnorm((h + p).astype(np.float32), w, eps), what="add_rmsnorm", **TOL)
    out = K.rmsnorm(B, D, eps)(_cuda(h), _cuda(w)).cpu().numpy()
    assert_close(out, rmsnorm(h, w, eps), what="rmsnorm", **TOL)


@pytest.mark.parametrize("B", [1, 2, 8, 64])
@pytest.mark.parametrize("I,D", [(2048, 1024), (3072, 1024)])
def test_swiglu_gemv(K, B, I, D):
    g = np.random.default_rng(3)
    x = _rand(g, B, D, std=1.0)
    wg, wu = _rand(g, I, D), _rand(g, I, D)
    out = K.swiglu_gemv(B, I, D)(_cuda(x), _cuda(wg), _cuda(wu)).cpu().numpy()
    ref = (silu((x @ wg.T).astype(np.float32)) * (x @ wu.T)).astype(np.float32)
    assert_close(out, ref, what="swiglu_gemv", **TOL)


@pytest.mark.parametrize("B", [1, 2, 8, 64])
@pytest.mark.parametrize("D,I", [(1024, 2048), (1024, 3072)])
def test_down_residual_gemv(K, B, D, I):
    g = np.random.default_rng(4)
    act, wd, res = _rand(g, B, I, std=0.5), _rand(g, D, I), _rand(g, B, D, std=1.0)
    out = K.down_residual_gemv(B, D, I)(_cuda(act), _cuda(wd), _cuda(res)).cpu().numpy()
    assert_close(out, (act @ wd.T + res).astype(np.float32), what="down_residual_gemv", **TOL)


@pytest.mark.parametrize("B", [1, 2, 8, 64])
@pytest.mark.parametrize("V", [2051, 2048])
def test_classifier_gemv(K, B, V):
    g = np.random.default_rng(5)
    D = 1024
    body, wq, bias = _rand(g, B, D, std=1.0), _rand(g, V, D), _rand(g, V, std=0.1)
    out = K.classifier_gemv(B, V, D)(_cuda(body), _cuda(wq), _cuda(bias)).cpu().numpy()
    assert_close(out, (body @ wq.T + bias).astype(np.float32), what="classifier_gemv", **TOL)


@pytest.mark.parametrize("R", [1, 73])
def test_frame_embed(K, R):
    g = np.random.default_rng(6)
    Q, V, D = 16, 2051, 1024
    table = _rand(g, Q, V, D)
    codes = g.integers(0, V, size=(R, Q)).astype(np.int64)
    out = K.frame_embed(R, Q, V, D, 0.25)(_cuda(codes), _cuda(table)).cpu().numpy()
    ref = sum(table[q][codes[:, q]] for q in range(Q)) * np.float32(0.25)
    assert_close(out, ref, what="frame_embed", rtol=1e-6, atol=1e-7)


def test_prefix_add(K):
    g = np.random.default_rng(7)
    B, V, D = 2, 2051, 1024
    prefix, tq = _rand(g, B, D), _rand(g, V, D)
    code = np.array([1234], dtype=np.int64)
    out = K.prefix_add(B, V, D, 0.25)(_cuda(prefix), _cuda(tq), _cuda(code)).cpu().numpy()
    np.testing.assert_array_equal(out, (prefix + tq[1234] * np.float32(0.25)).astype(np.float32))


@pytest.mark.parametrize("mask", [0, 1])
def test_sampling_prep(K, mask):
    g = np.random.default_rng(8)
    V = 2051
    logits = _rand(g, V, std=3.0)
    temp = np.array([0.9], dtype=np.float32)
    out = K.sampling_prep(V, 2048, 2050, 2049)(_cuda(logits), _cuda(temp),
                                               _cuda(np.array([mask], dtype=np.int32))).cpu().numpy()
    ref = (logits / temp[0]).astype(np.float32)
    ref[2048] = ref[2050] = -1e30
    if mask:
        ref[2049] = -1e30
    np.testing.assert_array_equal(out, ref)


def test_shape_errors_raise_value_error(K):
    with pytest.raises(ValueError):
        K.swiglu_gemv(2, 2048, 1022)(torch.zeros(2, 1022, device="cuda"), torch.zeros(2048, 1022, device="cuda"),
                                     torch.zeros(2048, 1022, device="cuda"))
    with pytest.raises(ValueError):
        K.rmsnorm(2, 1024, 1e-6)(torch.zeros(3, 1024, device="cuda"), torch.ones(1024, device="cuda"))
    with pytest.raises(ValueError):
        K.rmsnorm(2, 1024, 1e-6)(torch.zeros(2, 1024), torch.ones(1024))  # CPU tensors: no CPU path
