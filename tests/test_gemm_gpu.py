"""The batched / prefill GEMM (out = x @ w^T, FP32 operands) on the GPU
against a float64 reference: the 3xTF32 tcgen05 kernel (K splits chosen by
occupancy, none, 3 and 8 per tile: a cluster reduction in distributed shared
memory), the FP32 FFMA few-row kernel, the choice by rows, and the SIMT FP32
kernel, at shapes with partial row and column tiles and fewer K stages than
splits.  Tolerance: 1e-5 relative to the row scale (3xTF32 keeps ~21
mantissa bits per product; FFMA is plain FP32)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def lib():
    from soraku_tts_b200 import _lib

    return _lib


@pytest.mark.parametrize("tensor_cores,splits", [(2, 0), (2, 1), (2, 3), (2, 8), (1, 0), (0, 0)])
@pytest.mark.parametrize("M,N,K", [(128, 64, 32), (200, 320, 1024), (7, 1000, 2048), (388, 4096, 1024),
                                   (128, 1024, 3072), (130, 100, 160)])
def test_gemm_matches_float64(lib, tensor_cores, splits, M, N, K):
    g = np.random.default_rng(M * 7 + N + K)
    x = g.standard_normal((M, K)).astype(np.float32)
    w = (g.standard_normal((N, K)) * 0.02).astype(np.float32)
    xd, wd = torch.from_numpy(x).cuda(), torch.from_numpy(w).cuda()
    out = torch.full((M, N), np.nan, dtype=torch.float32, device="cuda")
    lib.call("skb_test_gemm", xd.data_ptr(), wd.data_ptr(), out.data_ptr(), M, N, K, tensor_cores, splits,
             lib.stream_ptr())
    got = out.cpu().numpy()
    ref = x.astype(np.float64) @ w.astype(np.float64).T
    scale = np.sqrt((x.astype(np.float64) ** 2).sum(1, keepdims=True) * (w.astype(np.float64) ** 2).sum(1)[None])
    err = np.abs(got - ref) / np.maximum(scale, 1e-30)
    assert np.isfinite(got).all()
    assert err.max() < 1e-5, f"max scaled error {err.max():.3g}"


@pytest.mark.parametrize("M", [1, 5, 8, 16, 17, 32])
@pytest.mark.parametrize("N,K", [(4096, 1024), (1000, 2048), (2051, 1024), (1024, 3072), (7, 256), (300, 512)])
def test_ffma_few_row_kernel_matches_float64(lib, M, N, K):
    """The FP32 FFMA kernel for few rows (one lane per output row, warps
    splitting K): every unit count per CTA from 1 to 28, so every lanes-per-
    unit split (1 to 32), and row counts on both sides of its 8 / 16 / 32
    row capacities."""
    g = np.random.default_rng(M * 13 + N + K)
    x = g.standard_normal((M, K)).astype(np.float32)
    w = (g.standard_normal((N, K)) * 0.02).astype(np.float32)
    xd, wd = torch.from_numpy(x).cuda(), torch.from_numpy(w).cuda()
    out = torch.full((M, N), np.nan, dtype=torch.float32, device="cuda")
    lib.call("skb_test_gemm", xd.data_ptr(), wd.data_ptr(), out.data_ptr(), M, N, K, 3, 0, lib.stream_ptr())
    got = out.cpu().numpy()
    ref = x.astype(np.float64) @ w.astype(np.float64).T
    scale = np.sqrt((x.astype(np.float64) ** 2).sum(1, keepdims=True) * (w.astype(np.float64) ** 2).sum(1)[None])
    err = np.abs(got - ref) / np.maximum(scale, 1e-30)
    assert np.isfinite(got).all()
    assert err.max() < 1e-5, f"max scaled error {err.max():.3g}"


def test_ffma_kernel_rejects_more_than_32_rows(lib):
    x = torch.zeros((33, 256), device="cuda")
    w = torch.zeros((8, 256), device="cuda")
    out = torch.zeros((33, 8), device="cuda")
    with pytest.raises(ValueError):
        lib.call("skb_test_gemm", x.data_ptr(), w.data_ptr(), out.data_ptr(), 33, 8, 256, 3, 0, lib.stream_ptr())
