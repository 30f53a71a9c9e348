"""ctypes wrapper of oracle/sampler.c (test infrastructure only)."""

from __future__ import annotations

import ctypes
import math

import numpy as np

from .build import build

_lib = None


def lib():
    global _lib
    if _lib is None:
        _lib = ctypes.CDLL(build())
        _lib.orc_exp.argtypes = [ctypes.c_float]
        _lib.orc_exp.restype = ctypes.c_float
        _lib.orc_uniform.argtypes = [ctypes.c_uint64, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32]
        _lib.orc_uniform.restype = ctypes.c_float
        _lib.orc_philox4x32_10.argtypes = [ctypes.POINTER(ctypes.c_uint32)] * 3
        _lib.orc_philox4x32_10.restype = None
        _lib.orc_sample.argtypes = [
            ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_float,
            ctypes.c_int, ctypes.c_float, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
            ctypes.c_float, ctypes.c_void_p, ctypes.c_void_p,
        ]
        _lib.orc_sample.restype = ctypes.c_int
    return _lib


def exp(x: float) -> float:
    return float(lib().orc_exp(ctypes.c_float(x)))


def philox4x32_10(ctr, key):
    c = (ctypes.c_uint32 * 4)(*[int(v) & 0xFFFFFFFF for v in ctr])
    k = (ctypes.c_uint32 * 2)(*[int(v) & 0xFFFFFFFF for v in key])
    o = (ctypes.c_uint32 * 4)()
    lib().orc_philox4x32_10(c, k, o)
    return [int(v) for v in o]


def uniform(seed: int, request: int, frame: int, q: int) -> float:
    return float(lib().orc_uniform(int(seed) & 0xFFFFFFFFFFFFFFFF, request, frame, q))


def norm_top_k(top_k, V: int) -> int:
    """Host rule shared with the product: top-k is active iff 0 < k < V."""
    return int(top_k) if top_k is not None and 0 < int(top_k) < V else 0


def norm_top_p(top_p) -> float:
    """Host rule shared with the product: top-p is active iff 0 < p < 1."""
    return float(top_p) if top_p is not None and 0.0 < float(top_p) < 1.0 else -1.0


def sample(cond, uncond, *, cfg: float, temperature: float, top_k, top_p, mask_eos: bool,
           bos: int, pad: int, eos: int, u: float, return_info: bool = False):
    """Draw one code.  See sampler.c for the exact contract."""
    cond = np.ascontiguousarray(cond, dtype=np.float32)
    V = cond.shape[0]
    un = None if uncond is None else np.ascontiguousarray(uncond, dtype=np.float32)
    merged = np.empty(V, dtype=np.float32)
    info = np.zeros(4, dtype=np.int32)
    code = lib().orc_sample(
        cond.ctypes.data, None if un is None else un.ctypes.data, V,
        ctypes.c_float(cfg), ctypes.c_float(temperature), norm_top_k(top_k, V),
        ctypes.c_float(norm_top_p(top_p)), 1 if mask_eos else 0, bos, pad, eos,
        ctypes.c_float(u), merged.ctypes.data, info.ctypes.data,
    )
    if return_info:
        return int(code), {"merged": merged, "n_candidates": int(info[0]), "n_kept": int(info[1]),
                           "pick_rank": int(info[2]), "greedy": bool(info[3])}
    return int(code)


def kept_set(cond, uncond, *, cfg, temperature, top_k, top_p, mask_eos, bos, pad, eos):
    """Indices the restatement keeps after top-k/top-p (u-independent), in
    (value desc, index asc) order, with their final probabilities."""
    code, info = sample(cond, uncond, cfg=cfg, temperature=temperature, top_k=top_k, top_p=top_p,
                        mask_eos=mask_eos, bos=bos, pad=pad, eos=eos, u=0.0, return_info=True)
    f = info["merged"] / np.float32(temperature)
    V = f.shape[0]
    k = norm_top_k(top_k, V)
    if k:
        cutoff = np.sort(f)[::-1][k - 1]
        idx = np.nonzero(~(f < cutoff))[0]
    else:
        idx = np.arange(V)
    order = sorted(idx.tolist(), key=lambda i: (-float(f[i]), i))
    keep = order[: info["n_kept"]]
    e = np.array([exp(float(np.float32(f[i] - f[order[0]]))) for i in keep], dtype=np.float64)
    return keep, e / e.sum()


__all__ = ["exp", "philox4x32_10", "uniform", "sample", "kept_set", "norm_top_k", "norm_top_p",
           "math"]
