"""CPU checks of the drop-in boundary: the library loads without a GPU, exports
every entry point include/soraku_b200.h declares, and the ctypes mirrors of
its structs have the header's layout.  No compute is called."""

from __future__ import annotations

import ctypes
import os
import re
import subprocess
import tempfile

import pytest

from tests.conftest import REPO

HEADER = os.path.join(REPO, "include", "soraku_b200.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(skb_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    from soraku_tts_b200 import _lib
    from soraku_tts_b200.build import build

    build()
    return _lib


def test_library_exports_every_declared_symbol(lib):
    names = declared_functions()
    assert len(names) >= 25
    out = subprocess.run(["nm", "-D", "--defined-only", lib.LIB_PATH], capture_output=True, text=True).stdout
    exported = set(re.findall(r"\bT (skb_[a-z0-9_]+)", out))
    missing = [n for n in names if n not in exported]
    assert not missing, f"declared but not exported: {missing}"
    handle = lib.lib()
    for n in names:
        assert getattr(handle, n) is not None


def test_python_binding_covers_the_header(lib):
    assert sorted(lib.SIGNATURES) == declared_functions()


def test_struct_layouts_match_header(lib):
    src = r'''
#include <stdio.h>
#include <stddef.h>
#include "soraku_b200.h"
int main(void) {
  printf("%zu %zu %zu\n", sizeof(skb_sample_params), sizeof(skb_model_desc), sizeof(skb_engine_opts));
  printf("%zu %zu %zu %zu\n", offsetof(skb_sample_params, seed), offsetof(skb_model_desc, embed_tokens),
         offsetof(skb_model_desc, speaker_slot_mode), offsetof(skb_model_desc, layers));
  return 0;
}
'''
    with tempfile.TemporaryDirectory() as d:
        c = os.path.join(d, "probe.c")
        exe = os.path.join(d, "probe")
        open(c, "w").write(src)
        subprocess.check_call(["gcc", "-I", os.path.dirname(HEADER), c, "-o", exe])
        lines = subprocess.check_output([exe], text=True).split("\n")
    sizes = [int(v) for v in lines[0].split()]
    offs = [int(v) for v in lines[1].split()]
    assert sizes == [ctypes.sizeof(lib.skb_sample_params), ctypes.sizeof(lib.skb_model_desc),
                     ctypes.sizeof(lib.skb_engine_opts)]
    assert offs == [lib.skb_sample_params.seed.offset, lib.skb_model_desc.embed_tokens.offset,
                    lib.skb_model_desc.speaker_slot_mode.offset, lib.skb_model_desc.layers.offset]


def test_abi_version_and_error_string_without_gpu(lib):
    assert lib.lib().skb_abi_version() == 5
    assert isinstance(lib.last_error(), str)
    # argument validation happens before any CUDA call: a bad call fails cleanly on CPU
    st = lib.lib().skb_swiglu_gemv(None, None, None, None, 2, 2048, 1022, None)
    assert st == lib.SKB_ERR_ARG
    assert "multiple of 4" in lib.last_error()
    with pytest.raises(ValueError):
        lib.check(st, "swiglu_gemv")


def test_status_mapping(lib):
    lib.check(lib.SKB_OK)
    with pytest.raises(RuntimeError):
        lib.check(lib.SKB_ERR_CAPACITY)
    with pytest.raises(RuntimeError):
        lib.check(lib.SKB_ERR_STATE)


def test_op_surface_rejects_cpu_tensors():
    import torch

    from soraku_tts_b200 import kernels

    with pytest.raises(ValueError, match="CUDA"):
        kernels.rmsnorm(2, 8, 1e-6)(torch.zeros(2, 8), torch.ones(8))
    with pytest.raises(ValueError, match="tensor"):
        kernels.add_rmsnorm(2, 8, 1e-6)([0.0] * 16, torch.zeros(2, 8), torch.ones(8))


def test_sample_param_packing_normalises_filters():
    import numpy as np

    from soraku_tts_b200 import _lib

    arr = (_lib.skb_sample_params * 3)()
    rows = [dict(temperature=0.9, top_k=50, top_p=0.95, V=2051), dict(temperature=0.9, top_k=2051, top_p=1.0, V=2051),
            dict(temperature=0.0, top_k=None, top_p=None)]
    for i, r in enumerate(rows):
        V = r.get("V", 1 << 30)
        k, p = r.get("top_k"), r.get("top_p")
        arr[i] = _lib.skb_sample_params(1.0, r["temperature"], k if k and 0 < k < V else 0,
                                        p if p and 0 < p < 1 else -1.0, 0, 0, 0, 0, 0)
    assert [arr[i].top_k for i in range(3)] == [50, 0, 0]
    assert np.allclose([arr[i].top_p for i in range(3)], [0.95, -1.0, -1.0])


def test_fast_generator_validates_before_touching_the_gpu():
    import torch

    from soraku_tts_b200.config import ModelDims, TrunkConfig
    from soraku_tts_b200.fast_generate import FastGenerator
    from soraku_tts_b200.model import SorakuModel

    dims = ModelDims(trunk=TrunkConfig(num_hidden_layers=1, vocab_size=64))
    sd = {k: torch.zeros(1) for k in ["x"]}
    model = SorakuModel(dims, sd, "cpu")
    gen = FastGenerator(model, device=torch.device("cpu"))
    with pytest.raises(ValueError, match="shape"):
        gen.generate(input_ids=torch.zeros(2, 3, dtype=torch.long))
    with pytest.raises(ValueError, match="guidance"):
        gen.generate(input_ids=torch.zeros(1, 3, dtype=torch.long), cfg_scale=1.5)
