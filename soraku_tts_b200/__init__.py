"""B200 (sm_100a) backend for soraku-TTS's per-frame autoregressive token loop.

Public surface (mirrors of the reference's acceleration plugin):
  kernels          -- the eight TileLang op factories (tilelang_kernels.py)
  GraphFrameEngine -- the whole-frame CUDA-graph engine (graph_frame.py)
  FastGenerator    -- the fast/graph generator (fast_generate.py)
  SorakuModel      -- FP32 CUDA weights under the reference's state-dict names

The compute runs in libsoraku_b200.so (hand-written sm_100a CUDA behind the C
ABI of include/soraku_b200.h); there is no CPU path.
"""

from .config import ModelDims, SorakuV2Config, TrunkConfig  # noqa: F401


def __getattr__(name):
    if name in ("GraphFrameEngine", "NativeEngine"):
        from . import graph_frame

        return getattr(graph_frame, name)
    if name == "FastGenerator":
        from .fast_generate import FastGenerator

        return FastGenerator
    if name == "SorakuModel":
        from .model import SorakuModel

        return SorakuModel
    raise AttributeError(name)
