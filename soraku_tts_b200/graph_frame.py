"""Drop-in for soraku_inference/acceleration/graph_frame.py's GraphFrameEngine.

Same constructor, attributes (``graph``, ``max_len``, ``cfg``) and methods
(``prefill``, ``capture``, ``step_frame``, ``set_temperature``,
``set_sampling``, ``set_seed``).  Underneath, the whole frame -- 16 depth
steps with CFG and sampling, the frame embedding and one 28-layer trunk step
-- is a native engine (libsoraku_b200.so) recorded as one CUDA graph of
sm_100a kernels; the trunk's KV cache is a paged FP32 pool with per-row
lengths, so the uncond branch needs no left padding.

Differences from the reference, all semantics-preserving:
* prefill embeds text with ``embed_text``'s language-ID substitution
  (model.py:326-338); the reference's graph prefill uses the raw text table
  (graph_frame.py:137);
* the draw is the Philox4x32-10 inverse-CDF rule of the fused sampler, not
  ``torch.multinomial``; greedy decoding (``sampled=False``) is argmax as in
  the reference;
* ``top_k``/``top_p`` are runtime parameters, so changing them needs no
  recapture.
"""

from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import _lib
from .model import as_soraku_model


class _GraphHandle:
    """Truthy stand-in for the reference's ``torch.cuda.CUDAGraph`` attribute."""

    def __init__(self, frames_per_graph: int):
        self.frames_per_graph = frames_per_graph


class NativeEngine:
    """Thin owner of an ``skb_engine*`` (the C ABI of include/soraku_b200.h)."""

    def __init__(self, model, *, max_requests=1, rows_per_request=2, max_len=1024, max_frames=1024,
                 max_prefill=None, page_size=64, attn_splits=0, use_pdl=True, l2_prefetch=True, gemm_min_rows=0,
                 prefill_batch=1, kv_pages=0, split_depth_head=False):
        self.model = model
        opts = _lib.skb_engine_opts(max_requests, rows_per_request, max_len, max_frames,
                                    max_prefill if max_prefill else max_len, page_size, attn_splits,
                                    1 if use_pdl else 0, 1 if l2_prefetch else 0, int(gemm_min_rows),
                                    int(prefill_batch), int(kv_pages),
                                    1 if split_depth_head else 0)
        self.prefill_batch = max(1, int(prefill_batch))
        self.page_size = page_size
        handle = ctypes.c_void_p()
        desc = model.model_desc()
        _lib.call("skb_engine_create", ctypes.byref(desc), ctypes.byref(opts), ctypes.byref(handle))
        self.h = handle
        self.rows_per_request = rows_per_request
        self.max_requests = max_requests
        self.max_len = max_len
        self.max_frames = max_frames
        self.Q = model.config.num_codebooks

    def close(self):
        if getattr(self, "h", None) is not None and self.h.value:
            _lib.lib().skb_engine_destroy(self.h)
            self.h = None

    def __del__(self):  # pragma: no cover - interpreter shutdown order
        try:
            self.close()
        except Exception:
            pass

    def prefill(self, request, cond_ids, uncond_ids, prompt_codes, speaker=None, stream=None):
        cond = _host_ids(cond_ids)
        unc = _host_ids(uncond_ids) if uncond_ids is not None else None
        pc = None
        n_prompt = 0
        if prompt_codes is not None and torch.as_tensor(prompt_codes).numel():
            pc = torch.as_tensor(prompt_codes).to("cpu", torch.int64).reshape(-1, self.Q).contiguous()
            n_prompt = pc.shape[0]
        spk = None
        if speaker is not None:
            spk = torch.as_tensor(speaker).to("cpu", torch.float32).reshape(-1).contiguous()
        _lib.call("skb_engine_prefill", self.h, request, cond.data_ptr(), cond.numel(),
                  unc.data_ptr() if unc is not None else None, unc.numel() if unc is not None else 0,
                  pc.data_ptr() if pc is not None else None, n_prompt,
                  spk.data_ptr() if spk is not None else None, _lib.stream_ptr(stream))

    def prefill_many(self, requests, cond_ids, uncond_ids, prompt_codes, stream=None):
        """Prompts of several requests in one pass (no speaker vectors):
        sequences of per-request cond ids, uncond ids and prompt codes."""
        n = len(requests)
        conds = [_host_ids(c) for c in cond_ids]
        uncs = [_host_ids(u) for u in uncond_ids]
        pcs = []
        for pc in prompt_codes:
            t = torch.as_tensor(pc if pc is not None else np.zeros((0, self.Q), np.int64))
            pcs.append(t.to("cpu", torch.int64).reshape(-1, self.Q).contiguous())
        P = ctypes.c_void_p
        req_a = (ctypes.c_int * n)(*[int(r) for r in requests])
        c_ptr = (P * n)(*[c.data_ptr() for c in conds])
        c_n = (ctypes.c_int * n)(*[c.numel() for c in conds])
        u_ptr = (P * n)(*[u.data_ptr() for u in uncs])
        u_n = (ctypes.c_int * n)(*[u.numel() for u in uncs])
        p_ptr = (P * n)(*[(p.data_ptr() if p.numel() else None) for p in pcs])
        p_n = (ctypes.c_int * n)(*[p.shape[0] for p in pcs])
        _lib.call("skb_engine_prefill_many", self.h, n, ctypes.addressof(req_a), ctypes.addressof(c_ptr),
                  ctypes.addressof(c_n), ctypes.addressof(u_ptr), ctypes.addressof(u_n), ctypes.addressof(p_ptr),
                  ctypes.addressof(p_n), _lib.stream_ptr(stream))

    def set_sampling(self, request, *, cfg, temperature, temperature_q0, top_k, top_p, top_k_q0, top_p_q0,
                     seed, min_new_frames=0, eos_rule=0):
        _lib.call("skb_engine_set_sampling", self.h, request, float(cfg), float(temperature),
                  float(temperature_q0), int(top_k or 0), float(top_p if top_p is not None else -1.0),
                  int(top_k_q0 or 0), float(top_p_q0 if top_p_q0 is not None else -1.0),
                  int(seed) & 0xFFFFFFFFFFFFFFFF, int(min_new_frames), int(eos_rule))

    def capture(self, n_active=1, frames_per_graph=1, stream=None):
        _lib.call("skb_engine_capture", self.h, n_active, frames_per_graph, _lib.stream_ptr(stream))

    def step(self, mask_eos_q0=True, stream=None):
        _lib.call("skb_engine_step", self.h, 1 if mask_eos_q0 else 0, _lib.stream_ptr(stream))

    def step_eager(self, n_active=1, mask_eos_q0=True, stream=None):
        _lib.call("skb_engine_step_eager", self.h, n_active, 1 if mask_eos_q0 else 0, _lib.stream_ptr(stream))

    def frames(self, request=0) -> int:
        return int(_lib.lib().skb_engine_frames(self.h, request))

    def set_rng_stream(self, request: int, stream: int) -> None:
        """Philox stream word of a request (counter = (stream, frame, q))."""
        _lib.call("skb_engine_set_rng_stream", self.h, request, int(stream) & 0xFFFFFFFF)

    def status(self, n: int, stream=None) -> tuple[list[int], list[int]]:
        """Device frame counters and EOS flags of requests [0, n)."""
        frames = (ctypes.c_int32 * max(n, 1))()
        done = (ctypes.c_int32 * max(n, 1))()
        _lib.call("skb_engine_status", self.h, n, ctypes.addressof(frames), ctypes.addressof(done),
                  _lib.stream_ptr(stream))
        return list(frames[:n]), list(done[:n])

    def map_pages(self, row: int, first: int, pages) -> None:
        """Shared KV pool: logical pages [first, first + len(pages)) of a row
        become these pool pages (-1 unmaps)."""
        arr = (ctypes.c_int32 * max(len(pages), 1))(*[int(p) for p in pages])
        _lib.call("skb_engine_map_pages", self.h, row, first, len(pages), ctypes.addressof(arr))

    def move_request(self, dst: int, src: int, stream=None) -> None:
        """Move request ``src``'s decode state into slot ``dst`` (slot compaction)."""
        _lib.call("skb_engine_move_request", self.h, dst, src, _lib.stream_ptr(stream))

    def read_codes(self, request, first, n, out=None, stream=None, sync=True) -> torch.Tensor:
        """Codes [n, Q] of frames first..first+n-1.  The copy is asynchronous on
        the stream; with sync=True (default) the stream is synchronised before
        returning, so the host buffer holds the codes."""
        if out is None:
            out = torch.empty((n, self.Q), dtype=torch.int64, pin_memory=True)
        _lib.call("skb_engine_read_codes", self.h, request, first, n, out.data_ptr(), _lib.stream_ptr(stream))
        if sync:
            (torch.cuda.current_stream() if stream is None else stream).synchronize()
        return out

    def view(self, which: int, dtype=torch.float32) -> torch.Tensor:
        ptr = ctypes.c_void_p()
        numel = ctypes.c_int64()
        _lib.call("skb_engine_view", self.h, which, ctypes.byref(ptr), ctypes.byref(numel))
        return _device_view(ptr.value, int(numel.value), dtype)

    def set_debug(self, on: bool):
        _lib.call("skb_engine_set_debug", self.h, 1 if on else 0)

    def kernels_per_frame(self) -> int:
        return int(_lib.lib().skb_engine_kernels_per_frame(self.h))

    def launches_per_step(self) -> int:
        """Kernel launches of one step() of the captured graph."""
        return int(_lib.lib().skb_engine_launches_per_step(self.h))


def _host_ids(ids) -> torch.Tensor:
    t = torch.as_tensor(ids).to("cpu", torch.int64).reshape(-1).contiguous()
    if t.numel() == 0:
        raise ValueError("empty id sequence")
    return t


def _device_view(ptr: int, numel: int, dtype) -> torch.Tensor:
    """A torch tensor aliasing engine-owned device memory (read-only use)."""
    class _Cai:
        def __init__(self):
            typestr = {torch.float32: "<f4", torch.int32: "<i4", torch.int64: "<i8"}[dtype]
            self.__cuda_array_interface__ = {"shape": (numel,), "typestr": typestr, "data": (ptr, False),
                                             "version": 3, "strides": None}
    return torch.as_tensor(_Cai(), device="cuda")


class GraphFrameEngine:
    """graph_frame.py:23-328, backed by the native engine."""

    def __init__(self, model, *, device: torch.device, max_cache_len: int, cfg_scale: float = 1.5,
                 batch: int = 2, max_frames: int | None = None, use_pdl: bool = True,
                 l2_prefetch: bool = True) -> None:
        if batch not in (1, 2):
            raise ValueError("batch must be 1 (no CFG) or 2 (cond + uncond)")
        self.model = as_soraku_model(model, device)
        self.config = self.model.config
        self.device = torch.device(device)
        self.batch = batch
        self.d_model = self.model.d_model
        self.Q = int(self.config.num_codebooks)
        self.V = int(self.config.audio_vocab_size)
        self.max_len = int(max_cache_len)
        self.native = NativeEngine(self.model, max_requests=1, rows_per_request=batch, max_len=self.max_len,
                                   max_frames=max_frames or self.max_len, max_prefill=self.max_len,
                                   use_pdl=use_pdl, l2_prefetch=l2_prefetch)
        self.cfg = torch.tensor([cfg_scale], device=self.device, dtype=torch.float32)
        self.graph = None
        self.top_k: int | None = None
        self.top_p: float | None = None
        self._temp = 1.0
        self._temp_q0 = 1.0
        self._sampled = False
        self._seed = 0
        self._frame = 0

    # --------------------------------------------------------------- state
    def _push(self):
        samp = self._sampled
        self.native.set_sampling(
            0, cfg=float(self.cfg.item()), temperature=self._temp if samp else 0.0,
            temperature_q0=self._temp_q0 if samp else 0.0,
            top_k=self.top_k if samp else None, top_p=self.top_p if samp else None,
            top_k_q0=self.top_k if samp else None, top_p_q0=self.top_p if samp else None,
            seed=self._seed, eos_rule=0)

    def set_temperature(self, value: float, *, q0: float | None = None) -> None:
        self._temp = float(value)
        self._temp_q0 = float(value if q0 is None else q0)

    def set_sampling(self, *, sampled: bool, top_k: int | None, top_p: float | None) -> None:
        self._sampled = bool(sampled)
        self.top_k = top_k
        self.top_p = top_p

    def set_seed(self, seed: int | None) -> None:
        if seed is not None:
            self._seed = int(seed)

    # ------------------------------------------------------------- prefill
    @torch.inference_mode()
    def prefill(self, cond_ids, uncond_ids, prompt_codes, speaker_embedding=None) -> torch.Tensor:
        """Prefill both branches; returns the [B, d] final hidden state."""
        if uncond_ids is None and self.batch == 2:
            uncond_ids = cond_ids
        self._push()
        self.native.prefill(0, cond_ids, uncond_ids if self.batch == 2 else None, prompt_codes,
                            speaker_embedding)
        self._frame = 0
        # the hidden state is the final-normed residual; the engine folds the final
        # norm into the first depth kernel, so compute it here for the caller
        x = self.native.view(0).view(self.batch, self.d_model)
        w = self.model.params["trunk.norm.weight"]
        eps = self.model.dims.trunk.rms_norm_eps
        hidden = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w
        return hidden.clone()

    # ------------------------------------------------------------- capture
    @torch.inference_mode()
    def capture(self, warmup: int = 3, frames_per_graph: int = 1) -> None:
        """Record the frame graph.  ``warmup`` is accepted for signature
        compatibility: stream capture executes nothing, so no state needs to be
        warmed up or restored (graph_frame.py:274-296 needs both)."""
        if self.graph is not None and self.graph.frames_per_graph == frames_per_graph:
            return
        self.native.capture(1, frames_per_graph)
        self.graph = _GraphHandle(frames_per_graph)

    @torch.inference_mode()
    def step_frame(self, *, mask_eos_q0: bool) -> torch.Tensor:
        """One replay; returns this frame's codes as a CPU int64 [Q] tensor."""
        if self.graph is None:
            raise RuntimeError("call capture() first")
        self._push_if_changed()
        self.native.step(mask_eos_q0)
        first = self.native.frames(0) - self.graph.frames_per_graph
        out = self.native.read_codes(0, first, self.graph.frames_per_graph)
        torch.cuda.current_stream().synchronize()
        return out[-1].clone()

    def _push_if_changed(self):
        key = (float(self.cfg.item()), self._temp, self._temp_q0, self._sampled, self.top_k, self.top_p,
               self._seed)
        if getattr(self, "_pushed", None) != key:
            self._push()
            self._pushed = key
