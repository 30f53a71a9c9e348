"""Continuous batching of ragged multi-request decode on one GPU.

The reference decodes one utterance per ``FastGenerator.generate`` call with
a fixed batch of the two CFG rows (``fast_generate.py:387-396``,
``graph_frame.py:31``).  ``ContinuousBatcher`` runs many requests through one
engine: a request joins the running batch as soon as a slot is free (its
prompt is prefilled into the slot), every active request advances by
``frames_per_graph`` frames per graph replay, and a request leaves when q0
draws EOS (from ``min_new_frames`` on, decided on the device) or its frame
budget is spent -- without stopping the others.  Finished slots are
compacted (the highest active request moves into the hole: its sampling
state, codes, residual stream and positions are copied, its KV pages change
hands by a page-table exchange), so the captured graph always covers a
contiguous prefix of the slots.  With ``kv_pages`` the KV cache is one shared
pool of pages: a request is admitted when the pool holds the pages its
prompt and frame budget need (both CFG rows), which it keeps until it
finishes, so short requests do not reserve a full ``max_len`` per row.

Determinism: every request draws from its own Philox stream (counter =
(stream 0, frame, q) under the request's seed), the engine runs the
tensor-core GEMM path for every batch width and fixes the attention kernel
variant, so a request's decode does not depend on its slot or on the
requests beside it.  Requests admitted together share one prompt pass
(``prefill_many``); while that pass holds at most 128 tokens its arithmetic
per token is the same as a pass of one prompt, beyond that the GEMM's K
split follows the token count and the prompt's hidden state can differ in
the last FP32 bits (``prefill_per_pass=1`` keeps one prompt per pass).

Semantics per request are ``FastGenerator.generate``'s: CFG ``u + s (c - u)``,
EOS only at q0 from frame ``min_new_frames`` on, which ends the utterance
without emitting that frame; frames a chunk computes past the end are
discarded.
"""

from __future__ import annotations

from collections import deque
from dataclasses import dataclass, field
from typing import Any, Callable, Hashable

import numpy as np
import torch

from .graph_frame import NativeEngine
from .model import as_soraku_model

UNCOND_TEXT_ID = 151643  # the uncond prompt [[151643]] of runtime.py:144


@dataclass
class DecodeRequest:
    """One utterance: prompt, sampling parameters and frame budget."""

    rid: Hashable
    input_ids: Any                     # [1, Lc] int64 cond ids
    uncond_ids: Any = None             # [1, Lu] int64; default [[text BOS]]
    prompt_codes: Any = None           # [R, Q] int64 reference frames
    speaker: Any = None                # [speaker_dim] float (route D)
    max_new_frames: int = 384
    min_new_frames: int = 4
    cfg_scale: float = 1.5
    temperature: float = 0.9
    temperature_q0: float | None = None
    top_k: int | None = 50
    top_p: float | None = 0.95
    seed: int = 0
    on_frame: Callable[[Hashable, np.ndarray], None] | None = None  # (rid, codes [Q]) per emitted frame


@dataclass
class _Slot:
    req: DecodeRequest
    emitted: int = 0
    frames: list = field(default_factory=list)
    pages: list = field(default_factory=list)  # shared pool: per CFG row, its pool pages in order


class PagePool:
    """Free list of a shared KV pool's pages (ids 0..n-1, lowest first)."""

    def __init__(self, n_pages: int):
        self.n = int(n_pages)
        self._free = list(range(self.n - 1, -1, -1))

    def available(self) -> int:
        return len(self._free)

    def take(self, k: int) -> list[int]:
        if k > len(self._free):
            raise RuntimeError(f"KV pool exhausted: {k} pages wanted, {len(self._free)} free")
        return [self._free.pop() for _ in range(k)]

    def give(self, pages) -> None:
        self._free.extend(sorted(pages, reverse=True))
        self._free.sort(reverse=True)


class ContinuousBatcher:
    """Continuous-batching scheduler over one ``NativeEngine`` with ``slots``
    request slots (2 CFG rows each)."""

    def __init__(self, model, *, slots: int, max_len: int, max_frames: int, frames_per_graph: int = 4,
                 max_prefill: int | None = None, kv_pages: int | None = None, page_size: int = 64,
                 prefill_per_pass: int = 8, device: Any = "cuda", engine_factory=None, **engine_kw):
        self.model = as_soraku_model(model, torch.device(device)) if engine_factory is None else model
        cfg = self.model.config
        self.Q = int(cfg.num_codebooks)
        self.eos = int(cfg.audio_eos_id)
        self.fpg = int(frames_per_graph)
        self.max_len = int(max_len)
        self.max_frames = int(max_frames)
        self.max_prefill = int(max_prefill or max_len)
        if self.fpg < 1:
            raise ValueError("frames_per_graph must be >= 1")
        make = engine_factory or (lambda **kw: NativeEngine(self.model, **kw))
        # every batch width on the tensor-core path; one attention split per
        # (row, kv head): a row's arithmetic is the same at every width
        kw = dict(gemm_min_rows=1, attn_splits=1, prefill_batch=max(1, min(slots, prefill_per_pass)))
        kw.update(engine_kw)
        self.page_size = int(page_size)
        self.max_pages = -(-self.max_len // self.page_size)
        self.pool = PagePool(kv_pages) if kv_pages else None
        if kv_pages:
            kw["kv_pages"] = int(kv_pages)
        self.engine = make(max_requests=slots, rows_per_request=2, max_len=self.max_len,
                           max_frames=self.max_frames, max_prefill=self.max_prefill, page_size=self.page_size,
                           **kw)
        self.slots: list[_Slot | None] = [None] * slots
        self.queue: deque[DecodeRequest] = deque()
        self.results: dict[Hashable, np.ndarray] = {}
        self.stop_reason: dict[Hashable, str] = {}
        self._graph: tuple[int, int] | None = None
        self.stats = {"replays": 0, "captures": 0, "moves": 0, "admitted": 0}

    # ------------------------------------------------------------------ API
    def submit(self, req: DecodeRequest) -> None:
        """Queue a request; raises if it can never fit the engine."""
        ids = torch.as_tensor(req.input_ids)
        if ids.ndim != 2 or ids.shape[0] != 1 or ids.numel() == 0:
            raise ValueError("input_ids must have shape [1, L] with L >= 1")
        if req.max_new_frames < 0 or req.min_new_frames < 0:
            raise ValueError("frame counts must be >= 0")
        unc = self._uncond(req)
        n_prompt = 0 if req.prompt_codes is None else int(torch.as_tensor(req.prompt_codes).numel() // self.Q)
        slot = 1 if req.speaker is not None and getattr(self.model.config, "speaker_condition_mode", "") == "slot" \
            else 0
        prompt_len = max(ids.shape[1], unc.numel()) + slot + 1 + n_prompt
        if prompt_len > self.max_prefill:
            raise ValueError(f"request {req.rid!r}: prompt of {prompt_len} positions exceeds max_prefill "
                             f"{self.max_prefill}")
        # a chunk may run up to frames_per_graph - 1 frames past the budget
        if prompt_len + req.max_new_frames + self.fpg > self.max_len:
            raise ValueError(f"request {req.rid!r}: {prompt_len} + {req.max_new_frames} frames exceed max_len "
                             f"{self.max_len}")
        if req.max_new_frames + self.fpg > self.max_frames:
            raise ValueError(f"request {req.rid!r}: {req.max_new_frames} frames exceed max_frames "
                             f"{self.max_frames}")
        if self.pool is not None and sum(self._pages_needed(req)) > self.pool.n:
            raise ValueError(f"request {req.rid!r} needs {sum(self._pages_needed(req))} KV pages, the pool has "
                             f"{self.pool.n}")
        if req.rid in self.results or any(s is not None and s.req.rid == req.rid for s in self.slots) or \
                any(q.rid == req.rid for q in self.queue):
            raise ValueError(f"request id {req.rid!r} already submitted")
        self.queue.append(req)

    def pending(self) -> int:
        return len(self.queue)

    def active(self) -> int:
        return sum(s is not None for s in self.slots)

    def step(self) -> bool:
        """Compact, admit, then one graph replay (frames_per_graph frames) of
        the active requests and their results; False when nothing is left."""
        self._compact()
        self._admit()
        n = self.active()
        if n == 0:
            return False
        if self._graph != (n, self.fpg):
            self.engine.capture(n, self.fpg)
            self._graph = (n, self.fpg)
            self.stats["captures"] += 1
        self.engine.step(True)
        self.stats["replays"] += 1
        frames, _ = self.engine.status(n)
        for j in range(n):
            self._collect(j, frames[j])
        return True

    def run(self) -> dict[Hashable, np.ndarray]:
        """Decode until the queue is empty and every request has finished;
        returns {rid: codes [frames, Q] int64}."""
        while self.step():
            pass
        return self.results

    def close(self) -> None:
        self.engine.close()

    # ------------------------------------------------------------ internals
    def _pages_needed(self, req: DecodeRequest) -> tuple[int, int]:
        """Pages of the cond and uncond rows for the prompt, the frame budget
        and one chunk of overrun."""
        slot = 1 if req.speaker is not None and getattr(self.model.config, "speaker_condition_mode", "") == "slot" \
            else 0
        n_prompt = 0 if req.prompt_codes is None else int(torch.as_tensor(req.prompt_codes).numel() // self.Q)
        tail = slot + 1 + n_prompt + req.max_new_frames + self.fpg
        lens = (torch.as_tensor(req.input_ids).shape[-1] + tail, self._uncond(req).numel() + tail)
        return tuple(-(-n // self.page_size) for n in lens)

    def _uncond(self, req: DecodeRequest) -> torch.Tensor:
        if req.uncond_ids is None:
            return torch.tensor([[UNCOND_TEXT_ID]], dtype=torch.int64)
        return torch.as_tensor(req.uncond_ids)

    def _compact(self) -> None:
        lo, hi = 0, len(self.slots) - 1
        while True:
            while lo < len(self.slots) and self.slots[lo] is not None:
                lo += 1
            while hi >= 0 and self.slots[hi] is None:
                hi -= 1
            if lo >= hi:
                return
            self.engine.move_request(lo, hi)  # also exchanges the two slots' page-table rows
            self.slots[lo], self.slots[hi] = self.slots[hi], None
            self.stats["moves"] += 1

    def _admit(self) -> None:
        """Fill free slots from the queue (in arrival order), then prefill the
        admitted prompts, several per pass over the trunk."""
        batch = []
        for j in range(len(self.slots)):
            if self.slots[j] is not None:
                continue
            while self.queue:
                req = self.queue.popleft()
                if req.max_new_frames == 0:  # nothing to decode
                    self.results[req.rid] = np.zeros((0, self.Q), np.int64)
                    self.stop_reason[req.rid] = "max_frames"
                    continue
                pages = []
                if self.pool is not None:
                    need = self._pages_needed(req)
                    if sum(need) > self.pool.available():  # wait for pages, keeping arrival order
                        self.queue.appendleft(req)
                        break
                    for b, k in enumerate(need):
                        got = self.pool.take(k)
                        self.engine.map_pages(2 * j + b, 0, got + [-1] * (self.max_pages - k))
                        pages.append(got)
                self.engine.set_sampling(
                    j, cfg=req.cfg_scale, temperature=req.temperature,
                    temperature_q0=req.temperature if req.temperature_q0 is None else req.temperature_q0,
                    top_k=req.top_k, top_p=req.top_p, top_k_q0=req.top_k, top_p_q0=req.top_p, seed=req.seed,
                    min_new_frames=req.min_new_frames, eos_rule=1)
                self.engine.set_rng_stream(j, 0)
                self.slots[j] = _Slot(req, pages=pages)
                self.stats["admitted"] += 1
                batch.append((j, req))
                break
            else:
                break  # queue empty
            if self.slots[j] is None:
                break  # the head request waits for pages
        per_pass = max(1, int(getattr(self.engine, "prefill_batch", 1)))
        plain = [(j, r) for j, r in batch if r.speaker is None]
        for i in range(0, len(plain), per_pass):
            chunk = plain[i:i + per_pass]
            self.engine.prefill_many([j for j, _ in chunk], [r.input_ids for _, r in chunk],
                                     [self._uncond(r) for _, r in chunk], [r.prompt_codes for _, r in chunk])
        for j, r in batch:
            if r.speaker is not None:
                self.engine.prefill(j, r.input_ids, self._uncond(r), r.prompt_codes, r.speaker)

    def _collect(self, j: int, frames: int) -> None:
        s = self.slots[j]
        req = s.req
        limit = min(frames, req.max_new_frames)
        stop = None
        if limit > s.emitted:
            new = self.engine.read_codes(j, s.emitted, limit - s.emitted).numpy()
            for i in range(new.shape[0]):
                f = s.emitted
                if f >= req.min_new_frames and int(new[i, 0]) == self.eos:
                    stop = "eos"
                    break
                codes = new[i].copy()
                s.frames.append(codes)
                s.emitted += 1
                if req.on_frame is not None:
                    req.on_frame(req.rid, codes)
        if stop is None and s.emitted >= req.max_new_frames:
            stop = "max_frames"
        if stop is not None:
            self.results[req.rid] = (np.stack(s.frames) if s.frames else np.zeros((0, self.Q), np.int64))
            self.stop_reason[req.rid] = stop
            if self.pool is not None:
                for b, pages in enumerate(s.pages):  # back to the pool; the rows map nothing
                    self.engine.map_pages(2 * j + b, 0, [-1] * self.max_pages)
                    self.pool.give(pages)
            self.slots[j] = None
