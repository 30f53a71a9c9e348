"""Drop-in for soraku_inference/acceleration/fast_generate.py's FastGenerator.

``FastGenerator(model, device=..., use_graph=True).generate(**kwargs)`` takes
the keyword arguments of the reference (fast_generate.py:331-350) plus
``speaker_embedding`` (route D, which the reference's fast path refuses,
fast_generate.py:42-45) and returns ``(codes [T, Q] int64 CPU, info)``.

Semantics follow the native loop (model.py:515-621): CFG
``u + s (c - u)``, BOS/PAD masked, EOS only at q0 from frame
``min_new_frames`` on, which ends the utterance without emitting that frame.
EOS masking is decided on the device from the frame counter, so frames run
in chunks of ``frames_per_graph`` per graph replay with one device-to-host
copy per chunk; frames computed after an EOS inside a chunk are discarded,
which leaves every returned code exactly as a frame-by-frame loop produces
it.  With ``on_frame`` the chunk is one frame, so the callback streams.
"""

from __future__ import annotations

import os
from typing import Any

import torch

from .graph_frame import NativeEngine
from .model import as_soraku_model


class FastGenerator:
    def __init__(self, model, *, device: torch.device, use_tilelang: bool = True, compile_trunk: bool = False,
                 batch_branches: bool = True, native_sampling: bool = True, use_graph: bool = True,
                 frames_per_graph: int = 8, use_pdl: bool = True, l2_prefetch: bool = True):
        self.model = as_soraku_model(model, device)
        self.config = self.model.config
        self.device = torch.device(device)
        self.Q = int(self.config.num_codebooks)
        self.V = int(self.config.audio_vocab_size)
        self.frames_per_graph = int(frames_per_graph)
        self.use_pdl = use_pdl
        self.l2_prefetch = l2_prefetch
        self._engine: NativeEngine | None = None
        self._graph_key = None
        self.last_timing: dict[str, float] = {}

    def _get_engine(self, rows: int, max_len: int, max_frames: int) -> NativeEngine:
        e = self._engine
        if e is None or e.rows_per_request != rows or e.max_len < max_len or e.max_frames < max_frames:
            if e is not None:
                e.close()
            self._engine = NativeEngine(self.model, max_requests=1, rows_per_request=rows,
                                        max_len=max(max_len, 512), max_frames=max(max_frames, 512),
                                        max_prefill=max(max_len, 512), use_pdl=self.use_pdl,
                                        l2_prefetch=self.l2_prefetch)
            self._graph_key = None
        return self._engine

    @torch.inference_mode()
    def generate(self, *, input_ids, prompt_codes=None, max_new_frames: int = 384, min_new_frames: int = 4,
                 temperature: float = 0.9, top_k: int | None = 50, top_p: float | None = 0.95,
                 temperature_q0: float | None = None, top_k_q0: int | None = None,
                 top_p_q0: float | None = None, cfg_scale: float = 1.0, uncond_input_ids=None,
                 seed: int | None = None, on_frame: Any = None, use_graph: bool | None = None,
                 speaker_embedding=None) -> tuple[torch.LongTensor, dict[str, Any]]:
        ids = torch.as_tensor(input_ids)
        if ids.ndim != 2 or ids.shape[0] != 1:
            raise ValueError("generate expects input_ids of shape [1,L]")
        if cfg_scale != 1.0 and uncond_input_ids is None:
            raise ValueError("classifier-free guidance requires uncond_input_ids")
        if max_new_frames < 0:
            raise ValueError("max_new_frames must be >= 0")
        rows = 2 if cfg_scale != 1.0 else 1
        n_prompt = 0 if prompt_codes is None else int(torch.as_tensor(prompt_codes).numel() // self.Q)
        slot = 1 if (speaker_embedding is not None and self.config.speaker_condition_mode == "slot") else 0
        lens = [ids.shape[1]] + ([torch.as_tensor(uncond_input_ids).numel()] if rows == 2 else [])
        prompt_len = max(lens) + slot + 1 + n_prompt
        fpg = 1 if on_frame is not None else max(1, min(self.frames_per_graph, max_new_frames or 1))
        eng = self._get_engine(rows, prompt_len + max_new_frames + fpg, max_new_frames + fpg)
        if seed is None:
            seed = int.from_bytes(os.urandom(8), "little")
        eng.set_sampling(0, cfg=cfg_scale, temperature=temperature,
                         temperature_q0=temperature if temperature_q0 is None else temperature_q0,
                         top_k=top_k, top_p=top_p, top_k_q0=top_k if top_k_q0 is None else top_k_q0,
                         top_p_q0=top_p if top_p_q0 is None else top_p_q0, seed=seed,
                         min_new_frames=min_new_frames, eos_rule=1)
        eng.prefill(0, ids, uncond_input_ids if rows == 2 else None, prompt_codes, speaker_embedding)
        if self._graph_key != (1, fpg):
            eng.capture(1, fpg)
            self._graph_key = (1, fpg)
        frames: list[torch.Tensor] = []
        stop_reason = "max_frames"
        done = 0
        eos = self.config.audio_eos_id
        while done < max_new_frames:
            eng.step(True)
            chunk = eng.read_codes(0, done, fpg)
            torch.cuda.current_stream().synchronize()
            take = min(fpg, max_new_frames - done)
            hit = None
            for i in range(take):
                if done + i >= min_new_frames and int(chunk[i, 0]) == eos:
                    hit = i
                    break
            keep = take if hit is None else hit
            for i in range(keep):
                f = chunk[i].clone()
                frames.append(f)
                if on_frame is not None:
                    on_frame(f.view(1, 1, self.Q))
            done += take
            if hit is not None:
                stop_reason = "eos"
                break
        codes = torch.stack(frames) if frames else torch.empty(0, self.Q, dtype=torch.long)
        return codes, {"stop_reason": stop_reason, "num_frames": int(codes.shape[0]), "cfg_scale": cfg_scale,
                       "backend": "b200", "sampled": temperature > 0, "temperature": temperature}
