"""Weights container and the engine's model descriptor.

``SorakuModel`` holds FP32 CUDA tensors under the reference's state-dict
names (soraku_inference/model.py:93-211 and transformers' Qwen3Model).
``as_soraku_model`` also accepts the reference's own ``SorakuTTSv2`` module
(anything with ``.config``, ``.trunk.config`` and ``.state_dict()``): its
parameters are borrowed, not copied, when they already are contiguous FP32
CUDA tensors, as the reference's engine borrows them (graph_frame.py:39-41).
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib
from .config import DEPTH_NORM_EPS, ModelDims, SorakuV2Config, TrunkConfig
from .weights import random_state_dict, rope_inv_freq

LAYER_KEYS = ("self_attn.q_proj.weight", "self_attn.k_proj.weight", "self_attn.v_proj.weight",
              "self_attn.o_proj.weight", "self_attn.q_norm.weight", "self_attn.k_norm.weight",
              "mlp.gate_proj.weight", "mlp.up_proj.weight", "mlp.down_proj.weight",
              "input_layernorm.weight", "post_attention_layernorm.weight")


class SorakuModel:
    def __init__(self, dims: ModelDims, state_dict, device="cuda"):
        self.dims = dims
        self.config = dims.soraku
        self.d_model = dims.d_model
        self.device = torch.device(device)
        self.params = {}
        for k, v in state_dict.items():
            t = v if isinstance(v, torch.Tensor) else torch.as_tensor(v)
            if t.device != self.device or t.dtype != torch.float32 or not t.is_contiguous():
                t = t.to(device=self.device, dtype=torch.float32).contiguous()
            self.params[k] = t
        self._desc = None

    @classmethod
    def random(cls, dims: ModelDims, seed: int = 42, device="cuda", **kw) -> "SorakuModel":
        return cls(dims, random_state_dict(dims, seed, **kw), device)

    def state_dict(self):
        return self.params

    # -------------------------------------------------------------- engine
    def model_desc(self):
        """skb_model_desc for the C ABI (kept alive with the host arrays it points to)."""
        if self._desc is not None:
            return self._desc[0]
        d, t, s = self.dims, self.dims.trunk, self.dims.soraku
        p = self.params
        desc = _lib.skb_model_desc()
        desc.n_layers = t.num_hidden_layers
        desc.d_model = t.hidden_size
        desc.n_heads = t.num_attention_heads
        desc.n_kv_heads = t.num_key_value_heads
        desc.head_dim = t.head_dim
        desc.ffn_dim = t.intermediate_size
        desc.text_vocab = t.vocab_size
        desc.n_codebooks = s.num_codebooks
        desc.audio_vocab = s.audio_vocab_size
        desc.depth_inner = d.depth_inner
        desc.speaker_dim = s.speaker_dim if s.speaker_conditioning else 0
        desc.rms_eps = t.rms_norm_eps
        desc.depth_eps = DEPTH_NORM_EPS
        desc.frame_scale = s.num_codebooks ** -0.5
        desc.bos_id, desc.eos_id, desc.pad_id = s.audio_bos_id, s.audio_eos_id, s.audio_pad_id
        langs = tuple(s.language_token_ids)
        desc.n_lang = len(langs)
        for i, v in enumerate(langs[:4]):
            desc.lang_ids[i] = int(v)

        def ptr(name):
            return p[name].data_ptr() if name in p else None

        desc.embed_tokens = ptr("trunk.embed_tokens.weight")
        desc.lang_embed = ptr("language_embeddings.weight")
        desc.final_norm = ptr("trunk.norm.weight")
        desc.table = ptr("audio_codebooks.table")
        desc.depth_bias = ptr("depth_head.bias")
        desc.depth_norm_in = ptr("depth_head.norm_in.weight")
        desc.depth_norm_out = ptr("depth_head.norm_out.weight")
        desc.depth_gate = ptr("depth_head.mlp.gate_proj.weight")
        desc.depth_up = ptr("depth_head.mlp.up_proj.weight")
        desc.depth_down = ptr("depth_head.mlp.down_proj.weight")
        desc.speaker_proj = ptr("speaker_projection.weight") if s.speaker_conditioning else None
        desc.speaker_slot = ptr("speaker_slot_embedding") if s.speaker_conditioning else None
        desc.speaker_slot_mode = 1 if s.speaker_condition_mode == "slot" else 0
        inv = rope_inv_freq(d).to(torch.float32).contiguous()
        inv_arr = (ctypes.c_float * inv.numel())(*inv.tolist())
        desc.rope_inv_freq = ctypes.cast(inv_arr, ctypes.c_void_p)
        ptrs = []
        for i in range(t.num_hidden_layers):
            for key in LAYER_KEYS:
                ptrs.append(p[f"trunk.layers.{i}.{key}"].data_ptr())
        layer_arr = (ctypes.c_void_p * len(ptrs))(*ptrs)
        desc.layers = ctypes.cast(layer_arr, ctypes.c_void_p)
        self._desc = (desc, inv_arr, layer_arr)
        return desc


def dims_from_reference(model) -> ModelDims:
    """ModelDims of a reference SorakuTTSv2 (model.config + model.trunk.config)."""
    c = model.config
    tc = model.trunk.config
    s = SorakuV2Config(num_codebooks=c.num_codebooks, codebook_size=c.codebook_size,
                       depth_ffn_mult=c.depth_ffn_mult, tie_audio_head=c.tie_audio_head,
                       speaker_conditioning=c.speaker_conditioning, speaker_dim=c.speaker_dim,
                       speaker_condition_mode=c.speaker_condition_mode,
                       language_token_ids=tuple(c.language_token_ids))
    rope = getattr(tc, "rope_parameters", None) or {}
    theta = rope.get("rope_theta", getattr(tc, "rope_theta", 1e6))
    t = TrunkConfig(hidden_size=tc.hidden_size, num_hidden_layers=tc.num_hidden_layers,
                    num_attention_heads=tc.num_attention_heads, num_key_value_heads=tc.num_key_value_heads,
                    head_dim=getattr(tc, "head_dim", tc.hidden_size // tc.num_attention_heads),
                    intermediate_size=tc.intermediate_size, rms_norm_eps=tc.rms_norm_eps,
                    rope_theta=float(theta), vocab_size=tc.vocab_size)
    return ModelDims(s, t)


def as_soraku_model(model, device="cuda") -> SorakuModel:
    if isinstance(model, SorakuModel):
        return model
    if hasattr(model, "state_dict") and hasattr(model, "trunk") and hasattr(model, "config"):
        if not model.config.tie_audio_head:
            raise ValueError("untied depth-head output projections are not supported")
        return SorakuModel(dims_from_reference(model), model.state_dict(), device)
    raise ValueError("expected a SorakuModel or a soraku_inference SorakuTTSv2 module")
