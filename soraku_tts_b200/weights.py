"""Seeded random-init weights under the reference's state-dict names.

No checkpoint is available offline, so benchmarks and parity runs use random
weights with the reference's layout (soraku_inference/model.py:93-211 for the
audio modules, transformers Qwen3Model for ``trunk.*``).  Every matrix, table
and embedding is N(0, 0.02) (``initializer_range``, model.py:42,103,145,195);
RMSNorm gains are 1 and the depth-head bias is 0 as the reference initialises
them (model.py:138-140), unless ``random_norms`` / ``random_bias`` ask for
non-trivial values, which the parity tests use so that a wrong gain or bias
index cannot hide behind a 1 or a 0.  The speaker projection and slot vector,
which the reference zero-initialises (model.py:205,209), are drawn N(0, 0.02)
so that the slot is not a no-op.

The tensors are drawn from one CPU ``torch.Generator`` in a fixed order, so a
seed names the same weights on every machine with the same torch build.
"""

from __future__ import annotations

from collections import OrderedDict

import torch

from .config import ModelDims


def state_dict_names(dims: ModelDims) -> list[tuple[str, tuple[int, ...], str]]:
    """(name, shape, kind) for every tensor, in generation order.

    kind is "normal" (N(0, std)), "norm" (RMSNorm gain) or "bias".
    """
    t, s = dims.trunk, dims.soraku
    d = t.hidden_size
    out: list[tuple[str, tuple[int, ...], str]] = []
    out.append(("trunk.embed_tokens.weight", (t.vocab_size, d), "normal"))
    for i in range(t.num_hidden_layers):
        p = f"trunk.layers.{i}."
        out += [
            (p + "self_attn.q_proj.weight", (t.q_dim, d), "normal"),
            (p + "self_attn.k_proj.weight", (t.kv_dim, d), "normal"),
            (p + "self_attn.v_proj.weight", (t.kv_dim, d), "normal"),
            (p + "self_attn.o_proj.weight", (d, t.q_dim), "normal"),
            (p + "self_attn.q_norm.weight", (t.head_dim,), "norm"),
            (p + "self_attn.k_norm.weight", (t.head_dim,), "norm"),
            (p + "mlp.gate_proj.weight", (t.intermediate_size, d), "normal"),
            (p + "mlp.up_proj.weight", (t.intermediate_size, d), "normal"),
            (p + "mlp.down_proj.weight", (d, t.intermediate_size), "normal"),
            (p + "input_layernorm.weight", (d,), "norm"),
            (p + "post_attention_layernorm.weight", (d,), "norm"),
        ]
    out.append(("trunk.norm.weight", (d,), "norm"))
    out.append(("audio_codebooks.table", (s.num_codebooks, s.audio_vocab_size, d), "normal"))
    inner = dims.depth_inner
    out += [
        ("depth_head.bias", (s.num_codebooks, s.audio_vocab_size), "bias"),
        ("depth_head.norm_in.weight", (d,), "norm"),
        ("depth_head.mlp.gate_proj.weight", (inner, d), "normal"),
        ("depth_head.mlp.up_proj.weight", (inner, d), "normal"),
        ("depth_head.mlp.down_proj.weight", (d, inner), "normal"),
        ("depth_head.norm_out.weight", (d,), "norm"),
    ]
    if not s.tie_audio_head:
        out.append(("depth_head.out_proj", (s.num_codebooks, s.audio_vocab_size, d), "normal"))
    if s.language_token_ids:
        out.append(("language_embeddings.weight", (4, d), "normal"))
    if s.speaker_conditioning:
        out.append(("speaker_projection.weight", (d, s.speaker_dim), "normal"))
        if s.speaker_condition_mode == "slot":
            out.append(("speaker_slot_embedding", (d,), "normal"))
    return out


def random_state_dict(
    dims: ModelDims,
    seed: int = 42,
    *,
    random_norms: bool = False,
    random_bias: bool = False,
) -> "OrderedDict[str, torch.Tensor]":
    """Draw a full FP32 state dict on the CPU.  See the module docstring."""
    gen = torch.Generator(device="cpu").manual_seed(int(seed))
    std = float(dims.soraku.initializer_range)
    out: "OrderedDict[str, torch.Tensor]" = OrderedDict()
    for name, shape, kind in state_dict_names(dims):
        if kind == "normal":
            tensor = torch.empty(shape, dtype=torch.float32).normal_(0.0, std, generator=gen)
        elif kind == "norm":
            if random_norms:
                tensor = 1.0 + torch.empty(shape, dtype=torch.float32).normal_(0.0, 0.1, generator=gen)
            else:
                tensor = torch.ones(shape, dtype=torch.float32)
        elif kind == "bias":
            if random_bias:
                tensor = torch.empty(shape, dtype=torch.float32).normal_(0.0, 0.05, generator=gen)
            else:
                tensor = torch.zeros(shape, dtype=torch.float32)
        else:  # pragma: no cover - table is closed
            raise AssertionError(kind)
        out[name] = tensor
    return out


def rope_inv_freq(dims: ModelDims) -> torch.Tensor:
    """RoPE inverse frequencies computed exactly as transformers' default rope
    init does (modeling_qwen3.py ``compute_default_rope_parameters``): FP32
    ``1 / theta ** (arange(0, hd, 2) / hd)``."""
    hd = dims.trunk.head_dim
    base = dims.trunk.rope_theta
    return 1.0 / (base ** (torch.arange(0, hd, 2, dtype=torch.int64).to(dtype=torch.float) / hd))
