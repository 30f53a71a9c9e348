"""Model dimensions of the soraku-TTS v2 talker and depth head.

``SorakuV2Config`` mirrors the reference dataclass field for field
(soraku_inference/model.py:34-66): the audio vocabulary is the 2048 codec
entries plus BOS (2048), EOS (2049) and PAD (2050), so every codebook table and
classifier has 2051 rows.  ``TrunkConfig`` holds the Qwen3 dimensions the
reference reads from ``text_config.json`` (soraku_inference/runtime.py:26-34);
the defaults are Qwen3-0.6B's.
"""

from __future__ import annotations

from dataclasses import asdict, dataclass, field


@dataclass(frozen=True)
class SorakuV2Config:
    """Mirror of ``soraku_inference.model.SorakuV2Config`` (model.py:34-66)."""

    text_model_path: str = "pre_train_models/Qwen3-0.6B-Base"
    num_codebooks: int = 16
    codebook_size: int = 2048
    depth_ffn_mult: int = 2
    tie_audio_head: bool = True
    freeze_text_embedding: bool = True
    initializer_range: float = 0.02
    speaker_conditioning: bool = False
    speaker_dim: int = 192
    speaker_condition_mode: str = "bos"
    language_token_ids: tuple[int, ...] = ()

    @property
    def audio_bos_id(self) -> int:
        return self.codebook_size

    @property
    def audio_eos_id(self) -> int:
        return self.codebook_size + 1

    @property
    def audio_pad_id(self) -> int:
        return self.codebook_size + 2

    @property
    def audio_vocab_size(self) -> int:
        return self.codebook_size + 3

    def to_dict(self) -> dict:
        return asdict(self)


@dataclass(frozen=True)
class TrunkConfig:
    """Qwen3 trunk dimensions (transformers Qwen3Config fields of the same name)."""

    hidden_size: int = 1024
    num_hidden_layers: int = 28
    num_attention_heads: int = 16
    num_key_value_heads: int = 8
    head_dim: int = 128
    intermediate_size: int = 3072
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1_000_000.0
    vocab_size: int = 151936

    @property
    def q_dim(self) -> int:
        return self.num_attention_heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.num_key_value_heads * self.head_dim

    def to_hf_kwargs(self) -> dict:
        """Keyword arguments for ``transformers.Qwen3Config`` with these dimensions."""
        return dict(
            hidden_size=self.hidden_size,
            num_hidden_layers=self.num_hidden_layers,
            num_attention_heads=self.num_attention_heads,
            num_key_value_heads=self.num_key_value_heads,
            head_dim=self.head_dim,
            intermediate_size=self.intermediate_size,
            rms_norm_eps=self.rms_norm_eps,
            rope_theta=self.rope_theta,
            vocab_size=self.vocab_size,
            max_position_embeddings=40960,
            tie_word_embeddings=False,
            attention_bias=False,
        )


# torch.finfo(torch.float32).eps: the depth head's nn.RMSNorm() is built without
# an eps (model.py:135,137), and torch then uses the dtype's machine epsilon.
DEPTH_NORM_EPS = 1.1920928955078125e-07


@dataclass(frozen=True)
class ModelDims:
    """Both configs together, as the engine consumes them."""

    soraku: SorakuV2Config = field(default_factory=SorakuV2Config)
    trunk: TrunkConfig = field(default_factory=TrunkConfig)

    @property
    def d_model(self) -> int:
        return self.trunk.hidden_size

    @property
    def depth_inner(self) -> int:
        return self.trunk.hidden_size * self.soraku.depth_ffn_mult
