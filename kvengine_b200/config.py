"""Model shapes for the Qwen2-architecture draft and target models.

The reference reads these numbers off a HuggingFace `Qwen2Config`
(kvengine/loader.py:55-73, `model_shape_info`); here they are a plain
dataclass so the device path never needs a HuggingFace object. `from_hf`
accepts anything that looks like a `Qwen2Config` (or a model carrying one).
"""

from __future__ import annotations

from dataclasses import asdict, dataclass, replace

VOCAB_QWEN2 = 151936


@dataclass(frozen=True)
class ModelConfig:
    num_layers: int
    hidden_size: int
    num_heads: int
    num_kv_heads: int
    head_dim: int
    intermediate_size: int
    vocab_size: int = VOCAB_QWEN2
    rope_theta: float = 1e6
    rms_norm_eps: float = 1e-6
    tie_word_embeddings: bool = True
    max_position: int = 32768

    @property
    def q_size(self) -> int:
        return self.num_heads * self.head_dim

    @property
    def kv_size(self) -> int:
        return self.num_kv_heads * self.head_dim

    @property
    def qkv_size(self) -> int:
        return self.q_size + 2 * self.kv_size

    @property
    def group(self) -> int:
        return self.num_heads // self.num_kv_heads

    @property
    def scaling(self) -> float:
        return self.head_dim ** -0.5

    def body_params(self) -> int:
        h, i = self.hidden_size, self.intermediate_size
        per_layer = (
            h * self.qkv_size + self.qkv_size  # q/k/v weights + biases
            + self.q_size * h                  # o_proj
            + 3 * h * i                        # gate, up, down
            + 2 * h                            # two RMSNorm weights
        )
        return self.num_layers * per_layer + h

    def embed_params(self) -> int:
        return self.vocab_size * self.hidden_size

    def kv_bytes_per_token(self, elem_bytes: int) -> int:
        """K+V bytes one token occupies across all layers of the paged pool."""
        return self.num_layers * 2 * self.kv_size * elem_bytes

    def to_dict(self) -> dict:
        return asdict(self)

    @classmethod
    def from_hf(cls, cfg) -> "ModelConfig":
        cfg = getattr(cfg, "config", cfg)
        n_heads = cfg.num_attention_heads
        head_dim = getattr(cfg, "head_dim", None) or cfg.hidden_size // n_heads
        rope = getattr(cfg, "rope_parameters", None) or {}
        theta = rope.get("rope_theta", getattr(cfg, "rope_theta", 1e6))
        return cls(
            num_layers=cfg.num_hidden_layers,
            hidden_size=cfg.hidden_size,
            num_heads=n_heads,
            num_kv_heads=getattr(cfg, "num_key_value_heads", n_heads),
            head_dim=head_dim,
            intermediate_size=cfg.intermediate_size,
            vocab_size=cfg.vocab_size,
            rope_theta=float(theta),
            rms_norm_eps=float(cfg.rms_norm_eps),
            tie_word_embeddings=bool(getattr(cfg, "tie_word_embeddings", True)),
            max_position=int(getattr(cfg, "max_position_embeddings", 32768)),
        )

    def to_hf(self):
        """A `transformers.Qwen2Config` with these shapes (used by test fixtures)."""
        from transformers import Qwen2Config

        return Qwen2Config(
            vocab_size=self.vocab_size,
            hidden_size=self.hidden_size,
            intermediate_size=self.intermediate_size,
            num_hidden_layers=self.num_layers,
            num_attention_heads=self.num_heads,
            num_key_value_heads=self.num_kv_heads,
            head_dim=self.head_dim,
            max_position_embeddings=self.max_position,
            rope_theta=self.rope_theta,
            rms_norm_eps=self.rms_norm_eps,
            tie_word_embeddings=self.tie_word_embeddings,
            initializer_range=0.02,
        )


# Qwen2.5-0.5B architecture (draft, and the CPU-runnable self-spec model).
QWEN2_0_5B = ModelConfig(
    num_layers=24, hidden_size=896, num_heads=14, num_kv_heads=2, head_dim=64,
    intermediate_size=4864,
)

# Qwen2.5-3B architecture (target).
QWEN2_3B = ModelConfig(
    num_layers=36, hidden_size=2048, num_heads=16, num_kv_heads=2, head_dim=128,
    intermediate_size=11008,
)

# A two-layer model with the same structure (GQA, biases, tied head) that the
# CPU oracle finishes in milliseconds; used for exhaustive parity sweeps.
TINY = ModelConfig(
    num_layers=2, hidden_size=256, num_heads=4, num_kv_heads=2, head_dim=64,
    intermediate_size=512, vocab_size=1024,
)

TINY_HD128 = ModelConfig(
    num_layers=2, hidden_size=256, num_heads=2, num_kv_heads=1, head_dim=128,
    intermediate_size=512, vocab_size=1024,
)

# The benchmark models' layer shapes (heads, head_dim, hidden, intermediate,
# full vocabulary) at two layers: the reference runs them on CPU in well under a
# second per pass, so the bf16 hot path of the 3B target (head_dim 128, 16/2
# heads) and of the 0.5B draft is pinned to reference outputs at these shapes.
QWEN2_3B_L2 = replace(QWEN2_3B, num_layers=2)
QWEN2_0_5B_L2 = replace(QWEN2_0_5B, num_layers=2)

PRESETS = {
    "qwen2.5-0.5b": QWEN2_0_5B,
    "qwen2.5-3b": QWEN2_3B,
    "qwen2.5-0.5b-2layer": QWEN2_0_5B_L2,
    "qwen2.5-3b-2layer": QWEN2_3B_L2,
    "tiny": TINY,
    "tiny-hd128": TINY_HD128,
}
