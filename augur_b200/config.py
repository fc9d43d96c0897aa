"""Model shape configuration the caches are sized from.

Same fields, defaults and validation as augur's QwenConfig
(augur/config.py:4-39), so a config built for augur builds the same caches
here. Only num_hidden_layers, num_key_value_heads and head_dim are read by
the cache code.
"""

from dataclasses import dataclass


@dataclass(frozen=True)
class QwenConfig:
    vocab_size: int = 151936
    hidden_size: int = 896
    intermediate_size: int = 4864
    num_hidden_layers: int = 24
    num_attention_heads: int = 14
    num_key_value_heads: int = 2
    hidden_act: str = "silu"
    max_position_embeddings: int = 32768
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1_000_000.0
    tie_word_embeddings: bool = True
    attention_bias: bool = False

    def __post_init__(self) -> None:
        if self.hidden_act != "silu":
            raise ValueError(f"only silu Qwen MLP is supported, got {self.hidden_act!r}")
        if self.hidden_size % self.num_attention_heads != 0:
            raise ValueError(
                f"hidden_size ({self.hidden_size}) must be divisible by "
                f"num_attention_heads ({self.num_attention_heads})"
            )
        if self.num_attention_heads % self.num_key_value_heads != 0:
            raise ValueError(
                f"num_attention_heads ({self.num_attention_heads}) must be divisible by "
                f"num_key_value_heads ({self.num_key_value_heads})"
            )

    @property
    def head_dim(self) -> int:
        return self.hidden_size // self.num_attention_heads

    @property
    def num_key_value_groups(self) -> int:
        return self.num_attention_heads // self.num_key_value_heads
