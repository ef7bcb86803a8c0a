"""Architecture description of the Qwen3.5 hybrid text decoder.

Field names follow the checkpoint ``config.json`` keys the reference reads
(main.py:354-370).  ``qwen35_4b()`` is the Qwen3.5-4B text decoder
(README.md:17-33): 32 layers in a 3 linear : 1 full pattern, hidden 2560,
MLP 9216, 16Q/4KV full-attention heads of 256 with 64-dim partial RoPE,
16-key / 32-value GatedDeltaNet heads of 128, vocab 248320.
"""

from __future__ import annotations

from dataclasses import dataclass, field


def hybrid_layer_types(n_layers: int, full_every: int = 4) -> list[str]:
    """Every ``full_every``-th layer is full attention, the rest linear (3:1)."""
    return ["full_attention" if (i + 1) % full_every == 0 else "linear_attention"
            for i in range(n_layers)]


@dataclass
class Qwen35Config:
    hidden_size: int = 2560
    intermediate_size: int = 9216
    num_hidden_layers: int = 32
    vocab_size: int = 248320
    num_attention_heads: int = 16
    num_key_value_heads: int = 4
    head_dim: int = 256
    partial_rotary_factor: float = 0.25
    rope_theta: float = 10_000_000.0
    linear_num_key_heads: int = 16
    linear_num_value_heads: int = 32
    linear_key_head_dim: int = 128
    linear_value_head_dim: int = 128
    linear_conv_kernel_dim: int = 4
    rms_norm_eps: float = 1e-6
    fp8_lm_head: bool = True
    layer_types: list = field(default_factory=list)

    def __post_init__(self):
        if not self.layer_types:
            self.layer_types = hybrid_layer_types(self.num_hidden_layers)
        assert len(self.layer_types) == self.num_hidden_layers

    @property
    def rotary_dim(self) -> int:
        return int(self.head_dim * self.partial_rotary_factor)

    @property
    def linear_key_dim(self) -> int:
        return self.linear_num_key_heads * self.linear_key_head_dim

    @property
    def linear_value_dim(self) -> int:
        return self.linear_num_value_heads * self.linear_value_head_dim

    @property
    def conv_dim(self) -> int:
        return 2 * self.linear_key_dim + self.linear_value_dim


def qwen35_4b(**kw) -> Qwen35Config:
    return Qwen35Config(**kw)


def qwen35_tiny(**kw) -> Qwen35Config:
    """A small member of the same family for oracle-speed parity runs.

    Every dimension keeps the 4B model's structure (head dims, head ratios,
    conv width, 3:1 pattern) at widths the CPU oracle finishes in seconds.
    """
    base = dict(hidden_size=512, intermediate_size=1536, num_hidden_layers=4, vocab_size=4096,
                num_attention_heads=4, num_key_value_heads=1, head_dim=256,
                linear_num_key_heads=2, linear_num_value_heads=4,
                linear_key_head_dim=128, linear_value_head_dim=128)
    base.update(kw)
    return Qwen35Config(**base)
