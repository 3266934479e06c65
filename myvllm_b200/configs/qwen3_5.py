"""Attention-stack shapes of the Qwen3.5-style hybrid text models served by myvllm
(the fields of ``m/configs/qwen3_5.py`` that the attention path reads; MoE and vision
fields are out of scope).  Defaults describe the reference's text config."""

from __future__ import annotations

from dataclasses import dataclass


@dataclass
class HybridAttentionConfig:
    hidden_size: int = 2048
    num_hidden_layers: int = 40
    full_attention_interval: int = 4  # every 4th layer is full attention, the rest GDN
    # gated DeltaNet
    linear_num_key_heads: int = 16
    linear_num_value_heads: int = 32
    linear_key_head_dim: int = 128
    linear_value_head_dim: int = 128
    linear_conv_kernel_dim: int = 4
    # gated full attention
    num_attention_heads: int = 16
    num_key_value_heads: int = 2
    head_dim: int = 256
    partial_rotary_factor: float = 0.25
    rope_theta: float = 10_000_000.0
    attention_bias: bool = False
    rms_norm_eps: float = 1e-6

    def layer_types(self) -> list[str]:
        return ["full_attention" if (i + 1) % self.full_attention_interval == 0 else "linear_attention"
                for i in range(self.num_hidden_layers)]
