"""Target-model configuration for the block-verify path.

The fields and their validation follow the reference's ``_configuration``
(model/qwen35_moe_dflash/fused/model.py:36-83) and the locked target config
(specs/target-config.json ``text_config``).  Two extra fields describe this
library's weight format: ``quant_group`` (W4A16 symmetric group size along K)
and ``feature_layers`` (the DFlash feature taps, model/qwen35_moe_dflash/config.py:219-232).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field, replace


@dataclass(frozen=True)
class TargetConfig:
    hidden_size: int
    num_hidden_layers: int
    vocab_size: int
    num_attention_heads: int
    num_key_value_heads: int
    head_dim: int
    linear_num_key_heads: int
    linear_num_value_heads: int
    linear_key_head_dim: int
    linear_value_head_dim: int
    linear_conv_kernel_dim: int
    num_experts: int
    num_experts_per_tok: int
    moe_intermediate_size: int
    shared_expert_intermediate_size: int
    layer_types: tuple[str, ...]
    feature_layers: tuple[int, ...]
    rms_norm_eps: float = 1e-6
    rope_theta: float = 10_000_000.0
    partial_rotary_factor: float = 0.25
    quant_group: int = 128
    max_position_embeddings: int = 262144

    def __post_init__(self):
        positive = ("hidden_size", "num_hidden_layers", "vocab_size", "num_attention_heads",
                    "num_key_value_heads", "head_dim", "linear_num_key_heads",
                    "linear_num_value_heads", "linear_key_head_dim", "linear_value_head_dim",
                    "linear_conv_kernel_dim", "num_experts", "num_experts_per_tok",
                    "moe_intermediate_size", "shared_expert_intermediate_size", "quant_group")
        for name in positive:
            v = getattr(self, name)
            if isinstance(v, bool) or not isinstance(v, int) or v <= 0:
                raise ValueError(f"{name} must be a positive integer")
        if len(self.layer_types) != self.num_hidden_layers or set(self.layer_types) - {
                "linear_attention", "full_attention"}:
            raise ValueError("layer_types must declare every full/linear attention layer")
        if (self.num_attention_heads % self.num_key_value_heads
                or self.linear_num_value_heads % self.linear_num_key_heads):
            raise ValueError("query/value head counts must be multiples of KV/key heads")
        if self.num_experts_per_tok > self.num_experts:
            raise ValueError("top-k exceeds expert count")
        if not math.isfinite(self.rms_norm_eps) or self.rms_norm_eps <= 0:
            raise ValueError("rms_norm_eps must be finite and positive")
        width = self.rotary_dim
        if width < 2 or width % 2 or not math.isfinite(self.rope_theta) or self.rope_theta <= 0:
            raise ValueError("RoPE requires positive even rotary width and positive finite theta")
        fl = self.feature_layers
        if (not fl or tuple(sorted(set(fl))) != tuple(fl) or fl[0] < 0
                or fl[-1] >= self.num_hidden_layers):
            raise ValueError("feature_layers must be sorted unique valid decoder layer IDs")

    # derived sizes -------------------------------------------------------------------
    @property
    def rotary_dim(self) -> int:
        return int(self.head_dim * self.partial_rotary_factor)

    @property
    def key_width(self) -> int:  # GDN q or k channels
        return self.linear_num_key_heads * self.linear_key_head_dim

    @property
    def value_width(self) -> int:  # GDN v / z channels
        return self.linear_num_value_heads * self.linear_value_head_dim

    @property
    def conv_channels(self) -> int:
        return 2 * self.key_width + self.value_width

    @property
    def feature_width(self) -> int:
        return len(self.feature_layers) * self.hidden_size

    @property
    def gdn_layers(self) -> tuple[int, ...]:
        return tuple(i for i, k in enumerate(self.layer_types) if k == "linear_attention")

    @property
    def attn_layers(self) -> tuple[int, ...]:
        return tuple(i for i, k in enumerate(self.layer_types) if k == "full_attention")

    def to_hf_text_config(self) -> dict:
        """The dict shape the reference's ``FusedTargetModel`` reads (text_config keys)."""
        return {
            "hidden_size": self.hidden_size, "num_hidden_layers": self.num_hidden_layers,
            "vocab_size": self.vocab_size, "num_attention_heads": self.num_attention_heads,
            "num_key_value_heads": self.num_key_value_heads, "head_dim": self.head_dim,
            "linear_num_key_heads": self.linear_num_key_heads,
            "linear_num_value_heads": self.linear_num_value_heads,
            "linear_key_head_dim": self.linear_key_head_dim,
            "linear_value_head_dim": self.linear_value_head_dim,
            "linear_conv_kernel_dim": self.linear_conv_kernel_dim,
            "num_experts": self.num_experts, "num_experts_per_tok": self.num_experts_per_tok,
            "moe_intermediate_size": self.moe_intermediate_size,
            "shared_expert_intermediate_size": self.shared_expert_intermediate_size,
            "max_position_embeddings": self.max_position_embeddings,
            "layer_types": list(self.layer_types), "rms_norm_eps": self.rms_norm_eps,
            "rope_parameters": {"rope_type": "default", "rope_theta": self.rope_theta,
                                "partial_rotary_factor": self.partial_rotary_factor},
            "attention_bias": False, "attention_dropout": 0.0, "hidden_act": "silu",
            "norm_topk_prob": True,
        }


def _interleaved(n_layers: int, interval: int = 4) -> tuple[str, ...]:
    return tuple("full_attention" if (i + 1) % interval == 0 else "linear_attention"
                 for i in range(n_layers))


# Qwen3.5-35B-A3B target (specs/target-config.json), W4A16 group 128.
QWEN35_35B_A3B = TargetConfig(
    hidden_size=2048, num_hidden_layers=40, vocab_size=248320,
    num_attention_heads=16, num_key_value_heads=2, head_dim=256,
    linear_num_key_heads=16, linear_num_value_heads=32,
    linear_key_head_dim=128, linear_value_head_dim=128, linear_conv_kernel_dim=4,
    num_experts=256, num_experts_per_tok=8, moe_intermediate_size=512,
    shared_expert_intermediate_size=512, layer_types=_interleaved(40),
    feature_layers=(1, 6, 11, 16, 22, 27, 32, 37), rope_theta=10_000_000.0,
    partial_rotary_factor=0.25, quant_group=128,
)

# The CPU-runnable tiny target of the benchmark's first configuration: 4 layers
# (3 GDN + 1 attention), hidden 256, 16 experts top-4 + shared, expert FFN 128,
# GDN 4 QK / 8 V heads of 64, attention 4 Q / 1 KV heads of 64, vocab 4096,
# int4 group 32.
TINY = TargetConfig(
    hidden_size=256, num_hidden_layers=4, vocab_size=4096,
    num_attention_heads=4, num_key_value_heads=1, head_dim=64,
    linear_num_key_heads=4, linear_num_value_heads=8,
    linear_key_head_dim=64, linear_value_head_dim=64, linear_conv_kernel_dim=4,
    num_experts=16, num_experts_per_tok=4, moe_intermediate_size=128,
    shared_expert_intermediate_size=128, layer_types=_interleaved(4),
    feature_layers=(1, 2), rope_theta=10_000_000.0, partial_rotary_factor=0.25,
    quant_group=32, max_position_embeddings=4096,
)


# The tiny target shaped for an original group-256 checkpoint (every contraction
# dimension a multiple of 256, every quantised projection a multiple of 16 rows):
# expert FFN and shared expert 256, GDN 8 QK / 16 V heads, group 128.
TINY_G256 = replace(TINY, moe_intermediate_size=256, shared_expert_intermediate_size=256, quant_group=128,
                    linear_num_key_heads=8, linear_num_value_heads=16)


def with_layers(config: TargetConfig, n_layers: int) -> TargetConfig:
    """Same architecture with fewer decoder layers (for tests), taps clipped."""
    taps = tuple(i for i in config.feature_layers if i < n_layers) or (n_layers - 1,)
    return replace(config, num_hidden_layers=n_layers, layer_types=_interleaved(n_layers),
                   feature_layers=taps)


@dataclass(frozen=True)
class DraftConfig:
    """The DFlash draft (model/qwen35_moe_dflash/config.py:11-140; the locked checkpoint
    specs/draft-config.json): a dense Qwen3-style decoder over a 16-token block (anchor +
    mask tokens) attending to the target's tapped features, sliding-window causal layers
    and a last full-attention layer that is bidirectional over the block."""
    hidden_size: int
    intermediate_size: int
    num_hidden_layers: int
    num_attention_heads: int
    num_key_value_heads: int
    head_dim: int
    layer_types: tuple[str, ...]
    target_layer_ids: tuple[int, ...]
    mask_token_id: int
    sliding_window: int
    use_sliding_window: bool = True
    block_size: int = 16
    rms_norm_eps: float = 1e-6
    rope_theta: float = 10_000_000.0
    input_embedding_scale: float = 1.0

    def __post_init__(self):
        if self.num_attention_heads % self.num_key_value_heads:
            raise ValueError("attention heads must be divisible by KV heads")
        if len(self.layer_types) != self.num_hidden_layers or set(self.layer_types) - {
                "sliding_attention", "full_attention"}:
            raise ValueError("layer_types must name one sliding_attention / full_attention per layer")
        if not self.target_layer_ids or tuple(sorted(set(self.target_layer_ids))) != self.target_layer_ids:
            raise ValueError("target_layer_ids must be sorted and unique")
        if min(self.hidden_size, self.intermediate_size, self.head_dim, self.sliding_window, self.block_size) <= 0:
            raise ValueError("DFlash configuration values must be positive")
        if self.input_embedding_scale != 1.0:
            raise ValueError("the draft block embedding is used unscaled (input_embedding_scale 1)")

    @property
    def feature_size(self) -> int:
        return len(self.target_layer_ids) * self.hidden_size

    def window(self, layer: int) -> int:
        """Sliding window of a layer's causal mask (0: none)."""
        sliding = self.layer_types[layer] == "sliding_attention"
        return self.sliding_window if sliding and self.use_sliding_window else 0

    def causal(self, layer: int) -> bool:
        """Sliding layers are causal; the full-attention layer is bidirectional over the
        block (model/qwen35_moe_dflash/model.py:134-141)."""
        return self.layer_types[layer] == "sliding_attention"

    def to_reference_dict(self, vocab_size: int, num_target_layers: int) -> dict:
        """The config.json shape the reference's Qwen35DFlashConfig.from_dict reads."""
        return {
            "hidden_size": self.hidden_size, "intermediate_size": self.intermediate_size,
            "vocab_size": vocab_size, "num_hidden_layers": self.num_hidden_layers,
            "num_attention_heads": self.num_attention_heads, "num_key_value_heads": self.num_key_value_heads,
            "head_dim": self.head_dim, "num_target_layers": num_target_layers,
            "layer_types": list(self.layer_types), "rms_norm_eps": self.rms_norm_eps,
            "rope_parameters": {"rope_theta": self.rope_theta, "rope_type": "default"},
            "max_position_embeddings": 262144, "sliding_window": self.sliding_window,
            "use_sliding_window": self.use_sliding_window, "attention_bias": False, "attention_dropout": 0.0,
            "hidden_act": "silu", "dtype": "bfloat16",
            "dflash_config": {"block_size": self.block_size, "mask_token_id": self.mask_token_id,
                              "target_layer_ids": list(self.target_layer_ids)},
        }


# The Qwen3.5-35B-A3B DFlash draft (specs/draft-config.json).
QWEN35_DFLASH_DRAFT = DraftConfig(
    hidden_size=2048, intermediate_size=6144, num_hidden_layers=6, num_attention_heads=32,
    num_key_value_heads=8, head_dim=128,
    layer_types=("sliding_attention",) * 5 + ("full_attention",),
    target_layer_ids=(1, 6, 11, 16, 22, 27, 32, 37), mask_token_id=248077, sliding_window=4096,
)

# The draft of the tiny configuration: 2 layers (sliding, full), a window of 8 positions
# so that the window cuts into the context in tests; taps = TINY.feature_layers.
TINY_DRAFT = DraftConfig(
    hidden_size=256, intermediate_size=512, num_hidden_layers=2, num_attention_heads=4,
    num_key_value_heads=1, head_dim=64, layer_types=("sliding_attention", "full_attention"),
    target_layer_ids=(1, 2), mask_token_id=4095, sliding_window=8,
)
