"""Seeded random-init weights and states for the target (no checkpoint is available).

Names and shapes follow the reference's canonical inventory
(model/qwen35_moe_dflash/target/weight_shapes.py:7-44).  Values follow the
benchmark's configuration: every matrix N(0, 0.02); RMSNorm weights stored
zero-centred (0, effective 1) except the GDN gated norm (stored effective, 1);
``A_log`` and ``dt_bias`` as the reference's deterministic tiny generator
(model/qwen35_moe_dflash/graph/weights.py:194-198).  Values outside the W4 scope
are rounded to bf16; matrices inside it are quantized by the caller.

Each tensor is drawn from its own generator seeded with (seed, crc32(name)), so a
model with fewer layers shares its tensors with the full one.
"""
from __future__ import annotations

import math
import zlib

import numpy as np

from .config import TargetConfig

# Matrices stored as W4A16 (int4 symmetric, bf16 group scales).  The router, the
# shared-expert gate, the GDN a/b predictors, the embedding and lm_head stay bf16
# (model/qwen35_moe_dflash/reference/quantization.py:92-97).
W4_SUFFIXES = (
    ".linear_attn.in_proj_qkv.weight", ".linear_attn.in_proj_z.weight",
    ".linear_attn.out_proj.weight", ".self_attn.q_proj.weight", ".self_attn.k_proj.weight",
    ".self_attn.v_proj.weight", ".self_attn.o_proj.weight", ".mlp.experts.gate_up_proj",
    ".mlp.experts.down_proj", ".mlp.shared_expert.gate_proj.weight",
    ".mlp.shared_expert.up_proj.weight", ".mlp.shared_expert.down_proj.weight",
)


def is_w4(name: str) -> bool:
    return name.endswith(W4_SUFFIXES)


def weight_shapes(c: TargetConfig) -> dict[str, tuple[int, ...]]:
    h, d = c.hidden_size, c.head_dim
    shapes = {"target.embed_tokens.weight": (c.vocab_size, h),
              "target.norm.weight": (h,), "target.lm_head.weight": (c.vocab_size, h)}
    for i, kind in enumerate(c.layer_types):
        p = f"target.layers.{i}"
        shapes[p + ".input_layernorm.weight"] = (h,)
        shapes[p + ".post_attention_layernorm.weight"] = (h,)
        if kind == "linear_attention":
            q = p + ".linear_attn"
            vh = c.linear_num_value_heads
            shapes.update({q + ".in_proj_qkv.weight": (c.conv_channels, h),
                           q + ".in_proj_z.weight": (c.value_width, h),
                           q + ".in_proj_b.weight": (vh, h), q + ".in_proj_a.weight": (vh, h),
                           q + ".A_log": (vh,), q + ".dt_bias": (vh,),
                           q + ".conv1d.weight": (c.conv_channels, 1, c.linear_conv_kernel_dim),
                           q + ".norm.weight": (c.linear_value_head_dim,),
                           q + ".out_proj.weight": (h, c.value_width)})
        else:
            q = p + ".self_attn"
            shapes.update({q + ".q_proj.weight": (c.num_attention_heads * d * 2, h),
                           q + ".k_proj.weight": (c.num_key_value_heads * d, h),
                           q + ".v_proj.weight": (c.num_key_value_heads * d, h),
                           q + ".o_proj.weight": (h, c.num_attention_heads * d),
                           q + ".q_norm.weight": (d,), q + ".k_norm.weight": (d,)})
        e, m, s = c.num_experts, c.moe_intermediate_size, c.shared_expert_intermediate_size
        q = p + ".mlp"
        shapes.update({q + ".gate.weight": (e, h),
                       q + ".experts.gate_up_proj": (e, 2 * m, h),
                       q + ".experts.down_proj": (e, h, m),
                       q + ".shared_expert.gate_proj.weight": (s, h),
                       q + ".shared_expert.up_proj.weight": (s, h),
                       q + ".shared_expert.down_proj.weight": (h, s),
                       q + ".shared_expert_gate.weight": (1, h)})
    return shapes


def _bf16(x: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(x, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32).view(np.float32)


def _rng(seed: int, name: str) -> np.random.Generator:
    return np.random.default_rng([seed, zlib.crc32(name.encode())])


def init_value(name: str, shape, seed: int, std: float = 0.02) -> np.ndarray:
    """float32 value of one tensor (bf16-rounded unless it is a W4 matrix)."""
    n = math.prod(shape)
    if name.endswith(".A_log"):
        value = np.log(np.arange(1, n + 1, dtype=np.float64)).reshape(shape)
    elif name.endswith(".dt_bias"):
        dt = np.exp(_rng(seed, name).uniform(math.log(.001), math.log(.1), shape))
        value = dt + np.log(-np.expm1(-dt))
    elif name.endswith("norm.weight") or name.endswith("layernorm.weight"):
        value = np.full(shape, 1.0 if ".linear_attn.norm." in name else 0.0)
    else:
        value = _rng(seed, name).normal(0.0, std, shape)
    value = value.astype(np.float32)
    return value if is_w4(name) else _bf16(value)


def init_weights(c: TargetConfig, seed: int = 17, std: float = 0.02) -> dict[str, np.ndarray]:
    """All target.* tensors as float32 numpy arrays (small configurations only)."""
    return {name: init_value(name, shape, seed, std) for name, shape in weight_shapes(c).items()}


def draft_weight_shapes(d) -> dict[str, tuple[int, ...]]:
    """Tensors of the DFlash draft by the reference's parameter names
    (model/qwen35_moe_dflash/model.py:310-391): layers.*, norm, fc, hidden_norm."""
    h, hd = d.hidden_size, d.head_dim
    q, kv = d.num_attention_heads * hd, d.num_key_value_heads * hd
    shapes = {"norm.weight": (h,), "fc.weight": (h, d.feature_size), "hidden_norm.weight": (h,)}
    for i in range(d.num_hidden_layers):
        p = f"layers.{i}"
        shapes.update({p + ".input_layernorm.weight": (h,), p + ".post_attention_layernorm.weight": (h,),
                       p + ".self_attn.q_proj.weight": (q, h), p + ".self_attn.k_proj.weight": (kv, h),
                       p + ".self_attn.v_proj.weight": (kv, h), p + ".self_attn.o_proj.weight": (h, q),
                       p + ".self_attn.q_norm.weight": (hd,), p + ".self_attn.k_norm.weight": (hd,),
                       p + ".mlp.gate_proj.weight": (d.intermediate_size, h),
                       p + ".mlp.up_proj.weight": (d.intermediate_size, h),
                       p + ".mlp.down_proj.weight": (h, d.intermediate_size)})
    return shapes


def init_draft_weights(d, seed: int = 29, std: float = 0.04) -> dict[str, np.ndarray]:
    """Seeded draft weights (bf16 values): matrices N(0, std), norm weights (stored as
    the effective scale) 1 + N(0, 0.1)."""
    out = {}
    for name, shape in draft_weight_shapes(d).items():
        if name.endswith("norm.weight"):
            value = 1.0 + _rng(seed, name).normal(0.0, 0.1, shape)
        else:
            value = _rng(seed, name).normal(0.0, std, shape)
        out[name] = _bf16(value.astype(np.float32))
    return out
