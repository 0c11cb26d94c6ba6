"""Drop-in fused-ops adapter module backed by libqw_b200.so (sm_100a).

Bind it exactly like the reference's host oracle::

    ModuleFusedOps(qwen35_dflash_b200.fused_ops)          # allow_reference not needed

It declares ``FUSED_OPS_ABI = 1``, a non-empty ``BACKEND_ID`` and
``IS_REFERENCE_BACKEND = False`` (model/qwen35_moe_dflash/fused/ops.py:138-176) and
defines the seven operators with the signatures, argument meaning, validation errors
(ValueError) and output dtypes of reference/fused_ops.py:28-173.  Inputs must be CUDA
tensors; outputs are new tensors and inputs are never written.  There is no CPU or
dtype fallback: a missing library or a CPU tensor raises.

Extra entry points (ignored by ModuleFusedOps): ``moe_with_routing``, ``qlinear_w4a16``,
``linear_b16``.
"""
from __future__ import annotations

import math

import torch
from torch import Tensor

from . import lib

FUSED_OPS_ABI = 1
BACKEND_ID = "b200-sm100a"
IS_REFERENCE_BACKEND = False

_FLOAT = (torch.float32, torch.float16, torch.bfloat16)


def _cuda(*values: Tensor | None) -> None:
    for value in values:
        if value is not None and (not isinstance(value, Tensor) or value.device.type != "cuda"):
            raise ValueError(f"{BACKEND_ID} requires CUDA tensors")


def _s(t: Tensor) -> int:
    return lib.stream_ptr(t.device)


def rms_norm(x: Tensor, gamma: Tensor, eps: float) -> Tensor:
    """reference/fused_ops.py:28-34 — gamma is effective (never adds one)."""
    _cuda(x, gamma)
    if not math.isfinite(eps) or eps <= 0 or gamma.shape != x.shape[-1:]:
        raise ValueError("RMSNorm needs positive epsilon and one gamma per feature")
    if x.dtype not in _FLOAT or gamma.dtype not in _FLOAT:
        raise ValueError("rms_norm: floating tensors required")
    out_dtype = torch.promote_types(x.dtype, gamma.dtype)
    if gamma.dtype != x.dtype and gamma.dtype != torch.float32:
        gamma = gamma.to(out_dtype)
        out_dtype = torch.promote_types(x.dtype, gamma.dtype)
    xc = x.contiguous()
    gc = gamma.contiguous()
    y = torch.empty(x.shape, dtype=out_dtype, device=x.device)
    dim = x.shape[-1]
    rows = x.numel() // dim if dim else 0
    lib.call("qw_rms_norm", xc.data_ptr(), lib.dtype_code(x.dtype), gc.data_ptr(),
             lib.dtype_code(gc.dtype), y.data_ptr(), lib.dtype_code(out_dtype), rows, dim,
             float(eps), _s(x))
    return y


def conv_state_update(projected: Tensor, history: Tensor) -> tuple[Tensor, Tensor]:
    """reference/fused_ops.py:37-47 — [B,S,C], [B,C,K-1] -> (history', padded [B,C,S+K-1])."""
    _cuda(projected, history)
    if (projected.ndim != 3 or history.ndim != 3 or projected.shape[1] < 1
            or projected.shape[0] != history.shape[0] or projected.shape[2] != history.shape[1]
            or projected.dtype != history.dtype):
        raise ValueError("conv state requires projected [B,S,C] and matching history [B,C,K-1]")
    b, s, c = projected.shape
    k1 = history.shape[-1]
    padded = torch.empty(b, c, s + k1, dtype=projected.dtype, device=projected.device)
    updated = torch.empty(b, c, k1, dtype=projected.dtype, device=projected.device)
    p, h = projected.contiguous(), history.contiguous()
    lib.call("qw_conv_state_update", p.data_ptr(), h.data_ptr(), updated.data_ptr(),
             padded.data_ptr(), lib.dtype_code(p.dtype), b, s, c, k1, _s(p))
    return updated, padded


def causal_conv1d(padded: Tensor, weight: Tensor) -> Tensor:
    """reference/fused_ops.py:50-56 — depthwise, [B,C,S+K-1] x [C,1,K] -> [B,S,C], no SiLU."""
    _cuda(padded, weight)
    if (padded.ndim != 3 or weight.ndim != 3 or weight.shape[1] != 1
            or padded.shape[1] != weight.shape[0] or weight.shape[-1] < 1
            or padded.shape[-1] < weight.shape[-1] or padded.dtype != weight.dtype):
        raise ValueError("depthwise conv requires [B,C,S+K-1] and [C,1,K]")
    b, c, length = padded.shape
    k = weight.shape[-1]
    out = torch.empty(b, length - k + 1, c, dtype=padded.dtype, device=padded.device)
    p, w = padded.contiguous(), weight.contiguous()
    lib.call("qw_causal_conv1d", p.data_ptr(), w.data_ptr(), out.data_ptr(),
             lib.dtype_code(p.dtype), b, c, length, k, _s(p))
    return out


def chunk_gated_delta_rule(query: Tensor, key: Tensor, value: Tensor, g: Tensor, beta: Tensor,
                           initial_state: Tensor, effective_length: Tensor, *, chunk_size: int,
                           use_qk_l2norm_in_kernel: bool) -> tuple[Tensor, Tensor]:
    """reference/fused_ops.py:59-107 — sequential gated delta rule; fp16/fp32 inputs
    as in the reference, plus bf16 (this build's activation dtype)."""
    _cuda(query, key, value, g, beta, initial_state, effective_length)
    if isinstance(chunk_size, bool) or chunk_size not in (1, 64):
        raise ValueError("chunk_size must be 1 or 64")
    if not isinstance(use_qk_l2norm_in_kernel, bool):
        raise ValueError("use_qk_l2norm_in_kernel must be bool")
    if (query.ndim != 4 or key.shape != query.shape or value.ndim != 4
            or value.shape[:3] != query.shape[:3] or g.shape != query.shape[:3]
            or beta.shape != query.shape[:3] or any(d < 1 for d in query.shape)
            or value.shape[-1] < 1):
        raise ValueError("GDN requires compatible [B,S,H,D] tensors and [B,S,H] gates")
    batch, sequence, heads, key_width = query.shape
    if (initial_state.shape != (batch, heads, key_width, value.shape[-1])
            or initial_state.dtype not in (torch.float16, torch.float32)):
        raise ValueError("initial_state must be FP16/FP32 [B,H,Dk,Dv]")
    if (effective_length.dtype != torch.int16 or effective_length.shape != (batch,)
            or bool(((effective_length < 0) | (effective_length > sequence)).any())):
        raise ValueError("effective_length must be INT16 [B] within [0,S]")
    if query.dtype not in _FLOAT or any(t.dtype != query.dtype for t in (key, value, g, beta)):
        raise ValueError("GDN floating inputs must share FP16, BF16 or FP32 dtype")
    q, k, v, gg, bb = (t.contiguous() for t in (query, key, value, g, beta))
    s0 = initial_state.contiguous()
    lens = effective_length.contiguous()
    core = torch.empty(value.shape, dtype=query.dtype, device=query.device)
    state = torch.empty_like(s0)
    lib.call("qw_gated_delta_rule", q.data_ptr(), k.data_ptr(), v.data_ptr(), gg.data_ptr(),
             bb.data_ptr(), lib.dtype_code(q.dtype), s0.data_ptr(), lib.dtype_code(s0.dtype),
             lens.data_ptr(), core.data_ptr(), state.data_ptr(), batch, sequence, heads,
             key_width, value.shape[-1], int(use_qk_l2norm_in_kernel), _s(q))
    return core, state


def cache_update(key: Tensor | None, value: Tensor | None, new_key: Tensor,
                 new_value: Tensor) -> tuple[Tensor, Tensor]:
    """reference/fused_ops.py:110-124 — privately owned appended ND caches."""
    _cuda(key, value, new_key, new_value)
    if ((key is None) != (value is None) or new_key.ndim != 4
            or new_value.ndim != 4 or new_key.shape[:3] != new_value.shape[:3]):
        raise ValueError("KV caches must appear together and use [B,H,T,D]")
    if new_key.dtype != new_value.dtype or new_key.shape != new_value.shape:
        raise ValueError("new key and value must match")
    if key is not None:
        for old, new in ((key, new_key), (value, new_value)):
            if (old.ndim != 4 or old.shape[:2] != new.shape[:2] or old.shape[-1] != new.shape[-1]
                    or old.dtype != new.dtype):
                raise ValueError("old and new KV cache dimensions/dtypes do not match")
        if key.shape[-2] != value.shape[-2]:
            raise ValueError("old key and value cache lengths differ")
    b, h, t_new, d = new_key.shape
    t_old = 0 if key is None else key.shape[-2]
    out_k = torch.empty(b, h, t_old + t_new, d, dtype=new_key.dtype, device=new_key.device)
    out_v = torch.empty_like(out_k)
    k0 = None if key is None else key.contiguous()
    v0 = None if value is None else value.contiguous()
    nk, nv = new_key.contiguous(), new_value.contiguous()
    lib.call("qw_cache_update", lib.ptr(k0), lib.ptr(v0), nk.data_ptr(), nv.data_ptr(),
             out_k.data_ptr(), out_v.data_ptr(), lib.dtype_code(nk.dtype), b, h, t_old, t_new, d,
             _s(nk))
    return out_k, out_v


def attention(query: Tensor, key: Tensor, value: Tensor, *, query_start: int,
              scale: float) -> Tensor:
    """reference/fused_ops.py:127-145 — causal GQA, row i sees keys <= query_start + i."""
    _cuda(query, key, value)
    if (query.ndim != 4 or key.ndim != 4 or value.ndim != 4
            or query.shape[0] != key.shape[0] or key.shape[:3] != value.shape[:3]
            or query.shape[-1] != key.shape[-1] or key.shape[1] < 1
            or query.shape[1] % key.shape[1] or isinstance(query_start, bool)
            or not isinstance(query_start, int) or query_start < 0
            or query_start + query.shape[-2] != key.shape[-2]
            or not math.isfinite(scale) or scale <= 0):
        raise ValueError("attention requires causal append-only GQA [B,H,S,D] inputs")
    if query.dtype not in (torch.bfloat16, torch.float16) or key.dtype != query.dtype or value.dtype != query.dtype:
        raise ValueError("attention: bf16 or fp16 tensors of one dtype required")
    b, h, s, d = query.shape
    q, k, v = query.contiguous(), key.contiguous(), value.contiguous()
    out = torch.empty_like(q)
    nbytes = lib.load().qw_attn_workspace_bytes(b, h, key.shape[1], s, d, key.shape[-2])
    if nbytes < 0:
        raise ValueError("attention requires causal append-only GQA [B,H,S,D] inputs")
    ws = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=q.device)
    lib.call("qw_attention", q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
             lib.dtype_code(q.dtype), b, h, key.shape[1], s, key.shape[-2], d, query_start,
             float(scale), ws.data_ptr(), _s(q))
    return out


def moe(hidden: Tensor, router_weight: Tensor, gate_up: Tensor, down: Tensor, *,
        top_k: int) -> Tensor:
    """reference/fused_ops.py:148-173 — routed SwiGLU experts (dense weights)."""
    out, _ = moe_with_routing(hidden, router_weight, gate_up, down, top_k=top_k)
    return out


def moe_with_routing(hidden: Tensor, router_weight: Tensor, gate_up: Tensor, down: Tensor, *,
                     top_k: int) -> tuple[Tensor, Tensor]:
    """``moe`` that also returns the selected expert indices (int32 [T, k])."""
    _cuda(hidden, router_weight, gate_up, down)
    if (hidden.ndim != 3 or router_weight.ndim != 2 or gate_up.ndim != 3
            or down.ndim != 3 or gate_up.shape[1] % 2
            or router_weight.shape[0] != gate_up.shape[0] or down.shape[0] != gate_up.shape[0]
            or router_weight.shape[1] != hidden.shape[-1] or gate_up.shape[2] != hidden.shape[-1]
            or down.shape[1:] != (hidden.shape[-1], gate_up.shape[1] // 2)
            or isinstance(top_k, bool) or not isinstance(top_k, int)
            or not 0 < top_k <= router_weight.shape[0]):
        raise ValueError("MoE needs compatible expert weights and a valid top_k")
    dt = hidden.dtype
    if dt not in (torch.bfloat16, torch.float16) or any(t.dtype != dt for t in (router_weight, gate_up, down)):
        raise ValueError("moe: bf16 or fp16 tensors of one dtype required")
    flat = hidden.reshape(-1, hidden.shape[-1]).contiguous()
    t, hdim = flat.shape
    e, two_i, _ = gate_up.shape
    out = torch.empty_like(flat)
    idx = torch.empty(t, top_k, dtype=torch.int32, device=hidden.device)
    r, gu, dn = router_weight.contiguous(), gate_up.contiguous(), down.contiguous()
    nbytes = lib.load().qw_moe_workspace_bytes(t, hdim, e, two_i // 2, top_k)
    ws = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=hidden.device)
    lib.call("qw_moe", flat.data_ptr(), r.data_ptr(), gu.data_ptr(), dn.data_ptr(), out.data_ptr(),
             lib.dtype_code(dt), t, hdim, e, two_i // 2, top_k, idx.data_ptr(), ws.data_ptr(), _s(flat))
    return out.reshape_as(hidden), idx


# ------------------------------------------------------------------ W4A16 / bf16 linears
def qlinear_w4a16(x: Tensor, stream: Tensor, n: int, group: int, *, out_dtype=torch.bfloat16) -> Tensor:
    """y = x . W^T for a W4 stream of an [n, K] matrix (K = x.shape[-1]); x bf16."""
    _cuda(x, stream)
    if x.dtype != torch.bfloat16:
        raise ValueError("qlinear_w4a16: x must be bf16")
    k = x.shape[-1]
    flat = x.reshape(-1, k).contiguous()
    mode = lib.QW_OUT_F32 if out_dtype == torch.float32 else lib.QW_OUT_BF16
    y = torch.empty(flat.shape[0], n, dtype=torch.float32 if mode == lib.QW_OUT_F32 else torch.bfloat16,
                    device=x.device)
    lib.call("qw_w4_linear", flat.data_ptr(), stream.data_ptr(), y.data_ptr(), mode, n,
             flat.shape[0], n, k, group, _s(x))
    return y.reshape(*x.shape[:-1], n)


def linear_b16(x: Tensor, stream: Tensor, n: int, *, out_dtype=torch.bfloat16) -> Tensor:
    """y = x . W^T for a B16 stream of a bf16 [n, K] matrix; x bf16."""
    _cuda(x, stream)
    if x.dtype != torch.bfloat16:
        raise ValueError("linear_b16: x must be bf16")
    k = x.shape[-1]
    flat = x.reshape(-1, k).contiguous()
    mode = lib.QW_OUT_F32 if out_dtype == torch.float32 else lib.QW_OUT_BF16
    y = torch.empty(flat.shape[0], n, dtype=torch.float32 if mode == lib.QW_OUT_F32 else torch.bfloat16,
                    device=x.device)
    lib.call("qw_b16_linear", flat.data_ptr(), stream.data_ptr(), y.data_ptr(), mode, n,
             flat.shape[0], n, k, _s(x))
    return y.reshape(*x.shape[:-1], n)
