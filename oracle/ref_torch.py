"""The reference's CPU path in torch, for the timed CPU baseline — TEST INFRASTRUCTURE.

The reference computes its host oracle with torch on CPU (``reference/fused_ops.py``,
composed by ``model/qwen35_moe_dflash/fused/model.py``).  This module restates the same
arithmetic with torch CPU tensors so that ``bench.py``'s ``cpu_baseline`` leg and its
``--impl reference`` arm time the reference's algorithm at the speed of the reference's
own library (multi-threaded ATen), not at numpy's.  Only ``bench.py`` (those two legs)
and ``tests/`` use it; its results are checked against the numpy oracle, which is pinned
to the reference's own outputs (``tests/test_oracle_golden.py``,
``tests/test_ref_torch.py``).

Precision follows the reference's CPU run as planned for the baseline: dense bf16
weights and activations for the projections, attention and experts (the W4A16 weights
dequantized), fp32 for the gated delta rule (its operator takes fp16/fp32 only).
"""
from __future__ import annotations

import torch
import torch.nn.functional as F


def rms_norm(x, gamma, eps):
    """reference/fused_ops.py:28-34: fp32 statistics, cast back, times the given gamma."""
    xf = x.float()
    inv = torch.rsqrt(xf.pow(2).mean(dim=-1, keepdim=True) + eps)
    return (xf * inv).to(x.dtype) * gamma


def conv_silu(projected, history, weight):
    """fused_ops.py:37-56 + fused/model.py:238-239: history ++ block, depthwise causal
    conv (no bias), SiLU.  projected [B,S,C], history [B,C,K-1], weight [C,1,K]."""
    padded = torch.cat([history, projected.transpose(1, 2)], dim=2)
    conv = F.conv1d(padded, weight, groups=weight.shape[0])      # [B, C, S]
    new_history = padded[:, :, padded.shape[2] - history.shape[2]:].clone()
    return F.silu(conv.transpose(1, 2)), new_history


def gated_delta_rule(q, k, v, g, beta, state, length):
    """fused_ops.py:59-107, sequential form, fp32: per token t < length[b]
    S <- e^g S; delta = beta (v - S^T k); S <- S + k delta^T; o = S^T q."""
    q = q.float()
    k = k.float()
    q = q * torch.rsqrt((q * q).sum(-1, keepdim=True) + 1e-6) * (q.shape[-1] ** -0.5)
    k = k * torch.rsqrt((k * k).sum(-1, keepdim=True) + 1e-6)
    v, g, beta = v.float(), g.float(), beta.float()
    s = state.float().clone()
    out = torch.zeros(v.shape, dtype=torch.float32)
    for t in range(q.shape[1]):
        live = (t < length).view(-1, 1, 1, 1)
        dec = s * torch.exp(g[:, t]).unsqueeze(-1).unsqueeze(-1)
        pred = torch.einsum("bhkv,bhk->bhv", dec, k[:, t])
        delta = (v[:, t] - pred) * beta[:, t].unsqueeze(-1)
        upd = dec + k[:, t].unsqueeze(-1) * delta.unsqueeze(-2)
        s = torch.where(live, upd, s)
        o = torch.einsum("bhkv,bhk->bhv", s, q[:, t])
        out[:, t] = torch.where(live.view(-1, 1, 1), o, torch.zeros_like(o))
    return out, s


def gdn_layer(x, w, conv_hist, state, *, kh, vh, dk, dv, eps=1e-6):
    """One gated-DeltaNet mixer (fused/model.py:232-263) on x [B,S,H] (bf16)."""
    b, s, _ = x.shape
    kw = kh * dk
    proj = F.linear(x, w["qkv"])
    mixed, hist = conv_silu(proj, conv_hist, w["conv"])
    q = mixed[..., :kw].reshape(b, s, kh, dk).repeat_interleave(vh // kh, dim=2)
    k = mixed[..., kw:2 * kw].reshape(b, s, kh, dk).repeat_interleave(vh // kh, dim=2)
    v = mixed[..., 2 * kw:].reshape(b, s, vh, dv)
    xf = x.float()
    beta = torch.sigmoid(xf @ w["b"].float().t())
    g = -torch.exp(w["A_log"]) * F.softplus(xf @ w["a"].float().t() + w["dt_bias"])
    core, new_state = gated_delta_rule(q, k, v, g, beta, state, torch.full((b,), s))
    z = F.linear(x, w["z"]).reshape(b, s, vh, dv)
    normed = rms_norm(core.to(x.dtype), w["norm"], eps) * F.silu(z)
    return F.linear(normed.reshape(b, s, vh * dv), w["out"]), hist, new_state


def _rope(x, start, rot, theta):
    half = rot // 2
    inv = 1.0 / (theta ** (torch.arange(0, half, dtype=torch.float32) * 2 / rot))
    ang = torch.arange(start, start + x.shape[-2], dtype=torch.float32)[:, None] * inv[None]
    ang = torch.cat([ang, ang], dim=-1)
    cos, sin = ang.cos().to(x.dtype), ang.sin().to(x.dtype)
    head, tail = x[..., :rot], x[..., rot:]
    swapped = torch.cat([-head[..., half:], head[..., :half]], dim=-1)
    return torch.cat([head * cos + swapped * sin, tail], dim=-1)


def attention_layer(x, w, key, value, start, *, heads, kv_heads, dim, rot, theta, eps=1e-6):
    """One full-attention mixer (fused/model.py:265-294): q|gate projection, q/k RMSNorm
    (+1 gamma), partial RoPE, causal GQA over cache ++ block (fused_ops.py:110-145, fp32
    scores), sigmoid output gate, o_proj.  key/value [B,Hkv,ctx,D]."""
    b, s, _ = x.shape
    qg = F.linear(x, w["q"]).reshape(b, s, heads, 2 * dim)
    q = rms_norm(qg[..., :dim], w["q_norm"] + 1, eps).transpose(1, 2)
    gate = qg[..., dim:].reshape(b, s, heads * dim)
    k = rms_norm(F.linear(x, w["k"]).reshape(b, s, kv_heads, dim), w["k_norm"] + 1, eps).transpose(1, 2)
    vv = F.linear(x, w["v"]).reshape(b, s, kv_heads, dim).transpose(1, 2)
    q, k = _rope(q, start, rot, theta), _rope(k, start, rot, theta)
    keys = torch.cat([key, k], dim=2)
    vals = torch.cat([value, vv], dim=2)
    rep = heads // kv_heads
    kf = keys.repeat_interleave(rep, dim=1).float()
    vf = vals.repeat_interleave(rep, dim=1).float()
    scores = (q.float() @ kf.transpose(-1, -2)) * dim ** -0.5
    pos = torch.arange(s) + start
    mask = torch.arange(keys.shape[2])[None, :] > pos[:, None]
    probs = torch.softmax(scores.masked_fill(mask, float("-inf")), dim=-1)
    mixed = (probs @ vf).to(x.dtype).transpose(1, 2).reshape(b, s, heads * dim)
    return F.linear(mixed * torch.sigmoid(gate), w["o"])


def moe_layer(x, w, experts, *, top_k):
    """Routed SwiGLU experts (fused_ops.py:148-173: fp32 softmax, top-k, renormalised,
    ascending-expert accumulation) plus the gated shared expert (fused/model.py:305-307).
    ``experts(e)`` returns expert e's (gate_up [2I,H], down [H,I]) weights."""
    flat = x.reshape(-1, x.shape[-1])
    probs = torch.softmax(F.linear(flat, w["router"]).float(), dim=-1)
    top_w, top_i = torch.topk(probs, top_k, dim=-1)
    top_w = (top_w / top_w.sum(-1, keepdim=True)).to(x.dtype)
    out = torch.zeros_like(flat)
    for e in torch.unique(top_i).tolist():
        rows, slots = torch.nonzero(top_i == e, as_tuple=True)
        gu, dn = experts(e)
        gate, up = F.linear(flat[rows], gu).chunk(2, dim=-1)
        out[rows] += F.linear(F.silu(gate) * up, dn) * top_w[rows, slots].unsqueeze(-1)
    sg, su = F.linear(flat, w["shared_gu"]).chunk(2, dim=-1)
    shared = F.linear(F.silu(sg) * su, w["shared_down"])
    return (out + shared * torch.sigmoid(F.linear(flat, w["shared_gate"]))).reshape(x.shape)
