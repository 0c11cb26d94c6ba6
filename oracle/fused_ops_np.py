"""numpy restatement of the reference host oracle ``reference/fused_ops.py``.

Test infrastructure only (see ``oracle/__init__.py``).  Every function computes in
float32 like the reference and rounds its result to the dtype the reference would
return, named by a tag ``"f32" | "f16" | "bf16"``.  Inputs are float32 arrays
holding values that are exactly representable in that dtype.
"""
from __future__ import annotations

import math

import numpy as np

from .numerics import round_to, topk_indices


def rms_norm(x, gamma, eps: float, dtype: str = "f32") -> np.ndarray:
    """reference/fused_ops.py:28-34 — normalize in fp32, cast to x.dtype, then times gamma."""
    x = np.asarray(x, np.float32)
    gamma = np.asarray(gamma, np.float32)
    if not math.isfinite(eps) or eps <= 0 or gamma.shape != x.shape[-1:]:
        raise ValueError("RMSNorm needs positive epsilon and one gamma per feature")
    ms = np.mean(np.square(x, dtype=np.float32), axis=-1, keepdims=True, dtype=np.float32)
    normalized = x * (np.float32(1.0) / np.sqrt(ms + np.float32(eps)))
    return round_to(round_to(normalized, dtype) * gamma, dtype)


def conv_state_update(projected, history):
    """reference/fused_ops.py:37-47 — padded = [history | projected^T]; history' = last K-1 columns."""
    projected = np.asarray(projected, np.float32)
    history = np.asarray(history, np.float32)
    if (projected.ndim != 3 or history.ndim != 3 or projected.shape[1] < 1
            or projected.shape[0] != history.shape[0] or projected.shape[2] != history.shape[1]):
        raise ValueError("conv state requires projected [B,S,C] and matching history [B,C,K-1]")
    padded = np.concatenate((history, projected.transpose(0, 2, 1)), axis=-1)
    count = history.shape[-1]
    updated = padded[..., padded.shape[-1] - count:] if count else padded[..., :0]
    return updated.copy(), padded


def causal_conv1d(padded, weight, dtype: str = "f32") -> np.ndarray:
    """reference/fused_ops.py:50-56 — depthwise cross-correlation, [B,C,S+K-1] x [C,1,K] -> [B,S,C]."""
    padded = np.asarray(padded, np.float32)
    weight = np.asarray(weight, np.float32)
    if (padded.ndim != 3 or weight.ndim != 3 or weight.shape[1] != 1
            or padded.shape[1] != weight.shape[0] or padded.shape[-1] < weight.shape[-1]):
        raise ValueError("depthwise conv requires [B,C,S+K-1] and [C,1,K]")
    k = weight.shape[-1]
    s = padded.shape[-1] - k + 1
    out = np.zeros((padded.shape[0], padded.shape[1], s), np.float32)
    for j in range(k):
        out += padded[:, :, j:j + s] * weight[None, :, 0, j:j + 1]
    return round_to(out.transpose(0, 2, 1), dtype).copy()


def chunk_gated_delta_rule(query, key, value, g, beta, initial_state, effective_length, *,
                           chunk_size: int, use_qk_l2norm_in_kernel: bool,
                           dtype: str = "f32", state_dtype: str = "f32"):
    """reference/fused_ops.py:59-107 — sequential gated delta rule.

    Per token t < effective_length[b]:  S <- exp(g) S;  delta = beta (v - S^T k);
    S <- S + k delta^T;  o = S^T q.  Outputs at t >= effective_length are zero and the
    state stops updating (fused_ops.py:99-106).  q,k are L2-normalized (eps 1e-6 inside
    the rsqrt, :92-94) and q is scaled by Dk^-1/2 (:95).
    """
    if isinstance(chunk_size, bool) or chunk_size not in (1, 64):
        raise ValueError("chunk_size must be 1 or 64")
    if not isinstance(use_qk_l2norm_in_kernel, bool):
        raise ValueError("use_qk_l2norm_in_kernel must be bool")
    q, k, v, decay, gate = [np.asarray(t, np.float32) for t in (query, key, value, g, beta)]
    if (q.ndim != 4 or k.shape != q.shape or v.ndim != 4 or v.shape[:3] != q.shape[:3]
            or decay.shape != q.shape[:3] or gate.shape != q.shape[:3]):
        raise ValueError("GDN requires compatible [B,S,H,D] tensors and [B,S,H] gates")
    batch, sequence, heads, dk = q.shape
    state = np.array(initial_state, dtype=np.float32, copy=True)
    if state.shape != (batch, heads, dk, v.shape[-1]):
        raise ValueError("initial_state must be [B,H,Dk,Dv]")
    length = np.asarray(effective_length).astype(np.int64)
    if length.shape != (batch,) or (length < 0).any() or (length > sequence).any():
        raise ValueError("effective_length must be [B] within [0,S]")
    if use_qk_l2norm_in_kernel:
        q = q / np.sqrt(np.sum(q * q, -1, keepdims=True) + np.float32(1e-6))
        k = k / np.sqrt(np.sum(k * k, -1, keepdims=True) + np.float32(1e-6))
    q = q * np.float32(dk ** -0.5)
    outputs = np.zeros((batch, sequence, heads, v.shape[-1]), np.float32)
    for t in range(sequence):
        valid = t < length  # [B]
        decayed = state * np.exp(decay[:, t])[..., None, None]
        prediction = np.einsum("bhkv,bhk->bhv", decayed, k[:, t])
        delta = (v[:, t] - prediction) * gate[:, t, :, None]
        candidate = decayed + k[:, t, :, :, None] * delta[:, :, None, :]
        state = np.where(valid[:, None, None, None], candidate, state)
        output = np.einsum("bhkv,bhk->bhv", state, q[:, t])
        outputs[:, t] = np.where(valid[:, None, None], output, 0.0)
    return round_to(outputs, dtype), round_to(state, state_dtype)


def cache_update(key, value, new_key, new_value):
    """reference/fused_ops.py:110-124 — append along T; never writes the inputs."""
    if (key is None) != (value is None):
        raise ValueError("KV caches must appear together and use [B,H,T,D]")
    if key is None:
        return np.array(new_key, copy=True), np.array(new_value, copy=True)
    return np.concatenate((key, new_key), -2), np.concatenate((value, new_value), -2)


def attention(query, key, value, *, query_start: int, scale: float, dtype: str = "f32") -> np.ndarray:
    """reference/fused_ops.py:127-145 — causal GQA; row i sees keys <= query_start + i."""
    q = np.asarray(query, np.float32)
    k = np.asarray(key, np.float32)
    v = np.asarray(value, np.float32)
    if (q.ndim != 4 or k.ndim != 4 or q.shape[0] != k.shape[0] or k.shape[:3] != v.shape[:3]
            or q.shape[1] % k.shape[1] or query_start < 0
            or query_start + q.shape[-2] != k.shape[-2] or not scale > 0):
        raise ValueError("attention requires causal append-only GQA [B,H,S,D] inputs")
    groups = q.shape[1] // k.shape[1]
    rk = np.repeat(k, groups, axis=1)
    rv = np.repeat(v, groups, axis=1)
    scores = np.einsum("bhsd,bhtd->bhst", q, rk) * np.float32(scale)
    positions = np.arange(q.shape[-2]) + query_start
    visible = np.arange(k.shape[-2])[None, :] <= positions[:, None]
    scores = np.where(visible[None, None], scores, -np.inf)
    scores = scores - scores.max(-1, keepdims=True)
    p = np.exp(scores)
    p = p / p.sum(-1, keepdims=True)
    return round_to(np.einsum("bhst,bhtd->bhsd", p, rv), dtype)


def silu(x):
    x = np.asarray(x, np.float32)
    return x / (np.float32(1.0) + np.exp(-x))


def sigmoid(x):
    x = np.asarray(x, np.float32)
    return np.float32(1.0) / (np.float32(1.0) + np.exp(-x))


def softplus(x):
    x = np.asarray(x, np.float32)
    return np.where(x > 20, x, np.log1p(np.exp(np.minimum(x, 20)))).astype(np.float32)


def route(logits, top_k: int, dtype: str = "f32"):
    """reference/fused_ops.py:161-164 — fp32 softmax, torch.topk, renormalize, cast.

    ``logits`` are the router outputs already rounded to the hidden dtype.
    Returns (indices int64 [T,k], weights [T,k] rounded to ``dtype``).
    """
    logits = np.asarray(logits, np.float32)
    shifted = logits - logits.max(-1, keepdims=True)
    e = np.exp(shifted)
    probabilities = e / e.sum(-1, keepdims=True)
    selected = topk_indices(probabilities, top_k)
    weights = np.take_along_axis(probabilities, selected, -1)
    weights = weights / weights.sum(-1, keepdims=True)
    return selected, round_to(weights, dtype)


def moe(hidden, router_weight, gate_up, down, *, top_k: int, dtype: str = "f32",
        emulate_rounding: bool = True, logits=None, return_routing: bool = False,
        return_magnitude: bool = False):
    """reference/fused_ops.py:148-173 — routed SwiGLU experts, ascending expert order.

    With ``emulate_rounding`` each intermediate is rounded to ``dtype`` where the
    reference's torch ops return ``dtype`` tensors; otherwise everything stays fp32
    and only the result is rounded.  ``logits`` replaces the router GEMV when given
    (the W4A16 microbench feeds router logits directly).  ``return_magnitude`` appends
    the elementwise largest |value| the accumulation passes through (each weighted
    expert term and each running sum): one rounding step of the sum is one ulp of
    that magnitude, which bounds how far two correct implementations can part.
    """
    hidden = np.asarray(hidden, np.float32)
    flat = hidden.reshape(-1, hidden.shape[-1])
    r = (lambda a: round_to(a, dtype)) if emulate_rounding else (lambda a: np.asarray(a, np.float32))
    if logits is None:
        logits = round_to(flat @ np.asarray(router_weight, np.float32).T, dtype)
    logits = np.asarray(logits, np.float32).reshape(flat.shape[0], -1)
    selected, weights = route(logits, top_k, dtype)
    result = np.zeros_like(flat)
    magnitude = np.zeros_like(flat)
    experts = logits.shape[-1]
    for expert in range(experts):
        tokens, slots = np.nonzero(selected == expert)
        if not tokens.size:
            continue
        gu = r(flat[tokens] @ np.asarray(gate_up[expert], np.float32).T)
        inter = gu.shape[-1] // 2
        gate, up = gu[:, :inter], gu[:, inter:]
        act = r(r(silu(gate)) * up)
        values = r(act @ np.asarray(down[expert], np.float32).T)
        term = r(values * weights[tokens, slots][:, None])
        result[tokens] = r(result[tokens] + term)
        if return_magnitude:
            magnitude[tokens] = np.maximum(magnitude[tokens], np.maximum(np.abs(term), np.abs(result[tokens])))
    out = round_to(result, dtype).reshape(hidden.shape)
    extra = ()
    if return_routing:
        extra += (selected, weights)
    if return_magnitude:
        extra += (magnitude.reshape(hidden.shape),)
    return (out,) + extra if extra else out
