"""Shared test helpers: tolerance checks, numpy<->torch, oracle compositions."""
from __future__ import annotations

import ctypes

import numpy as np
import torch

from oracle import fused_ops_np as F
from oracle.numerics import bf16_round

# The stated tolerance for bf16 outputs after dequant: |a - b| <= 2e-2 + 1e-2 |b|
ATOL, RTOL = 2e-2, 1e-2


def assert_close(got, want, atol=ATOL, rtol=RTOL, what="", row_scale=False, strict_frac=None, magnitude=None):
    """|got - want| <= atol + rtol * |want| elementwise.

    row_scale: the relative term uses max(|want|, RMS of want's last-axis row), for
    outputs that are sums of bf16-rounded partial sums (the reference's MoE accumulates
    experts in bf16, so a one-ulp difference in an expert's output carries the row's
    scale into a small, cancelled result).  magnitude: an explicit elementwise magnitude
    for the relative term (e.g. the largest intermediate of a bf16 accumulation).
    strict_frac: additionally require that fraction of elements to meet the plain
    elementwise bound.
    """
    a = np.asarray(got, np.float64)
    b = np.asarray(want, np.float64)
    assert a.shape == b.shape, (what, a.shape, b.shape)
    mag = np.abs(b)
    if strict_frac is not None:
        ok = np.abs(a - b) <= atol + rtol * mag
        assert ok.mean() >= strict_frac, f"{what}: only {ok.mean():.5f} of elements within the strict bound"
    if row_scale:
        mag = np.maximum(mag, np.sqrt(np.mean(b * b, axis=-1, keepdims=True)))
    if magnitude is not None:
        mag = np.maximum(mag, np.asarray(magnitude, np.float64))
    excess = np.abs(a - b) - (atol + rtol * mag)
    worst = np.unravel_index(np.argmax(excess), excess.shape) if excess.size else ()
    assert excess.size == 0 or excess.max() <= 0, (
        f"{what}: max excess {excess.max():.3e} at {worst}: got {a[worst]:.6g} want {b[worst]:.6g}; "
        f"max abs diff {np.abs(a - b).max():.3e}")


def to_np(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


def bf16_tensor(a, device="cuda") -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(device).to(torch.bfloat16)


def struct_array_to_device(structs, device="cuda") -> torch.Tensor:
    """ctypes structure array -> uint8 device tensor holding the same bytes."""
    raw = bytes(memoryview(structs).cast("B"))
    return torch.frombuffer(bytearray(raw), dtype=torch.uint8).to(device)


def oracle_gdn_layer(proj, ab, hist, conv_w, a_log, dt_bias, norm_w, state_rowmajor, *,
                     k_heads, v_heads, dk, dv, eps, accepted=None):
    """The GDN layer body of fused/model.py:232-262 from its projections, bf16 semantics.

    proj [B,S,ldp] (bf16 values), ab [B,S,2H] fp32, hist [B,C,K-1], state [B,H,Dk,Dv].
    Returns (out [B,S,H*Dv], state after S tokens, {r: (state_r, hist_r)} for accepted).
    """
    b, s, _ = proj.shape
    kw, vw = k_heads * dk, v_heads * dv
    c = 2 * kw + vw
    projected = proj[..., :c]
    _, padded = F.conv_state_update(projected, hist)
    mixed = bf16_round(F.silu(F.causal_conv1d(padded, conv_w[:, None, :], "bf16")))
    q = np.repeat(mixed[..., :kw].reshape(b, s, k_heads, dk), v_heads // k_heads, axis=2)
    k = np.repeat(mixed[..., kw:2 * kw].reshape(b, s, k_heads, dk), v_heads // k_heads, axis=2)
    v = mixed[..., 2 * kw:].reshape(b, s, v_heads, dv)
    beta = F.sigmoid(ab[..., :v_heads])
    g = -np.exp(a_log) * F.softplus(ab[..., v_heads:] + dt_bias)
    full = np.full((b,), s, np.int16)
    core, state = F.chunk_gated_delta_rule(q, k, v, g, beta, state_rowmajor, full, chunk_size=64,
                                           use_qk_l2norm_in_kernel=True, dtype="bf16")
    z = proj[..., c:c + vw].reshape(b, s, v_heads, dv)
    out = bf16_round(F.rms_norm(core, norm_w, eps, "bf16") * bf16_round(F.silu(z)))
    commits = {}
    for r in (accepted or []):
        lens = np.full((b,), r, np.int16)
        _, st_r = F.chunk_gated_delta_rule(q, k, v, g, beta, state_rowmajor, lens, chunk_size=64,
                                           use_qk_l2norm_in_kernel=True)
        commits[r] = (st_r, padded[..., r:r + hist.shape[-1]].copy())
    return out.reshape(b, s, vw), state, commits
