"""W4A16 quantization and packing into the kernels' weight streams.

Quantizer: int4 symmetric per group of ``group`` along K with bf16 scales — the
arithmetic of the reference's portable quantizer
(model/qwen35_moe_dflash/graph/quant_weights.py:135-146: scale = max|w|/7, zero group
-> 1, q = clip(rint(w/scale), -8, 7)) with the W4A16 group size and bf16 scale storage
of the DOPT plan (model/qwen35_moe_dflash/reference/quantization.py:87-103).  The
scale is rounded to bf16 before q is chosen so that the stored pair dequantizes to
exactly q * scale.

Stream layouts (see csrc/stream_gemm.cuh): every function here is a pure
permutation / bit packing implemented with torch tensor ops, so it runs on the
device that holds the weights.  K is permuted within 32-wide blocks
(``physical_k``) so that the kernels read activations with 16-byte loads.
"""
from __future__ import annotations

import torch

TILE = 16


def quantize(weight: torch.Tensor, group: int) -> tuple[torch.Tensor, torch.Tensor]:
    """float [..., N, K] -> (int8 q in [-8,7] [..., N, K], bf16 scales [..., N, K/group])."""
    w = weight.float()
    if w.shape[-1] % group:
        raise ValueError(f"K={w.shape[-1]} must be divisible by group={group}")
    g = w.reshape(*w.shape[:-1], w.shape[-1] // group, group)
    scale = (g.abs().amax(-1) / 7.0).to(torch.bfloat16)
    scale = torch.where(scale == 0, torch.ones_like(scale), scale)
    q = torch.clamp(torch.round(g / scale.float()[..., None]), -8, 7).to(torch.int8)
    return q.reshape(w.shape), scale


def dequantize(q: torch.Tensor, scale: torch.Tensor, group: int) -> torch.Tensor:
    return (q.float() * scale.float().repeat_interleave(group, -1))


def physical_k(step, tig, second, e):
    """Physical K offset (within the chunk) of the mma-logical element k = 16*step + 2*tig
    + 8*second + e.  Within each 32-wide block the streams are permuted so that lane tig's
    B fragments of steps 2p and 2p+1 are the 8 contiguous activations 32p + 8*tig .. +7."""
    return 32 * (step // 2) + 8 * tig + 4 * (step % 2) + 2 * second + e


def _lane_maps(steps: int, device):
    """Row-in-tile and (physical) column-in-group of nibble j of word (lane, step)."""
    lane = torch.arange(32, device=device).view(32, 1, 1)
    s = torch.arange(steps, device=device).view(1, steps, 1)
    j = torch.arange(8, device=device).view(1, 1, 8)
    gid, tig = lane // 4, lane % 4
    row = gid + 8 * (j & 1)
    col = physical_k(s, tig, (j >> 1) & 1, j >> 2)
    return row.expand(32, steps, 8), col.expand(32, steps, 8)


def pack_w4(q: torch.Tensor, scale: torch.Tensor, group: int) -> torch.Tensor:
    """int8 q [N, K] (or [E, N, K]) + scales -> uint8 W4 stream (experts concatenated)."""
    if q.dim() == 3:  # expert bank: per-expert streams back to back == one [E*N, K] stream
        if q.shape[1] % TILE:
            raise ValueError("pack_w4 needs N % 16 == 0")
        return pack_w4(q.reshape(-1, q.shape[-1]), scale.reshape(-1, scale.shape[-1]), group)
    n, k = q.shape
    if n % TILE or k % group or group not in (32, 64, 128):
        raise ValueError("pack_w4 needs N % 16 == 0, K % group == 0, group in {32,64,128}")
    nt, ng, steps = n // TILE, k // group, group // 16
    dev = q.device
    u = (q.to(torch.int16) + 8).to(torch.int64)                   # offset binary 0..15
    u = u.view(nt, TILE, ng, group).permute(0, 2, 1, 3)          # [nt, ng, 16, group]
    row, col = _lane_maps(steps, dev)
    vals = u[:, :, row, col]                                     # [nt, ng, 32, steps, 8]
    shifts = (4 * torch.arange(8, device=dev, dtype=torch.int64))
    words = (vals << shifts).sum(-1)                             # [nt, ng, 32, steps]
    vw = min(4, steps)
    nv = steps // vw
    words = words.view(nt, ng, 32, nv, vw).permute(0, 1, 3, 2, 4).reshape(nt, ng, steps * 32)
    words = torch.where(words >= 2 ** 31, words - 2 ** 32, words).to(torch.int32)
    nib = words.contiguous().view(torch.uint8).view(nt, ng, 8 * group)
    # scales: position p = 2*gid + h <-> row gid + 8h
    p = torch.arange(16, device=dev)
    srow = (p >> 1) + 8 * (p & 1)
    sc = scale.to(torch.bfloat16).view(nt, TILE, ng).permute(0, 2, 1)[:, :, srow]
    scb = sc.contiguous().view(torch.uint8).view(nt, ng, 32)
    return torch.cat((nib, scb), -1).reshape(-1).contiguous()


def unpack_w4(stream: torch.Tensor, n: int, k: int, group: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Inverse of pack_w4 for one [N, K] matrix (tests)."""
    nt, ng, steps = n // TILE, k // group, group // 16
    dev = stream.device
    chunk = stream.view(nt, ng, 8 * group + 32)
    words = chunk[:, :, :8 * group].contiguous().view(torch.int32).to(torch.int64) & 0xFFFFFFFF
    vw = min(4, steps)
    nv = steps // vw
    words = words.view(nt, ng, nv, 32, vw).permute(0, 1, 3, 2, 4).reshape(nt, ng, 32, steps)
    shifts = 4 * torch.arange(8, device=dev, dtype=torch.int64)
    vals = (words[..., None] >> shifts) & 15                      # [nt, ng, 32, steps, 8]
    row, col = _lane_maps(steps, dev)
    q = torch.empty(nt, ng, TILE, group, dtype=torch.int64, device=dev)
    q[:, :, row, col] = vals
    q = (q - 8).permute(0, 2, 1, 3).reshape(n, k).to(torch.int8)
    sc = chunk[:, :, 8 * group:].contiguous().view(torch.bfloat16).view(nt, ng, 16)
    p = torch.arange(16, device=dev)
    srow = (p >> 1) + 8 * (p & 1)
    scale = torch.empty(nt, ng, 16, dtype=torch.bfloat16, device=dev)
    scale[:, :, srow] = sc
    return q, scale.permute(0, 2, 1).reshape(n, ng)


def pack_b16(weight: torch.Tensor) -> torch.Tensor:
    """bf16 [N, K] (or [E, N, K]) -> uint8 B16 stream; N % 16 == 0, K % 64 == 0."""
    if weight.dim() == 3:
        if weight.shape[1] % TILE:
            raise ValueError("pack_b16 needs N % 16 == 0")
        return pack_b16(weight.reshape(-1, weight.shape[-1]))
    n, k = weight.shape
    if n % TILE or k % 64:
        raise ValueError("pack_b16 needs N % 16 == 0 and K % 64 == 0")
    nt, nc = n // TILE, k // 64
    w = weight.to(torch.bfloat16).contiguous().view(torch.int16).view(nt, TILE, nc, 64)
    w = w.permute(0, 2, 1, 3)                                   # [nt, nc, 16, 64]
    dev = weight.device
    lane = torch.arange(32, device=dev).view(32, 1, 1, 1)
    s = torch.arange(4, device=dev).view(1, 4, 1, 1)
    reg = torch.arange(4, device=dev).view(1, 1, 4, 1)
    half = torch.arange(2, device=dev).view(1, 1, 1, 2)
    gid, tig = lane // 4, lane % 4
    row = gid + 8 * (reg & 1)
    col = physical_k(s, tig, reg >> 1, half)
    row, col = torch.broadcast_tensors(row, col)
    vals = w[:, :, row, col]                                    # [nt, nc, 32, 4(step), 4(reg), 2]
    vals = vals.permute(0, 1, 3, 2, 4, 5).contiguous()          # [nt, nc, step, lane, reg, 2]
    return vals.view(torch.uint8).reshape(-1)


def pad_rows(weight: torch.Tensor, multiple: int = TILE) -> torch.Tensor:
    n = weight.shape[-2]
    pad = (-n) % multiple
    if not pad:
        return weight
    z = torch.zeros(*weight.shape[:-2], pad, weight.shape[-1], dtype=weight.dtype, device=weight.device)
    return torch.cat((weight, z), -2)
