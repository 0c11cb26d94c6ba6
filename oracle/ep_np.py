"""numpy restatement of the expert-parallel exchange -- TEST INFRASTRUCTURE ONLY (see
``oracle/__init__.py``).

The reference plans multi-GPU serving with the routed experts sharded over the GPUs
(rank g owns experts [g E/G, (g+1) E/G)) and dispatch/combine by all-to-all (its
serving plan; there is no multi-GPU code in the reference to pin against, so this is
the protocol the CUDA kernels of ``qw_moe_ep_*`` implement, stated plainly):

* pack: pair p = t * k + s (token t, slot s) of expert e goes to rank d = e // (E/G),
  at position = number of earlier pairs for d; segment d of the send buffers holds
  cap rows [cap, H] and a header meta[d] = [count, (p << 8) | (e - d E/G), ...];
* the receiving rank runs local expert ``meta & 0xFF`` on each received row;
* the outputs return in the same segment positions and land in slot (t, s).
"""
from __future__ import annotations

import numpy as np


def pack(topk: np.ndarray, x: np.ndarray, experts: int, ranks: int, cap: int):
    """topk int [T, k], x [T, H] -> (rows [ranks, cap, H], meta int32 [ranks, cap + 1])."""
    T, k = topk.shape
    el = experts // ranks
    rows = np.zeros((ranks, cap, x.shape[1]), x.dtype)
    meta = np.zeros((ranks, cap + 1), np.int32)
    for p in range(T * k):
        e = int(topk.flat[p])
        d = e // el
        pos = int(meta[d, 0])
        if pos >= cap:
            raise ValueError("segment overflow")
        rows[d, pos] = x[p // k]
        meta[d, 1 + pos] = (p << 8) | (e - d * el)
        meta[d, 0] += 1
    return rows, meta


def recv_experts(meta: np.ndarray) -> np.ndarray:
    """Local expert of every received row (-1 past each segment's count): [ranks * cap]."""
    ranks, cap1 = meta.shape
    out = np.full((ranks, cap1 - 1), -1, np.int64)
    for g in range(ranks):
        n = int(meta[g, 0])
        out[g, :n] = meta[g, 1:1 + n] & 0xFF
    return out.reshape(-1)


def scatter(topk: np.ndarray, back: np.ndarray, experts: int, ranks: int) -> np.ndarray:
    """Returned outputs [ranks, cap, H] -> per-(token, slot) outputs [T, k, H]."""
    T, k = topk.shape
    el = experts // ranks
    out = np.zeros((T, k, back.shape[2]), back.dtype)
    filled = np.zeros(ranks, np.int64)
    for p in range(T * k):
        d = int(topk.flat[p]) // el
        out[p // k, p % k] = back[d, filled[d]]
        filled[d] += 1
    return out
