"""numpy restatement of the expert-parallel exchange -- TEST INFRASTRUCTURE ONLY (see
``oracle/__init__.py``).

The reference plans multi-GPU serving with the routed experts sharded over the GPUs
(rank g owns experts [g E/G, (g+1) E/G)) and dispatch/combine by all-to-all (its
serving plan; there is no multi-GPU code in the reference to pin against, so this is
the protocol the CUDA kernels of ``qw_moe_ep_*`` implement, stated plainly):

* pack: pair p = t * k + s (token t, slot s) of expert e goes to rank d = e // (E/G),
  at position = number of earlier pairs for d; segment d of the send buffer is cap + 1
  rows [cap + 1, H]: row 0 the header, int32 words [count, (p << 8) | (e - d E/G), ...]
  laid into the row's bytes, row 1 + position the pair's activation row;
* the receiving rank runs local expert ``word & 0xFF`` on each received pair row;
* the outputs return in the same rows of segments of the same layout and land in slot
  (t, s).
"""
from __future__ import annotations

import numpy as np


def header_words(seg: np.ndarray, cap: int) -> np.ndarray:
    """int32 header words [ranks, cap + 1] of 16-bit segments [ranks, cap + 1, H]."""
    head = np.ascontiguousarray(seg[:, 0])
    return head.view(np.int32)[:, : cap + 1]


def pack(topk: np.ndarray, x16: np.ndarray, experts: int, ranks: int, cap: int) -> np.ndarray:
    """topk int [T, k], x16 16-bit rows [T, H] (bf16 bits as uint16) -> send segments
    uint16 [ranks, cap + 1, H]."""
    T, k = topk.shape
    H = x16.shape[1]
    if (cap + 1) * 2 > H:
        raise ValueError("the header does not fit in one row")
    el = experts // ranks
    seg = np.zeros((ranks, cap + 1, H), np.uint16)
    words = np.zeros((ranks, cap + 1), np.int32)
    for p in range(T * k):
        e = int(topk.flat[p])
        d = e // el
        pos = int(words[d, 0])
        if pos >= cap:
            raise ValueError("segment overflow")
        seg[d, 1 + pos] = x16[p // k]
        words[d, 1 + pos] = (p << 8) | (e - d * el)
        words[d, 0] += 1
    seg[:, 0, : 2 * (cap + 1)] = words.view(np.uint16).reshape(ranks, 2 * (cap + 1))
    return seg


def recv_experts(seg: np.ndarray, cap: int) -> np.ndarray:
    """Local expert of every received row, rows taken as they lie (-1 for the header rows
    and past each segment's count): [ranks * (cap + 1)]."""
    words = header_words(seg, cap)
    ranks = seg.shape[0]
    out = np.full((ranks, cap + 1), -1, np.int64)
    for g in range(ranks):
        n = int(words[g, 0])
        out[g, 1:1 + n] = words[g, 1:1 + n] & 0xFF
    return out.reshape(-1)


def scatter(topk: np.ndarray, back: np.ndarray, experts: int, ranks: int) -> np.ndarray:
    """Returned output segments [ranks, cap + 1, H] -> per-(token, slot) outputs [T, k, H]."""
    T, k = topk.shape
    el = experts // ranks
    out = np.zeros((T, k, back.shape[2]), back.dtype)
    filled = np.zeros(ranks, np.int64)
    for p in range(T * k):
        d = int(topk.flat[p]) // el
        out[p // k, p % k] = back[d, 1 + filled[d]]
        filled[d] += 1
    return out
