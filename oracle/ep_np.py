"""numpy restatement of the expert-parallel exchange -- TEST INFRASTRUCTURE ONLY (see
``oracle/__init__.py``).

The reference plans multi-GPU serving with the routed experts sharded over the GPUs
(rank g owns experts [g E/G, (g+1) E/G)) and dispatch/combine between them (its serving
plan; there is no multi-GPU code in the reference to pin against, so this is the
protocol the ``qw_moe_ep_*`` kernels implement, stated plainly):

* dispatch: pair p = t * k + s (token t, slot s) of expert e goes to rank d = e // (E/G),
  at position = number of earlier pairs for d; the source g writes, into d's window,
  rows[g][position] = x[t] and meta[g][position] = (p << 9) | (e - d E/G), and
  count[g] = its number of pairs for d;
* with the shared expert exchanged, it is every rank's local expert E/G and token t
  sends one more pair, p = T k + t, to its own rank, after its routed pairs there;
* the receiving rank takes the valid rows source by source (rows [s][0, count[s])) and
  runs local expert ``meta & 0x1FF`` on each;
* combine: the output of received row (s, j) goes to source s's ``back`` row
  ``meta[s][j] >> 9`` (its own pair index); the source's pair p output lands in slot
  (p // k, p % k), a shared pair's in slot (p - T k, k).
"""
from __future__ import annotations

import numpy as np


def dispatch(topk: np.ndarray, x16: np.ndarray, experts: int, ranks: int, rank: int = 0, shared: bool = False):
    """topk int [T, k], x16 16-bit rows [T, H] of source ``rank`` -> per destination d the
    block this source writes into d's window: (rows uint16 [cap, H], meta int32 [cap],
    count), cap = T (k + shared)."""
    T, k = topk.shape
    H = x16.shape[1]
    cap = T * (k + int(shared))
    el = experts // ranks
    rows = np.zeros((ranks, cap, H), np.uint16)
    meta = np.zeros((ranks, cap), np.int32)
    count = np.zeros(ranks, np.int64)
    pairs = [(p, int(topk.flat[p]) // el, int(topk.flat[p]) % el, p // k) for p in range(T * k)]
    if shared:
        pairs += [(T * k + t, rank, el, t) for t in range(T)]
    for p, d, local, t in pairs:
        pos = int(count[d])
        rows[d, pos] = x16[t]
        meta[d, pos] = (p << 9) | local
        count[d] += 1
    return [(rows[d], meta[d], int(count[d])) for d in range(ranks)]


def received(blocks) -> list[tuple[int, int, int]]:
    """The blocks a rank received, one per source s (rows, meta, count), as its valid rows
    in order: (source, row j, local expert)."""
    out = []
    for s, (_, meta, count) in enumerate(blocks):
        for j in range(count):
            out.append((s, j, int(meta[j]) & 0x1FF))
    return out


def combine(blocks, outputs: dict, cap: int, H: int, dtype=np.uint16):
    """Received rows' outputs {(s, j): row} -> per source s the rows written into its
    ``back`` array [cap, H] (at the source's pair index) and the mask of rows written."""
    ranks = len(blocks)
    back = np.zeros((ranks, cap, H), dtype)
    written = np.zeros((ranks, cap), bool)
    for (s, j), row in outputs.items():
        pair = int(blocks[s][1][j]) >> 9
        back[s, pair] = row
        written[s, pair] = True
    return back, written


def scatter(back: np.ndarray, T: int, k: int, shared: bool = False) -> np.ndarray:
    """The source's ``back`` [cap, H] -> per-(token, slot) outputs [T, k + shared, H]."""
    routed = back[: T * k].reshape(T, k, back.shape[-1])
    if not shared:
        return routed
    return np.concatenate([routed, back[T * k: T * k + T, None]], axis=1)
