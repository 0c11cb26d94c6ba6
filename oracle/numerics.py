"""Rounding helpers, the W4A16 quantizer and torch's CPU top-k selection order.

Test infrastructure only (see ``oracle/__init__.py``).
"""
from __future__ import annotations

import numpy as np


def bf16_round(x) -> np.ndarray:
    """Round float32 values to the nearest bfloat16 (ties to even), kept as float32."""
    a = np.ascontiguousarray(np.asarray(x, dtype=np.float32))
    u = a.view(np.uint32).astype(np.uint64)
    rounded = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    out = rounded.astype(np.uint32).view(np.float32)
    return np.where(np.isnan(a), a, out).reshape(a.shape)


def f16_round(x) -> np.ndarray:
    return np.asarray(x, dtype=np.float32).astype(np.float16).astype(np.float32)


def round_to(x, dtype: str) -> np.ndarray:
    if dtype == "bf16":
        return bf16_round(x)
    if dtype == "f16":
        return f16_round(x)
    if dtype == "f32":
        return np.asarray(x, dtype=np.float32)
    raise ValueError(f"unknown dtype tag {dtype!r}")


def bf16_bits(x) -> np.ndarray:
    """bfloat16 bit patterns (uint16) of float32 values after rounding."""
    return (bf16_round(x).view(np.uint32) >> 16).astype(np.uint16)


def bf16_from_bits(bits) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint32) << 16).view(np.float32)


# --------------------------------------------------------------------------------------
# W4A16 symmetric group quantizer.
# Arithmetic follows the reference's portable symmetric quantizer
# (model/qwen35_moe_dflash/graph/quant_weights.py:135-146: scale = max|group| / 7, zero
# group -> scale 1, q = clip(rint(w / scale), -8, 7), ties to even), with the group size
# (128, or 32 for the tiny fixture) and bf16 scale storage of the W4A16 plan
# (model/qwen35_moe_dflash/reference/quantization.py:87-103).  The scale is rounded to
# bf16 first and the integer is chosen against the stored scale, so that the stored pair
# dequantizes to exactly q * scale.
# --------------------------------------------------------------------------------------

def quantize_w4(weight, group: int):
    """float [..., N, K] -> (int8 q in [-8, 7], bf16-valued float32 scales [..., N, K/group])."""
    w = np.asarray(weight, dtype=np.float32)
    if w.shape[-1] % group:
        raise ValueError(f"K={w.shape[-1]} must be divisible by group={group}")
    grouped = w.reshape(*w.shape[:-1], w.shape[-1] // group, group)
    maxima = np.max(np.abs(grouped), axis=-1)
    scale = bf16_round(maxima / np.float32(7.0))
    scale = np.where(scale == 0, np.float32(1.0), scale).astype(np.float32)
    q = np.clip(np.rint(grouped / scale[..., None]), -8, 7).astype(np.int8)
    return q.reshape(w.shape), scale


def dequantize_w4(q, scale, group: int) -> np.ndarray:
    q = np.asarray(q, dtype=np.float32)
    s = np.repeat(np.asarray(scale, dtype=np.float32), group, axis=-1)
    return (q * s).astype(np.float32)


# --------------------------------------------------------------------------------------
# torch.topk(largest=True, sorted=True) on CPU, restated.
# The reference router calls torch.topk on float32 probabilities
# (reference/fused_ops.py:163).  ATen's CPU kernel copies (value, index) pairs into a
# queue in index order and, when k*64 > n, runs std::nth_element at k-1 followed by
# std::sort of the first k-1 entries; otherwise std::partial_sort.  Both use the
# comparator  a.value > b.value.  The C++ library is GNU libstdc++ (the one torch
# 2.11.0+cu128 was built against); its introselect / heap-select / insertion-sort
# steps are restated below so that ties resolve in the same order.  Pinned against
# torch.topk by tests/golden/topk_*.npz.
# --------------------------------------------------------------------------------------

def _gt(a, b):
    return a[0] > b[0]


def _move_median_to_first(q, result, a, b, c):
    if _gt(q[a], q[b]):
        if _gt(q[b], q[c]):
            q[result], q[b] = q[b], q[result]
        elif _gt(q[a], q[c]):
            q[result], q[c] = q[c], q[result]
        else:
            q[result], q[a] = q[a], q[result]
    elif _gt(q[a], q[c]):
        q[result], q[a] = q[a], q[result]
    elif _gt(q[b], q[c]):
        q[result], q[c] = q[c], q[result]
    else:
        q[result], q[b] = q[b], q[result]


def _unguarded_partition(q, first, last, pivot):
    while True:
        while _gt(q[first], q[pivot]):
            first += 1
        last -= 1
        while _gt(q[pivot], q[last]):
            last -= 1
        if not first < last:
            return first
        q[first], q[last] = q[last], q[first]
        first += 1


def _insertion_sort(q, first, last):
    for i in range(first + 1, last):
        val = q[i]
        if _gt(val, q[first]):
            q[first + 1:i + 1] = q[first:i]
            q[first] = val
        else:
            hole, prev = i, i - 1
            while _gt(val, q[prev]):
                q[hole] = q[prev]
                hole, prev = prev, prev - 1
            q[hole] = val


def _push_heap(q, first, hole, top, value):
    parent = (hole - 1) // 2
    while hole > top and _gt(q[first + parent], value):
        q[first + hole] = q[first + parent]
        hole = parent
        parent = (hole - 1) // 2
    q[first + hole] = value


def _adjust_heap(q, first, hole, length, value):
    top = hole
    child = hole
    while child < (length - 1) // 2:
        child = 2 * (child + 1)
        if _gt(q[first + child], q[first + child - 1]):
            child -= 1
        q[first + hole] = q[first + child]
        hole = child
    if (length & 1) == 0 and child == (length - 2) // 2:
        child = 2 * (child + 1)
        q[first + hole] = q[first + child - 1]
        hole = child - 1
    _push_heap(q, first, hole, top, value)


def _make_heap(q, first, last):
    length = last - first
    if length < 2:
        return
    parent = (length - 2) // 2
    while True:
        _adjust_heap(q, first, parent, length, q[first + parent])
        if parent == 0:
            return
        parent -= 1


def _heap_select(q, first, middle, last):
    _make_heap(q, first, middle)
    for i in range(middle, last):
        if _gt(q[i], q[first]):
            value = q[i]
            q[i] = q[first]
            _adjust_heap(q, first, 0, middle - first, value)


def _introselect(q, first, nth, last, depth):
    while last - first > 3:
        if depth == 0:
            _heap_select(q, first, nth + 1, last)
            q[first], q[nth] = q[nth], q[first]
            return
        depth -= 1
        mid = first + (last - first) // 2
        _move_median_to_first(q, first, first + 1, mid, last - 1)
        cut = _unguarded_partition(q, first + 1, last, first)
        if cut <= nth:
            first = cut
        else:
            last = cut
    _insertion_sort(q, first, last)


def topk_indices_row(values, k: int) -> list[int]:
    """Indices torch.topk(values, k) returns on CPU for one row (float values)."""
    n = len(values)
    if not 0 < k <= n:
        raise ValueError("invalid k")
    if k - 1 > 16:
        # std::sort of more than 16 entries switches to introsort; not restated here
        raise NotImplementedError("top-k order restated for k <= 17 only")
    q = [(float(v), i) for i, v in enumerate(values)]
    if k * 64 <= n:
        _heap_select(q, 0, k, n)
        last = k
        while last > 1:
            last -= 1
            value = q[last]
            q[last] = q[0]
            _adjust_heap(q, 0, 0, last, value)
    else:
        _introselect(q, 0, k - 1, n, 2 * (n.bit_length() - 1))
        _insertion_sort(q, 0, k - 1)
    return [i for _, i in q[:k]]


def topk_indices(values, k: int) -> np.ndarray:
    v = np.asarray(values, dtype=np.float32)
    flat = v.reshape(-1, v.shape[-1])
    out = np.array([topk_indices_row(row, k) for row in flat], dtype=np.int64)
    return out.reshape(*v.shape[:-1], k)


def stable_argmax(values) -> np.ndarray:
    """Row argmax with ties to the lowest index (targets/cpro/ops/draft-top1/src/reference/top1_cpu.cpp:39)."""
    v = np.asarray(values, dtype=np.float32)
    return np.argmax(v, axis=-1).astype(np.int32)  # numpy returns the first maximum
