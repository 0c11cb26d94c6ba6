"""Synthetic checkpoints in the original group-256 quantised layout (tests only).

``write_original`` quantises float weights the way the original checkpoint stores them
(int4 values one per int8, one fp16 scale per 256 along K: scale = max|w| / 7 rounded
to fp16, a zero group -> 1, q = clip(rint(w / scale), -8, 7)), writes them as two
``data*.safetensors`` shards, the embedding as int8 rows + fp32 row scales, and the
remaining weights as an HF-layout model file, and returns the weights the library must
reproduce from those files (the oracle's input).
"""
from __future__ import annotations

import json
import struct
from pathlib import Path

import numpy as np

from oracle.numerics import bf16_round

_DT = {np.dtype("i1"): "I8", np.dtype("<f2"): "F16", np.dtype("<f4"): "F32", np.dtype("<u2"): "BF16"}


def write_safetensors(path, tensors: dict) -> None:
    header, blobs, off = {}, [], 0
    for key, arr in tensors.items():
        arr = np.ascontiguousarray(arr)
        b = arr.tobytes()
        header[key] = {"dtype": _DT[arr.dtype], "shape": list(arr.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    h = json.dumps(header).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def quantize_g256(w: np.ndarray):
    w = np.asarray(w, np.float32)
    g = w.reshape(*w.shape[:-1], w.shape[-1] // 256, 256)
    s = (np.abs(g).max(-1) / np.float32(7)).astype(np.float16)
    s = np.where(s == 0, np.float16(1), s)
    q = np.clip(np.rint(g / s.astype(np.float32)[..., None]), -8, 7).astype(np.int8)
    return q.reshape(w.shape), s


def write_original(cfg, raw: dict, root) -> dict:
    """Write ``raw`` (target name -> float array) as an original checkpoint under
    ``root``; returns {"quant_dir", "base", "embed_w", "embed_s", "expected"}."""
    from qwen35_dflash_b200 import original
    root = Path(root)
    qdir = root / "quant"
    qdir.mkdir(parents=True, exist_ok=True)
    shards, base, expected = [{}, {}], {}, {}
    i = 0
    for name, w in raw.items():
        if name == "target.embed_tokens.weight":
            w = np.asarray(w, np.float32)
            s = (np.abs(w).max(-1, keepdims=True) / np.float32(127)).astype(np.float32)
            s = np.where(s == 0, np.float32(1), s)
            q = np.clip(np.rint(w / s), -127, 127).astype(np.int8)
            q.tofile(root / "embed_w.bin")
            s.astype("<f4").tofile(root / "embed_s.bin")
            expected[name] = bf16_round(q.astype(np.float32) * s)
            continue
        if not original.is_original_quantized(name):
            base[original.checkpoint_name(name)] = np.asarray(w, np.float32)
            expected[name] = np.asarray(w, np.float32)
            continue
        q, s = quantize_g256(w)
        wkey, skey = original.original_keys(name)
        expert = name.endswith(tuple(original.EXPERTS))
        shards[i % 2][wkey] = q
        shards[i % 2][skey] = s if expert else s[..., None]
        i += 1
        s32 = np.repeat(s.astype(np.float32), 256, -1)
        if name.endswith(("in_proj_a.weight", "in_proj_b.weight", "mlp.gate.weight", "lm_head.weight")):
            expected[name] = bf16_round(q.astype(np.float32) * s32)        # bf16-streamed
        else:
            expected[name] = q.astype(np.float32) * np.repeat(bf16_round(s.astype(np.float32)), 256, -1)
    write_safetensors(qdir / "data-00001.safetensors", shards[0])
    write_safetensors(qdir / "data-00002.safetensors", shards[1])
    write_safetensors(root / "model.safetensors", base)
    return {"quant_dir": qdir, "base": root / "model.safetensors", "embed_w": root / "embed_w.bin",
            "embed_s": root / "embed_s.bin", "expected": expected}
