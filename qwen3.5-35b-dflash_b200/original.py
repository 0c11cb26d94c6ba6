"""Import of the original group-256 quantised target checkpoint.

The original checkpoint (read by the reference in
model/qwen35_moe_dflash/target/original_quant.py:152-297, ``OriginalQuantWeights``)
keeps every quantised projection as signed int4 values stored one per int8 in
``data*.safetensors`` shards, with one non-negative fp16 or fp32 scale per group of 256
along K:

* ``<stem>_quant_weight``: int8 ``[N, K]`` (experts ``[E, N, K]``), values in [-8, 7];
* ``<stem>_quant_scale``: ``[N, K/256, 1]`` (experts ``[E, N, K/256]``);
* stems (``canonicalkeys``, original_quant.py:34-48): ``lm_head`` and
  ``model.layers.{i}.<module>`` for the linear projections (GDN in_proj_qkv / z / b /
  a and out_proj, attention q / k / v / o, the router ``mlp.gate`` and the shared
  expert's three projections) and the expert banks ``mlp.experts.gate_up_proj`` /
  ``down_proj``;
* the embedding lives outside the shards: int8 rows ``[V, H]`` and one fp32 scale
  per row (``load_embedding``, original_quant.py:301-313);
* norms, conv taps, A_log, dt_bias and the shared-expert gate come from the HF model
  file under ``model.language_model.<name>`` (fused/quantization.py:205-221,
  graph/weights.py:180-186).

This module reads those files (its own safetensors header reader, with the
reference's validation rules: header bounds, unique keys across shards, exact and
non-overlapping extents, regular files inside the directory, int4 range, finite
non-negative scales) and converts them without requantising a single value:

* W4 projections keep their int4 values; each group-256 scale becomes the scale of
  the two group-128 groups it covers (the library's W4A16 format), rounded to bf16
  (relative change at most 2^-9; fp16 scales whose significand fits 8 bits are kept
  exactly);
* the projections the library streams in bf16 (router, GDN in_proj_b / in_proj_a,
  lm_head) are dequantised, q * scale in fp32 rounded once to bf16;
* the embedding rows are dequantised the same way (the reference keeps them, and
  its residual stream, in fp32; this library's residual stream is bf16).
"""
from __future__ import annotations

import json
import math
import re
import struct
from pathlib import Path

import numpy as np
import torch

from . import w4
from .config import TargetConfig

ORIGINAL_GROUP = 256
_CHUNK = 1 << 20
_WIDTHS = {"BOOL": 1, "U8": 1, "I8": 1, "I16": 2, "U16": 2, "I32": 4, "U32": 4, "I64": 8, "U64": 8,
           "F16": 2, "BF16": 2, "F32": 4, "F64": 8}
_NP = {"I8": np.dtype("i1"), "F16": np.dtype("<f2"), "F32": np.dtype("<f4"), "BF16": np.dtype("<u2")}
# module suffixes of the quantised linear projections and of the expert banks
# (original_quant.py:24-31)
LINEARS = frozenset({
    "linear_attn.in_proj_qkv", "linear_attn.in_proj_z", "linear_attn.in_proj_b",
    "linear_attn.in_proj_a", "linear_attn.out_proj", "self_attn.q_proj",
    "self_attn.k_proj", "self_attn.v_proj", "self_attn.o_proj", "mlp.gate",
    "mlp.shared_expert.gate_proj", "mlp.shared_expert.up_proj", "mlp.shared_expert.down_proj",
})
EXPERTS = frozenset({"mlp.experts.gate_up_proj", "mlp.experts.down_proj"})


def original_keys(name: str) -> tuple[str, str]:
    """Target weight name -> (int4 value key, scale key) in the original shards
    (original_quant.py:34-48)."""
    if name == "target.lm_head.weight":
        stem = "lm_head"
    else:
        m = re.fullmatch(r"target\.layers\.([0-9]+)\.(.+)", name)
        if m is None:
            raise ValueError(f"not an original target quantized weight: {name}")
        suffix = m[2]
        if suffix.endswith(".weight") and suffix[:-7] in LINEARS:
            suffix = suffix[:-7]
        elif suffix not in EXPERTS:
            raise ValueError(f"not an original target quantized weight: {name}")
        stem = f"model.layers.{m[1]}.{suffix}"
    return stem + "_quant_weight", stem + "_quant_scale"


def is_original_quantized(name: str) -> bool:
    try:
        original_keys(name)
        return True
    except ValueError:
        return False


def _unique(pairs):
    out = {}
    for k, v in pairs:
        if k in out:
            raise ValueError("duplicate safetensors JSON key: " + k)
        out[k] = v
    return out


def read_header(path: Path) -> dict:
    """One safetensors file's tensors: key -> {dtype, shape, offset (absolute), bytes}."""
    size = path.stat().st_size
    with path.open("rb") as f:
        prefix = f.read(8)
        if len(prefix) != 8:
            raise ValueError(f"{path.name}: truncated safetensors prefix")
        hlen = struct.unpack("<Q", prefix)[0]
        if not 2 <= hlen <= min(32 << 20, size - 8):
            raise ValueError(f"{path.name}: invalid safetensors header length")
        header = json.loads(f.read(hlen), object_pairs_hook=_unique)
    if not isinstance(header, dict):
        raise ValueError(f"{path.name}: safetensors header must be an object")
    start, out, extents = 8 + hlen, {}, []
    for key, spec in header.items():
        if key == "__metadata__":
            continue
        if not isinstance(spec, dict):
            raise ValueError(f"{key}: invalid safetensors tensor descriptor")
        dtype, shape, offs = spec.get("dtype"), spec.get("shape"), spec.get("data_offsets")
        if (dtype not in _WIDTHS or not isinstance(shape, list) or any(type(x) is not int or x < 0 for x in shape)
                or not isinstance(offs, list) or len(offs) != 2 or any(type(x) is not int for x in offs)):
            raise ValueError(f"{key}: invalid dtype, shape or offsets")
        nbytes = math.prod(shape) * _WIDTHS[dtype]
        if offs[0] < 0 or offs[1] - offs[0] != nbytes or start + offs[1] > size:
            raise ValueError(f"{key}: invalid safetensors data extent")
        if nbytes:
            extents.append((offs[0], offs[1], key))
        out[key] = {"dtype": dtype, "shape": tuple(shape), "offset": start + offs[0], "bytes": nbytes,
                    "file": path}
    end = 0
    for b, e, key in sorted(extents):
        if b < end:
            raise ValueError(f"{key}: overlapping safetensors data extents")
        end = e
    return out


def _view(rec) -> np.ndarray:
    if rec["dtype"] not in _NP:
        raise ValueError(f"unsupported tensor dtype {rec['dtype']}")
    if rec["bytes"] == 0:
        return np.zeros(rec["shape"], _NP[rec["dtype"]])
    return np.memmap(rec["file"], mode="r", dtype=_NP[rec["dtype"]], offset=rec["offset"], shape=rec["shape"])


def _float(rec) -> np.ndarray:
    v = np.asarray(_view(rec))
    if rec["dtype"] == "BF16":
        return (v.astype(np.uint32) << 16).view(np.float32)
    return v.astype(np.float32)


class OriginalCheckpoint:
    """The original quantised shards of one directory (``data*.safetensors``)."""

    def __init__(self, root):
        self.root = Path(root).resolve()
        paths = sorted(self.root.glob("data*.safetensors"))
        if not 0 < len(paths) <= 4096:
            raise ValueError("original quantized directory must contain 1..4096 data*.safetensors shards")
        self.tensors = {}
        for p in paths:
            real = p.resolve()
            if p.is_symlink() or self.root not in real.parents or not real.is_file():
                raise ValueError("quantized shard must be a regular file inside the supplied directory")
            for key, rec in read_header(real).items():
                if key in self.tensors:
                    raise ValueError(f"duplicate quantized tensor across shards: {key}")
                self.tensors[key] = rec

    def describe(self, name: str, shape) -> dict:
        """Validate the records of ``name`` (target weight name, logical shape [N,K] or
        [E,N,K]) from the headers alone (original_quant.py:214-242)."""
        shape = tuple(shape)
        if len(shape) not in (2, 3) or any(type(x) is not int or x <= 0 for x in shape):
            raise ValueError("weight shape must have positive integer dimensions and rank two or three")
        wkey, skey = original_keys(name)
        expert = name.endswith(tuple(EXPERTS))
        if len(shape) != (3 if expert else 2):
            raise ValueError(f"{name}: rank does not match linear/expert role")
        n, k = shape[-2:]
        if k % ORIGINAL_GROUP or n % 16:
            raise ValueError(f"{name}: group-256 I4ZN requires K%256=0 and N%16=0")
        sshape = (*shape[:-1], k // ORIGINAL_GROUP) if expert else (n, k // ORIGINAL_GROUP, 1)
        for key, want, types in ((wkey, shape, {"I8"}), (skey, sshape, {"F16", "F32"})):
            rec = self.tensors.get(key)
            if rec is None:
                raise ValueError("original quantized tensor missing: " + key)
            if rec["shape"] != want or rec["dtype"] not in types:
                raise ValueError(f"{key}: expected {list(want)} with dtype in {sorted(types)}")
        return {"kind": "expert" if expert else "linear", "weight": self.tensors[wkey], "scale": self.tensors[skey],
                "scale_shape": (*shape[:-1], k // ORIGINAL_GROUP)}

    def logical(self, name: str, shape) -> tuple[np.ndarray, np.ndarray]:
        """(int8 values [.., N, K] in [-8, 7], float32 scales [.., N, K/256]) of ``name``,
        validated (original_quant.py:254-268)."""
        meta = self.describe(name, shape)
        q = _view(meta["weight"])
        flat = q.reshape(-1)
        for i in range(0, flat.size, _CHUNK):
            v = flat[i:i + _CHUNK]
            if v.min() < -8 or v.max() > 7:
                raise ValueError("original quantized weight contains values outside signed I4 [-8,7]")
        s = _float(meta["scale"]).reshape(meta["scale_shape"])
        if not np.isfinite(s).all() or (s < 0).any():
            raise ValueError("original quantization scales must be finite and nonnegative")
        return q, s


def load_embedding(weight_path, scale_path, shape) -> tuple[np.ndarray, np.ndarray]:
    """The original external embedding: int8 rows [V, H] and fp32 row scales [V, 1]
    (original_quant.py:301-313)."""
    shape = tuple(shape)
    weight_path, scale_path = Path(weight_path).resolve(), Path(scale_path).resolve()
    for path, size in ((weight_path, math.prod(shape)), (scale_path, shape[0] * 4)):
        if not path.is_file() or path.stat().st_size != size:
            raise ValueError(f"original embedding file size mismatch: {path}")
    weight = np.memmap(weight_path, mode="r", dtype="i1", shape=shape)
    scale = np.memmap(scale_path, mode="r", dtype="<f4", shape=(shape[0], 1))
    if not np.isfinite(scale).all() or (np.asarray(scale) < 0).any():
        raise ValueError("embedding scales must be finite and nonnegative")
    return weight, scale


def scales_g128(scale256: torch.Tensor, group: int) -> torch.Tensor:
    """Group-256 scales [.., K/256] -> bf16 scales of ``group``-wide groups [.., K/group]."""
    if ORIGINAL_GROUP % group:
        raise ValueError("the library group must divide 256")
    return scale256.to(torch.bfloat16).repeat_interleave(ORIGINAL_GROUP // group, -1)


def dequantize_bf16(q: torch.Tensor, scale256: torch.Tensor) -> torch.Tensor:
    """q * scale in fp32 (exact), rounded once to bf16."""
    s = scale256.float().repeat_interleave(ORIGINAL_GROUP, -1)
    return (q.float() * s).to(torch.bfloat16)


def checkpoint_name(name: str) -> str:
    """Target weight name -> its key in the HF model file (graph/weights.py:180-186)."""
    if not name.startswith("target."):
        raise ValueError(f"unknown weight namespace: {name}")
    suffix = name[len("target."):]
    return suffix if suffix == "lm_head.weight" else "model.language_model." + suffix


class BaseWeights:
    """The unquantised weights (norms, conv taps, A_log, dt_bias, shared-expert gate)
    from HF ``*.safetensors`` files (one file or every file of a directory), by target
    weight name."""

    def __init__(self, path):
        p = Path(path).resolve()
        files = sorted(p.glob("*.safetensors")) if p.is_dir() else [p]
        if not files:
            raise ValueError(f"no safetensors files at {path}")
        self.tensors = {}
        for f in files:
            for key, rec in read_header(f).items():
                if key in self.tensors:
                    raise ValueError(f"duplicate tensor across files: {key}")
                self.tensors[key] = rec

    def __getitem__(self, name: str) -> np.ndarray:
        rec = self.tensors.get(checkpoint_name(name))
        if rec is None:
            raise KeyError(name)
        return _float(rec)


def load_original_target(cfg: TargetConfig, quant_dir, base, embedding_weight_path, embedding_scale_path,
                         device="cuda"):
    """Packed weights (``engine.pack_weights``'s result) from the original checkpoint.

    ``base``: a mapping target-name -> float array for the unquantised weights, or a
    path to the HF model file(s) (``BaseWeights``)."""
    from .engine import pack_weights
    from .synthetic import weight_shapes
    if ORIGINAL_GROUP % cfg.quant_group:
        raise ValueError("the configuration's quant_group must divide 256")
    ckpt = OriginalCheckpoint(quant_dir)
    base = BaseWeights(base) if isinstance(base, (str, Path)) else base
    shapes = weight_shapes(cfg)
    dev = torch.device(device)

    def logical(name):
        q, s = ckpt.logical(name, shapes[name])
        return torch.from_numpy(np.array(q)).to(dev), torch.from_numpy(np.array(s)).to(dev)

    def get(name):
        if name == "target.embed_tokens.weight":
            ew, es = load_embedding(embedding_weight_path, embedding_scale_path, shapes[name])
            rows = torch.from_numpy(np.array(ew)).to(dev).float()
            return (rows * torch.from_numpy(np.array(es)).to(dev)).to(torch.bfloat16).float()
        if is_original_quantized(name):
            return dequantize_bf16(*logical(name)).float()
        v = base[name]
        t = v if isinstance(v, torch.Tensor) else torch.from_numpy(np.ascontiguousarray(v, np.float32))
        return t.to(dev).float().reshape(shapes[name])

    def quantized(name):
        q, s = logical(name)
        return q, scales_g128(s, cfg.quant_group)

    return pack_weights(cfg, get, dev, quantized=quantized)
