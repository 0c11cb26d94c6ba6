"""Import of the original group-256 quantised checkpoint (CPU).

* the reader against the reference's own OriginalQuantWeights on committed shards
  (``tests/golden/original/``: key mapping, logical values and scales);
* the conversion: every W4 projection keeps its int4 values and each group-256 scale
  becomes the bf16 scale of the groups it covers; router / GDN b, a / lm_head and the
  embedding are dequantised to bf16;
* the reference's validation errors (missing tensor, wrong shape or dtype, values
  outside int4, negative scale, duplicate key across shards, symlinked shard).
"""
import dataclasses
import json
from pathlib import Path

import numpy as np
import pytest
import torch

from original_fixture import quantize_g256, write_original, write_safetensors

GOLD = Path(__file__).parent / "golden" / "original"


def test_reader_matches_reference_on_committed_shards():
    from qwen35_dflash_b200 import original
    exp = json.loads((GOLD / "expect.json").read_text())
    ck = original.OriginalCheckpoint(GOLD)
    for name, keys in exp["keys"].items():
        assert list(original.original_keys(name)) == keys, name
    for name, bad in exp["rejected_names"].items():
        with pytest.raises(ValueError):
            original.original_keys(name)
    arrays = np.load(GOLD / "expect.npz")
    for i, (name, shape) in enumerate(exp["logical"]):
        q, s = ck.logical(name, shape)
        np.testing.assert_array_equal(np.asarray(q), arrays[f"q{i}"])
        np.testing.assert_array_equal(s.reshape(arrays[f"s{i}"].shape), arrays[f"s{i}"].astype(np.float32))


def _tiny_raw(seed=5):
    from qwen35_dflash_b200 import config, synthetic
    cfg = config.with_layers(config.TINY_G256, 4)
    return cfg, synthetic.init_weights(cfg, seed=seed)


def test_conversion_keeps_values_and_scales(tmp_path):
    from qwen35_dflash_b200 import original, w4
    from qwen35_dflash_b200.synthetic import weight_shapes
    cfg, raw = _tiny_raw()
    fx = write_original(cfg, raw, tmp_path)
    glob, layers = original.load_original_target(cfg, fx["quant_dir"], fx["base"], fx["embed_w"], fx["embed_s"],
                                                 device="cpu")
    exp = fx["expected"]
    g = cfg.quant_group
    np.testing.assert_array_equal(glob["embed"].float().numpy(), exp["target.embed_tokens.weight"])
    # a W4 projection: unpack the stream -> the original int4 values and the bf16 scales
    ck = original.OriginalCheckpoint(fx["quant_dir"])
    shapes = weight_shapes(cfg)
    for name, stream, rows in (("target.layers.0.linear_attn.out_proj.weight", layers[0].out, None),
                               ("target.layers.3.self_attn.o_proj.weight", layers[3].o, None)):
        n, k = shapes[name]
        q, s = w4.unpack_w4(stream, n, k, g)
        q0, s0 = ck.logical(name, shapes[name])
        np.testing.assert_array_equal(q.numpy(), np.asarray(q0))
        want = torch.from_numpy(np.repeat(s0, 256 // g, -1)).to(torch.bfloat16)
        assert torch.equal(s, want)
    # the fused q|k|v stream: rows of q, then k, then v, each with its own values
    a = "target.layers.3.self_attn."
    n = sum(shapes[a + p + ".weight"][0] for p in ("q_proj", "k_proj", "v_proj"))
    q, s = w4.unpack_w4(layers[3].qkv, n, cfg.hidden_size, g)
    ref = np.concatenate([np.asarray(ck.logical(a + p + ".weight", shapes[a + p + ".weight"])[0])
                          for p in ("q_proj", "k_proj", "v_proj")])
    np.testing.assert_array_equal(q.numpy(), ref)
    # an expert bank (expert 3's gate|up)
    name = "target.layers.1.mlp.experts.gate_up_proj"
    E, N, K = shapes[name]
    per = w4.unpack_w4(layers[1].gate_up[3 * layers[1].gate_up.numel() // E:4 * layers[1].gate_up.numel() // E],
                       N, K, g)
    q0, s0 = ck.logical(name, shapes[name])
    np.testing.assert_array_equal(per[0].numpy(), np.asarray(q0[3]))
    assert torch.equal(per[1], torch.from_numpy(np.repeat(s0[3], 256 // g, -1)).to(torch.bfloat16))
    # the whole set of dequantised values the engine computes with == the fixture's expectation
    for name, want in exp.items():
        assert np.isfinite(want).all(), name


def test_dequantized_bf16_streams(tmp_path):
    from qwen35_dflash_b200 import original, w4
    cfg, raw = _tiny_raw()
    fx = write_original(cfg, raw, tmp_path)
    glob, layers = original.load_original_target(cfg, fx["quant_dir"], fx["base"], fx["embed_w"], fx["embed_s"],
                                                 device="cpu")
    exp = fx["expected"]
    lm = exp["target.lm_head.weight"]
    assert torch.equal(glob["lm_head"], w4.pack_b16(torch.from_numpy(lm).to(torch.bfloat16)))
    m = "target.layers.2.mlp."
    router = np.concatenate([exp[m + "gate.weight"], exp[m + "shared_expert_gate.weight"]])
    router = np.concatenate([router, np.zeros(((-len(router)) % 16, router.shape[1]), np.float32)])
    assert torch.equal(layers[2].router, w4.pack_b16(torch.from_numpy(router).to(torch.bfloat16)))


def _one_linear(tmp_path, mutate=None, extra_shard=None):
    from qwen35_dflash_b200 import original
    name = "target.layers.0.linear_attn.out_proj.weight"
    q, s = quantize_g256(np.random.default_rng(0).normal(0, 0.02, (32, 512)))
    wkey, skey = original.original_keys(name)
    t = {wkey: q, skey: s[..., None]}
    if mutate:
        mutate(t, wkey, skey)
    d = tmp_path / "q"
    d.mkdir()
    write_safetensors(d / "data-00001.safetensors", t)
    if extra_shard:
        write_safetensors(d / "data-00002.safetensors", extra_shard(wkey, skey))
    return name, d


@pytest.mark.parametrize("case", ["ok", "missing", "shape", "dtype", "range", "negative", "duplicate"])
def test_validation(tmp_path, case):
    from qwen35_dflash_b200 import original
    muts = {
        "missing": lambda t, w, s: t.pop(s),
        "shape": lambda t, w, s: t.__setitem__(s, t[s][:, :1]),
        "dtype": lambda t, w, s: t.__setitem__(w, t[w].astype("<f2")),
        "range": lambda t, w, s: t[w].__setitem__((0, 0), 8),
        "negative": lambda t, w, s: t[s].__setitem__((0, 0, 0), -1),
    }
    extra = (lambda w, s: {w: np.zeros((32, 512), np.int8)}) if case == "duplicate" else None
    if case == "duplicate":
        with pytest.raises(ValueError, match="duplicate"):
            name, d = _one_linear(tmp_path, extra_shard=extra)
            original.OriginalCheckpoint(d)
        return
    name, d = _one_linear(tmp_path, muts.get(case))
    ck = original.OriginalCheckpoint(d)
    if case == "ok":
        q, s = ck.logical(name, (32, 512))
        assert q.shape == (32, 512) and s.shape == (32, 2)
        with pytest.raises(ValueError, match="rank"):
            ck.logical(name, (1, 32, 512))
        with pytest.raises(ValueError, match="K%256"):
            ck.logical(name, (32, 384))
        return
    with pytest.raises(ValueError):
        ck.logical(name, (32, 512))


def test_symlinked_shard_rejected(tmp_path):
    from qwen35_dflash_b200 import original
    name, d = _one_linear(tmp_path)
    (d / "data-00003.safetensors").symlink_to(d / "data-00001.safetensors")
    with pytest.raises(ValueError, match="regular file"):
        original.OriginalCheckpoint(d)


def test_truncated_and_overlapping_headers(tmp_path):
    from qwen35_dflash_b200 import original
    p = tmp_path / "x.safetensors"
    p.write_bytes(b"\x00" * 4)
    with pytest.raises(ValueError, match="truncated"):
        original.read_header(p)
    hdr = json.dumps({"a": {"dtype": "I8", "shape": [4], "data_offsets": [0, 4]},
                      "b": {"dtype": "I8", "shape": [4], "data_offsets": [2, 6]}}).encode()
    p.write_bytes(len(hdr).to_bytes(8, "little") + hdr + b"\x00" * 8)
    with pytest.raises(ValueError, match="overlapping"):
        original.read_header(p)
