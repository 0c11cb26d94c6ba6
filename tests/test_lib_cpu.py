"""CPU checks of the C-ABI library and the host-side packing (no GPU needed)."""
import os
import re

import numpy as np
import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared_functions():
    text = open(os.path.join(ROOT, "include", "qw_b200.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(qw_[a-z0-9_]+)\s*\(", text)))


def test_library_loads_and_exports_every_declared_symbol():
    from qwen35_dflash_b200 import lib
    so = lib.load()
    declared = _declared_functions()
    assert len(declared) >= 20
    missing = [name for name in declared if not hasattr(so, name)]
    assert not missing, missing
    # every declared symbol has a typed ctypes signature
    assert not [n for n in declared if n not in lib.SIGNATURES]
    assert so.qw_abi_version() == 1


def test_size_queries_without_gpu():
    from qwen35_dflash_b200 import lib
    so = lib.load()
    assert so.qw_w4_stream_bytes(2048, 4096, 128) == 2048 // 16 * 32 * 1056
    assert so.qw_w4_stream_bytes(100, 4096, 128) == -1
    assert so.qw_b16_stream_bytes(272, 2048) == 17 * 32 * 2048
    assert so.qw_moe_workspace_bytes(16, 2048, 256, 512, 8) > 16 * 9 * 2048 * 4
    assert so.qw_attn_workspace_bytes(1, 16, 2, 16, 256, 4112) > 0


def test_argument_errors_raise_value_error_without_launch():
    from qwen35_dflash_b200 import lib
    with pytest.raises(ValueError):
        lib.call("qw_w4_linear", 16, 16, 16, 0, 15, 1, 15, 128, 128, None)  # N not a multiple of 16
    with pytest.raises(ValueError):
        lib.call("qw_rms_norm", 16, 0, 16, 0, 16, 0, 1, 8, -1.0, None)       # eps <= 0


@pytest.mark.parametrize("group", [32, 64, 128])
def test_w4_pack_roundtrip_and_size(group):
    from qwen35_dflash_b200 import lib, w4
    torch.manual_seed(group)
    q = torch.randint(-8, 8, (64, 512), dtype=torch.int8)
    s = (torch.rand(64, 512 // group) * 0.01 + 0.004).to(torch.bfloat16)
    stream = w4.pack_w4(q, s, group)
    assert stream.numel() == lib.load().qw_w4_stream_bytes(64, 512, group)
    q2, s2 = w4.unpack_w4(stream, 64, 512, group)
    assert torch.equal(q, q2) and torch.equal(s, s2)


def test_w4_stream_fragment_layout():
    """Word (lane, step) of a W4 stream holds A-fragment nibbles in the documented order."""
    from qwen35_dflash_b200 import w4
    n, k, g = 16, 128, 128
    q = (torch.arange(n * k).reshape(n, k) % 16 - 8).to(torch.int8)
    s = torch.ones(n, 1, dtype=torch.bfloat16)
    words = w4.pack_w4(q, s, g)[:8 * g].view(torch.int32).numpy().astype(np.int64) & 0xFFFFFFFF
    for lane in (0, 5, 31):
        gid, tig = lane // 4, lane % 4
        for step in (0, 3, 7):
            word = words[(step // 4) * 128 + lane * 4 + step % 4]
            for j in range(8):
                row = gid + 8 * (j & 1)
                # mma-logical k = 16*step + 2*tig + 8*second + e, stored permuted in 32-blocks
                second, e = (j >> 1) & 1, j >> 2
                col = 32 * (step // 2) + 8 * tig + 4 * (step % 2) + 2 * second + e
                assert (word >> (4 * j)) & 15 == int(q[row, col]) + 8


def test_b16_stream_fragment_layout():
    from qwen35_dflash_b200 import w4
    w = torch.arange(16 * 64, dtype=torch.float32).reshape(16, 64).to(torch.bfloat16)
    st = w4.pack_b16(w).view(torch.bfloat16).float().numpy()
    for lane in (0, 9, 31):
        gid, tig = lane // 4, lane % 4
        for step in range(4):
            base = step * 256 + lane * 8
            for reg in range(4):
                row = gid + 8 * (reg & 1)
                col = 32 * (step // 2) + 8 * tig + 4 * (step % 2) + 2 * (reg >> 1)
                assert st[base + reg * 2] == float(w[row, col])
                assert st[base + reg * 2 + 1] == float(w[row, col + 1])


def test_quantizer_matches_oracle():
    from qwen35_dflash_b200 import w4
    from oracle.numerics import quantize_w4
    rng = np.random.default_rng(3)
    w = rng.normal(0, 0.02, (32, 512)).astype(np.float32)
    w[1, :128] = 0
    q, s = w4.quantize(torch.from_numpy(w), 128)
    qo, so = quantize_w4(w, 128)
    np.testing.assert_array_equal(q.numpy(), qo)
    np.testing.assert_array_equal(s.float().numpy(), so)


def test_k_permutation_is_a_bijection_per_block():
    from qwen35_dflash_b200 import w4
    cols = sorted(w4.physical_k(s, t, sec, e) for s in range(2) for t in range(4) for sec in range(2) for e in range(2))
    assert cols == list(range(32))


def test_fused_ops_module_binds_like_the_reference_adapter():
    from qwen35_dflash_b200 import fused_ops
    assert fused_ops.FUSED_OPS_ABI == 1 and type(fused_ops.FUSED_OPS_ABI) is int
    assert isinstance(fused_ops.BACKEND_ID, str) and fused_ops.BACKEND_ID.strip()
    assert fused_ops.IS_REFERENCE_BACKEND is False
    for name in ("rms_norm", "conv_state_update", "causal_conv1d", "chunk_gated_delta_rule",
                 "cache_update", "attention", "moe"):
        assert callable(getattr(fused_ops, name))


def test_binding_trace_fixture_is_complete(golden):
    """The recorded reference calls (tests/golden/binding_trace.npz) that the GPU replay
    test drives through the module: every operator of the adapter contract occurs, every
    argument resolves (a recorded array, or a weight of the tiny target by name, with
    the shape the call needs), and the decode step came after the prefill."""
    import json
    from qwen35_dflash_b200 import config as qcfg, synthetic
    d = golden("binding_trace.npz")
    calls = json.loads(str(d["calls"]))
    ops = [c["op"] for c in calls]
    assert set(ops) == {"rms_norm", "conv_state_update", "causal_conv1d", "chunk_gated_delta_rule",
                        "cache_update", "attention", "moe"}
    shapes = {k: v.shape for k, v in synthetic.init_weights(qcfg.TINY, seed=17).items()}
    seen = set()

    def check(e):
        if "weight" in e:
            assert e["weight"] in shapes, e["weight"]
            seen.add(e["weight"])
        elif "array" in e:
            assert e["array"] in d.files and e["dtype"] in ("float16", "bfloat16", "float32", "int16", "int32", "int64")
        elif "seq" in e:
            for x in e["seq"]:
                check(x)
        else:
            assert "value" in e
    for c in calls:
        for a in c["args"]:
            check(a)
        for v in c["kwargs"].values():
            check(v)
        check(c["out"])
    # the MoE calls pass the router and expert banks of every MoE layer by name
    moe = [c for c in calls if c["op"] == "moe"]
    assert len(moe) == 2 * qcfg.TINY.num_hidden_layers
    e, i, h = qcfg.TINY.num_experts, qcfg.TINY.moe_intermediate_size, qcfg.TINY.hidden_size
    for c in moe:
        assert shapes[c["args"][2]["weight"]] == (e, 2 * i, h)
        assert shapes[c["args"][3]["weight"]] == (e, h, i)
    # attention: the prefill sees keys from 0, the decode step after the 16 prompt tokens
    starts = [c["kwargs"]["query_start"]["value"] for c in calls if c["op"] == "attention"]
    assert starts == [0, 16]
    assert len(d["next_tokens"]) == 2


def test_fused_ops_rejects_cpu_tensors():
    from qwen35_dflash_b200 import fused_ops
    x = torch.zeros(2, 8)
    with pytest.raises(ValueError):
        fused_ops.rms_norm(x, torch.ones(8), 1e-6)
    with pytest.raises(ValueError):
        fused_ops.chunk_gated_delta_rule(x, x, x, x, x, x, x, chunk_size=3, use_qk_l2norm_in_kernel=True)
