"""CUDA kernels vs the oracle / the reference's golden outputs (GPU)."""
import ctypes

import numpy as np
import pytest
import torch

from helpers import assert_close, to_np, bf16_tensor, struct_array_to_device, oracle_gdn_layer
from oracle import fused_ops_np as F
from oracle.numerics import bf16_round

pytestmark = pytest.mark.gpu

DT = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}


def _t(a, dtype):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda().to(dtype)


def _lowp(golden, tag):
    return {k[len(tag) + 1:]: v for k, v in golden("ops_lowp.npz").items() if k.startswith(tag + "_")}


@pytest.mark.parametrize("tag", ["f32", "bf16", "f16"])
def test_rms_norm_matches_reference(golden, cuda_lib, tag):
    from qwen35_dflash_b200 import fused_ops as Q
    d = dict(golden("ops_fp32.npz")) if tag == "f32" else _lowp(golden, tag)
    ulp = {"f32": 1e-6, "bf16": 2 ** -8, "f16": 2 ** -11}[tag]
    for i in range(2):
        y = Q.rms_norm(_t(d[f"rms{i}_x"], DT[tag]), _t(d[f"rms{i}_g"], DT[tag]), 1e-6)
        assert y.dtype == DT[tag]
        assert_close(to_np(y), d[f"rms{i}_y"], 1e-6, 2 * ulp, f"rms{i}")


@pytest.mark.parametrize("tag", ["f32", "bf16", "f16"])
def test_conv_ops_match_reference(golden, cuda_lib, tag):
    from qwen35_dflash_b200 import fused_ops as Q
    d = dict(golden("ops_fp32.npz")) if tag == "f32" else _lowp(golden, tag)
    nh, padded = Q.conv_state_update(_t(d["conv_proj"], DT[tag]), _t(d["conv_hist"], DT[tag]))
    np.testing.assert_array_equal(to_np(padded), d["conv_padded"])
    if "conv_newhist" in d:
        np.testing.assert_array_equal(to_np(nh), d["conv_newhist"])
    out = Q.causal_conv1d(padded, _t(d["conv_w"], DT[tag]))
    ulp = {"f32": 1e-6, "bf16": 2 ** -8, "f16": 2 ** -11}[tag]
    assert_close(to_np(out), d["conv_out"], 1e-6, 2 * ulp, "conv")
    k, v = Q.cache_update(_t(d["cache_k0"], DT[tag]), _t(d["cache_v0"], DT[tag]),
                          _t(d["cache_k1"], DT[tag]), _t(d["cache_v1"], DT[tag]))
    np.testing.assert_array_equal(to_np(k), d["cache_k"])
    np.testing.assert_array_equal(to_np(v), d["cache_v"])
    k0, v0 = Q.cache_update(None, None, _t(d["cache_k1"], DT[tag]), _t(d["cache_v1"], DT[tag]))
    np.testing.assert_array_equal(to_np(k0), d["cache_k1"])


@pytest.mark.parametrize("tag", ["f32", "f16"])
def test_gated_delta_rule_matches_reference(golden, cuda_lib, tag):
    from qwen35_dflash_b200 import fused_ops as Q
    d = dict(golden("ops_fp32.npz")) if tag == "f32" else _lowp(golden, tag)
    args = [_t(d[n], DT[tag]) for n in ("gdn_q", "gdn_k", "gdn_v", "gdn_g", "gdn_beta")]
    s0 = _t(d["gdn_s0"], torch.float32)
    lens = torch.from_numpy(d["gdn_len"]).cuda()
    for norm in (0, 1):
        core, st = Q.chunk_gated_delta_rule(*args, s0, lens, chunk_size=64,
                                            use_qk_l2norm_in_kernel=bool(norm))
        tol = 1e-5 if tag == "f32" else 2e-3
        assert_close(to_np(core), d[f"gdn_core_{norm}"], tol, tol * 10, "core")
        if tag == "f32":
            assert_close(to_np(st), d[f"gdn_state_{norm}"], 1e-5, 1e-4, "state")


@pytest.mark.parametrize("batch", [1, 8, 32])
def test_gated_delta_rule_config3_shapes(cuda_lib, batch):
    """Full head shape (32 heads x 128) with ragged effective lengths, fp32 in and out."""
    from qwen35_dflash_b200 import fused_ops as Q
    rng = np.random.default_rng(batch)
    b, s, h, dk = batch, 16, 32, 128
    q, k, v = (rng.normal(0, 1, (b, s, h, dk)).astype(np.float32) for _ in range(3))
    g = -F.softplus(rng.normal(0, 1, (b, s, h))).astype(np.float32)
    beta = F.sigmoid(rng.normal(0, 1, (b, s, h))).astype(np.float32)
    s0 = rng.normal(0, 0.02, (b, h, dk, dk)).astype(np.float32)
    lens = np.array([(16, 0, 7, 1, 16, 15, 3, 9)[i % 8] for i in range(b)], np.int16)
    core, st = F.chunk_gated_delta_rule(q, k, v, g, beta, s0, lens, chunk_size=64,
                                        use_qk_l2norm_in_kernel=True)
    gc, gs = Q.chunk_gated_delta_rule(*[_t(a, torch.float32) for a in (q, k, v, g, beta)],
                                      _t(s0, torch.float32), torch.from_numpy(lens).cuda(),
                                      chunk_size=64, use_qk_l2norm_in_kernel=True)
    assert_close(to_np(gc), core, 1e-4, 1e-3, "core")
    assert_close(to_np(gs), st, 1e-5, 1e-4, "state")


W4_SHAPES = [(12288, 2048, 128), (2048, 4096, 128), (9216, 2048, 128), (1024, 256, 32), (512, 512, 64)]


@pytest.mark.parametrize("n,k,group", W4_SHAPES)
@pytest.mark.parametrize("tokens", [1, 16, 33])
def test_w4_linear_matches_dequantized_matmul(cuda_lib, n, k, group, tokens):
    from qwen35_dflash_b200 import fused_ops as Q, w4
    torch.manual_seed(n + k + tokens)
    q = torch.randint(-8, 8, (n, k), dtype=torch.int8, device="cuda")
    scale = (torch.rand(n, k // group, device="cuda") * 0.015 + 0.005).to(torch.bfloat16)
    stream = w4.pack_w4(q, scale, group)
    x = torch.randn(tokens, k, device="cuda").to(torch.bfloat16)
    ref = x.float() @ w4.dequantize(q, scale, group).T
    y32 = Q.qlinear_w4a16(x, stream, n, group, out_dtype=torch.float32)
    assert_close(to_np(y32), to_np(ref), 1e-3, 1e-4, "w4 f32")
    y = Q.qlinear_w4a16(x, stream, n, group)
    assert_close(to_np(y), to_np(ref.to(torch.bfloat16)), 1e-2, 8e-3, "w4 bf16")


@pytest.mark.parametrize("n,k", [(272, 2048), (64, 2048), (4096, 256), (248320 // 16, 2048)])
@pytest.mark.parametrize("tokens", [1, 16])
def test_b16_linear_matches_matmul(cuda_lib, n, k, tokens):
    from qwen35_dflash_b200 import fused_ops as Q, w4
    torch.manual_seed(n + tokens)
    w = (torch.randn(n, k, device="cuda") * 0.02).to(torch.bfloat16)
    x = torch.randn(tokens, k, device="cuda").to(torch.bfloat16)
    ref = x.float() @ w.float().T
    y = Q.linear_b16(x, w4.pack_b16(w), n, out_dtype=torch.float32)
    assert_close(to_np(y), to_np(ref), 1e-4, 1e-4, "b16")


def test_residual_mode_adds_in_place(cuda_lib):
    from qwen35_dflash_b200 import lib, w4
    torch.manual_seed(3)
    n, k, g, t = 256, 512, 128, 16
    q = torch.randint(-8, 8, (n, k), dtype=torch.int8, device="cuda")
    scale = (torch.rand(n, k // g, device="cuda") * 0.01 + 0.005).to(torch.bfloat16)
    stream = w4.pack_w4(q, scale, g)
    x = torch.randn(t, k, device="cuda").to(torch.bfloat16)
    resid = torch.randn(t, n, device="cuda").to(torch.bfloat16)
    before = resid.clone()
    lib.call("qw_w4_linear", x.data_ptr(), stream.data_ptr(), resid.data_ptr(), lib.QW_OUT_RESID_BF16,
             n, t, n, k, g, lib.stream_ptr())
    mixed = (x.float() @ w4.dequantize(q, scale, g).T).to(torch.bfloat16)
    want = (before.float() + mixed.float()).to(torch.bfloat16)
    assert_close(to_np(resid), to_np(want), 1e-2, 8e-3, "resid")


def _gdn_case(batch, seq, k_heads, v_heads, dk, dv, slots, seed):
    rng = np.random.default_rng(seed)
    kw, vw = k_heads * dk, v_heads * dv
    c = 2 * kw + vw
    ldp = c + vw
    nslot = max(slots) + 1
    proj = bf16_round(rng.normal(0, 1, (batch, seq, ldp)))
    ab = rng.normal(0, 1, (batch, seq, 2 * v_heads)).astype(np.float32)
    hist = bf16_round(rng.normal(0, 1, (nslot, c, 3)))
    conv_w = bf16_round(rng.normal(0, 0.3, (c, 4)))
    a_log = np.log(np.arange(1, v_heads + 1, dtype=np.float32))
    dt_bias = rng.normal(0, 0.5, (v_heads,)).astype(np.float32)
    norm_w = bf16_round(1 + rng.normal(0, 0.1, (dv,)))
    state = rng.normal(0, 0.02, (nslot, v_heads, dk, dv)).astype(np.float32)
    return dict(proj=proj, ab=ab, hist=hist, conv_w=conv_w, a_log=a_log, dt_bias=dt_bias,
                norm_w=norm_w, state=state, ldp=ldp, c=c)


def _gdn_device(case, batch, seq, k_heads, v_heads, dk, dv, slots):
    from qwen35_dflash_b200 import lib
    dev = {
        "proj": bf16_tensor(case["proj"].reshape(batch * seq, -1)),
        "ab": torch.from_numpy(case["ab"].reshape(batch * seq, -1)).cuda(),
        "hist": bf16_tensor(case["hist"]),
        "conv_w": bf16_tensor(case["conv_w"]),
        "a_log": torch.from_numpy(case["a_log"]).cuda(),
        "dt_bias": torch.from_numpy(case["dt_bias"]).cuda(),
        "norm_w": bf16_tensor(case["norm_w"]),
        # bank layout: [slot, head, dv, dk]
        "state": torch.from_numpy(np.ascontiguousarray(case["state"].transpose(0, 1, 3, 2))).cuda(),
        "out": torch.zeros(batch * seq, v_heads * dv, dtype=torch.bfloat16, device="cuda"),
        "slots": torch.tensor(slots, dtype=torch.int32, device="cuda"),
    }
    layer = (lib.GdnLayer * 1)()
    layer[0] = lib.GdnLayer(dev["proj"].data_ptr(), dev["ab"].data_ptr(), dev["hist"].data_ptr(),
                            dev["conv_w"].data_ptr(), dev["a_log"].data_ptr(), dev["dt_bias"].data_ptr(),
                            dev["norm_w"].data_ptr(), dev["state"].data_ptr(), dev["out"].data_ptr())
    dev["layers"] = struct_array_to_device(layer)
    dims = lib.GdnDims(batch, seq, k_heads, v_heads, dk, dv, case["c"], 4, case["ldp"], 1e-6,
                       dev["slots"].data_ptr(), None)
    return dev, dims


@pytest.mark.parametrize("batch,k_heads,v_heads,dk", [(1, 16, 32, 128), (3, 4, 8, 64), (8, 16, 32, 128),
                                                    (32, 16, 32, 128)])
def test_gdn_verify_and_commit(cuda_lib, batch, k_heads, v_heads, dk):
    from qwen35_dflash_b200 import lib
    seq, dv = 16, dk
    # distinct bank slots, scattered over twice the batch
    slots = [int(i) for i in np.random.default_rng(batch + 100).permutation(2 * batch + 1)[:batch]]
    case = _gdn_case(batch, seq, k_heads, v_heads, dk, dv, slots, seed=batch)
    dev, dims = _gdn_device(case, batch, seq, k_heads, v_heads, dk, dv, slots)
    accepted = [(16, 0, 5, 1, 9, 16, 3, 12)[i % 8] for i in range(batch)]
    sl = np.asarray(slots)
    out, _, commits = oracle_gdn_layer(
        case["proj"], case["ab"], case["hist"][sl], case["conv_w"], case["a_log"], case["dt_bias"],
        case["norm_w"], case["state"][sl], k_heads=k_heads, v_heads=v_heads, dk=dk, dv=dv,
        eps=1e-6, accepted=sorted(set(accepted)))
    st = lib.stream_ptr()
    lib.check(cuda_lib.qw_gdn_verify(ctypes.byref(dims), dev["layers"].data_ptr(), 0, st), "verify")
    got = to_np(dev["out"]).reshape(batch, seq, -1)
    assert_close(got, out, what="gdn verify out")
    # verify must not touch the banks
    np.testing.assert_array_equal(to_np(dev["state"]), case["state"].transpose(0, 1, 3, 2))
    acc_t = torch.tensor(accepted, dtype=torch.int32, device="cuda")
    dims.accepted = acc_t.data_ptr()
    lib.check(cuda_lib.qw_gdn_commit(ctypes.byref(dims), dev["layers"].data_ptr(), 1, st), "commit")
    torch.cuda.synchronize()
    bank = to_np(dev["state"]).transpose(0, 1, 3, 2)
    hist = to_np(dev["hist"])
    for i, r in enumerate(accepted):
        want_state = case["state"][slots[i]] if r == 0 else commits[r][0][i]
        want_hist = case["hist"][slots[i]] if r == 0 else commits[r][1][i]
        assert_close(bank[slots[i]], want_state, 1e-5, 1e-4, f"state seq {i} r={r}")
        np.testing.assert_array_equal(hist[slots[i]], want_hist)


def _stable_top1_bits(logits_bf16: torch.Tensor) -> np.ndarray:
    """Row argmax of bf16 logits by the stable top-1 rule of the reference
    (targets/cpro/ops/draft-top1/src/reference/top1_cpu.cpp:12-46): the larger value
    wins, -0 and +0 are equal, ties go to the lowest index."""
    bits = logits_bf16.view(torch.int16).cpu().numpy().astype(np.int64) & 0xFFFF
    bits = np.where((bits & 0x7FFF) == 0, 0, bits)
    key = np.where(bits & 0x8000, (~bits) & 0xFFFF, bits ^ 0x8000)
    return np.argmax(key, axis=-1).astype(np.int32)   # numpy: the first maximum


@pytest.mark.parametrize("n", [32768, 248320])
def test_lmhead_argmax_stable_ties(cuda_lib, n):
    """qw_lmhead_argmax + qw_accept against the stable top-1 rule with planted ties:
    rows 0-7 have an exact tie of three duplicated lm_head rows at their maximum, in
    different CTAs (the lowest index must win); rows 8-11 have their maximum at 0 with a
    -0 logit below a +0 one in index order (an activation pair whose products cancel to a
    negative value under bf16's smallest subnormal, so the bf16 logit is -0); rows 12-15
    have x = 0, every logit +0 (index 0 wins).  The kernel's logits come back too: its
    top-1 must equal the rule applied to them, and the planted maxima must be where
    they were planted."""
    from qwen35_dflash_b200 import lib, w4
    torch.manual_seed(n)
    k, t = 2048, 16
    dup = [17, n // 3 + 5, n - 40]          # three equal rows, far apart (different CTAs)
    neg0, pos0 = 40, (41, 3001)              # the -0 row below the +0 rows
    base = torch.randn(k, device="cuda")
    x = torch.zeros(t, k, device="cuda")
    x[:8] = base + 0.05 * torch.randn(8, k, device="cuda")
    # rows 8-11: only k = 0 and k = 256 are nonzero (positive), bf16-exact
    x[8:12, 0] = (1 + 2 ** -6) * 2.0 ** -62
    x[8:12, 256] = (1 + 2 ** -7) * 2.0 ** -62
    w = torch.randn(n, k, device="cuda") * 0.02
    w[:, 0] = -w[:, 0].abs() - 0.01         # rows 8-11: every ordinary logit < 0
    w[:, 256] = -w[:, 256].abs() - 0.01
    best = base * 0.5
    best[0] = best[256] = -1.0
    for r in dup:
        w[r] = best
    w[neg0] = 0.0                             # products (1+2^-6)2^-125 and -(1+2^-7)^2 2^-125
    w[neg0, 0] = 2.0 ** -63
    w[neg0, 256] = -(1 + 2 ** -7) * 2.0 ** -63
    for r in pos0:
        w[r] = 0.0
    x = x.to(torch.bfloat16)
    w = w.to(torch.bfloat16)
    assert float(x[8, 0]) == (1 + 2 ** -6) * 2.0 ** -62 and float(w[neg0, 256]) == -(1 + 2 ** -7) * 2.0 ** -63
    stream = w4.pack_b16(w)
    nblk = cuda_lib.qw_lmhead_blocks(n)
    keys = torch.zeros(nblk, t, dtype=torch.int64, device="cuda")
    logits = torch.empty(t, n, dtype=torch.bfloat16, device="cuda")
    st = lib.stream_ptr()
    lib.call("qw_lmhead_argmax", x.data_ptr(), stream.data_ptr(), logits.data_ptr(), keys.data_ptr(), t, n, k, st)
    props = torch.zeros(t, dtype=torch.int32, device="cuda")
    top1 = torch.empty(t, dtype=torch.int32, device="cuda")
    maxacc = torch.empty(1, dtype=torch.int32, device="cuda")
    nxt = torch.zeros(1, dtype=torch.int32, device="cuda")
    lib.call("qw_accept", keys.data_ptr(), nblk, props.data_ptr(), top1.data_ptr(), maxacc.data_ptr(),
             nxt.data_ptr(), None, None, 1, t, 0, st)
    torch.cuda.synchronize()
    got = top1.cpu().numpy()
    np.testing.assert_array_equal(got, _stable_top1_bits(logits))
    lg = logits.float().cpu().numpy()
    for i in range(8):       # the duplicated rows are the maximum, bit-equal
        assert lg[i, dup[0]] == lg[i, dup[1]] == lg[i, dup[2]] == lg[i].max(), i
    assert (got[:8] == dup[0]).all(), got[:8]
    bits = logits.view(torch.int16).cpu().numpy().astype(np.int64) & 0xFFFF
    for i in range(8, 12):   # maximum 0 with the -0 logit first; the rule takes the -0 row
        # the planted row is -0 when the fp32 accumulator keeps the subnormal sum (it is
        # +0 if the sum is flushed; either way the lowest index holds the maximum)
        assert bits[i, neg0] in (0x8000, 0) and bits[i, pos0[0]] == 0 and bits[i, pos0[1]] == 0, i
        assert lg[i].max() == 0.0, i
    print(f"\nplanted -0 logit came out as 0x{int(bits[8, neg0]):04x}")
    assert (got[8:12] == neg0).all(), got[8:12]
    assert (got[12:] == 0).all(), got[12:]
