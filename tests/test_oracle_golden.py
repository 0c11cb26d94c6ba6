"""Pin the CPU oracle to outputs of the reference itself (fixtures from make_golden.py)."""
import numpy as np
import torch
import pytest

from oracle import fused_ops_np as F
from oracle.numerics import topk_indices, bf16_round, quantize_w4, dequantize_w4
from oracle.model_np import OracleTarget, verify, commit


def _close(a, b, atol, rtol):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    assert a.shape == b.shape, (a.shape, b.shape)
    err = np.abs(a - b) - (atol + rtol * np.abs(b))
    assert err.max() <= 0, f"max excess {err.max():.3e}, max abs diff {np.abs(a - b).max():.3e}"


def test_fp32_ops(golden):
    d = golden("ops_fp32.npz")
    for i in range(2):
        _close(F.rms_norm(d[f"rms{i}_x"], d[f"rms{i}_g"], 1e-6), d[f"rms{i}_y"], 1e-6, 1e-5)
    nh, padded = F.conv_state_update(d["conv_proj"], d["conv_hist"])
    np.testing.assert_array_equal(nh, d["conv_newhist"])
    np.testing.assert_array_equal(padded, d["conv_padded"])
    _close(F.causal_conv1d(padded, d["conv_w"]), d["conv_out"], 1e-6, 1e-5)
    k, v = F.cache_update(d["cache_k0"], d["cache_v0"], d["cache_k1"], d["cache_v1"])
    np.testing.assert_array_equal(k, d["cache_k"])
    np.testing.assert_array_equal(v, d["cache_v"])
    _close(F.attention(d["attn_q"], d["attn_k"], d["attn_v"], query_start=8, scale=32 ** -0.5),
           d["attn_o"], 1e-6, 1e-5)
    for norm in (0, 1):
        core, state = F.chunk_gated_delta_rule(
            d["gdn_q"], d["gdn_k"], d["gdn_v"], d["gdn_g"], d["gdn_beta"], d["gdn_s0"], d["gdn_len"],
            chunk_size=64, use_qk_l2norm_in_kernel=bool(norm))
        _close(core, d[f"gdn_core_{norm}"], 1e-5, 1e-4)
        _close(state, d[f"gdn_state_{norm}"], 1e-5, 1e-4)
    _close(F.moe(d["moe_x"], d["moe_router"], d["moe_gu"], d["moe_down"], top_k=4),
           d["moe_y"], 1e-5, 1e-4)


@pytest.mark.parametrize("tag", ["bf16", "f16"])
def test_lowp_ops(golden, tag):
    """Rounding points of the reference at bf16 / fp16 (one final-ulp slack)."""
    d = {k[len(tag) + 1:]: v for k, v in golden("ops_lowp.npz").items() if k.startswith(tag + "_")}
    ulp = 2.0 ** -8 if tag == "bf16" else 2.0 ** -11
    for i in range(2):
        _close(F.rms_norm(d[f"rms{i}_x"], d[f"rms{i}_g"], 1e-6, tag), d[f"rms{i}_y"], 1e-6, 2 * ulp)
    nh, padded = F.conv_state_update(d["conv_proj"], d["conv_hist"])
    np.testing.assert_array_equal(padded, d["conv_padded"])
    _close(F.causal_conv1d(padded, d["conv_w"], tag), d["conv_out"], 1e-6, 2 * ulp)
    _close(F.attention(d["attn_q"], d["attn_k"], d["attn_v"], query_start=8, scale=32 ** -0.5, dtype=tag),
           d["attn_o"], 1e-6, 2 * ulp)
    y = F.moe(d["moe_x"], d["moe_router"], d["moe_gu"], d["moe_down"], top_k=4, dtype=tag)
    _close(y, d["moe_y"], 4 * ulp, 4 * ulp)
    if tag == "f16":
        for norm in (0, 1):
            core, state = F.chunk_gated_delta_rule(
                d["gdn_q"], d["gdn_k"], d["gdn_v"], d["gdn_g"], d["gdn_beta"], d["gdn_s0"],
                d["gdn_len"], chunk_size=1, use_qk_l2norm_in_kernel=bool(norm), dtype="f16")
            _close(core, d[f"gdn_core_{norm}"], 1e-4, 2 * ulp)


def test_topk_matches_torch(golden):
    d = golden("topk.npz")
    for key in d.files:
        if key.startswith("p_"):
            _, e, k = key.split("_")
            got = topk_indices(d[key], int(k))
            np.testing.assert_array_equal(got, d[f"i_{e}_{k}"].astype(np.int64), err_msg=key)


@pytest.mark.parametrize("n,k", [(16, 4), (40, 6), (64, 8), (128, 8), (256, 8), (257, 8), (256, 2),
                                 (512, 8), (1024, 8), (96, 17)])
def test_topk_matches_live_torch_topk(n, k):
    """The oracle's restatement of torch.topk's CPU tie order against torch.topk itself
    (this process's torch), on seeded rows dense in ties: small integers, bf16-rounded
    normals and signed zeros; both of ATen's paths (nth_element + sort when k * 64 > n,
    partial_sort otherwise)."""
    g = torch.Generator().manual_seed(n * 31 + k)
    rows = [torch.randint(-3, 4, (24, n), generator=g).float(),
            torch.randn(24, n, generator=g).to(torch.bfloat16).float(),
            torch.where(torch.rand(8, n, generator=g) < 0.3, torch.ones(8, n),
                        torch.where(torch.rand(8, n, generator=g) < 0.5, torch.full((8, n), -0.0), torch.zeros(8, n)))]
    assert torch.signbit(rows[2]).any() and (rows[2] == 0).any()
    for x in rows:
        want = torch.topk(x, k, dim=-1).indices.numpy()
        got = topk_indices(x.numpy(), k)
        np.testing.assert_array_equal(got, want, err_msg=f"n={n} k={k}")


def test_quantizer_roundtrip():
    rng = np.random.default_rng(0)
    w = rng.normal(0, 0.02, (48, 256)).astype(np.float32)
    w[3, :128] = 0.0
    q, s = quantize_w4(w, 128)
    assert q.min() >= -8 and q.max() <= 7
    assert np.all(bf16_round(s) == s) and s[3, 0] == 1.0
    deq = dequantize_w4(q, s, 128)
    assert np.abs(deq - w).max() <= s.max() * 0.5 + 1e-7


def _rows_close_fraction(a, b, atol, rtol):
    """Fraction of rows (last axis) whose every element is within atol + rtol*|b|."""
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    ok = (np.abs(a - b) <= atol + rtol * np.abs(b)).all(-1)
    return float(ok.mean())


def _tiny_oracle(act, rope):
    from qwen35_dflash_b200 import config as qcfg, synthetic
    from oracle.numerics import f16_round
    cfg = qcfg.TINY
    raw = synthetic.init_weights(cfg, seed=17)
    weights = {}
    for name, value in raw.items():
        if synthetic.is_w4(name):
            q, s = quantize_w4(value, cfg.quant_group)
            value = dequantize_w4(q, s, cfg.quant_group)
        weights[name] = f16_round(value) if act == "f16" else value
    return cfg, OracleTarget(cfg.to_hf_text_config(), weights, cfg.feature_layers, act=act, rope=rope)


def test_tiny_layers_fp16_teacher_forced(golden):
    """Each decoder layer of the oracle (FP16), fed the reference's previous-layer output,
    reproduces the reference's layer output on the 64-token prompt.

    MoE routing is discontinuous: a one-ulp difference inside a layer (fp32 summation
    order) can swap a near-tied expert for one token, so rows are counted.
    """
    d = golden("tiny_session.npz")
    cfg, model = _tiny_oracle("f16", "f16")
    hidden_ref = d["layer_hidden"].astype(np.float32)
    prompt = d["prompt"]
    state = model.initial_state(1)
    x = model.w["target.embed_tokens.weight"][prompt][None]
    for layer in range(cfg.num_hidden_layers):
        out, _ = model.layer(layer, x, state.layers[layer], 0)
        if layer == cfg.num_hidden_layers - 1:
            out = model.norm(out, "target.norm.weight")
        frac = _rows_close_fraction(out[0], hidden_ref[layer], 1e-3, 1e-2)
        assert frac >= 0.95, (layer, frac)
        x = hidden_ref[layer][None]


def test_tiny_session_fp16_matches_reference(golden):
    """Free-running block verify / commit rounds against the reference FusedTargetSession.

    Teacher-forced layers agree to an ulp (test above); free-running, a near-tied
    routing decision resolved differently by fp32 summation order can move one
    token's logits, so >= 95% of predicted tokens and >= 6 of 8 acceptance counts
    must agree.  The session semantics (which row is compared, what commit keeps)
    are exact: rounds are replayed with the reference's own accepted counts.
    """
    d = golden("tiny_session.npz")
    cfg, model = _tiny_oracle("f16", "f16")
    prompt = d["prompt"]
    top1, feats, state, _ = model.forward(prompt[None, :])
    assert int(top1[0, -1]) == int(d["greedy"][0])
    next_token = int(top1[0, -1])
    agree = total = same_acc = 0
    for props, expected, accepted in zip(d["proposals"], d["expected"], d["accepted"]):
        exp, acc, _, _ = verify(model, state, next_token, props)
        agree += sum(int(a == b) for a, b in zip(exp, expected))
        total += len(expected)
        same_acc += int(acc == int(accepted))
        state = commit(model, state, props, int(accepted))
        next_token = int(expected[int(accepted)])
    assert agree >= 0.95 * total, (agree, total)
    assert same_acc >= 6, same_acc
    assert state.position == int(d["final_position"])


def test_draft_oracle_matches_reference_draft_model(golden):
    """The numpy draft forward against the reference's own DFlashDraftModel (bf16) on the
    tiny draft configuration, with a context shorter and longer than the sliding window:
    hidden rows within bf16 rounding drift, proposals equal except on near-ties."""
    from qwen35_dflash_b200 import config as qcfg, synthetic
    from oracle.draft_np import OracleDraft
    d = golden("draft.npz")
    tc, dc = qcfg.TINY, qcfg.TINY_DRAFT
    target = synthetic.init_weights(tc, seed=17)
    oracle = OracleDraft(dc, synthetic.init_draft_weights(dc))
    for case in (0, 1):
        feats = d[f"features_{case}"]
        C = len(feats)
        ctx = oracle.context(feats, np.arange(C))
        ids = [int(d[f"anchor_{case}"])] + [dc.mask_token_id] * (dc.block_size - 1)
        hidden = oracle.block(ids, C, ctx, target["target.embed_tokens.weight"])
        want = d[f"hidden_{case}"]
        diff = np.abs(hidden[1:] - want)
        tol = 2e-2 + 1e-2 * np.abs(want)
        assert (diff <= tol).mean() >= 0.995, (case, float(diff.max()))
        top, logits = oracle.draft(feats, ids[0], target["target.embed_tokens.weight"],
                                   target["target.lm_head.weight"], return_logits=True)
        ref = d[f"top1_{case}"]
        for i, (a, b) in enumerate(zip(top, ref)):
            if a != b:   # only where the oracle's two candidates are within 4 bf16 ulps
                assert abs(logits[i, a] - logits[i, b]) <= 4 * 2 ** -7 * max(1.0, abs(logits[i, b])), (case, i, a, b)
