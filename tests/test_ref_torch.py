"""The torch restatement used for the timed CPU baseline (oracle/ref_torch.py) agrees with
the numpy oracle, which the golden fixtures pin to the reference's own outputs (CPU)."""
import numpy as np
import torch

from oracle import fused_ops_np as F
from oracle import ref_torch as R


def _t(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32))


def test_rms_norm_and_conv():
    rng = np.random.default_rng(0)
    x, gamma = rng.normal(0, 1, (2, 5, 64)).astype(np.float32), rng.normal(1, 0.1, 64).astype(np.float32)
    np.testing.assert_allclose(R.rms_norm(_t(x), _t(gamma), 1e-6).numpy(), F.rms_norm(x, gamma, 1e-6),
                               rtol=1e-5, atol=1e-6)
    proj, hist = rng.normal(0, 1, (2, 7, 12)).astype(np.float32), rng.normal(0, 1, (2, 12, 3)).astype(np.float32)
    w = rng.normal(0, 0.3, (12, 1, 4)).astype(np.float32)
    got, new_hist = R.conv_silu(_t(proj), _t(hist), _t(w))
    want_hist, padded = F.conv_state_update(proj, hist)
    np.testing.assert_allclose(got.numpy(), F.silu(F.causal_conv1d(padded, w)), rtol=1e-5, atol=1e-6)
    np.testing.assert_array_equal(new_hist.numpy(), want_hist)


def test_gated_delta_rule():
    rng = np.random.default_rng(1)
    b, s, h, d = 3, 9, 4, 16
    q, k, v = (rng.normal(0, 1, (b, s, h, d)).astype(np.float32) for _ in range(3))
    g = -F.softplus(rng.normal(0, 1, (b, s, h))).astype(np.float32)
    beta = F.sigmoid(rng.normal(0, 1, (b, s, h))).astype(np.float32)
    s0 = rng.normal(0, 0.02, (b, h, d, d)).astype(np.float32)
    lens = np.array([9, 4, 0], np.int16)
    core, st = F.chunk_gated_delta_rule(q, k, v, g, beta, s0, lens, chunk_size=64, use_qk_l2norm_in_kernel=True)
    gc, gs = R.gated_delta_rule(_t(q), _t(k), _t(v), _t(g), _t(beta), _t(s0), torch.from_numpy(lens.astype(np.int64)))
    np.testing.assert_allclose(gc.numpy(), core, rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(gs.numpy(), st, rtol=1e-4, atol=1e-6)


def test_attention_core():
    rng = np.random.default_rng(2)
    b, hq, hkv, s, ctx, d = 1, 4, 1, 5, 11, 32
    x = rng.normal(0, 1, (b, s, 64)).astype(np.float32)
    w = {"q": rng.normal(0, 0.1, (hq * 2 * d, 64)), "k": rng.normal(0, 0.1, (hkv * d, 64)),
         "v": rng.normal(0, 0.1, (hkv * d, 64)), "o": rng.normal(0, 0.1, (64, hq * d)),
         "q_norm": np.zeros(d), "k_norm": np.zeros(d)}
    w = {n: _t(a) for n, a in w.items()}
    key, value = rng.normal(0, 1, (b, hkv, ctx, d)).astype(np.float32), rng.normal(0, 1, (b, hkv, ctx, d)).astype(np.float32)
    got = R.attention_layer(_t(x), w, _t(key), _t(value), ctx, heads=hq, kv_heads=hkv, dim=d, rot=8, theta=1e7)
    # the same composition from the numpy oracle's operators
    qg = (x @ w["q"].numpy().T).reshape(b, s, hq, 2 * d)
    q = F.rms_norm(qg[..., :d], np.ones(d, np.float32), 1e-6).transpose(0, 2, 1, 3)
    kk = F.rms_norm((x @ w["k"].numpy().T).reshape(b, s, hkv, d), np.ones(d, np.float32), 1e-6).transpose(0, 2, 1, 3)
    vv = (x @ w["v"].numpy().T).reshape(b, s, hkv, d).transpose(0, 2, 1, 3)
    q = R._rope(_t(q), ctx, 8, 1e7).numpy()
    kk = R._rope(_t(kk), ctx, 8, 1e7).numpy()
    keys, vals = F.cache_update(key, value, kk, vv)
    mixed = F.attention(q, keys, vals, query_start=ctx, scale=d ** -0.5).transpose(0, 2, 1, 3).reshape(b, s, -1)
    want = (mixed * F.sigmoid(qg[..., d:].reshape(b, s, -1))) @ w["o"].numpy().T
    np.testing.assert_allclose(got.numpy(), want, rtol=1e-4, atol=1e-5)


def test_moe_routed_part():
    rng = np.random.default_rng(3)
    t, h, e, i, k = 6, 32, 8, 16, 3
    x = rng.normal(0, 1, (1, t, h)).astype(np.float32)
    router = rng.normal(0, 0.3, (e, h)).astype(np.float32)
    gu = rng.normal(0, 0.1, (e, 2 * i, h)).astype(np.float32)
    dn = rng.normal(0, 0.1, (e, h, i)).astype(np.float32)
    zeros = {"shared_gu": torch.zeros(2 * i, h), "shared_down": torch.zeros(h, i), "shared_gate": torch.zeros(1, h)}
    got = R.moe_layer(_t(x), {"router": _t(router), **zeros}, lambda j: (_t(gu[j]), _t(dn[j])), top_k=k)
    np.testing.assert_allclose(got.numpy(), F.moe(x, router, gu, dn, top_k=k), rtol=1e-4, atol=1e-5)
