"""MoE routing/experts and attention kernels vs the oracle and the reference (GPU)."""
import numpy as np
import pytest
import torch

from helpers import assert_close, to_np, bf16_tensor
from oracle import fused_ops_np as F
from oracle.model_np import OracleTarget
from oracle.numerics import bf16_round

pytestmark = pytest.mark.gpu

DT = {"bf16": torch.bfloat16, "f16": torch.float16}


def _t(a, dtype):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda().to(dtype)


def _lowp(golden, tag):
    return {k[len(tag) + 1:]: v for k, v in golden("ops_lowp.npz").items() if k.startswith(tag + "_")}


@pytest.mark.parametrize("tag", ["bf16", "f16"])
def test_moe_operator_matches_reference(golden, cuda_lib, tag):
    from qwen35_dflash_b200 import fused_ops as Q
    d = _lowp(golden, tag)
    ulp = 2 ** -8 if tag == "bf16" else 2 ** -11
    out, idx = Q.moe_with_routing(_t(d["moe_x"], DT[tag]), _t(d["moe_router"], DT[tag]),
                                  _t(d["moe_gu"], DT[tag]), _t(d["moe_down"], DT[tag]), top_k=4)
    assert out.dtype == DT[tag]
    assert_close(to_np(out), d["moe_y"], 4 * ulp, 4 * ulp, "moe")
    _, sel, _ = F.moe(d["moe_x"], d["moe_router"], d["moe_gu"], d["moe_down"], top_k=4, dtype=tag,
                      return_routing=True)
    np.testing.assert_array_equal(idx.cpu().numpy(), sel)


def _tie_heavy_logits(t, e, seed):
    g = torch.Generator().manual_seed(seed)
    logits = torch.randn(t, e, generator=g)
    logits[::4] = torch.randint(-3, 3, (len(range(0, t, 4)), e), generator=g).float()
    return logits.to(torch.bfloat16)


@pytest.mark.parametrize("t,e,k,dt", [(16, 256, 8, "bf16"), (256, 256, 8, "bf16"), (64, 16, 4, "bf16"),
                                      (33, 128, 8, "bf16"), (40, 256, 2, "bf16"), (48, 256, 8, "f16"),
                                      (16, 256, 8, "f32"),
                                      # introselect ranges that start in registers: two per lane
                                      # (64 experts), and part-filled lanes (40 experts)
                                      (64, 64, 8, "bf16"), (48, 40, 6, "f16")])
def test_routing_indices_bit_exact_vs_torch_topk(cuda_lib, t, e, k, dt):
    """Router selection equals torch.topk on CPU (the reference's call) element for element,
    ties included (integer-valued rows, and rows whose largest logits are +0.0 and -0.0)."""
    from qwen35_dflash_b200 import lib
    logits = _tie_heavy_logits(t, e, seed=t * 7 + e).float()
    for r in range(2, t, 8):   # signed zeros on top: equal values for the selection
        logits[r] = -1.0 - torch.rand(e, generator=torch.Generator().manual_seed(r))
        logits[r, r % e] = 0.0
        logits[r, (3 * r + 1) % e] = -0.0
        logits[r, (5 * r + 2) % e] = -0.0
    torch_dt = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}[dt]
    code = {"bf16": lib.QW_BF16, "f16": lib.QW_F16, "f32": lib.QW_F32}[dt]
    logits = logits.to(torch_dt)
    probs = torch.softmax(logits.float(), -1)
    _, want = torch.topk(probs, k, dim=-1)
    dev = logits.cuda()
    nbytes = cuda_lib.qw_moe_workspace_bytes(t, 256, e, 128, k)
    ws = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    lib.call("qw_moe_route", dev.data_ptr(), code, e, t, e, k, -1, lib.QW_BF16, ws.data_ptr(),
             lib.stream_ptr())
    idx = ws[: t * k * 4].view(torch.int32).view(t, k).cpu()
    np.testing.assert_array_equal(idx.numpy(), want.numpy())
    w = ws[t * k * 4: 2 * t * k * 4].view(torch.float32).view(t, k).cpu()
    sel = torch.gather(probs, 1, want.long())
    ref_w = (sel / sel.sum(-1, keepdim=True)).to(torch.bfloat16).float()
    assert_close(w.numpy(), ref_w.numpy(), 2 ** -8, 2 ** -7, "route weights")
    # expert -> (token, slot) lists: active experts ascending, tokens ascending in each
    lib.call("qw_moe_route_lists", ws.data_ptr(), t, e, k, lib.stream_ptr())
    _check_lists(ws, t, e, k, want.numpy())


def _check_lists(ws, t, e, k, sel_np):
    """The workspace's per-expert lists against the top-k indices sel_np [t, k]."""
    torch.cuda.synchronize()
    ints = ws.view(torch.int32).cpu().numpy()
    na_max = min(e, t * k)
    o = 2 * t * k + t
    n_active = int(ints[o])
    active = ints[o + 4: o + 4 + na_max]
    off = ints[o + 4 + na_max: o + 5 + 2 * na_max]
    ptok = ints[o + 5 + 2 * na_max: o + 5 + 2 * na_max + t * k]
    pslot = ints[o + 5 + 2 * na_max + t * k: o + 5 + 2 * na_max + 2 * t * k]
    experts = sorted(set(sel_np.ravel().tolist()))
    assert n_active == len(experts) and active[:n_active].tolist() == experts
    assert off[0] == 0 and off[n_active] == t * k
    for a, ex in enumerate(experts):
        toks, slots = np.nonzero(sel_np == ex)
        assert ptok[off[a]:off[a + 1]].tolist() == toks.tolist()
        assert pslot[off[a]:off[a + 1]].tolist() == slots.tolist()


class _LazyDequant:
    def __init__(self, q, s, group):
        self.q, self.s, self.group = q, s, group

    def __getitem__(self, e):
        return (self.q[e].astype(np.float32) * np.repeat(self.s[e], self.group, -1)).astype(np.float32)


@pytest.mark.parametrize("t,skew,dense", [(16, 0, 128), (64, 0, 128), (256, 0, 128), (256, 0, 0), (256, 12, 32),
                                          (64, 5, 32), (200, 3, 32), (256, 12, 0), (512, 8, 128), (256, 16, 64)])
def test_moe_w4a16_matches_oracle(cuda_lib, t, skew, dense):
    """Config-2 microbench shapes (T = 16, 64, 256): H 2048, 256 experts top-8 + shared,
    I 512, W4 g128, scales U(0.005, 0.02).  ``skew`` experts get +4 on every token's
    router logits (they receive nearly every token: dense contractions of up to 256
    pairs); ``dense`` is the tensor-core threshold (tokens per expert; 0 = grouped
    mma.sync kernels only).  With T > 16 the skewed routed experts with at least that
    many pairs run on the tcgen05 kernels when they make at least 128 gate/up items
    (cases 256/12/32, 512/8/128, 256/16/64); the others check the rule's fallback."""
    from qwen35_dflash_b200 import lib, w4
    torch.manual_seed(t)
    h, e, k, inter, g = 2048, 256, 8, 512, 128
    x = torch.randn(t, h, device="cuda").to(torch.bfloat16)
    logits = torch.cat([_tie_heavy_logits(t, e, seed=t).cuda(),
                        torch.randn(t, 1, device="cuda").to(torch.bfloat16)], 1).contiguous()
    if skew:
        hot = torch.randperm(e, generator=torch.Generator().manual_seed(skew))[:skew].cuda()
        logits[:, hot] = (logits[:, hot].float() + 4.0).to(torch.bfloat16)
    prev = cuda_lib.qw_moe_dense_threshold(dense)
    qgu = torch.randint(-8, 8, (e, 2 * inter, h), dtype=torch.int8, device="cuda")
    sgu = (torch.rand(e, 2 * inter, h // g, device="cuda") * 0.015 + 0.005).to(torch.bfloat16)
    qdn = torch.randint(-8, 8, (e, h, inter), dtype=torch.int8, device="cuda")
    sdn = (torch.rand(e, h, inter // g, device="cuda") * 0.015 + 0.005).to(torch.bfloat16)
    qsgu = torch.randint(-8, 8, (2 * inter, h), dtype=torch.int8, device="cuda")
    ssgu = (torch.rand(2 * inter, h // g, device="cuda") * 0.015 + 0.005).to(torch.bfloat16)
    qsdn = torch.randint(-8, 8, (h, inter), dtype=torch.int8, device="cuda")
    ssdn = (torch.rand(h, inter // g, device="cuda") * 0.015 + 0.005).to(torch.bfloat16)
    gu_s, dn_s = w4.pack_w4(qgu, sgu, g), w4.pack_w4(qdn, sdn, g)
    sgu_s, sdn_s = w4.pack_w4(qsgu, ssgu, g), w4.pack_w4(qsdn, ssdn, g)
    ws = torch.zeros(cuda_lib.qw_moe_workspace_bytes(t, h, e, inter, k), dtype=torch.uint8, device="cuda")
    out = torch.empty(t, h, dtype=torch.bfloat16, device="cuda")
    st = lib.stream_ptr()
    lib.call("qw_moe_route", logits.data_ptr(), lib.QW_BF16, e + 1, t, e, k, e, lib.QW_BF16, ws.data_ptr(), st)
    lib.call("qw_moe_experts_w4", x.data_ptr(), gu_s.data_ptr(), dn_s.data_ptr(), sgu_s.data_ptr(),
             sdn_s.data_ptr(), t, h, e, inter, k, g, ws.data_ptr(), st)
    lib.call("qw_moe_combine", ws.data_ptr(), out.data_ptr(), 0, t, h, e, inter, k, 1, st)
    torch.cuda.synchronize()
    cuda_lib.qw_moe_dense_threshold(prev)
    lib.call("qw_check_wait_status", 1, st)
    # oracle (bf16 rounding points of fused_ops.moe + the shared expert of fused/model.py:305-307)
    xn = to_np(x)
    ln = to_np(logits)
    routed, sel, _, mag = F.moe(xn, None, _LazyDequant(qgu.cpu().numpy(), sgu.float().cpu().numpy(), g),
                                _LazyDequant(qdn.cpu().numpy(), sdn.float().cpu().numpy(), g), top_k=k,
                                dtype="bf16", logits=ln[:, :e], return_routing=True, return_magnitude=True)
    wsg = to_np(w4.dequantize(qsgu, ssgu, g))
    wsd = to_np(w4.dequantize(qsdn, ssdn, g))
    gate = bf16_round(xn @ wsg[:inter].T)
    up = bf16_round(xn @ wsg[inter:].T)
    act = bf16_round(bf16_round(F.silu(gate)) * up)
    shared = bf16_round(act @ wsd.T)
    sgate = bf16_round(F.sigmoid(ln[:, e:e + 1]))
    sterm = bf16_round(shared * sgate)
    want = bf16_round(routed + sterm)
    idx = ws[: t * k * 4].view(torch.int32).view(t, k).cpu().numpy()
    np.testing.assert_array_equal(idx, sel)
    _check_lists(ws, t, e, k, sel)   # as the expert kernels built (and published) them
    # The stated bound, |got - want| <= 2e-2 + 1e-2 M, with M the largest magnitude the
    # reference's bf16 expert accumulation passes through at that element (the routed
    # terms and running sums, the shared term): the sum is rounded to bf16 after every
    # add, so one ulp of a large term survives cancellation; >= 99.9 % of elements must
    # also meet the plain elementwise bound.  The sum rounds to bf16 after each of its
    # k + 1 adds, so two kernels whose fp32 expert outputs differ in the last bits may
    # part by two flipped roundings: up to two bf16 ulps of M is allowed as well.
    mag = np.maximum(mag, np.abs(sterm))
    ulp2 = 2.0 * np.exp2(np.floor(np.log2(np.maximum(np.maximum(mag, np.abs(want)), 2.0 ** -100))) - 7)
    assert_close(to_np(out), want, what="moe w4a16", magnitude=np.maximum(mag, (ulp2 - 2e-2) / 1e-2),
                 strict_frac=0.999)


@pytest.mark.parametrize("t,g", [(16, 128), (5, 64), (16, 32)])
def test_moe_route_x_staging_is_bit_identical(cuda_lib, t, g):
    """qw_moe_route_x stages x for the gate/up kernel; the experts' output must be the
    bits of the unstaged path (qw_moe_route), and a different x than the staged one
    must be converted afresh, not taken from the stage."""
    from qwen35_dflash_b200 import lib, w4
    torch.manual_seed(t + g)
    h, e, k, inter = 2048, 64, 8, 256
    x = torch.randn(t, h, device="cuda").to(torch.bfloat16)
    x2 = torch.randn(t, h, device="cuda").to(torch.bfloat16)
    logits = torch.randn(t, e + 1, device="cuda").to(torch.bfloat16)
    gu = w4.pack_w4(torch.randint(-8, 8, (e, 2 * inter, h), dtype=torch.int8, device="cuda"),
                    (torch.rand(e, 2 * inter, h // g, device="cuda") * 0.02).to(torch.bfloat16), g)
    dn = w4.pack_w4(torch.randint(-8, 8, (e, h, inter), dtype=torch.int8, device="cuda"),
                    (torch.rand(e, h, inter // g, device="cuda") * 0.02).to(torch.bfloat16), g)
    sgu = w4.pack_w4(torch.randint(-8, 8, (2 * inter, h), dtype=torch.int8, device="cuda"),
                     (torch.rand(2 * inter, h // g, device="cuda") * 0.02).to(torch.bfloat16), g)
    sdn = w4.pack_w4(torch.randint(-8, 8, (h, inter), dtype=torch.int8, device="cuda"),
                     (torch.rand(h, inter // g, device="cuda") * 0.02).to(torch.bfloat16), g)
    st = lib.stream_ptr()

    def run(stage_x, x_in):
        ws = torch.zeros(cuda_lib.qw_moe_workspace_bytes(t, h, e, inter, k), dtype=torch.uint8, device="cuda")
        out = torch.empty(t, h, dtype=torch.bfloat16, device="cuda")
        if stage_x is None:
            lib.call("qw_moe_route", logits.data_ptr(), lib.QW_BF16, e + 1, t, e, k, e, lib.QW_BF16, ws.data_ptr(), st)
        else:
            lib.call("qw_moe_route_x", logits.data_ptr(), lib.QW_BF16, e + 1, t, e, k, e, lib.QW_BF16,
                     stage_x.data_ptr(), h, g, ws.data_ptr(), st, 1)
        lib.call("qw_moe_experts_w4", x_in.data_ptr(), gu.data_ptr(), dn.data_ptr(), sgu.data_ptr(),
                 sdn.data_ptr(), t, h, e, inter, k, g, ws.data_ptr(), st)
        lib.call("qw_moe_combine", ws.data_ptr(), out.data_ptr(), 0, t, h, e, inter, k, 1, st)
        torch.cuda.synchronize()
        return out

    assert torch.equal(run(x, x), run(None, x))
    assert torch.equal(run(x, x2), run(None, x2))


@pytest.mark.parametrize("t,e,k,combine", [(16, 256, 8, "norm"), (16, 64, 8, "plain"), (48, 40, 6, "plain")])
def test_route_tie_order_zero_same_selection_and_outputs(cuda_lib, t, e, k, combine):
    """qw_moe_route_x with tie_order 0 (the engine's routing) on tie-heavy logits: per
    token the same selected experts with the same weights as torch.topk, ties at the
    k / k+1 boundary resolved in torch's order, and the MoE output (experts + combine,
    plain or fused with the next RMSNorm) bit-identical to the tie_order 1 routing."""
    from qwen35_dflash_b200 import lib, w4
    g, h, inter = 128, 2048, 256
    gen = torch.Generator().manual_seed(t * 31 + e)
    logits = _tie_heavy_logits(t, e, seed=t * 7 + e + 1).float()
    logits[1::4] = torch.randint(-2, 3, (len(range(1, t, 4)), e), generator=gen).float() * 0.5
    logits = torch.cat([logits, torch.randn(t, 1, generator=gen)], 1).to(torch.bfloat16).cuda()
    probs = torch.softmax(logits[:, :e].cpu().float(), -1)
    _, want = torch.topk(probs, k, dim=-1)
    x = torch.randn(t, h, device="cuda").to(torch.bfloat16)
    gu = w4.pack_w4(torch.randint(-8, 8, (e, 2 * inter, h), dtype=torch.int8, device="cuda"),
                    (torch.rand(e, 2 * inter, h // g, device="cuda") * 0.02).to(torch.bfloat16), g)
    dn = w4.pack_w4(torch.randint(-8, 8, (e, h, inter), dtype=torch.int8, device="cuda"),
                    (torch.rand(e, h, inter // g, device="cuda") * 0.02).to(torch.bfloat16), g)
    sgu = w4.pack_w4(torch.randint(-8, 8, (2 * inter, h), dtype=torch.int8, device="cuda"),
                     (torch.rand(2 * inter, h // g, device="cuda") * 0.02).to(torch.bfloat16), g)
    sdn = w4.pack_w4(torch.randint(-8, 8, (h, inter), dtype=torch.int8, device="cuda"),
                     (torch.rand(h, inter // g, device="cuda") * 0.02).to(torch.bfloat16), g)
    gamma = (torch.randn(h, device="cuda") * 0.1).to(torch.bfloat16)
    resid = torch.randn(t, h, device="cuda").to(torch.bfloat16)
    st = lib.stream_ptr()

    def run(order):
        ws = torch.zeros(cuda_lib.qw_moe_workspace_bytes(t, h, e, inter, k), dtype=torch.uint8, device="cuda")
        lib.call("qw_moe_route_x", logits.data_ptr(), lib.QW_BF16, e + 1, t, e, k, e, lib.QW_BF16,
                 x.data_ptr(), h, g, ws.data_ptr(), st, order)
        lib.call("qw_moe_experts_w4", x.data_ptr(), gu.data_ptr(), dn.data_ptr(), sgu.data_ptr(),
                 sdn.data_ptr(), t, h, e, inter, k, g, ws.data_ptr(), st)
        hidden = resid.clone()
        normed = torch.empty(t, h, dtype=torch.bfloat16, device="cuda")
        if combine == "norm":
            lib.call("qw_moe_combine_norm", ws.data_ptr(), hidden.data_ptr(), t, h, e, inter, k, 1,
                     gamma.data_ptr(), normed.data_ptr(), 1e-6, None, 0, 0, st)
        else:
            lib.call("qw_moe_combine", ws.data_ptr(), normed.data_ptr(), 0, t, h, e, inter, k, 1, st)
        torch.cuda.synchronize()
        idx = ws[: t * k * 4].view(torch.int32).view(t, k).cpu()
        w = ws[t * k * 4: 2 * t * k * 4].view(torch.float32).view(t, k).cpu()
        return idx, w, hidden, normed

    i1, w1, h1, n1 = run(1)
    i0, w0, h0, n0 = run(0)
    np.testing.assert_array_equal(i1.numpy(), want.numpy())
    for r in range(t):
        assert sorted(i0[r].tolist()) == sorted(want[r].tolist()), r
        m1 = dict(zip(i1[r].tolist(), w1[r].tolist()))
        m0 = dict(zip(i0[r].tolist(), w0[r].tolist()))
        assert m0 == m1, r
    assert torch.equal(h0, h1) and torch.equal(n0, n1)


@pytest.mark.parametrize("tag", ["bf16", "f16"])
def test_attention_operator_matches_reference(golden, cuda_lib, tag):
    from qwen35_dflash_b200 import fused_ops as Q
    d = _lowp(golden, tag)
    ulp = 2 ** -8 if tag == "bf16" else 2 ** -11
    out = Q.attention(_t(d["attn_q"], DT[tag]), _t(d["attn_k"], DT[tag]), _t(d["attn_v"], DT[tag]),
                      query_start=8, scale=32 ** -0.5)
    assert_close(to_np(out), d["attn_o"], 4 * ulp, 4 * ulp, "attention")


@pytest.mark.parametrize("b,h,hkv,s,ctx,dim", [(1, 16, 2, 16, 4096, 256), (2, 4, 1, 16, 100, 64),
                                               (1, 8, 2, 64, 64, 128), (3, 16, 2, 1, 37, 256)])
def test_attention_operator_shapes(cuda_lib, b, h, hkv, s, ctx, dim):
    from qwen35_dflash_b200 import fused_ops as Q
    rng = np.random.default_rng(ctx + s)
    q = bf16_round(rng.normal(0, 1, (b, h, s, dim)))
    k = bf16_round(rng.normal(0, 1, (b, hkv, ctx + s, dim)))
    v = bf16_round(rng.normal(0, 1, (b, hkv, ctx + s, dim)))
    want = F.attention(q, k, v, query_start=ctx, scale=dim ** -0.5, dtype="bf16")
    got = Q.attention(bf16_tensor(q), bf16_tensor(k), bf16_tensor(v), query_start=ctx, scale=dim ** -0.5)
    assert_close(to_np(got), want, what="attention")


@pytest.mark.parametrize("b,ctx", [(1, 4096), (3, 40)])
def test_paged_attention_layer_matches_oracle(cuda_lib, b, ctx):
    """q/k norm + RoPE + paged KV append + causal GQA + sigmoid gate (fused/model.py:278-293)."""
    from qwen35_dflash_b200 import lib
    h, hkv, dim, s, page = 16, 2, 256, 16, 16
    rot, theta, eps = 64, 1e7, 1e-6
    rng = np.random.default_rng(b + ctx)
    ldq = h * 2 * dim + 2 * hkv * dim
    qkv = bf16_round(rng.normal(0, 1, (b, s, ldq)))
    qn = bf16_round(rng.normal(0, 0.1, (dim,)))
    kn = bf16_round(rng.normal(0, 0.1, (dim,)))
    qpos = np.array([ctx - 7 * i for i in range(b)], np.int32)
    max_len = int(qpos.max()) + s
    max_pages = (max_len + page - 1) // page
    npages = b * max_pages + 3
    perm = rng.permutation(npages)[: b * max_pages].reshape(b, max_pages).astype(np.int32)
    kcache = bf16_round(rng.normal(0, 1, (npages, hkv, page, dim)))
    vcache = bf16_round(rng.normal(0, 1, (npages, hkv, page, dim)))
    # oracle
    cfg = {"head_dim": dim, "rope_parameters": {"partial_rotary_factor": rot / dim, "rope_theta": theta}}
    orc = OracleTarget(cfg, {}, (0,), act="bf16", rope="f32")
    want = np.zeros((b, s, h * dim), np.float32)
    new_k = np.zeros((b, hkv, s, dim), np.float32)
    new_v = np.zeros((b, hkv, s, dim), np.float32)
    for i in range(b):
        x = qkv[i]
        qg = x[:, : h * 2 * dim].reshape(s, h, 2 * dim)
        qh, gate = qg[..., :dim], qg[..., dim:]
        qh = F.rms_norm(qh, bf16_round(qn + 1), eps, "bf16").transpose(1, 0, 2)[None]
        kh = F.rms_norm(x[:, h * 2 * dim: h * 2 * dim + hkv * dim].reshape(s, hkv, dim), bf16_round(kn + 1),
                        eps, "bf16").transpose(1, 0, 2)[None]
        vh = x[:, h * 2 * dim + hkv * dim:].reshape(s, hkv, dim).transpose(1, 0, 2)[None]
        qh, kh = orc.rotary(qh, int(qpos[i])), orc.rotary(kh, int(qpos[i]))
        new_k[i], new_v[i] = kh[0], vh[0]
        pos = np.arange(qpos[i])
        old_k = kcache[perm[i][pos // page], :, pos % page].transpose(1, 0, 2)[None]
        old_v = vcache[perm[i][pos // page], :, pos % page].transpose(1, 0, 2)[None]
        kk, vv = F.cache_update(old_k, old_v, kh, vh)
        o = F.attention(qh, kk, vv, query_start=int(qpos[i]), scale=dim ** -0.5, dtype="bf16")
        o = o[0].transpose(1, 0, 2).reshape(s, h * dim)
        want[i] = bf16_round(o * bf16_round(F.sigmoid(gate.reshape(s, h * dim))))
    # device
    qkv_d = bf16_tensor(qkv.reshape(b * s, ldq))
    kc, vc = bf16_tensor(kcache), bf16_tensor(vcache)
    pages_d = torch.from_numpy(perm).cuda()
    qpos_d = torch.from_numpy(qpos).cuda()
    qout = torch.empty(b, h, s, dim, dtype=torch.bfloat16, device="cuda")
    out = torch.empty(b * s, h * dim, dtype=torch.bfloat16, device="cuda")
    ws = torch.empty(cuda_lib.qw_attn_workspace_bytes(b, h, hkv, s, dim, max_len), dtype=torch.uint8, device="cuda")
    st = lib.stream_ptr()
    qn_d, kn_d = bf16_tensor(qn), bf16_tensor(kn)  # keep the tensors alive across the launch
    lib.call("qw_attn_prep", qkv_d.data_ptr(), ldq, qn_d.data_ptr(), kn_d.data_ptr(), eps,
             theta, rot, qpos_d.data_ptr(), pages_d.data_ptr(), max_pages, page, kc.data_ptr(), vc.data_ptr(),
             qout.data_ptr(), b, s, h, hkv, dim, st)
    gate_ptr = qkv_d.data_ptr() + dim * 2
    lib.call("qw_attn_paged", qout.data_ptr(), kc.data_ptr(), vc.data_ptr(), pages_d.data_ptr(), max_pages, page,
             qpos_d.data_ptr(), max_len, gate_ptr, ldq, out.data_ptr(), b, s, h, hkv, dim, dim ** -0.5,
             ws.data_ptr(), st)
    torch.cuda.synchronize()
    kc_h = to_np(kc)
    for i in range(b):
        pos = qpos[i] + np.arange(s)
        got_k = kc_h[perm[i][pos // page], :, pos % page].transpose(1, 0, 2)
        assert_close(got_k, new_k[i], what="k append")
        np.testing.assert_array_equal(to_np(vc)[perm[i][pos // page], :, pos % page].transpose(1, 0, 2), new_v[i])
    assert_close(to_np(out).reshape(b, s, h * dim), want, what="paged attention")


@pytest.mark.parametrize("t,g,e,inter", [(16, 128, 256, 512), (16, 32, 64, 128), (7, 64, 32, 256)])
def test_moe_ep_kernels_one_rank_bit_identical(cuda_lib, t, g, e, inter):
    """The expert-parallel kernels with one rank (the window is its own peer, allocated
    here as a plain device tensor) and the shared expert exchanged as local expert E:
    dispatch, receive routing, the receiving experts (the streaming kernels over the
    window's rows), combine and scatter must give the one-GPU MoE (the bulk kernels at 16
    tokens) bit for bit, twice in a row (the epoch advances), and the window must hold the
    protocol's rows and descriptors (oracle/ep_np.py)."""
    from qwen35_dflash_b200 import lib, w4
    from oracle import ep_np
    torch.manual_seed(t + g + e)
    h, k = 2048, 8
    x = torch.randn(t, h, device="cuda").to(torch.bfloat16)
    logits = torch.cat([_tie_heavy_logits(t, e, seed=t + e).cuda(),
                        torch.randn(t, 1, device="cuda").to(torch.bfloat16)], 1).contiguous()

    def bank(n, kk, *lead):
        return w4.pack_w4(torch.randint(-8, 8, (*lead, n, kk), dtype=torch.int8, device="cuda"),
                          (torch.rand(*lead, n, kk // g, device="cuda") * 0.015 + 0.005).to(torch.bfloat16), g)
    gu, dn = bank(2 * inter, h, e), bank(h, inter, e)
    sgu, sdn = bank(2 * inter, h), bank(h, inter)
    st = lib.stream_ptr()
    nbytes = cuda_lib.qw_moe_workspace_bytes(t, h, e, inter, k)

    ws1 = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    out1 = torch.empty(t, h, dtype=torch.bfloat16, device="cuda")
    lib.call("qw_moe_route", logits.data_ptr(), lib.QW_BF16, e + 1, t, e, k, e, lib.QW_BF16, ws1.data_ptr(), st)
    lib.call("qw_moe_experts_w4", x.data_ptr(), gu.data_ptr(), dn.data_ptr(), sgu.data_ptr(), sdn.data_ptr(),
             t, h, e, inter, k, g, ws1.data_ptr(), st)
    lib.call("qw_moe_combine", ws1.data_ptr(), out1.data_ptr(), 0, t, h, e, inter, k, 1, st)

    cap = t * (k + 1)                      # routed pairs + one shared-expert row per token
    window = torch.zeros(cuda_lib.qw_ep_window_bytes(1, cap, h), dtype=torch.uint8, device="cuda")
    peers = torch.tensor([window.data_ptr()], dtype=torch.int64, device="cuda")
    ws_r = torch.zeros(cuda_lib.qw_moe_ep_recv_workspace_bytes(1, cap, h, e + 1, inter), dtype=torch.uint8,
                       device="cuda")
    gu_l, dn_l = torch.cat([gu.view(-1), sgu.view(-1)]), torch.cat([dn.view(-1), sdn.view(-1)])
    for rep in range(2):
        ws2 = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
        out2 = torch.empty(t, h, dtype=torch.bfloat16, device="cuda")
        lib.call("qw_moe_route", logits.data_ptr(), lib.QW_BF16, e + 1, t, e, k, e, lib.QW_BF16, ws2.data_ptr(), st)
        lib.call("qw_moe_ep_dispatch", ws2.data_ptr(), x.data_ptr(), t, h, e, k, 1, 0, cap, 1, peers.data_ptr(),
                 window.data_ptr(), st)
        lib.call("qw_moe_ep_recv_route", window.data_ptr(), 1, cap, h, e + 1, ws_r.data_ptr(), st)
        lib.call("qw_moe_ep_experts", window.data_ptr(), gu_l.data_ptr(), dn_l.data_ptr(), 1, 0, cap, h, e + 1,
                 inter, g, peers.data_ptr(), ws_r.data_ptr(), st)
        lib.call("qw_moe_ep_scatter", ws2.data_ptr(), window.data_ptr(), t, h, e, inter, k, 1, cap, 1, st)
        lib.call("qw_moe_combine", ws2.data_ptr(), out2.data_ptr(), 0, t, h, e, inter, k, 1, st)
        lib.call("qw_check_wait_status", 1, st)
        torch.cuda.synchronize()
        # the window holds the protocol's rows and descriptors
        words = window.view(torch.int32).cpu().numpy()
        assert words[0] == rep + 1                                    # epoch of the finished exchange
        topk = ws2[: t * k * 4].view(torch.int32).view(t, k).cpu().numpy()
        rows_w, meta_w, count_w = ep_np.dispatch(topk, x.cpu().view(torch.int16).numpy().view("uint16"), e, 1, 0,
                                                 shared=True)[0]
        assert words[320] == count_w == cap                            # count[0] at byte 1280
        counters = window[256:256 + 2 * 64 * 8].view(torch.int64).cpu().numpy()
        assert counters[0] == counters[64] == (rep + 1) << 20          # dispatch / result arrivals
        assert (words[512:512 + count_w] == meta_w[:count_w]).all()   # meta [1][cap] at byte 2048
        rows_off = 2048 + (cap * 4 + 255) // 256 * 256
        got = window[rows_off: rows_off + cap * h * 2].view(torch.int16).cpu().numpy().view("uint16").reshape(cap, h)
        assert (got[:count_w] == rows_w[:count_w]).all()
        if not torch.equal(out1, out2):
            raise AssertionError(f"rep {rep}: {(out1 != out2).sum().item()} elements differ")
