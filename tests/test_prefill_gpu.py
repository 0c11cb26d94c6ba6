"""Prefill in chunks of 64 tokens per forward (GPU).

The reference prefills a prompt in one forward (fused/session.py:282-296).  Here a
prefill engine (``TargetEngine.prefill_engine``) runs 64-token chunks on the verify
engine's weights and state; its GDN kernels take a chunk in sub-blocks of 16 with the
state in registers.  Checked on the tiny target:

* the GDN kernels on a 64-token sequence equal four 16-token verify + commit blocks, bit
  for bit (outputs, recurrent state, conv tails);
* a prompt prefilled in 64-token chunks leaves the same state as one prefilled in
  16-token blocks (GDN state and conv tails within fp32 rounding, KV cache within bf16
  rounding) and predicts the oracle's next token (or a counted near-tie);
* DFlash with 64-token prefill chunks still emits the target's greedy continuation.
"""
import ctypes

import numpy as np
import pytest
import torch

from helpers import to_np
from oracle.model_np import OracleTarget
from oracle.numerics import quantize_w4, dequantize_w4

pytestmark = pytest.mark.gpu


def _gdn_case(seq, seed):
    from qwen35_dflash_b200 import lib
    g = torch.Generator(device="cuda").manual_seed(seed)
    kh, vh, d = 4, 8, 64
    kw, vw = kh * d, vh * d
    C = 2 * kw + vw
    ldp = C + vw
    proj = torch.randn(seq, ldp, device="cuda", generator=g).to(torch.bfloat16)
    ab = torch.randn(seq, 2 * vh, device="cuda", generator=g)
    hist = torch.randn(1, C, 3, device="cuda", generator=g).to(torch.bfloat16)
    conv_w = (torch.randn(C, 4, device="cuda", generator=g) * 0.3).to(torch.bfloat16)
    a_log = torch.log(torch.arange(1, vh + 1, dtype=torch.float32, device="cuda"))
    dt_bias = torch.randn(vh, device="cuda", generator=g) * 0.5
    norm_w = (1 + 0.1 * torch.randn(d, device="cuda", generator=g)).to(torch.bfloat16)
    state = torch.randn(1, vh, d, d, device="cuda", generator=g) * 0.05
    return dict(kh=kh, vh=vh, d=d, C=C, ldp=ldp, proj=proj, ab=ab, hist=hist, conv_w=conv_w, a_log=a_log,
                dt_bias=dt_bias, norm_w=norm_w, state=state, lib=lib)


def _gdn_run(c, lo, n, hist, state):
    """Verify tokens [lo, lo + n) of the case's projections, then commit them all."""
    lib, so = c["lib"], c["lib"].load()
    out = torch.zeros(n, c["vh"] * c["d"], dtype=torch.bfloat16, device="cuda")
    proj = c["proj"][lo:lo + n].contiguous()
    ab = c["ab"][lo:lo + n].contiguous()
    slots = torch.zeros(1, dtype=torch.int32, device="cuda")
    accepted = torch.full((1,), n, dtype=torch.int32, device="cuda")
    layer = (lib.GdnLayer * 1)()
    layer[0] = lib.GdnLayer(proj.data_ptr(), ab.data_ptr(), hist.data_ptr(), c["conv_w"].data_ptr(),
                            c["a_log"].data_ptr(), c["dt_bias"].data_ptr(), c["norm_w"].data_ptr(),
                            state.data_ptr(), out.data_ptr())
    desc = torch.frombuffer(bytearray(bytes(memoryview(layer).cast("B"))), dtype=torch.uint8).cuda()
    dims = lib.GdnDims(1, n, c["kh"], c["vh"], c["d"], c["d"], c["C"], 4, c["ldp"], 1e-6, slots.data_ptr(),
                       accepted.data_ptr())
    st = lib.stream_ptr()
    lib.check(so.qw_gdn_verify(ctypes.byref(dims), desc.data_ptr(), 0, st))
    lib.check(so.qw_gdn_commit(ctypes.byref(dims), desc.data_ptr(), 1, st))
    torch.cuda.synchronize()
    return out


@pytest.mark.parametrize("seq", [64, 45])
def test_gdn_long_sequence_equals_blocks_of_16(cuda_lib, seq):
    c = _gdn_case(seq, seed=seq)
    h1, s1 = c["hist"].clone(), c["state"].clone()
    out1 = _gdn_run(c, 0, seq, h1, s1)
    h2, s2 = c["hist"].clone(), c["state"].clone()
    outs = [_gdn_run(c, lo, min(16, seq - lo), h2, s2) for lo in range(0, seq, 16)]
    assert torch.equal(out1, torch.cat(outs))
    assert torch.equal(s1, s2)
    assert torch.equal(h1, h2)


def _tiny(seed=17):
    from qwen35_dflash_b200 import config as qcfg, synthetic
    cfg = qcfg.TINY
    raw = synthetic.init_weights(cfg, seed=seed)
    deq = {}
    for name, value in raw.items():
        if synthetic.is_w4(name):
            q, s = quantize_w4(value, cfg.quant_group)
            value = dequantize_w4(q, s, cfg.quant_group)
        deq[name] = value
    return cfg, raw, deq


def _prefill(eng, prompt, block):
    e = eng if block == eng.S else eng.prefill_engine(block)
    eng.qpos.zero_(); eng.state.zero_(); eng.conv_hist.zero_()
    for i in range(0, len(prompt), block):
        chunk = prompt[i:i + block]
        e.tokens.copy_(torch.tensor(chunk + [0] * (block - len(chunk)), dtype=torch.int32))
        e.forward()
        e.accept(auto_commit=False)
        e.commit([len(chunk)])
    torch.cuda.synchronize()
    return e


def test_prefill_chunks_equal_verify_blocks_and_oracle(cuda_lib):
    from qwen35_dflash_b200 import engine as E
    cfg, raw, deq = _tiny()
    prompt = [int(t) for t in np.random.default_rng(5).integers(0, cfg.vocab_size, 150)]
    engines = []
    for block in (16, 64):
        te = E.TargetEngine(cfg, E.weights_from_arrays(cfg, raw), batch=1, block=16, capacity=512)
        pe = _prefill(te, prompt, block)
        engines.append((te, pe))
    (a, _), (b, pb) = engines
    assert int(a.qpos.item()) == int(b.qpos.item()) == len(prompt)
    np.testing.assert_allclose(to_np(b.state), to_np(a.state), rtol=1e-4, atol=1e-5)
    assert torch.equal(b.conv_hist, a.conv_hist)
    n = len(prompt)
    for kc, kb in ((a.k_cache, b.k_cache), (a.v_cache, b.v_cache)):
        ka = to_np(kc).transpose(1, 0, 2, 3, 4).reshape(kc.shape[1], -1)[:(n + 15) // 16]
        kbb = to_np(kb).transpose(1, 0, 2, 3, 4).reshape(kb.shape[1], -1)[:(n + 15) // 16]
        np.testing.assert_allclose(kbb, ka, rtol=2e-2, atol=2e-2)
    oracle = OracleTarget(cfg.to_hf_text_config(), deq, cfg.feature_layers, act="bf16", rope="f32")
    top1, _, _, logits = oracle.forward(np.asarray([prompt]), return_logits=True)
    want = int(top1[0, -1])
    row = logits[0, -1]
    for te in (a, b):
        got = int(te.next_token.item())
        assert got == want or abs(float(row[got]) - float(row[want])) <= 4 * 2 ** -7 * max(1.0, abs(float(row[want])))
    # the chunk engine's feature taps of the last chunk: the committed rows' features
    last = n - (n - 1) // 64 * 64
    assert pb.features[:last].abs().sum().item() > 0


def test_dflash_prefill_in_chunks_then_greedy(cuda_lib):
    from qwen35_dflash_b200 import config, engine as E, synthetic
    from qwen35_dflash_b200.dflash import DFlash
    from qwen35_dflash_b200.draft import DraftEngine
    from qwen35_dflash_b200.session import TargetSession
    tc, dc = config.TINY, config.TINY_DRAFT
    raw = synthetic.init_weights(tc, seed=17)
    te = E.TargetEngine(tc, E.weights_from_arrays(tc, raw), batch=1, block=16, capacity=512)
    df = DFlash(te, DraftEngine(dc, te, synthetic.init_draft_weights(dc)), prefill_block=64)
    prompt = [int(t) for t in np.random.default_rng(9).integers(0, tc.vocab_size, 100)]
    sess = TargetSession(E.TargetEngine(tc, E.weights_from_arrays(tc, raw), batch=1, block=16, capacity=512))
    sess.prefill(list(prompt))
    greedy = [sess.next_token]
    while len(greedy) < 40:
        sess.step(greedy[-1])
        greedy.append(sess.next_token)
    res = df.generate(prompt, max_new_tokens=40, use_graph=True)
    # the first generated token comes from the chunked prefill, the rest from verify
    # blocks: equal to the plain greedy run unless a near-tie parts them (then the first
    # difference must be the chunked prefill's own prediction)
    if res.token_ids != greedy:
        first = next(i for i, (x, y) in enumerate(zip(res.token_ids, greedy)) if x != y)
        assert first == 0, (first, res.token_ids[:first + 2], greedy[:first + 2])
