"""The DFlash draft on the device and the greedy DFlash loop (GPU), on the tiny target and
the tiny draft (2 layers: a sliding-window layer with a window of 8 positions and a
full-attention layer).

* the draft's proposals against the numpy draft (pinned to the reference's
  DFlashDraftModel) run on the very target features the engine committed, with
  contexts shorter and longer than the window;
* the DFlash loop (draft -> verify -> accept -> commit -> extend the draft's context)
  emits exactly the target engine's plain greedy continuation, both when the draft
  proposes (random draft weights: mostly rejected) and when the verify blocks carry the
  greedy continuation with a corruption (long accepted prefixes, so the feature ring
  extends the draft's context by many rows at once), eager and as a CUDA graph.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _setup(capacity=512):
    from qwen35_dflash_b200 import config, engine as E, synthetic
    from qwen35_dflash_b200.dflash import DFlash
    from qwen35_dflash_b200.draft import DraftEngine
    tc, dc = config.TINY, config.TINY_DRAFT
    raw = synthetic.init_weights(tc, seed=17)
    dw = synthetic.init_draft_weights(dc)
    te = E.TargetEngine(tc, E.weights_from_arrays(tc, raw), batch=1, block=16, capacity=capacity)
    dr = DraftEngine(dc, te, dw)
    return tc, dc, raw, dw, te, dr, DFlash(te, dr)


def _greedy(tc, raw, prompt, n, capacity=512):
    """The target engine's plain greedy continuation (one token per block)."""
    from qwen35_dflash_b200 import engine as E
    from qwen35_dflash_b200.session import TargetSession
    sess = TargetSession(E.TargetEngine(tc, E.weights_from_arrays(tc, raw), batch=1, block=16, capacity=capacity))
    sess.prefill(list(prompt))
    out = [sess.next_token]
    while len(out) < n:
        sess.step(out[-1])
        out.append(sess.next_token)
    return out


def _near_tie(row, a, b, ulps=4):
    return abs(float(row[a]) - float(row[b])) <= ulps * 2 ** -7 * max(1.0, abs(float(row[b])))


def _check_proposals(dc, dw, raw, feats, anchor, got, what):
    from oracle.draft_np import OracleDraft
    oracle = OracleDraft(dc, dw)
    want, logits = oracle.draft(np.concatenate(feats, 0), anchor, raw["target.embed_tokens.weight"],
                                raw["target.lm_head.weight"], return_logits=True)
    flips = 0
    for i, (a, b) in enumerate(zip(got, want)):
        if a != b:
            assert _near_tie(logits[i], a, b), (what, i, a, b)
            flips += 1
    return flips


def test_dflash_loop_is_the_greedy_continuation_and_draft_matches_oracle(cuda_lib):
    from helpers import to_np
    tc, dc, raw, dw, te, dr, df = _setup()
    prompt = [int(t) for t in np.random.default_rng(17).integers(0, tc.vocab_size, 20)]
    G = _greedy(tc, raw, prompt, 120)
    # prefill by hand to keep the committed rows' target features (the draft's context)
    S = te.S
    feats = []
    te.qpos.zero_(); te.state.zero_(); te.conv_hist.zero_()
    for i in range(0, len(prompt), S):
        chunk = prompt[i:i + S]
        te.tokens.copy_(torch.tensor(chunk + [0] * (S - len(chunk)), dtype=torch.int32))
        te.forward()
        te.accept(auto_commit=False)
        te.commit([len(chunk)])
        dr.extend()
        feats.append(to_np(te.features[:len(chunk)]))
    assert int(te.next_token.item()) == G[0]
    rng = np.random.default_rng(3)
    emitted, checks, flips, long_accepts = [], 0, 0, 0
    while len(emitted) < 100:
        anchor = int(te.next_token.item())
        dr.propose()
        props = te.tokens.cpu().tolist()
        assert props[0] == anchor
        # the draft's proposals against the oracle draft over the same context features
        flips += _check_proposals(dc, dw, raw, feats, anchor, props[1:], len(emitted))
        checks += 1
        if rng.random() < 0.6:      # verify the greedy continuation instead, with a corruption
            pos = len(emitted)
            block = G[pos:pos + S]
            j = int(rng.integers(1, S + 2))
            if j < S:
                block[j] = (block[j] + 1) % tc.vocab_size
            te.tokens.copy_(torch.tensor(block, dtype=torch.int32))
        te.step()
        dr.extend()
        acc = int(te.accepted.item())
        committed = te.tokens[:acc].cpu().tolist()
        long_accepts += acc > 4
        feats.append(to_np(te.features[:acc]))
        emitted += committed
    assert emitted[:100] == G[:100]
    assert checks >= 10 and long_accepts >= 5, (checks, long_accepts)
    assert flips <= 0.05 * checks * (S - 1), (flips, checks)


def test_dflash_generate_graph_equals_greedy(cuda_lib):
    tc, dc, raw, dw, te, dr, df = _setup()
    prompt = [int(t) for t in np.random.default_rng(5).integers(0, tc.vocab_size, 37)]
    G = _greedy(tc, raw, prompt, 48)
    for use_graph in (False, True):
        res = df.generate(prompt, max_new_tokens=48, use_graph=use_graph)
        assert res.token_ids == G, (use_graph, res.token_ids[:8], G[:8])
        assert res.steps >= 1 and len(res.iterations) == res.steps
