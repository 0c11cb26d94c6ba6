"""The 40-layer-style block verify engine on the tiny configuration vs the oracle (GPU)."""
import dataclasses

import numpy as np
import pytest
import torch

from helpers import assert_close, to_np
from oracle.model_np import OracleTarget, verify as oracle_verify, commit as oracle_commit
from oracle.numerics import quantize_w4, dequantize_w4, bf16_round

pytestmark = pytest.mark.gpu


def _tiny(feature_layers=None, seed=17):
    from qwen35_dflash_b200 import config as qcfg, synthetic
    cfg = qcfg.TINY
    if feature_layers is not None:
        cfg = dataclasses.replace(cfg, feature_layers=tuple(feature_layers))
    raw = synthetic.init_weights(cfg, seed=seed)
    deq = {}
    for name, value in raw.items():
        if synthetic.is_w4(name):
            q, s = quantize_w4(value, cfg.quant_group)
            value = dequantize_w4(q, s, cfg.quant_group)
        deq[name] = value
    oracle = OracleTarget(cfg.to_hf_text_config(), deq, cfg.feature_layers, act="bf16", rope="f32")
    return cfg, raw, oracle


def _engine(cfg, raw, batch=1, capacity=256):
    from qwen35_dflash_b200 import engine as E
    weights = E.weights_from_arrays(cfg, raw)
    return E.TargetEngine(cfg, weights, batch=batch, block=16, capacity=capacity)


def _oracle_state_from_engine(oracle, eng, b=0):
    """The engine's committed banks of sequence b as an oracle State (teacher forcing)."""
    from oracle.model_np import LayerState, State
    cfg = eng.cfg
    pos = int(eng.qpos[b].item())
    layers = []
    for l, kind in enumerate(cfg.layer_types):
        if kind == "linear_attention":
            gi = eng.gdn_idx[l]
            layers.append(LayerState(conv=to_np(eng.conv_hist[gi, b:b + 1]),
                                     recurrent=to_np(eng.state[gi, b:b + 1]).transpose(0, 1, 3, 2).copy()))
        else:
            ai = eng.attn_idx[l]
            t = np.arange(pos)
            pg = eng.pages[b].cpu().numpy()[t // eng.P]
            k = to_np(eng.k_cache[ai])[pg, :, t % eng.P].transpose(1, 0, 2)[None]
            v = to_np(eng.v_cache[ai])[pg, :, t % eng.P].transpose(1, 0, 2)[None]
            layers.append(LayerState(key=k, value=v))
    return State(pos, layers)


def test_layers_teacher_forced(cuda_lib):
    """Every layer's output from the engine (taps on all layers) equals the oracle layer
    applied to the engine's previous-layer output and the engine's committed state
    (64-token prompt in 4 blocks, each committed)."""
    cfg, raw, oracle = _tiny(feature_layers=(0, 1, 2, 3))
    eng = _engine(cfg, raw)
    prompt = np.random.default_rng(17).integers(0, cfg.vocab_size, 64)
    H = cfg.hidden_size
    rows_ok = rows = 0
    for blk in range(4):
        ostate = _oracle_state_from_engine(oracle, eng)
        ids = prompt[blk * 16:(blk + 1) * 16]
        eng.tokens.copy_(torch.from_numpy(ids.astype(np.int32)))
        eng.forward()
        eng.accept(auto_commit=False)
        feats = to_np(eng.features)
        x = oracle.w["target.embed_tokens.weight"][ids][None]
        for layer in range(cfg.num_hidden_layers):
            out, _ = oracle.layer(layer, x, ostate.layers[layer], ostate.position)
            if layer == cfg.num_hidden_layers - 1:
                out = oracle.norm(out, "target.norm.weight")
            got = feats[:, layer * H:(layer + 1) * H]
            # a token whose routing sits on a near-tie may pick another expert (fp32
            # summation order of the router logits), which changes its whole row: count
            # rows, allow at most two such tokens per layer and 3% overall
            want = out[0]
            tol = 2e-2 + 1e-2 * np.maximum(np.abs(want), np.sqrt(np.mean(want * want, -1, keepdims=True)))
            ok = (np.abs(got - want) <= tol).all(-1)
            assert ok.sum() >= len(ok) - 2, (blk, layer, np.nonzero(~ok))
            rows_ok += int(ok.sum())
            rows += len(ok)
            x = got[None]
        eng.commit([16])
    assert rows_ok >= 0.97 * rows, (rows_ok, rows)


def _greedy_chain(sess, next_token, n=16):
    """Proposals equal to the engine's own greedy continuation from the committed state:
    iterate verify until the block is self-consistent (p[i+1] = prediction after p[i])."""
    props = [next_token] + [0] * (n - 1)
    for _ in range(n):
        v = sess.verify(props)
        new = [next_token] + list(v.expected_next_tokens[1:n])
        v.abort()
        if new == props:
            break
        props = new
    return props


def _near_tie(row, a, b, ulps=4):
    """Oracle logits of tokens a and b within ``ulps`` bf16 ulps (2^-7 relative) of each other."""
    return abs(float(row[a]) - float(row[b])) <= ulps * 2 ** -7 * max(1.0, abs(float(row[b])))


def test_session_rounds_match_oracle(cuda_lib, golden):
    """DFlash rounds (the engine's own greedy chain with a seeded corruption, then commit
    of the accepted prefix) vs the bf16 oracle run from the engine's own committed state
    each round.  A predicted token may differ from the oracle's only where the oracle's
    two candidate logits are within four bf16 ulps (2^-7 relative each: two
    implementations that round at the same points but sum in different fp32 orders drift
    by a few ulps over the layers), and an accepted count only where the first such
    near-tie sits inside the accepted prefix; >= 95% of the predictions must agree.
    A prediction may also differ where a token of the block at or before it sits on a
    routing near-tie (k-th and (k+1)-th router logits within two bf16 ulps in some
    layer of the oracle): the engine's router GEMV sums in another order and may pick
    the other expert, which moves that token's hidden state by more than a few ulps.
    Such rounds are counted and must stay rare."""
    from qwen35_dflash_b200.session import TargetSession
    cfg, raw, oracle = _tiny()
    eng = _engine(cfg, raw, capacity=2048)
    sess = TargetSession(eng)
    d = golden("tiny_session.npz")
    prompt = [int(t) for t in d["prompt"]]
    sess.prefill(prompt)
    top1, feats, _, _ = oracle.forward(np.asarray([prompt]))
    assert sess.next_token == int(top1[0, -1])
    assert_close(to_np(sess.last_features[0]), feats[0, -1:], 2e-2, 1e-2, "prefill features", row_scale=True)
    agree = total = same_acc = tie_acc = route_flips = 0
    rng = np.random.default_rng(11)
    rounds = 48
    for r in range(rounds):
        next_token = sess.next_token
        props = _greedy_chain(sess, next_token)
        j = int(rng.integers(1, 18))
        if j < 16:
            props[j] = int((props[j] + 1 + rng.integers(0, cfg.vocab_size - 1)) % cfg.vocab_size)
        ostate = _oracle_state_from_engine(oracle, eng)
        v = sess.verify(props)
        oracle.router_gaps = []
        o_top1, _, _, logits = oracle.forward(np.asarray([props]), ostate, return_logits=True)
        gaps = np.min(np.stack(oracle.router_gaps), 0)     # per token, over the MoE layers
        oracle.router_gaps = None
        exp = (next_token,) + tuple(int(t) for t in o_top1[0])
        ties = set()
        flipped = False
        for i, (a, b) in enumerate(zip(v.expected_next_tokens, exp)):
            total += 1
            if a == b:
                agree += 1
            else:
                assert i > 0, (r, i, a, b)
                if not _near_tie(logits[0, i - 1], a, b):
                    assert gaps[:i].min() <= 2.0, (r, i, a, b, gaps[:i].min())
                    flipped = True
                ties.add(i)
        route_flips += int(flipped)
        acc = 0
        for i, t in enumerate(props):
            if t != exp[i]:
                break
            acc += 1
        got = v.max_accepted_prefix
        if got == acc:
            same_acc += 1
        else:
            # the decisions part at the first position where the predictions differ
            assert min(got, acc) in ties, (r, got, acc, sorted(ties))
            tie_acc += 1
        v.commit(got)
    assert agree >= 0.95 * total, (agree, total)
    assert same_acc + tie_acc == rounds and same_acc >= 0.75 * rounds, (same_acc, tie_acc, rounds)
    assert route_flips <= 0.1 * rounds, (route_flips, rounds)


def test_verification_semantics(cuda_lib):
    from qwen35_dflash_b200.session import TargetSession
    cfg, raw, _ = _tiny()
    sess = TargetSession(_engine(cfg, raw))
    with pytest.raises(RuntimeError):
        sess.verify([1, 2])
    sess.prefill(list(range(20)))
    assert sess.position == 20
    v1 = sess.verify([sess.next_token, 5, 6])
    v2 = sess.verify([sess.next_token, 7])
    assert v1.max_accepted_prefix >= 1 and v2.max_accepted_prefix >= 1
    with pytest.raises(ValueError):
        v1.commit(v1.max_accepted_prefix + 1)
    v1.commit(1)             # v2 was the engine's last block: v1 is re-run before commit
    assert sess.position == 21
    with pytest.raises(RuntimeError):
        v2.commit(1)         # stale after v1 committed
    with pytest.raises(ValueError):
        sess.verify([])


def test_device_commit_equals_host_commit(cuda_lib):
    """The graph-capturable step (device-side accept + commit) equals verify + commit(max)."""
    cfg, raw, _ = _tiny()
    a = _engine(cfg, raw, batch=2, capacity=128)
    b = _engine(cfg, raw, batch=2, capacity=128)
    for e in (a, b):
        e.set_random_context(40, seed=5)
    rng = np.random.default_rng(0)
    for it in range(3):
        props = torch.from_numpy(rng.integers(0, cfg.vocab_size, (2, 16)).astype(np.int32)).cuda()
        props[:, 0] = a.next_token
        props[1, 1:4] = a.top1.view(2, 16)[1, :3] if it else props[1, 1:4]
        for e in (a, b):
            e.tokens.copy_(props.view(-1))
        a.step()
        b.forward()
        b.accept(auto_commit=False)
        b.commit(b.max_accepted.clone())
        torch.cuda.synchronize()
        assert torch.equal(a.accepted, b.accepted)
        assert torch.equal(a.qpos, b.qpos) and torch.equal(a.next_token, b.next_token)
        assert torch.equal(a.state, b.state) and torch.equal(a.conv_hist, b.conv_hist)


def test_cuda_graph_replay_matches_eager(cuda_lib):
    cfg, raw, _ = _tiny()
    a = _engine(cfg, raw, batch=2, capacity=128)
    b = _engine(cfg, raw, batch=2, capacity=128)
    for e in (a, b):
        e.set_random_context(30, seed=9)
    a.capture()
    for it in range(3):
        props = torch.randint(0, cfg.vocab_size, (32,), dtype=torch.int32, device="cuda")
        for e in (a, b):
            e.tokens.copy_(props)
        a.replay()
        b.step()
        torch.cuda.synchronize()
        assert torch.equal(a.top1, b.top1) and torch.equal(a.qpos, b.qpos)
        assert torch.equal(a.state, b.state) and torch.equal(a.features, b.features)


@pytest.mark.parametrize("batch", [3])
def test_batched_sequences_are_independent(cuda_lib, batch):
    """Sequences of one batch at different positions give the single-sequence results."""
    cfg, raw, _ = _tiny()
    big = _engine(cfg, raw, batch=batch, capacity=128)
    big.set_random_context(0, seed=1)
    ctx = [20, 33, 47]
    big.qpos.copy_(torch.tensor(ctx, dtype=torch.int32))
    props = torch.randint(0, cfg.vocab_size, (batch, 16), dtype=torch.int32, device="cuda")
    big.tokens.copy_(props.view(-1))
    big.forward()
    big.accept(auto_commit=False)
    for i in range(batch):
        one = _engine(cfg, raw, batch=1, capacity=128)
        one.state.copy_(big.state[:, i:i + 1])
        one.conv_hist.copy_(big.conv_hist[:, i:i + 1])
        mp = big.max_pages
        one.k_cache.copy_(big.k_cache[:, i * mp:(i + 1) * mp])
        one.v_cache.copy_(big.v_cache[:, i * mp:(i + 1) * mp])
        one.qpos.fill_(ctx[i])
        one.tokens.copy_(props[i])
        one.forward()
        one.accept(auto_commit=False)
        assert torch.equal(one.top1, big.top1.view(batch, 16)[i])
        assert torch.equal(one.features, big.features.view(batch, 16, -1)[i])


def test_greedy_dflash_free_running_matches_oracle(cuda_lib, golden):
    """Greedy DFlash rounds on config 1 (the tiny target, 64-token prompt), free-running:
    the engine (through TargetSession) and the bf16 oracle each keep their OWN state for
    the whole run -- the oracle's caches come from its own forwards over the committed
    tokens, never from the engine's banks -- and commit the same token stream (the
    engine's decisions).  Each round verifies one 16-token block (anchor + 15 drafts:
    the engine's own greedy continuation with a seeded corruption, or random drafts)
    and both sides' accepted sequences (accepted drafts + correction/bonus token) are
    compared.

    The stated greedy gate: identical accepted sequences on >= 99 % of rounds, where a round
    whose first differing prediction sits on a near-tie of the oracle's logits (<= 4
    bf16 ulps) or behind a routing near-tie (k-th and (k+1)-th router logits within 4
    bf16 ulps) of a token at or before it counts as explained: such rounds are counted
    and printed (<= 30 %: the logits are bf16, whose 8-bit significand makes near-ties
    of the top two of 4096 random-weight logits common; measured about 21 %); other
    differences count against the 99 %."""
    from qwen35_dflash_b200.session import TargetSession
    from oracle.model_np import commit as o_commit
    cfg, raw, oracle = _tiny()
    rounds, S = 160, 16
    eng = _engine(cfg, raw, capacity=64 + rounds * S + 2 * S)
    sess = TargetSession(eng)
    prompt = [int(t) for t in np.random.default_rng(17).integers(0, cfg.vocab_size, 64)]
    sess.prefill(prompt)
    o_top1, _, ostate, _ = oracle.forward(np.asarray([prompt]))
    assert sess.next_token == int(o_top1[0, -1])
    rng = np.random.default_rng(23)
    identical = exempt_logit = exempt_route = 0
    unexplained = []
    new_tokens = 0
    for r in range(rounds):
        anchor = sess.next_token
        if r % 4 == 3:
            props = [anchor] + [int(t) for t in rng.integers(0, cfg.vocab_size, S - 1)]
        else:
            props = _greedy_chain(sess, anchor, S)
            j = int(rng.integers(1, S + 2))
            if j < S:
                props[j] = int((props[j] + 1 + rng.integers(0, cfg.vocab_size - 1)) % cfg.vocab_size)
        v = sess.verify(props)
        oracle.router_gaps = []
        o_top1, _, _, logits = oracle.forward(np.asarray([props]), ostate.copy(), return_logits=True)
        gaps = np.min(np.stack(oracle.router_gaps), 0)
        oracle.router_gaps = None
        exp_o = (anchor,) + tuple(int(t) for t in o_top1[0])
        exp_e = tuple(v.expected_next_tokens)
        acc_e = v.max_accepted_prefix
        acc_o = 0
        while acc_o < S and props[acc_o] == exp_o[acc_o]:
            acc_o += 1
        seq_e = tuple(props[:acc_e]) + (exp_e[acc_e],)
        seq_o = tuple(props[:acc_o]) + (exp_o[acc_o],)
        if seq_e == seq_o:
            identical += 1
        else:
            # the first prediction (entry i, made after consuming proposal i-1) that differs
            i = next(i for i in range(1, S + 1) if exp_e[i] != exp_o[i])
            if _near_tie(logits[0, i - 1], exp_e[i], exp_o[i]):
                exempt_logit += 1
            elif gaps[:i].min() <= 4.0:
                exempt_route += 1
            else:
                unexplained.append((r, i, exp_e[i], exp_o[i], float(gaps[:i].min())))
        # both sides commit the engine's decision: the oracle from its own state
        ostate = o_commit(oracle, ostate, props, acc_e)
        v.commit(acc_e)
        new_tokens += acc_e
    exempt = exempt_logit + exempt_route
    print(f"\ngreedy DFlash free-running: {rounds} rounds, {new_tokens} committed tokens; "
          f"identical {identical}, near-tie exemptions {exempt} (logits {exempt_logit}, routing "
          f"{exempt_route}), unexplained {len(unexplained)} {unexplained}")
    assert new_tokens >= 64
    # >= 99 % of rounds identical, or different only on a counted near-tie
    assert identical + exempt >= 0.99 * rounds, (identical, exempt, unexplained)
    assert exempt <= 0.30 * rounds, (exempt_logit, exempt_route, rounds)
