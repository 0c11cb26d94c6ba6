"""The engine built from an original group-256 checkpoint vs the oracle (GPU).

A tiny target shaped like the original checkpoint (every K a multiple of 256) is
written in the original layout (tests/original_fixture.py), imported with
``original.load_original_target`` and run through the block verify engine; every
layer's output (taps on all layers, teacher forced from the engine's committed state)
must equal the oracle evaluated on the weights those files define: the int4 values
times their bf16-rounded scales, and bf16 for the dequantised router / b, a / lm_head /
embedding.  Then a greedy prefill must predict the oracle's next token.
"""
import dataclasses

import numpy as np
import pytest
import torch

from helpers import to_np
from oracle.model_np import OracleTarget
from original_fixture import write_original
from test_engine_gpu import _oracle_state_from_engine

pytestmark = pytest.mark.gpu


def test_imported_engine_matches_oracle(cuda_lib, tmp_path):
    from qwen35_dflash_b200 import config, engine as E, original, synthetic
    cfg = dataclasses.replace(config.TINY_G256, feature_layers=(0, 1, 2, 3))
    raw = synthetic.init_weights(cfg, seed=23)
    fx = write_original(cfg, raw, tmp_path)
    weights = original.load_original_target(cfg, fx["quant_dir"], fx["base"], fx["embed_w"], fx["embed_s"])
    eng = E.TargetEngine(cfg, weights, batch=1, block=16, capacity=256)
    oracle = OracleTarget(cfg.to_hf_text_config(), fx["expected"], cfg.feature_layers, act="bf16", rope="f32")
    prompt = np.random.default_rng(23).integers(0, cfg.vocab_size, 48)
    H = cfg.hidden_size
    rows_ok = rows = 0
    for blk in range(3):
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
            want = out[0]
            tol = 2e-2 + 1e-2 * np.maximum(np.abs(want), np.sqrt(np.mean(want * want, -1, keepdims=True)))
            ok = (np.abs(got - want) <= tol).all(-1)
            # a routing near-tie may move a token's whole row (see test_layers_teacher_forced)
            assert ok.sum() >= len(ok) - 2, (blk, layer, np.nonzero(~ok))
            rows_ok += int(ok.sum())
            rows += len(ok)
            x = got[None]
        eng.commit([16])
    assert rows_ok >= 0.97 * rows, (rows_ok, rows)
    # the prediction after the prompt: the oracle's, or a counted near-tie of its logits
    top1, _, _, logits = oracle.forward(np.asarray([prompt]), return_logits=True)
    got = int(eng.next_token.item())
    want = int(top1[0, -1])
    row = logits[0, -1]
    assert got == want or abs(float(row[got]) - float(row[want])) <= 4 * 2 ** -7 * max(1.0, abs(float(row[want])))
