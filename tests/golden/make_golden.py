"""Generate the golden fixtures in this directory from the reference itself.

Runs ONLY where a checkout of the reference is present, named by the environment
variable ``QW_REFERENCE`` (its root directory); the committed ``*.npz`` files are what
the tests read, on any machine.  Nothing here is imported by the library.

Fixtures:
  ops_fp32.npz        reference/fused_ops.py functions on seeded float32 inputs
  ops_lowp.npz        the same functions on bf16 / fp16 inputs (rounding points)
  topk.npz            torch.topk on tie-heavy float32 rows (the router's selection)
  tiny_session.npz    FusedTargetModel + FusedTargetSession (fp16, fp32 recurrent
                      state) on the tiny configuration: greedy decode, then
                      block verify / commit rounds with seeded proposals.
  draft.npz           the reference's DFlashDraftModel (bf16) of the tiny draft
                      configuration: context features -> draft hidden rows and the
                      proposals of the target's lm_head, for two context lengths.
  binding_trace.npz   every call the reference's FusedTargetModel makes through the
                      reference's ModuleFusedOps on the tiny configuration (a 16-token
                      prefill and one decode step), recorded at the adapter-module
                      boundary: op name, arguments (weights by name) and the reference
                      backend's outputs; replayed through qwen35_dflash_b200.fused_ops.
  original/           two small shards in the original group-256 quantised layout
                      (data-0000{1,2}.safetensors, written here) and what the
                      reference's OriginalQuantWeights / canonicalkeys make of them
                      (expect.json: key mapping, rejected names; expect.npz: the
                      logical int4 values and scales of each tensor).

Usage:  QW_REFERENCE=<reference checkout> python tests/golden/make_golden.py
        (QW_GOLDEN_ONLY=draft: only draft.npz; =original: only original/;
         =binding: only binding_trace.npz)
"""
from __future__ import annotations

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
REF = os.environ.get("QW_REFERENCE", "")


def _import_reference():
    if not REF or not os.path.isdir(REF):
        raise SystemExit("set QW_REFERENCE to the root of a checkout of the reference")
    for sub in ("model", "reference"):
        path = os.path.join(REF, sub)
        if path not in sys.path:
            sys.path.insert(0, path)
    import fused_ops  # reference/fused_ops.py
    from qwen35_moe_dflash.fused.ops import ModuleFusedOps
    from qwen35_moe_dflash.fused.model import FusedTargetModel
    from qwen35_moe_dflash.fused.session import FusedTargetSession
    return fused_ops, ModuleFusedOps, FusedTargetModel, FusedTargetSession


def _np(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().numpy()


def make_ops(fused_ops):
    g = torch.Generator().manual_seed(1234)
    out = {}

    def rn(*shape, std=1.0, dtype=torch.float32):
        return (torch.randn(*shape, generator=g) * std).to(dtype)

    for tag, dtype in (("f32", torch.float32), ("bf16", torch.bfloat16), ("f16", torch.float16)):
        d = {}
        # rms_norm [3,5,64] and [7,256]
        for i, shape in enumerate(((3, 5, 64), (7, 256))):
            x = rn(*shape, dtype=dtype)
            gamma = (1 + rn(shape[-1], std=0.1)).to(dtype)
            d[f"rms{i}_x"], d[f"rms{i}_g"] = _np(x), _np(gamma)
            d[f"rms{i}_y"] = _np(fused_ops.rms_norm(x, gamma, 1e-6))
        # conv_state_update + causal_conv1d: B=2, S=5, C=24, K=4
        proj = rn(2, 5, 24, dtype=dtype)
        hist = rn(2, 24, 3, dtype=dtype)
        w = rn(24, 1, 4, std=0.3, dtype=dtype)
        new_hist, padded = fused_ops.conv_state_update(proj, hist)
        d["conv_proj"], d["conv_hist"], d["conv_w"] = _np(proj), _np(hist), _np(w)
        d["conv_newhist"], d["conv_padded"] = _np(new_hist), _np(padded)
        d["conv_out"] = _np(fused_ops.causal_conv1d(padded, w))
        # cache_update
        k0, v0 = rn(2, 2, 7, 16, dtype=dtype), rn(2, 2, 7, 16, dtype=dtype)
        k1, v1 = rn(2, 2, 3, 16, dtype=dtype), rn(2, 2, 3, 16, dtype=dtype)
        kk, vv = fused_ops.cache_update(k0, v0, k1, v1)
        d["cache_k0"], d["cache_v0"], d["cache_k1"], d["cache_v1"] = map(_np, (k0, v0, k1, v1))
        d["cache_k"], d["cache_v"] = _np(kk), _np(vv)
        # attention: B=2, H=8, Hkv=2, S=5, T=13, D=32
        q = rn(2, 8, 5, 32, dtype=dtype)
        kc, vc = rn(2, 2, 13, 32, dtype=dtype), rn(2, 2, 13, 32, dtype=dtype)
        d["attn_q"], d["attn_k"], d["attn_v"] = _np(q), _np(kc), _np(vc)
        d["attn_o"] = _np(fused_ops.attention(q, kc, vc, query_start=8, scale=32 ** -0.5))
        # moe: T=2x5 tokens, H=64, E=16, I=32, top-4; router rows coarsened to force ties
        hidden = rn(2, 5, 64, dtype=dtype)
        router = (torch.round(rn(16, 64, std=0.5) * 4) / 4).to(dtype)
        gate_up = rn(16, 64, 64, std=0.125, dtype=dtype)
        down = rn(16, 64, 32, std=0.125, dtype=dtype)
        d["moe_x"], d["moe_router"], d["moe_gu"], d["moe_down"] = map(_np, (hidden, router, gate_up, down))
        d["moe_y"] = _np(fused_ops.moe(hidden, router, gate_up, down, top_k=4))
        out[tag] = d
    # gated delta rule: fp32 and fp16 only (the reference rejects bf16)
    for tag, dtype in (("f32", torch.float32), ("f16", torch.float16)):
        d = out[tag]
        b, s, h, dk, dv = 3, 6, 4, 16, 24
        q, k = rn(b, s, h, dk, dtype=dtype), rn(b, s, h, dk, dtype=dtype)
        v = rn(b, s, h, dv, dtype=dtype)
        gg = (-torch.nn.functional.softplus(rn(b, s, h))).to(dtype)
        beta = torch.sigmoid(rn(b, s, h)).to(dtype)
        state = rn(b, h, dk, dv, std=0.1)
        length = torch.tensor([6, 0, 4], dtype=torch.int16)
        for norm in (True, False):
            core, st = fused_ops.chunk_gated_delta_rule(
                q, k, v, gg, beta, state, length, chunk_size=64, use_qk_l2norm_in_kernel=norm)
            d[f"gdn_core_{int(norm)}"], d[f"gdn_state_{int(norm)}"] = _np(core), _np(st)
        d["gdn_q"], d["gdn_k"], d["gdn_v"], d["gdn_g"], d["gdn_beta"] = map(_np, (q, k, v, gg, beta))
        d["gdn_s0"], d["gdn_len"] = _np(state), length.numpy()
    np.savez_compressed(os.path.join(HERE, "ops_fp32.npz"), **out["f32"])
    np.savez_compressed(os.path.join(HERE, "ops_lowp.npz"),
                        **{f"bf16_{k}": v for k, v in out["bf16"].items()},
                        **{f"f16_{k}": v for k, v in out["f16"].items()})


def make_topk():
    g = torch.Generator().manual_seed(99)
    out = {}
    for e, k in ((256, 8), (16, 4), (64, 6), (256, 1), (128, 8)):
        logits = torch.randn(256, e, generator=g)
        logits[::3] = torch.randint(-3, 3, (len(range(0, 256, 3)), e), generator=g).float()
        logits = logits.to(torch.bfloat16)
        probs = torch.softmax(logits.float(), -1)
        _, idx = torch.topk(probs, k, dim=-1)
        out[f"p_{e}_{k}"] = probs.numpy()
        out[f"i_{e}_{k}"] = idx.numpy().astype(np.int16)
    np.savez_compressed(os.path.join(HERE, "topk.npz"), **out)


def tiny_weights():
    """The tiny target's fp16 weights as the reference model takes them (W4 matrices
    quantised and dequantised); tests/test_binding_replay_gpu.py rebuilds the same."""
    sys.path.insert(0, ROOT)
    import __graft_entry__
    __graft_entry__.load_package()
    from qwen35_dflash_b200 import config as qcfg, synthetic
    from oracle.numerics import quantize_w4, dequantize_w4
    cfg = qcfg.TINY
    raw = synthetic.init_weights(cfg, seed=17)
    weights = {}
    for name, value in raw.items():
        if synthetic.is_w4(name):
            q, s = quantize_w4(value, cfg.quant_group)
            value = dequantize_w4(q, s, cfg.quant_group)
        weights[name] = torch.from_numpy(value).to(torch.float16)
    return cfg, weights


def make_binding_trace(ModuleFusedOps, FusedTargetModel, FusedTargetSession, fused_ops):
    """Record the reference model's calls at the fused-ops module boundary."""
    import json
    import types
    cfg, weights = tiny_weights()
    calls, arrays, wmap = [], {}, {}

    def enc(x):
        if isinstance(x, torch.Tensor):
            if id(x) in wmap:
                return {"weight": wmap[id(x)]}
            key = f"a{len(arrays):04d}"
            arrays[key] = x.detach().cpu().float().numpy() if x.dtype == torch.bfloat16 else x.detach().cpu().numpy()
            return {"array": key, "dtype": str(x.dtype).replace("torch.", "")}
        if isinstance(x, (tuple, list)):
            return {"seq": [enc(v) for v in x]}
        if x is None or isinstance(x, (bool, int, float)):
            return {"value": x}
        raise TypeError(f"unrecorded argument type {type(x)}")

    rec = types.ModuleType("recording_fused_ops")
    rec.FUSED_OPS_ABI = fused_ops.FUSED_OPS_ABI
    rec.BACKEND_ID = "reference-recorder"
    rec.IS_REFERENCE_BACKEND = True
    for name in ModuleFusedOps.required_operations:
        def wrapper(*args, _fn=getattr(fused_ops, name), _name=name, **kwargs):
            entry = {"op": _name, "args": [enc(a) for a in args], "kwargs": {k: enc(v) for k, v in kwargs.items()}}
            out = _fn(*args, **kwargs)
            entry["out"] = enc(out)
            calls.append(entry)
            return out
        setattr(rec, name, wrapper)
    ops = ModuleFusedOps(rec, allow_reference=True)
    model = FusedTargetModel(cfg.to_hf_text_config(), weights, feature_layers=cfg.feature_layers,
                             ops=ops, recurrent_dtype=torch.float32)
    for name in model._weight_names:
        wmap[id(model.weight(name))] = name
    prompt = np.random.default_rng(23).integers(0, cfg.vocab_size, 16).tolist()
    session = FusedTargetSession(model)
    session.prefill(prompt)
    first = session.next_token
    session.step(first)
    np.savez_compressed(os.path.join(HERE, "binding_trace.npz"), calls=np.asarray(json.dumps(calls)),
                        prompt=np.asarray(prompt, np.int32),
                        next_tokens=np.asarray([first, session.next_token], np.int32), **arrays)
    print("binding trace:", len(calls), "calls,", len(arrays), "arrays")


def make_tiny_session(ModuleFusedOps, FusedTargetModel, FusedTargetSession, fused_ops):
    sys.path.insert(0, ROOT)
    import __graft_entry__
    pkg = __graft_entry__.load_package()
    from qwen35_dflash_b200 import config as qcfg, synthetic
    from oracle.numerics import quantize_w4, dequantize_w4

    cfg = qcfg.TINY
    raw = synthetic.init_weights(cfg, seed=17)
    weights = {}
    for name, value in raw.items():
        if synthetic.is_w4(name):
            q, s = quantize_w4(value, cfg.quant_group)
            value = dequantize_w4(q, s, cfg.quant_group)
        weights[name] = torch.from_numpy(value).to(torch.float16)
    ops = ModuleFusedOps(fused_ops, allow_reference=True)
    model = FusedTargetModel(cfg.to_hf_text_config(), weights, feature_layers=cfg.feature_layers,
                             ops=ops, recurrent_dtype=torch.float32)
    prompt = np.random.default_rng(17).integers(0, cfg.vocab_size, 64).tolist()
    # every layer's output on the prompt (teacher-forced per-layer pin)
    all_layers = tuple(range(cfg.num_hidden_layers))
    probe = FusedTargetModel(cfg.to_hf_text_config(), weights, feature_layers=all_layers,
                             ops=ops, recurrent_dtype=torch.float32)
    layer_hidden = probe(torch.tensor([prompt])).features[0].reshape(64, cfg.num_hidden_layers, -1)
    layer_hidden = layer_hidden.permute(1, 0, 2).numpy().astype(np.float16)
    # layer outputs of the last layer are replaced by the final norm; keep the raw one too
    last = probe._forward_hidden  # noqa: F841  (documented behaviour, fused/model.py:407-409)
    # ordinary greedy decode: G[i] = prediction after prompt + G[:i]
    session = FusedTargetSession(model)
    session.prefill(prompt)
    greedy = [session.next_token]
    for _ in range(79):
        session.step(greedy[-1])
        greedy.append(session.next_token)
    # block verify rounds with seeded proposals
    session = FusedTargetSession(model)
    pre = session.prefill(prompt)
    rng = np.random.default_rng(5)
    committed = 0
    rounds = {"proposals": [], "expected": [], "accepted": [], "features": []}
    corrupt_at = [3, 16, 1, 9, 15, 5, 12, 2]
    for j in corrupt_at:
        if committed + 16 > len(greedy):
            break
        props = list(greedy[committed:committed + 16])
        if j < 16:
            props[j] = int((props[j] + 1 + rng.integers(0, cfg.vocab_size - 1)) % cfg.vocab_size)
        verification = session.verify(props)
        accepted = verification.max_accepted_prefix
        rounds["proposals"].append(props)
        rounds["expected"].append(list(verification.expected_next_tokens))
        rounds["accepted"].append(accepted)
        feats = torch.cat([f for _, f in verification._snapshots[1:]], dim=1)[0]
        rounds["features"].append(feats.float().numpy())
        verification.commit(accepted)
        committed += accepted
    state = session.state
    sums = []
    for layer in state.layers:
        for name in ("conv", "recurrent", "key", "value"):
            t = getattr(layer, name)
            if t is not None:
                sums.append([float(t.double().sum()), float(t.double().square().sum())])
    np.savez_compressed(
        os.path.join(HERE, "tiny_session.npz"),
        prompt=np.asarray(prompt, np.int32), greedy=np.asarray(greedy, np.int32),
        layer_hidden=layer_hidden,
        prefill_features=pre.features[0].float().numpy().astype(np.float16),
        proposals=np.asarray(rounds["proposals"], np.int32),
        expected=np.asarray(rounds["expected"], np.int32),
        accepted=np.asarray(rounds["accepted"], np.int32),
        features=np.asarray(rounds["features"], np.float16),
        final_position=np.int32(state.position), state_sums=np.asarray(sums, np.float64))


def make_draft():
    sys.path.insert(0, ROOT)
    import __graft_entry__
    __graft_entry__.load_package()
    from qwen35_dflash_b200 import config as qcfg, synthetic
    from qwen35_moe_dflash.config import Qwen35DFlashConfig
    from qwen35_moe_dflash.model import DFlashDraftModel

    tc, dc = qcfg.TINY, qcfg.TINY_DRAFT
    raw = dc.to_reference_dict(tc.vocab_size, tc.num_hidden_layers)
    model = DFlashDraftModel(Qwen35DFlashConfig.from_dict(raw), dtype=torch.bfloat16).eval()
    weights = synthetic.init_draft_weights(dc)
    with torch.no_grad():
        for name, param in model.named_parameters():
            param.copy_(torch.from_numpy(weights[name]).to(torch.bfloat16))
    target = synthetic.init_weights(tc, seed=17)
    embed = torch.from_numpy(target["target.embed_tokens.weight"]).to(torch.bfloat16)
    lm_head = torch.from_numpy(target["target.lm_head.weight"]).to(torch.bfloat16)
    g = torch.Generator().manual_seed(31)
    out = {}
    for case, ctx in enumerate((5, 20)):
        feats = torch.randn(1, ctx, dc.feature_size, generator=g).to(torch.bfloat16)
        anchor = int(torch.randint(0, tc.vocab_size, (1,), generator=g))
        ids = torch.tensor([[anchor] + [dc.mask_token_id] * (dc.block_size - 1)])
        positions = torch.arange(ctx + dc.block_size).view(1, -1)
        with torch.inference_mode():
            noise = model.embed_block(ids, embed)
            hidden = model.draft_hidden(feats, noise, positions)
            top1 = torch.argmax(torch.nn.functional.linear(hidden, lm_head), -1)
        out[f"features_{case}"] = feats[0].float().numpy()
        out[f"anchor_{case}"] = np.int32(anchor)
        out[f"hidden_{case}"] = hidden[0].float().numpy()
        out[f"top1_{case}"] = top1[0].numpy().astype(np.int32)
    np.savez_compressed(os.path.join(HERE, "draft.npz"), **out)


def make_original():
    import json
    sys.path.insert(0, os.path.dirname(HERE))
    sys.path.insert(0, ROOT)
    from original_fixture import quantize_g256, write_safetensors
    from qwen35_moe_dflash.target.original_quant import OriginalQuantWeights, canonicalkeys

    rng = np.random.default_rng(41)
    d = os.path.join(HERE, "original")
    os.makedirs(d, exist_ok=True)
    tensors = [("target.layers.0.linear_attn.out_proj.weight", (32, 512), np.float16),
               ("target.layers.3.self_attn.q_proj.weight", (48, 256), np.float32),
               ("target.layers.1.mlp.experts.down_proj", (2, 32, 512), np.float16),
               ("target.layers.2.mlp.gate.weight", (16, 256), np.float32),
               ("target.lm_head.weight", (64, 256), np.float16)]
    shards = [{}, {}]
    for i, (name, shape, sdt) in enumerate(tensors):
        w = rng.normal(0, 0.02, shape).astype(np.float32)
        w[..., :256] *= 3.0
        q, sc = quantize_g256(w)
        wkey, skey = canonicalkeys(name)
        shards[i % 2][wkey] = q
        shards[i % 2][skey] = (sc if "experts" in name else sc[..., None]).astype(sdt)
    for i, t in enumerate(shards):
        write_safetensors(os.path.join(d, f"data-0000{i + 1}.safetensors"), t)
    ref = OriginalQuantWeights(d)
    arrays = {}
    for i, (name, shape, _) in enumerate(tensors):
        q, sc = ref.logical(name, shape)
        arrays[f"q{i}"] = np.asarray(q)
        arrays[f"s{i}"] = np.asarray(sc)
    names = [t[0] for t in tensors] + [
        "target.layers.7.linear_attn.in_proj_qkv.weight", "target.layers.7.linear_attn.in_proj_z.weight",
        "target.layers.7.linear_attn.in_proj_b.weight", "target.layers.7.linear_attn.in_proj_a.weight",
        "target.layers.39.self_attn.k_proj.weight", "target.layers.39.self_attn.v_proj.weight",
        "target.layers.39.self_attn.o_proj.weight", "target.layers.5.mlp.experts.gate_up_proj",
        "target.layers.5.mlp.shared_expert.gate_proj.weight", "target.layers.5.mlp.shared_expert.up_proj.weight",
        "target.layers.5.mlp.shared_expert.down_proj.weight"]
    rejected = {}
    for name in ("target.embed_tokens.weight", "target.layers.0.input_layernorm.weight",
                 "target.layers.5.mlp.shared_expert_gate.weight", "target.layers.0.linear_attn.A_log",
                 "target.layers.5.mlp.experts.gate_up_proj.weight", "draft.fc.weight", "target.norm.weight"):
        try:
            canonicalkeys(name)
        except ValueError as e:
            rejected[name] = str(e)
    exp = {"keys": {n: list(canonicalkeys(n)) for n in names}, "rejected_names": rejected,
           "logical": [[n, list(s)] for n, s, _ in tensors]}
    with open(os.path.join(d, "expect.json"), "w") as f:
        json.dump(exp, f, indent=1)
    np.savez_compressed(os.path.join(d, "expect.npz"), **arrays)


def main():
    fused_ops, ModuleFusedOps, FusedTargetModel, FusedTargetSession = _import_reference()
    if os.environ.get("QW_GOLDEN_ONLY") == "draft":
        make_draft()
        return
    if os.environ.get("QW_GOLDEN_ONLY") == "original":
        make_original()
        return
    if os.environ.get("QW_GOLDEN_ONLY") == "binding":
        make_binding_trace(ModuleFusedOps, FusedTargetModel, FusedTargetSession, fused_ops)
        return
    torch.set_num_threads(min(8, os.cpu_count() or 1))
    make_ops(fused_ops)
    make_topk()
    make_tiny_session(ModuleFusedOps, FusedTargetModel, FusedTargetSession, fused_ops)
    make_binding_trace(ModuleFusedOps, FusedTargetModel, FusedTargetSession, fused_ops)
    make_draft()
    make_original()
    for name in sorted(os.listdir(HERE)):
        if name.endswith(".npz"):
            print(name, os.path.getsize(os.path.join(HERE, name)))


if __name__ == "__main__":
    main()
