"""The DFlash draft on the device: its context cache and its block forward.

The reference's draft (model/qwen35_moe_dflash/model.py:102-522) is cache-free: every
call projects the target features of the whole context again.  Here the draft keeps a
paged K/V cache per layer (the same page table as the target's KV cache, positions are
the committed positions of the sequence), extended after every commit by the rows that
were committed (``extend``: fc + hidden_norm of their target features, then each layer's
k_proj / k_norm / rotary and v_proj) -- the feature ring that feeds the draft.  A
``propose`` runs the draft over the block [anchor, mask x 15] at the committed
positions, attending to that cache and to the block itself (sliding layers causal
within the window, the last layer bidirectional over the block), and writes the next
verify block -- the anchor and 15 proposals -- straight into the target engine's
tokens.  Everything is device-side and stream-ordered (graph-capturable).
"""
from __future__ import annotations

import torch

from . import lib, w4
from .config import DraftConfig

BF16 = torch.bfloat16


class DraftEngine:
    def __init__(self, dcfg: DraftConfig, target, weights, device="cuda"):
        """``target``: the TargetEngine whose features feed the draft and whose tokens
        receive the proposals; ``weights``: name -> array/tensor by the reference's draft
        parameter names (model.py), bf16 values."""
        te = target
        c = te.cfg
        if tuple(c.feature_layers) != tuple(dcfg.target_layer_ids):
            raise ValueError("the target's feature taps must be the draft's target_layer_ids")
        if dcfg.hidden_size != c.hidden_size or dcfg.block_size != te.S:
            raise ValueError("draft and target disagree on hidden size or block size")
        self.d, self.te, self.lib = dcfg, te, lib.load()
        self.dev = torch.device(device)
        d, dev = dcfg, self.dev
        B, S, H = te.B, te.S, d.hidden_size
        T = B * S
        Hq, Hkv, D, I = d.num_attention_heads, d.num_key_value_heads, d.head_dim, d.intermediate_size
        self.B, self.S, self.T, self.H, self.Hq, self.Hkv, self.D, self.I = B, S, T, H, Hq, Hkv, D, I

        def t(name):
            v = weights[name]
            v = v if isinstance(v, torch.Tensor) else torch.from_numpy(v)
            return v.to(device=dev, dtype=BF16).contiguous()

        self.fc = w4.pack_b16(t("fc.weight"))
        self.hidden_norm, self.final_norm = t("hidden_norm.weight"), t("norm.weight")
        self.layers = []
        tile_bytes = (H // 64) * 2048       # one 16-row tile of a bf16 stream with K = H
        for i in range(d.num_hidden_layers):
            p = f"layers.{i}"
            qkv = w4.pack_b16(torch.cat([t(p + ".self_attn.q_proj.weight"), t(p + ".self_attn.k_proj.weight"),
                                         t(p + ".self_attn.v_proj.weight")]))
            self.layers.append({
                "qkv": qkv, "kv_ptr": qkv.data_ptr() + (Hq * D // 16) * tile_bytes,   # the k | v rows
                "o": w4.pack_b16(t(p + ".self_attn.o_proj.weight")),
                "gate_up": w4.pack_b16(torch.cat([t(p + ".mlp.gate_proj.weight"), t(p + ".mlp.up_proj.weight")])),
                "down": w4.pack_b16(t(p + ".mlp.down_proj.weight")),
                "in_norm": t(p + ".input_layernorm.weight"), "post_norm": t(p + ".post_attention_layernorm.weight"),
                "q_norm": t(p + ".self_attn.q_norm.weight"), "k_norm": t(p + ".self_attn.k_norm.weight"),
            })
        L = d.num_hidden_layers
        self.ldq = (Hq + 2 * Hkv) * D
        kv_shape = (L, te.B * te.max_pages, Hkv, te.P, D)
        self.k_cache = torch.zeros(kv_shape, dtype=BF16, device=dev)
        self.v_cache = torch.zeros(kv_shape, dtype=BF16, device=dev)
        self.hidden = torch.zeros(T, H, dtype=BF16, device=dev)
        self.normed = torch.zeros(T, H, dtype=BF16, device=dev)
        self.qkv = torch.zeros(T, self.ldq, dtype=BF16, device=dev)
        self.qout = torch.zeros(B, Hq, S, D, dtype=BF16, device=dev)
        self.attn_out = torch.zeros(T, Hq * D, dtype=BF16, device=dev)
        self.gu = torch.zeros(T, 2 * I, dtype=BF16, device=dev)
        self.act = torch.zeros(T, I, dtype=BF16, device=dev)
        self.ext = torch.zeros(T, H, dtype=BF16, device=dev)
        self.ext_n = torch.zeros(T, H, dtype=BF16, device=dev)
        self.kvx = torch.zeros(T, 2 * Hkv * D, dtype=BF16, device=dev)
        self.keys = torch.zeros_like(te.keys)
        self.attn_ws = torch.zeros(max(16, self.lib.qw_attn_workspace_bytes(B, Hq, Hkv, S, D, te.capacity)),
                                   dtype=torch.uint8, device=dev)

    def _call(self, name, *args):
        self.te._call(name, *args)

    def _st(self):
        return torch.cuda.current_stream(self.dev).cuda_stream

    # ------------------------------------------------------------------ context
    def extend(self, valid: torch.Tensor | None = None, features: torch.Tensor | None = None,
               pos_sub: torch.Tensor | None = None):
        """Append the draft K/V of committed rows: row s of sequence b (s < valid[b],
        default the target's accepted counts) of ``features`` (default the target's
        feature taps of the last verify block, [B * S, F]) at position
        qpos[b] - pos_sub[b] + s (default pos_sub = valid: the rows are the last ones the
        target committed, its qpos already advanced past them)."""
        te, d, st = self.te, self.d, self._st()
        valid = te.accepted if valid is None else valid
        pos_sub = valid if pos_sub is None else pos_sub
        features = te.features if features is None else features
        if features.shape[0] != self.T or features.stride(-1) != 1:
            raise ValueError("features: one row per block position, contiguous rows")
        T, H, Hkv, D = self.T, self.H, self.Hkv, self.D
        self._call("qw_b16_linear", features.data_ptr(), self.fc.data_ptr(), self.ext.data_ptr(),
                   lib.QW_OUT_BF16, H, T, H, d.feature_size, st)
        self._call("qw_rms_norm", self.ext.data_ptr(), lib.QW_BF16, self.hidden_norm.data_ptr(), lib.QW_BF16,
                   self.ext_n.data_ptr(), lib.QW_BF16, T, H, d.rms_norm_eps, st)
        for i, lw in enumerate(self.layers):
            self._call("qw_b16_linear", self.ext_n.data_ptr(), lw["kv_ptr"], self.kvx.data_ptr(), lib.QW_OUT_BF16,
                       2 * Hkv * D, T, 2 * Hkv * D, H, st)
            self._call("qw_draft_prep", self.kvx.data_ptr(), 2 * Hkv * D, 0, None, lw["k_norm"].data_ptr(),
                       d.rms_norm_eps, d.rope_theta, te.qpos.data_ptr(), pos_sub.data_ptr(), valid.data_ptr(),
                       te.pages.data_ptr(), te.max_pages, te.P, self.k_cache[i].data_ptr(),
                       self.v_cache[i].data_ptr(), None, self.B, self.S, self.Hq, Hkv, D, st)

    # ------------------------------------------------------------------ block
    def propose(self):
        """The draft over [anchor = target next_token, mask x (S-1)] at the committed
        positions; writes [anchor, proposals] into the target's tokens."""
        te, d, st = self.te, self.d, self._st()
        T, H, Hq, Hkv, D, I = self.T, self.H, self.Hq, self.Hkv, self.D, self.I
        eps = d.rms_norm_eps
        self._call("qw_draft_block_embed", te.glob["embed"].data_ptr(), te.next_token.data_ptr(), d.mask_token_id,
                   self.hidden.data_ptr(), self.B, self.S, H, st)
        for i, lw in enumerate(self.layers):
            self._call("qw_rms_norm", self.hidden.data_ptr(), lib.QW_BF16, lw["in_norm"].data_ptr(), lib.QW_BF16,
                       self.normed.data_ptr(), lib.QW_BF16, T, H, eps, st)
            self._call("qw_b16_linear", self.normed.data_ptr(), lw["qkv"].data_ptr(), self.qkv.data_ptr(),
                       lib.QW_OUT_BF16, self.ldq, T, self.ldq, H, st)
            self._call("qw_draft_prep", self.qkv.data_ptr(), self.ldq, 1, lw["q_norm"].data_ptr(),
                       lw["k_norm"].data_ptr(), eps, d.rope_theta, te.qpos.data_ptr(), None, None,
                       te.pages.data_ptr(), te.max_pages, te.P, self.k_cache[i].data_ptr(),
                       self.v_cache[i].data_ptr(), self.qout.data_ptr(), self.B, self.S, Hq, Hkv, D, st)
            self._call("qw_attn_paged_masked", self.qout.data_ptr(), self.k_cache[i].data_ptr(),
                       self.v_cache[i].data_ptr(), te.pages.data_ptr(), te.max_pages, te.P, te.qpos.data_ptr(),
                       te.capacity, self.attn_out.data_ptr(), self.B, self.S, Hq, Hkv, D, D ** -0.5,
                       0 if d.causal(i) else 1, d.window(i), self.attn_ws.data_ptr(), st)
            self._call("qw_b16_linear", self.attn_out.data_ptr(), lw["o"].data_ptr(), self.hidden.data_ptr(),
                       lib.QW_OUT_RESID_BF16, H, T, H, Hq * D, st)
            self._call("qw_rms_norm", self.hidden.data_ptr(), lib.QW_BF16, lw["post_norm"].data_ptr(), lib.QW_BF16,
                       self.normed.data_ptr(), lib.QW_BF16, T, H, eps, st)
            self._call("qw_b16_linear", self.normed.data_ptr(), lw["gate_up"].data_ptr(), self.gu.data_ptr(),
                       lib.QW_OUT_BF16, 2 * I, T, 2 * I, H, st)
            self._call("qw_swiglu", self.gu.data_ptr(), self.act.data_ptr(), T, I, st)
            self._call("qw_b16_linear", self.act.data_ptr(), lw["down"].data_ptr(), self.hidden.data_ptr(),
                       lib.QW_OUT_RESID_BF16, H, T, H, I, st)
        self._call("qw_rms_norm", self.hidden.data_ptr(), lib.QW_BF16, self.final_norm.data_ptr(), lib.QW_BF16,
                   self.normed.data_ptr(), lib.QW_BF16, T, H, eps, st)
        self._call("qw_lmhead_argmax", self.normed.data_ptr(), te.glob["lm_head"].data_ptr(), None,
                   self.keys.data_ptr(), T, te.vocab_pad, H, st)
        self._call("qw_draft_propose", self.keys.data_ptr(), te.nblk, te.next_token.data_ptr(), te.tokens.data_ptr(),
                   self.B, self.S, st)
