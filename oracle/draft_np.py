"""numpy restatement of the DFlash draft forward -- TEST INFRASTRUCTURE ONLY (see
``oracle/__init__.py``).

Follows the reference's cache-free draft golden (model/qwen35_moe_dflash/model.py:102-522,
its primitive ops model/qwen35_moe_dflash/ops.py:58-128) and the draft graph's block
and context construction (model/qwen35_moe_dflash/reference/graphs.py:63-97), rounding to
bf16 where the reference's bf16 torch ops return bf16 tensors:

* target_hidden = hidden_norm(fc(features)) over the context positions [0, start);
* block = [anchor, mask x (S-1)] embedded, at positions start .. start + S - 1;
* per layer: x = RMSNorm(h); q = q_norm(q_proj(x)); k, v = k_norm(k_proj(.)),
  v_proj(.) of the context rows and of the block rows, concatenated; rotary on q and k
  (full head dim, theta from the config, bf16 cos/sin); attention with the layer's mask
  (sliding layers causal with the window, the full layer bidirectional over the block);
  h += o_proj(attn); h += down(silu(gate(x')) * up(x')) with x' = RMSNorm(h);
* the final RMSNorm; proposals = stable argmax of lm_head rows 1 .. S-1.

RMSNorm here is the draft's (model.py via ops.py:66-71): weight * normalized.to(dtype),
the weight being the effective scale.  The parity pin is ``tests/golden/draft.npz``, made
by the reference's own DFlashDraftModel (``tests/golden/make_golden.py``).
"""
from __future__ import annotations

import numpy as np

from .numerics import bf16_round, stable_argmax


class OracleDraft:
    def __init__(self, cfg, weights: dict):
        self.c = cfg
        self.w = {k: np.asarray(v, np.float32) for k, v in weights.items()}

    # primitives ----------------------------------------------------------------------
    @staticmethod
    def r(x):
        return bf16_round(x)

    def norm(self, x, name):
        x = np.asarray(x, np.float32)
        inv = 1.0 / np.sqrt(np.mean(x * x, -1, keepdims=True, dtype=np.float32) + np.float32(self.c.rms_norm_eps))
        return self.r(self.r(x * inv) * self.w[name])

    def linear(self, x, name):
        return self.r(np.asarray(x, np.float32) @ self.w[name].T)

    def rope(self, x, positions):
        """x [..., n, D] at positions [n] (model.py:80-99, ops.py:75-90)."""
        d = self.c.head_dim
        inv = (1.0 / (np.float32(self.c.rope_theta) ** (np.arange(0, d, 2, dtype=np.float32) / np.float32(d))))
        freq = np.asarray(positions, np.float32)[:, None] * inv.astype(np.float32)[None, :]
        emb = np.concatenate([freq, freq], -1)
        cos, sin = self.r(np.cos(emb)), self.r(np.sin(emb))
        half = d // 2
        rot = np.concatenate([-x[..., half:], x[..., :half]], -1)
        return self.r(self.r(x * cos) + self.r(rot * sin))

    # context ---------------------------------------------------------------------------
    def context(self, features, positions):
        """Per layer (K [Hkv, C, D], V [Hkv, C, D]) of the context rows (features [C, F])."""
        c = self.c
        th = self.norm(self.linear(features, "fc.weight"), "hidden_norm.weight")
        out = []
        for i in range(c.num_hidden_layers):
            p = f"layers.{i}.self_attn"
            k = self.norm(self.linear(th, p + ".k_proj.weight").reshape(-1, c.num_key_value_heads, c.head_dim),
                          p + ".k_norm.weight").transpose(1, 0, 2)
            v = self.linear(th, p + ".v_proj.weight").reshape(-1, c.num_key_value_heads, c.head_dim).transpose(1, 0, 2)
            out.append((self.rope(k, positions), v))
        return out

    # block ---------------------------------------------------------------------------
    def block(self, block_ids, start, ctx_kv, embed):
        """Final-normed hidden states [S, H] of the block at positions start .. start+S-1
        over the context keys/values of positions [0, start)."""
        c = self.c
        S = len(block_ids)
        pos = np.arange(start, start + S)
        h = np.asarray(embed, np.float32)[np.asarray(block_ids)]
        hq, hkv, d = c.num_attention_heads, c.num_key_value_heads, c.head_dim
        for i in range(c.num_hidden_layers):
            p = f"layers.{i}"
            x = self.norm(h, p + ".input_layernorm.weight")
            q = self.norm(self.linear(x, p + ".self_attn.q_proj.weight").reshape(S, hq, d),
                          p + ".self_attn.q_norm.weight").transpose(1, 0, 2)
            k = self.norm(self.linear(x, p + ".self_attn.k_proj.weight").reshape(S, hkv, d),
                          p + ".self_attn.k_norm.weight").transpose(1, 0, 2)
            v = self.linear(x, p + ".self_attn.v_proj.weight").reshape(S, hkv, d).transpose(1, 0, 2)
            q, k = self.rope(q, pos), self.rope(k, pos)
            kc, vc = ctx_kv[i]
            K = np.concatenate([kc, k], 1)
            V = np.concatenate([vc, v], 1)
            kpos = np.arange(K.shape[1])
            visible = np.ones((S, K.shape[1]), bool)
            if c.causal(i):
                visible &= kpos[None, :] <= pos[:, None]
            w = c.window(i)
            if w:
                visible &= (pos[:, None] - kpos[None, :]) < w
            rep = hq // hkv
            Kr, Vr = np.repeat(K, rep, 0), np.repeat(V, rep, 0)
            s = np.einsum("hsd,htd->hst", q, Kr) * np.float32(d ** -0.5)
            s = np.where(visible[None], s, -np.inf)
            s = s - s.max(-1, keepdims=True)
            pr = np.exp(s)
            pr = pr / pr.sum(-1, keepdims=True)
            attn = self.r(np.einsum("hst,htd->hsd", pr, Vr)).transpose(1, 0, 2).reshape(S, hq * d)
            h = self.r(h + self.linear(attn, p + ".self_attn.o_proj.weight"))
            x = self.norm(h, p + ".post_attention_layernorm.weight")
            g = self.linear(x, p + ".mlp.gate_proj.weight")
            u = self.linear(x, p + ".mlp.up_proj.weight")
            a = self.r(self.r(g / (1.0 + np.exp(-g))) * u)
            h = self.r(h + self.linear(a, p + ".mlp.down_proj.weight"))
        return self.norm(h, "norm.weight")

    def draft(self, features, next_token, embed, lm_head, *, return_logits=False):
        """Proposals [S-1] after a context of len(features) committed rows (positions
        0 .. C-1), the anchor next_token at position C (graphs.py:74-97)."""
        c = self.c
        C = len(features)
        ctx = self.context(features, np.arange(C))
        ids = [int(next_token)] + [c.mask_token_id] * (c.block_size - 1)
        hidden = self.block(ids, C, ctx, embed)
        logits = self.r(hidden[1:] @ np.asarray(lm_head, np.float32).T)
        top = stable_argmax(logits)
        return (top, logits) if return_logits else top
