"""numpy restatement of the target verify forward and of verify/commit semantics.

Test infrastructure only (see ``oracle/__init__.py``).

``OracleTarget.forward`` follows ``FusedTargetModel._forward_hidden``
(model/qwen35_moe_dflash/fused/model.py:386-427) with the layer bodies ``_gdn``
(:227-263), ``_attention`` (:278-294), ``_moe`` (:296-307), ``_norm`` (:206-217),
``_gated_norm`` (:219-225) and ``_rotary`` (:265-276).  Every activation tensor is
rounded to the activation dtype ``act`` ("f16" reproduces the reference's FP16
model, "bf16" the same semantics with bf16 activations) at the points where the
reference's torch ops return a tensor of that dtype.  The gated-delta-rule gates g
and beta are kept in fp32 when ``act == "bf16"`` (the reference's GDN operator does
not accept bf16 inputs, fused_ops.py:87-90; this build feeds it fp32 gates).
``rope`` selects the rotary arithmetic: "f16" is the reference's unquantized path
(FP16 positions and inverse frequencies, :135-136, :267), "f32" its quantized path.

``verify`` / ``commit`` restate ``FusedTargetSession.verify`` and
``TargetVerification.commit`` (model/qwen35_moe_dflash/fused/session.py:316-387)
for a block forward: proposal i is accepted while it equals the prediction made
before consuming it (row i-1, or the pre-block prediction for i = 0).
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

from . import fused_ops_np as F
from .numerics import round_to, stable_argmax


@dataclass
class LayerState:
    conv: np.ndarray | None = None       # [B, C, K-1]
    recurrent: np.ndarray | None = None  # [B, H, Dk, Dv] fp32
    key: np.ndarray | None = None        # [B, Hkv, T, D]
    value: np.ndarray | None = None

    def copy(self):
        return LayerState(*(None if a is None else a.copy()
                            for a in (self.conv, self.recurrent, self.key, self.value)))


@dataclass
class State:
    position: int
    layers: list = field(default_factory=list)

    def copy(self):
        return State(self.position, [layer.copy() for layer in self.layers])


class OracleTarget:
    def __init__(self, cfg: dict, weights: dict, feature_layers, *, act: str = "bf16",
                 rope: str = "f32"):
        self.c = dict(cfg)
        self.w = {k: np.asarray(v, np.float32) for k, v in weights.items()}
        self.feature_layers = tuple(feature_layers)
        self.act = act
        self.rope = rope
        rot = int(self.c["head_dim"] * self.c["rope_parameters"]["partial_rotary_factor"])
        theta = float(self.c["rope_parameters"]["rope_theta"])
        inv = 1.0 / (theta ** (np.arange(0, rot, 2, dtype=np.float32) / rot))
        self.inv_freq = inv.astype(np.float32)
        self.rotary_dim = rot
        # when a list: each MoE call appends, per token, the gap between the k-th and
        # (k+1)-th largest router logits in bf16 ulps of the k-th (a routing near-tie
        # is a gap of a few ulps; two implementations that sum the router GEMV in
        # different orders may select differently there)
        self.router_gaps = None

    # helpers -------------------------------------------------------------------------
    def r(self, x):
        return round_to(x, self.act)

    def linear(self, x, name):
        return self.r(np.asarray(x, np.float32) @ self.w[name].T)

    def norm(self, x, name, zero_centered=True):
        gamma = self.w[name] + (1.0 if zero_centered else 0.0)
        gamma = self.r(gamma)
        return F.rms_norm(x, gamma, self.c["rms_norm_eps"], self.act)

    def initial_state(self, batch: int = 1) -> State:
        c, layers = self.c, []
        kw = c["linear_num_key_heads"] * c["linear_key_head_dim"]
        vw = c["linear_num_value_heads"] * c["linear_value_head_dim"]
        for kind in c["layer_types"]:
            if kind == "linear_attention":
                layers.append(LayerState(
                    conv=np.zeros((batch, 2 * kw + vw, c["linear_conv_kernel_dim"] - 1), np.float32),
                    recurrent=np.zeros((batch, c["linear_num_value_heads"], c["linear_key_head_dim"],
                                        c["linear_value_head_dim"]), np.float32)))
            else:
                shape = (batch, c["num_key_value_heads"], 0, c["head_dim"])
                layers.append(LayerState(key=np.zeros(shape, np.float32), value=np.zeros(shape, np.float32)))
        return State(0, layers)

    # layer bodies --------------------------------------------------------------------
    def gdn(self, x, p, cache: LayerState):
        c = self.c
        b, s = x.shape[:2]
        kh, vh = c["linear_num_key_heads"], c["linear_num_value_heads"]
        kd, vd = c["linear_key_head_dim"], c["linear_value_head_dim"]
        kw, vw = kh * kd, vh * vd
        projected = self.linear(x, p + ".in_proj_qkv.weight")
        conv, padded = F.conv_state_update(projected, cache.conv)
        mixed = F.causal_conv1d(padded, self.w[p + ".conv1d.weight"], self.act)
        mixed = self.r(F.silu(mixed))
        q, k, v = mixed[..., :kw], mixed[..., kw:2 * kw], mixed[..., 2 * kw:]
        q = np.repeat(q.reshape(b, s, kh, kd), vh // kh, axis=2)
        k = np.repeat(k.reshape(b, s, kh, kd), vh // kh, axis=2)
        v = v.reshape(b, s, vh, vd)
        if self.act == "bf16":
            beta = F.sigmoid(x @ self.w[p + ".in_proj_b.weight"].T)
            a = x @ self.w[p + ".in_proj_a.weight"].T
            g = -np.exp(self.w[p + ".A_log"]) * F.softplus(a + self.w[p + ".dt_bias"])
        else:
            beta = self.r(F.sigmoid(self.linear(x, p + ".in_proj_b.weight")))
            a = self.r(self.linear(x, p + ".in_proj_a.weight") + self.w[p + ".dt_bias"])
            g = self.r(-self.r(np.exp(self.w[p + ".A_log"])) * self.r(F.softplus(a)))
        valid = np.full((b,), s, np.int16)
        core, recurrent = F.chunk_gated_delta_rule(
            q, k, v, g, beta, cache.recurrent, valid, chunk_size=1 if s == 1 else 64,
            use_qk_l2norm_in_kernel=True, dtype=self.act, state_dtype="f32")
        z = self.linear(x, p + ".in_proj_z.weight").reshape(b, s, vh, vd)
        core = self.r(self.norm(core, p + ".norm.weight", zero_centered=False) * self.r(F.silu(z)))
        out = self.linear(core.reshape(b, s, vw), p + ".out_proj.weight")
        return out, LayerState(conv=conv, recurrent=recurrent)

    def rotary(self, x, start):
        width = self.rotary_dim
        if self.rope == "f16":
            positions = np.arange(start, start + x.shape[-2]).astype(np.float16)
            inv = self.inv_freq.astype(np.float16)
            freq = (positions[:, None] * inv[None, :]).astype(np.float16).astype(np.float32)
            angle = np.concatenate((freq, freq), -1)
            cos = round_to(np.cos(angle), "f16")
            sin = round_to(np.sin(angle), "f16")
        else:
            positions = np.arange(start, start + x.shape[-2]).astype(np.float32)
            freq = positions[:, None] * self.inv_freq[None, :]
            angle = np.concatenate((freq, freq), -1)
            cos, sin = np.cos(angle).astype(np.float32), np.sin(angle).astype(np.float32)
            if self.act != "f32":
                cos, sin = self.r(cos), self.r(sin)
        a, tail = x[..., :width], x[..., width:]
        half = width // 2
        first, second = a[..., :half], a[..., half:]
        rotated = np.concatenate((-second, first), -1)
        a = self.r(self.r(a * cos) + self.r(rotated * sin))
        return np.concatenate((a, tail), -1)

    def attention(self, x, p, cache: LayerState, start):
        c = self.c
        b, s = x.shape[:2]
        heads, kv, d = c["num_attention_heads"], c["num_key_value_heads"], c["head_dim"]
        qg = self.linear(x, p + ".q_proj.weight").reshape(b, s, heads, 2 * d)
        q, gate = qg[..., :d], qg[..., d:]
        q = self.norm(q, p + ".q_norm.weight").transpose(0, 2, 1, 3)
        k = self.norm(self.linear(x, p + ".k_proj.weight").reshape(b, s, kv, d),
                      p + ".k_norm.weight").transpose(0, 2, 1, 3)
        v = self.linear(x, p + ".v_proj.weight").reshape(b, s, kv, d).transpose(0, 2, 1, 3)
        q, k = self.rotary(q, start), self.rotary(k, start)
        key, value = F.cache_update(cache.key, cache.value, k, v)
        mixed = F.attention(q, key, value, query_start=start, scale=d ** -0.5, dtype=self.act)
        mixed = mixed.transpose(0, 2, 1, 3).reshape(b, s, heads * d)
        mixed = self.r(mixed * self.r(F.sigmoid(gate.reshape(b, s, heads * d))))
        return self.linear(mixed, p + ".o_proj.weight"), LayerState(key=key, value=value)

    def moe(self, x, p):
        c = self.c
        if self.router_gaps is not None:
            flat = np.asarray(x, np.float32).reshape(-1, x.shape[-1])
            lg = self.r(flat @ self.w[p + ".gate.weight"].T)
            srt = -np.sort(-lg, -1)
            k = c["num_experts_per_tok"]
            top, nxt = srt[:, k - 1], srt[:, min(k, srt.shape[-1] - 1)]
            ulp = 2.0 ** (np.floor(np.log2(np.maximum(np.abs(top), 1e-30))) - 7)
            self.router_gaps.append((top - nxt) / ulp)
        routed = F.moe(x, self.w[p + ".gate.weight"], self.w[p + ".experts.gate_up_proj"],
                       self.w[p + ".experts.down_proj"], top_k=c["num_experts_per_tok"],
                       dtype=self.act, emulate_rounding=True)
        shared = self.r(self.r(F.silu(self.linear(x, p + ".shared_expert.gate_proj.weight")))
                        * self.linear(x, p + ".shared_expert.up_proj.weight"))
        shared = self.linear(shared, p + ".shared_expert.down_proj.weight")
        gate = self.r(F.sigmoid(self.linear(x, p + ".shared_expert_gate.weight")))
        return self.r(routed + self.r(shared * gate))

    def layer(self, index: int, hidden, cache: LayerState, position: int):
        """One decoder layer (fused/model.py:396-404): mixer + residual, MoE + residual."""
        p = f"target.layers.{index}"
        normed = self.norm(hidden, p + ".input_layernorm.weight")
        if self.c["layer_types"][index] == "linear_attention":
            mixed, new = self.gdn(normed, p + ".linear_attn", cache)
        else:
            mixed, new = self.attention(normed, p + ".self_attn", cache, position)
        hidden = self.r(hidden + mixed)
        hidden = self.r(hidden + self.moe(self.norm(hidden, p + ".post_attention_layernorm.weight"),
                                          p + ".mlp"))
        return hidden, new

    # forward -------------------------------------------------------------------------
    def forward(self, ids, state: State | None = None, *, return_logits: bool = False):
        """ids int [B,S] -> (top1 int32 [B,S], features [B,S,F], new state, logits|None)."""
        ids = np.asarray(ids)
        b, s = ids.shape
        state = self.initial_state(b) if state is None else state
        hidden = self.w["target.embed_tokens.weight"][ids]
        layers, features = [], {}
        for index in range(len(self.c["layer_types"])):
            hidden, new = self.layer(index, hidden, state.layers[index], state.position)
            layers.append(new)
            if index in self.feature_layers:
                features[index] = hidden
        hidden = self.norm(hidden, "target.norm.weight")
        last = self.c["num_hidden_layers"] - 1
        if last in features:
            features[last] = hidden
        logits = hidden @ self.w["target.lm_head.weight"].T
        logits = self.r(logits)
        top1 = stable_argmax(logits)
        captured = np.concatenate([features[i] for i in self.feature_layers], -1)
        return top1, captured, State(state.position + s, layers), (logits if return_logits else None)


def verify(model: OracleTarget, state: State, next_token: int, proposals):
    """Block verify of ``proposals`` [S] from ``state`` for one sequence.

    Returns (expected_next_tokens tuple[S+1], max_accepted_prefix, top1 [S], features [S,F]).
    """
    proposals = [int(t) for t in proposals]
    top1, features, _, _ = model.forward(np.asarray([proposals]), state.copy())
    expected = (int(next_token),) + tuple(int(t) for t in top1[0])
    accepted = 0
    for i, token in enumerate(proposals):
        if token != expected[i]:
            break
        accepted += 1
    return expected, accepted, top1[0], features[0]


def commit(model: OracleTarget, state: State, proposals, accepted: int) -> State:
    """State after the first ``accepted`` proposals (fused/session.py:166-175, :374-387)."""
    if accepted == 0:
        return state.copy()
    _, _, new_state, _ = model.forward(np.asarray([list(proposals)[:accepted]]), state.copy())
    return new_state
