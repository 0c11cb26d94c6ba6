"""Device-resident block-verify engine for the Qwen3.5-MoE target.

One ``TargetEngine`` owns, on one GPU:
  * the weights, packed for the streaming kernels (W4A16 streams for the quantized
    projections and experts, B16 streams for the router / GDN gate predictors /
    lm_head, plain bf16 for norms, conv taps and the embedding);
  * the recurrent-state banks (GDN conv tails and fp32 recurrent states, one row per
    sequence slot) and the paged bf16 KV cache of the attention layers;
  * the activation buffers of one verify block of ``batch`` sequences x ``block``
    tokens, and the per-layer GDN projections kept until commit.

``forward()`` runs the 40-layer composition of FusedTargetModel._forward_hidden
(model/qwen35_moe_dflash/fused/model.py:386-427) for every token of the block in one
launch sequence per layer (no per-token loop), ``accept()`` evaluates the block against
the pre-block prediction (fused/session.py:316-341) and ``commit()`` advances every
sequence's state by its accepted count (session.py:374-387): GDN states and conv tails
are recomputed for the accepted prefix in place, KV entries past the new position are
simply overwritten by the next block.  ``capture()`` records forward + accept + commit
as one CUDA graph.
"""
from __future__ import annotations

import ctypes
import math
import zlib
from dataclasses import dataclass

import numpy as np
import torch

from . import lib, w4
from .config import TargetConfig
from .synthetic import weight_shapes, init_value, is_w4

BF16 = torch.bfloat16


def _bf16(x) -> torch.Tensor:
    return x.to(BF16).contiguous() if isinstance(x, torch.Tensor) else torch.from_numpy(np.asarray(x, np.float32)).to(BF16)


def _pad16(rows: torch.Tensor) -> torch.Tensor:
    return w4.pad_rows(rows, 16)


@dataclass
class LayerWeights:
    kind: str
    in_norm: torch.Tensor
    post_norm: torch.Tensor
    # GDN
    qkvz: torch.Tensor | None = None
    ab: torch.Tensor | None = None
    conv_w: torch.Tensor | None = None
    a_log: torch.Tensor | None = None
    dt_bias: torch.Tensor | None = None
    gnorm: torch.Tensor | None = None
    out: torch.Tensor | None = None
    # attention
    qkv: torch.Tensor | None = None
    q_norm: torch.Tensor | None = None
    k_norm: torch.Tensor | None = None
    o: torch.Tensor | None = None
    # MoE
    router: torch.Tensor | None = None
    gate_up: torch.Tensor | None = None
    down: torch.Tensor | None = None
    shared_gu: torch.Tensor | None = None
    shared_down: torch.Tensor | None = None


def pack_weights(cfg: TargetConfig, get, device, quantized=None) -> tuple[dict, list[LayerWeights]]:
    """Pack all target weights.  ``get(name) -> float tensor on `device``` (bf16-exact
    values outside the W4 scope).  ``quantized(name) -> (int8 q, bf16 scales)``, when
    given, supplies the W4 projections already quantised (the original checkpoint's
    values); otherwise ``get``'s values are quantised here."""
    g = cfg.quant_group

    def q4(*names):
        if quantized is not None:
            parts = [quantized(n) for n in names]
            return w4.pack_w4(torch.cat([p[0] for p in parts], -2), torch.cat([p[1] for p in parts], -2), g)
        mats = [get(n).float() for n in names]
        mat = torch.cat(mats, -2) if len(mats) > 1 else mats[0]
        q, s = w4.quantize(mat, g)
        return w4.pack_w4(q, s, g)

    def experts(name):
        if quantized is not None:
            q, s = quantized(name)
            return torch.cat([w4.pack_w4(q[e0:e0 + 64], s[e0:e0 + 64], g) for e0 in range(0, q.shape[0], 64)])
        t = get(name)
        out = []
        for e0 in range(0, t.shape[0], 64):
            q, s = w4.quantize(t[e0:e0 + 64].float(), g)
            out.append(w4.pack_w4(q, s, g))
        return torch.cat(out)

    glob = {"embed": _bf16(get("target.embed_tokens.weight")),
            "final_norm": _bf16(get("target.norm.weight")),
            "lm_head": w4.pack_b16(_bf16(get("target.lm_head.weight")))}
    layers = []
    for i, kind in enumerate(cfg.layer_types):
        p = f"target.layers.{i}"
        lw = LayerWeights(kind, _bf16(get(p + ".input_layernorm.weight")),
                          _bf16(get(p + ".post_attention_layernorm.weight")))
        if kind == "linear_attention":
            a = p + ".linear_attn"
            lw.qkvz = q4(a + ".in_proj_qkv.weight", a + ".in_proj_z.weight")
            lw.ab = w4.pack_b16(_pad16(torch.cat([_bf16(get(a + ".in_proj_b.weight")),
                                                  _bf16(get(a + ".in_proj_a.weight"))])))
            lw.conv_w = _bf16(get(a + ".conv1d.weight").reshape(cfg.conv_channels, -1))
            lw.a_log = get(a + ".A_log").float().contiguous()
            lw.dt_bias = get(a + ".dt_bias").float().contiguous()
            lw.gnorm = _bf16(get(a + ".norm.weight"))
            lw.out = q4(a + ".out_proj.weight")
        else:
            a = p + ".self_attn"
            lw.qkv = q4(a + ".q_proj.weight", a + ".k_proj.weight", a + ".v_proj.weight")
            lw.q_norm = _bf16(get(a + ".q_norm.weight"))
            lw.k_norm = _bf16(get(a + ".k_norm.weight"))
            lw.o = q4(a + ".o_proj.weight")
        m = p + ".mlp"
        lw.router = w4.pack_b16(_pad16(torch.cat([_bf16(get(m + ".gate.weight")),
                                                  _bf16(get(m + ".shared_expert_gate.weight"))])))
        lw.gate_up = experts(m + ".experts.gate_up_proj")
        lw.down = experts(m + ".experts.down_proj")
        lw.shared_gu = q4(m + ".shared_expert.gate_proj.weight", m + ".shared_expert.up_proj.weight")
        lw.shared_down = q4(m + ".shared_expert.down_proj.weight")
        layers.append(lw)
    return glob, layers


def weights_from_arrays(cfg: TargetConfig, arrays: dict, device="cuda"):
    """Pack float weights given as numpy arrays / tensors (e.g. synthetic.init_weights)."""
    def get(name):
        v = arrays[name]
        t = v if isinstance(v, torch.Tensor) else torch.from_numpy(np.ascontiguousarray(v, np.float32))
        return t.to(device)
    return pack_weights(cfg, get, device)


def weights_random(cfg: TargetConfig, seed: int = 2, std: float = 0.02, device="cuda"):
    """Random-init weights generated on the device, N(0, std) for every matrix (the
    benchmark's configuration), deterministic per (seed, tensor name)."""
    shapes = weight_shapes(cfg)
    gen = torch.Generator(device=device)

    def get(name):
        shape = shapes[name]
        if math.prod(shape) < (1 << 20) or name.endswith(("A_log", "dt_bias", "norm.weight", "layernorm.weight")):
            return torch.from_numpy(init_value(name, shape, seed, std)).to(device)
        gen.manual_seed((seed * 1_000_003 + zlib.crc32(name.encode())) & 0x7FFFFFFFFFFF)
        t = torch.empty(shape, device=device, dtype=torch.float32).normal_(0.0, std, generator=gen)
        return t if is_w4(name) else t.to(BF16).float()
    return pack_weights(cfg, get, device)


class TargetEngine:
    def __init__(self, cfg: TargetConfig, weights, *, batch: int, block: int = 16, capacity: int = 4096,
                 page_size: int = 16, device="cuda", ep_group=None, share: "TargetEngine | None" = None):
        """``share``: another engine of the same configuration, batch, capacity and page
        size whose state (GDN and conv banks, paged KV cache, positions, next tokens) this
        one works on -- a prefill engine with longer blocks beside a verify engine."""
        if not 1 <= block <= lib.QW_MAX_SEQ:
            raise ValueError(f"block must be in [1, {lib.QW_MAX_SEQ}]")
        if share is not None and (share.cfg != cfg or share.B != batch or share.capacity != capacity
                                  or share.P != page_size or ep_group is not None):
            raise ValueError("a sharing engine needs the same configuration, batch, capacity and pages "
                             "(and no expert parallelism)")
        self.cfg, self.B, self.S, self.device = cfg, batch, block, torch.device(device)
        self.T = batch * block
        self.capacity = capacity
        self.P = page_size
        self.glob, self.layers = weights
        c, dev, T = cfg, self.device, self.T
        self.lib = lib.load()
        H = c.hidden_size
        self.gdn_idx = {l: i for i, l in enumerate(c.gdn_layers)}
        self.attn_idx = {l: i for i, l in enumerate(c.attn_layers)}
        ng, na = len(c.gdn_layers), len(c.attn_layers)
        # activations
        self.tokens = torch.zeros(T, dtype=torch.int32, device=dev)
        self.hidden = torch.zeros(T, H, dtype=BF16, device=dev)
        self.normed = torch.zeros(T, H, dtype=BF16, device=dev)
        self.ldp = c.conv_channels + c.value_width
        self.proj = torch.zeros(max(ng, 1), T, self.ldp, dtype=BF16, device=dev)
        self.nab = 2 * c.linear_num_value_heads
        if self.nab % 16:
            raise ValueError("the GDN gate predictors need a multiple of 8 value heads")
        self.nab_pad = self.nab
        self.ab = torch.zeros(max(ng, 1), T, self.nab_pad, dtype=torch.float32, device=dev)
        self.gdn_out = torch.zeros(T, c.value_width, dtype=BF16, device=dev)
        self.ldq = c.num_attention_heads * 2 * c.head_dim + 2 * c.num_key_value_heads * c.head_dim
        self.qkv = torch.zeros(T, self.ldq, dtype=BF16, device=dev)
        self.qout = torch.zeros(batch, c.num_attention_heads, block, c.head_dim, dtype=BF16, device=dev)
        self.attn_out = torch.zeros(T, c.num_attention_heads * c.head_dim, dtype=BF16, device=dev)
        self.attn_ws = torch.zeros(max(16, self.lib.qw_attn_workspace_bytes(
            batch, c.num_attention_heads, c.num_key_value_heads, block, c.head_dim, capacity)),
            dtype=torch.uint8, device=dev)
        self.nrouter = (c.num_experts + 1 + 15) // 16 * 16
        self.router_logits = torch.zeros(T, self.nrouter, dtype=BF16, device=dev)
        # optional per-expert router-logit bias (synthetic routing skew of a serving
        # benchmark); None in the model
        self.router_bias = None
        self.moe_ws = torch.zeros(self.lib.qw_moe_workspace_bytes(
            T, H, c.num_experts, c.moe_intermediate_size, c.num_experts_per_tok), dtype=torch.uint8, device=dev)
        self.features = torch.zeros(T, c.feature_width, dtype=BF16, device=dev)
        self.vocab_pad = (c.vocab_size + 15) // 16 * 16
        # expert parallelism: this rank keeps only its slice of every routed expert bank
        # (the shared weights object is not modified) and exchanges rows with the group
        self.ep_moe = None
        if ep_group is not None:
            from . import ep as _ep
            import torch.distributed as dist
            G, rank = dist.get_world_size(ep_group), dist.get_rank(ep_group)
            E = c.num_experts
            self.ep_moe = _ep.ExpertParallelMoE(ep_group, tokens=T, hidden=H, experts=E,
                                                inter=c.moe_intermediate_size, top_k=c.num_experts_per_tok,
                                                quant_group=c.quant_group, device=dev)
            banks = [self.ep_moe.local_banks(lw.gate_up, lw.down, lw.shared_gu, lw.shared_down) for lw in self.layers]
            self.ep_gu = [b[0] for b in banks]
            self.ep_dn = [b[1] for b in banks]
        self.nblk = self.lib.qw_lmhead_blocks(self.vocab_pad)
        self.keys = torch.zeros(self.nblk, T, dtype=torch.int64, device=dev)
        self.top1 = torch.zeros(T, dtype=torch.int32, device=dev)
        self.max_accepted = torch.zeros(batch, dtype=torch.int32, device=dev)
        self.accepted = torch.zeros(batch, dtype=torch.int32, device=dev)
        self.next_token = torch.zeros(batch, dtype=torch.int32, device=dev) if share is None else share.next_token
        self.qpos = torch.zeros(batch, dtype=torch.int32, device=dev) if share is None else share.qpos
        # QW_OK / QW_ERR_TIMEOUT of the bounded device waits of the last forward
        self.wait_status = torch.zeros(1, dtype=torch.int32, device=dev)
        self._wait_status_host = torch.zeros(1, dtype=torch.int32).pin_memory()
        self.slots = torch.arange(batch, dtype=torch.int32, device=dev)
        # state banks (a sharing engine works on the other engine's)
        self.max_pages = (capacity + page_size - 1) // page_size
        if share is not None:
            self.conv_hist, self.state = share.conv_hist, share.state
            self.pages, self.k_cache, self.v_cache = share.pages, share.k_cache, share.v_cache
        else:
            self.conv_hist = torch.zeros(max(ng, 1), batch, c.conv_channels, c.linear_conv_kernel_dim - 1,
                                         dtype=BF16, device=dev)
            self.state = torch.zeros(max(ng, 1), batch, c.linear_num_value_heads, c.linear_value_head_dim,
                                     c.linear_key_head_dim, dtype=torch.float32, device=dev)
            self.pages = torch.arange(batch * self.max_pages, dtype=torch.int32, device=dev).view(batch,
                                                                                                 self.max_pages)
            kv_shape = (max(na, 1), batch * self.max_pages, c.num_key_value_heads, page_size, c.head_dim)
            self.k_cache = torch.zeros(kv_shape, dtype=BF16, device=dev)
            self.v_cache = torch.zeros(kv_shape, dtype=BF16, device=dev)
        # GDN layer descriptors (device array) and dims
        descs = (lib.GdnLayer * max(ng, 1))()
        for l, gi in self.gdn_idx.items():
            lw = self.layers[l]
            descs[gi] = lib.GdnLayer(self.proj[gi].data_ptr(), self.ab[gi].data_ptr(), self.conv_hist[gi].data_ptr(),
                                     lw.conv_w.data_ptr(), lw.a_log.data_ptr(), lw.dt_bias.data_ptr(),
                                     lw.gnorm.data_ptr(), self.state[gi].data_ptr(), self.gdn_out.data_ptr())
        raw = bytes(memoryview(descs).cast("B"))
        self.gdn_desc = torch.frombuffer(bytearray(raw), dtype=torch.uint8).to(dev)
        self.gdn_dims = lib.GdnDims(batch, block, c.linear_num_key_heads, c.linear_num_value_heads,
                                    c.linear_key_head_dim, c.linear_value_head_dim, c.conv_channels,
                                    c.linear_conv_kernel_dim, self.ldp, c.rms_norm_eps,
                                    self.slots.data_ptr(), self.accepted.data_ptr())
        self.graph = None
        self._recording = None
        self.captured_calls = {}

    # ------------------------------------------------------------------ helpers
    def _st(self):
        return torch.cuda.current_stream(self.device).cuda_stream

    def _call(self, name, *args):
        if self._recording is not None:
            self._recording[name] = self._recording.get(name, 0) + 1
        lib.check(getattr(self.lib, name)(*args), name)

    # kernels each entry point launches (all others launch one)
    # (expert-parallel MoE layer: dispatch, receive routing, gate/up + down-and-send of the
    # received rows, and the combine + norm that reads the returned rows)
    KERNELS_PER_CALL = {"qw_attn_paged": 2, "qw_moe_experts_w4": 2, "qw_gdn_commit": 2, "qw_moe_ep": 5}

    def launches_per_step(self) -> int:
        """Kernels of this library in the captured step (counted from the entry calls)."""
        if not self.captured_calls:
            raise RuntimeError("capture() first")
        return sum(n * self.KERNELS_PER_CALL.get(name, 1) for name, n in self.captured_calls.items())

    def _tap(self, layer: int):
        c = self.cfg
        if layer in c.feature_layers:
            col = c.feature_layers.index(layer) * c.hidden_size
            return self.features.data_ptr() + col * 2
        return None

    # ------------------------------------------------------------------ the block
    def forward(self, after_moe_route=None):
        """All layers + final norm + lm_head argmax keys for the tokens in ``self.tokens``.

        ``after_moe_route(layer)`` (eager use only) is called after each layer's experts
        (the routing lists, e.g. ``active_experts()``, are valid then)."""
        c, T, H, st = self.cfg, self.T, self.cfg.hidden_size, self._st()
        eps = c.rms_norm_eps
        L = c.num_hidden_layers
        for l, lw in enumerate(self.layers):
            if l == 0:
                # embedding + input RMSNorm; later layers' input norms are fused into the
                # previous layer's MoE combine
                self._call("qw_residual_norm", self.hidden.data_ptr(), self.tokens.data_ptr(),
                           self.glob["embed"].data_ptr(), lw.in_norm.data_ptr(), self.normed.data_ptr(),
                           None, c.feature_width, 0, T, H, eps, st)
            if lw.kind == "linear_attention":
                gi = self.gdn_idx[l]
                self._call("qw_w4_linear", self.normed.data_ptr(), lw.qkvz.data_ptr(), self.proj[gi].data_ptr(),
                           lib.QW_OUT_BF16, self.ldp, T, self.ldp, H, c.quant_group, st)
                self._call("qw_b16_linear", self.normed.data_ptr(), lw.ab.data_ptr(), self.ab[gi].data_ptr(),
                           lib.QW_OUT_F32, self.nab_pad, T, self.nab_pad, H, st)
                self._call("qw_gdn_verify", ctypes.byref(self.gdn_dims), self.gdn_desc.data_ptr(), gi, st)
                self._call("qw_w4_linear", self.gdn_out.data_ptr(), lw.out.data_ptr(), self.hidden.data_ptr(),
                           lib.QW_OUT_RESID_BF16, H, T, H, c.value_width, c.quant_group, st)
            else:
                ai = self.attn_idx[l]
                D, Hq, Hkv = c.head_dim, c.num_attention_heads, c.num_key_value_heads
                self._call("qw_w4_linear", self.normed.data_ptr(), lw.qkv.data_ptr(), self.qkv.data_ptr(),
                           lib.QW_OUT_BF16, self.ldq, T, self.ldq, H, c.quant_group, st)
                self._call("qw_attn_prep", self.qkv.data_ptr(), self.ldq, lw.q_norm.data_ptr(),
                           lw.k_norm.data_ptr(), eps, c.rope_theta, c.rotary_dim, self.qpos.data_ptr(),
                           self.pages.data_ptr(), self.max_pages, self.P, self.k_cache[ai].data_ptr(),
                           self.v_cache[ai].data_ptr(), self.qout.data_ptr(), self.B, self.S, Hq, Hkv, D, st)
                self._call("qw_attn_paged", self.qout.data_ptr(), self.k_cache[ai].data_ptr(),
                           self.v_cache[ai].data_ptr(), self.pages.data_ptr(), self.max_pages, self.P,
                           self.qpos.data_ptr(), self.capacity, self.qkv.data_ptr() + D * 2, self.ldq,
                           self.attn_out.data_ptr(), self.B, self.S, Hq, Hkv, D, D ** -0.5,
                           self.attn_ws.data_ptr(), st)
                self._call("qw_w4_linear", self.attn_out.data_ptr(), lw.o.data_ptr(), self.hidden.data_ptr(),
                           lib.QW_OUT_RESID_BF16, H, T, H, Hq * D, c.quant_group, st)
            # MoE
            self._call("qw_residual_norm", self.hidden.data_ptr(), None, None, lw.post_norm.data_ptr(),
                       self.normed.data_ptr(), None, 0, 0, T, H, eps, st)
            self._call("qw_b16_linear", self.normed.data_ptr(), lw.router.data_ptr(),
                       self.router_logits.data_ptr(), lib.QW_OUT_BF16, self.nrouter, T, self.nrouter, H, st)
            E, k, I = c.num_experts, c.num_experts_per_tok, c.moe_intermediate_size
            if self.router_bias is not None:
                self.router_logits[:, :E].add_(self.router_bias)
            self._call("qw_moe_route_x", self.router_logits.data_ptr(), lib.QW_BF16, self.nrouter, T, E, k, E,
                       lib.QW_BF16, self.normed.data_ptr(), H, c.quant_group, self.moe_ws.data_ptr(), st, 0)
            if self.ep_moe is not None:
                if self._recording is not None:
                    self._recording["qw_moe_ep"] = self._recording.get("qw_moe_ep", 0) + 1
                self.ep_moe.experts(self.normed, self.moe_ws, self.ep_gu[l], self.ep_dn[l], scatter=False)
            else:
                self._call("qw_moe_experts_w4", self.normed.data_ptr(), lw.gate_up.data_ptr(), lw.down.data_ptr(),
                           lw.shared_gu.data_ptr(), lw.shared_down.data_ptr(), T, H, E, I, k, c.quant_group,
                           self.moe_ws.data_ptr(), st)
            if after_moe_route is not None:
                after_moe_route(l)
            # residual add of the MoE output + the next RMSNorm (next layer's input norm, or
            # the final norm) + the feature tap of this layer (normed after the last layer)
            last = l == L - 1
            gamma = self.glob["final_norm"] if last else self.layers[l + 1].in_norm
            if self.ep_moe is not None:
                self.ep_moe.combine_norm(self.moe_ws, self.hidden, gamma, self.normed, eps, self._tap(l),
                                         c.feature_width, int(last))
            else:
                self._call("qw_moe_combine_norm", self.moe_ws.data_ptr(), self.hidden.data_ptr(), T, H, E, I, k, 1,
                           gamma.data_ptr(), self.normed.data_ptr(), eps, self._tap(l), c.feature_width, int(last), st)
        self._call("qw_lmhead_argmax", self.normed.data_ptr(), self.glob["lm_head"].data_ptr(), None,
                   self.keys.data_ptr(), T, self.vocab_pad, H, st)
        # did a bounded wait of this block's kernels expire? (read back with the results)
        self._call("qw_wait_status", self.wait_status.data_ptr(), 1, st)

    def raise_on_wait_timeout(self, status: int | None = None):
        """TimeoutError if a bounded device wait of the last forward expired (its outputs
        are incomplete); ``status`` is an already-copied value of ``wait_status``."""
        value = int(self.wait_status.item()) if status is None else int(status)
        if value != lib.QW_OK:
            raise TimeoutError("a bounded device wait expired during the verify forward: "
                               "the block's outputs are incomplete")

    def accept(self, auto_commit: bool):
        self._call("qw_accept", self.keys.data_ptr(), self.nblk, self.tokens.data_ptr(), self.top1.data_ptr(),
                   self.max_accepted.data_ptr(), self.next_token.data_ptr(), self.accepted.data_ptr(),
                   self.qpos.data_ptr(), self.B, self.S, int(auto_commit), self._st())

    def commit_states(self):
        """Advance GDN states / conv tails by ``self.accepted`` (device) tokens."""
        ng = len(self.cfg.gdn_layers)
        if ng:
            self._call("qw_gdn_commit", ctypes.byref(self.gdn_dims), self.gdn_desc.data_ptr(), ng, self._st())

    def commit(self, accepted=None):
        """Host-chosen commit: accepted counts per sequence (sequence or tensor)."""
        if accepted is not None:
            self.accepted.copy_(torch.as_tensor(accepted, dtype=torch.int32), non_blocking=False)
        self.commit_states()
        self._call("qw_apply_commit", self.accepted.data_ptr(), self.top1.data_ptr(), self.next_token.data_ptr(),
                   self.qpos.data_ptr(), self.B, self.S, self._st())

    def step(self):
        """verify + device-side accept + commit of the block in ``self.tokens``."""
        self.forward()
        self.accept(auto_commit=True)
        self.commit_states()

    def active_experts(self) -> int:
        """Distinct routed experts of the last routed layer (reads the workspace; syncs);
        with expert parallelism, this rank's experts that received rows."""
        c = self.cfg
        if self.ep_moe is not None:
            m = self.ep_moe
            off = self.lib.qw_moe_active_experts(None, m.G * m.cap, m.local, 1)
            return int(m.ws_r[off:off + 4].view(torch.int32).item())
        off = self.lib.qw_moe_active_experts(None, self.T, c.num_experts, c.num_experts_per_tok)
        return int(self.moe_ws[off:off + 4].view(torch.int32).item())

    def algorithmic_bytes(self, active_per_layer) -> dict:
        """Bytes one verify step must move at least once (weights read once, the
        recurrent state read and written once, the KV context read once), given the
        distinct routed experts of each layer."""
        c = self.cfg
        g = c.quant_group
        w4b = lambda n, k: n * k // 2 + n * (k // g) * 2  # noqa: E731
        H, I, E = c.hidden_size, c.moe_intermediate_size, c.num_experts
        expert = w4b(2 * I, H) + w4b(H, I)
        ctx = int(self.qpos.float().mean().item()) + self.S
        parts = {"gdn_weights": 0, "attn_weights": 0, "moe_fixed": 0, "routed_experts": 0, "state": 0,
                 "kv": 0, "lm_head": 0}
        for l, kind in enumerate(c.layer_types):
            if kind == "linear_attention":
                parts["gdn_weights"] += (w4b(c.conv_channels + c.value_width, H) + 2 * c.linear_num_value_heads * H * 2
                                         + c.conv_channels * c.linear_conv_kernel_dim * 2 + w4b(H, c.value_width))
                parts["state"] += self.B * (2 * c.linear_num_value_heads * c.linear_key_head_dim
                                            * c.linear_value_head_dim * 4
                                            + 2 * c.conv_channels * (c.linear_conv_kernel_dim - 1) * 2)
            else:
                D, Hq, Hkv = c.head_dim, c.num_attention_heads, c.num_key_value_heads
                parts["attn_weights"] += w4b(Hq * 2 * D + 2 * Hkv * D, H) + w4b(H, Hq * D)
                parts["kv"] += self.B * 2 * Hkv * D * 2 * ctx
            parts["moe_fixed"] += (E + 1) * H * 2 + expert
            parts["routed_experts"] += active_per_layer[l] * expert
        parts["lm_head"] = c.vocab_size * H * 2
        parts["total"] = sum(parts.values())
        return parts

    def serve_step(self, host_tokens: torch.Tensor, host_out: torch.Tensor):
        """Public serving step: pinned host proposals [B*S] int32 in, device-side verify
        + accept + commit (the captured graph), then [accepted (B), next_token (B)] back
        into the pinned host buffer; returns after the copy completes."""
        self.tokens.copy_(host_tokens, non_blocking=True)
        self.graph.replay()
        host_out[: self.B].copy_(self.accepted, non_blocking=True)
        host_out[self.B: 2 * self.B].copy_(self.next_token, non_blocking=True)
        self._wait_status_host.copy_(self.wait_status, non_blocking=True)
        torch.cuda.current_stream(self.device).synchronize()
        self.raise_on_wait_timeout(self._wait_status_host[0])
        return host_out

    def serve_d2h_bytes(self) -> int:
        """Bytes ``serve_step`` copies back per step: accepted + next token + wait status."""
        return 4 * (2 * self.B + 1)

    # ------------------------------------------------------------------ graph
    def capture(self):
        """Record ``step()`` as a CUDA graph (buffers are static; inputs go to self.tokens)."""
        torch.cuda.synchronize(self.device)
        s = torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        snapshot = self.snapshot()
        with torch.cuda.stream(s):
            self.step()  # warm-up: lazy module loading and attribute setup outside capture
        torch.cuda.current_stream(self.device).wait_stream(s)
        torch.cuda.synchronize(self.device)
        self.restore(snapshot)
        g = torch.cuda.CUDAGraph()
        self._recording = {}
        try:
            with torch.cuda.graph(g, stream=s):
                self.step()
        finally:
            self.captured_calls, self._recording = self._recording, None
        torch.cuda.synchronize(self.device)
        self.graph = g
        return g

    def replay(self):
        self.graph.replay()

    def close(self):
        """Release the captured graph and, with expert parallelism, the exchange windows
        (collective: every rank of the group)."""
        self.graph = None
        if self.ep_moe is not None:
            self.ep_moe.close()

    def prefill_engine(self, block: int = 64) -> "TargetEngine":
        """An engine of ``block``-token blocks on this engine's weights and state: prompt
        chunks of ``block`` tokens per forward (the reference prefills the whole prompt in
        one forward, fused/session.py:282-296) instead of verify blocks of 16.  Its
        ``forward`` + ``accept(False)`` + ``commit([n])`` commits the first n tokens of a
        chunk into the shared banks and sets the shared next token."""
        return TargetEngine(self.cfg, (self.glob, self.layers), batch=self.B, block=block, capacity=self.capacity,
                            page_size=self.P, device=self.device, share=self)

    # ------------------------------------------------------------------ state utilities
    def snapshot(self):
        return {n: getattr(self, n).clone() for n in ("conv_hist", "state", "k_cache", "v_cache", "qpos",
                                                      "next_token", "hidden")}

    def restore(self, snap):
        for n, t in snap.items():
            getattr(self, n).copy_(t)

    def set_random_context(self, ctx: int, seed: int = 2, state_std: float = 0.02):
        """Synthetic committed context of ``ctx`` tokens per sequence: KV ~ N(0,1), GDN
        recurrent state ~ N(0, state_std), conv tails ~ N(0,1) (the benchmark's inputs)."""
        if ctx + self.S > self.capacity:
            raise ValueError("context exceeds capacity")
        gen = torch.Generator(device=self.device)
        gen.manual_seed(seed)
        self.k_cache.normal_(0, 1, generator=gen)
        self.v_cache.normal_(0, 1, generator=gen)
        self.state.normal_(0, state_std, generator=gen)
        self.conv_hist.normal_(0, 1, generator=gen)
        self.qpos.fill_(ctx)
        self.next_token.random_(0, self.cfg.vocab_size, generator=gen)

    def memory_bytes(self) -> dict:
        w = sum(t.numel() * t.element_size() for t in self.glob.values())
        for lw in self.layers:
            for v in lw.__dict__.values():
                if isinstance(v, torch.Tensor):
                    w += v.numel() * v.element_size()
        banks = sum(t.numel() * t.element_size() for t in (self.conv_hist, self.state, self.k_cache, self.v_cache))
        return {"weights": w, "state_banks": banks}
