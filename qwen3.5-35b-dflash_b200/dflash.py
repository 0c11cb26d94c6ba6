"""Greedy DFlash generation on the device: draft -> verify -> accept -> commit -> extend.

The reference's scheduler (model/qwen35_moe_dflash/execution/runtime.py:24-107; the
board loop targets/cpro/runtime/src/generation.cpp:178-294) recomputes the whole prefix
for every target and draft call and compares tokens on the host.  Here one step is a
fixed sequence of kernels on the device, capturable as one CUDA graph:

1. ``DraftEngine.propose``: the draft over [anchor, mask x 15] writes the verify block
   [anchor, 15 proposals] into the target engine's tokens;
2. ``TargetEngine.step``: the block verify, the longest accepted prefix (proposal i is
   accepted while it equals the target's greedy prediction after proposal i - 1), the
   commit of that prefix into the GDN / conv / KV state, and the next anchor (the
   target's prediction after the accepted prefix: the correction or the bonus token);
3. ``DraftEngine.extend``: the draft's context cache takes the committed rows' target
   features (the feature ring).

The host only reads, per step, how many tokens were committed and which (the verify
block's first ``accepted`` tokens): greedy DFlash emits exactly the target's greedy
continuation, whatever the draft proposes.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch

from .draft import DraftEngine
from .engine import TargetEngine


@dataclass
class Generation:
    """Result of ``DFlash.generate`` (the fields of the reference's Result)."""
    token_ids: list[int]
    stop_reason: str
    steps: int = 0
    drafted: int = 0
    accepted: int = 0
    iterations: list[dict] = field(default_factory=list)


PREFILL_BLOCK = 64   # prompt tokens per prefill forward


class DFlash:
    def __init__(self, target: TargetEngine, draft: DraftEngine, prefill_block: int = PREFILL_BLOCK):
        """``prefill_block``: prompt tokens per prefill forward (a multiple of the verify
        block; the target's prefill engine shares its state)."""
        if target.B != 1:
            raise ValueError("DFlash.generate drives one sequence (engine batch 1)")
        if prefill_block % target.S:
            raise ValueError("the prefill block must be a multiple of the verify block")
        self.te, self.dr = target, draft
        self.graph = None
        self._host = torch.zeros(1 + target.S, dtype=torch.int32).pin_memory()
        self.prefill_block = prefill_block
        self._pe = None
        self._valid = torch.zeros(1, dtype=torch.int32, device=target.device)
        self._pos_sub = torch.zeros(1, dtype=torch.int32, device=target.device)

    def prefill(self, prompt: list[int]) -> None:
        """Commit the prompt into the target and the draft's context, ``prefill_block``
        tokens per target forward; the target's next_token is then the first generated
        token (the first anchor).  The draft's context takes each chunk's committed rows
        one verify block of features at a time."""
        te, S, P = self.te, self.te.S, self.prefill_block
        if not prompt:
            raise ValueError("nonempty prompt required")
        if any(type(t) is not int or not 0 <= t < te.cfg.vocab_size for t in prompt):
            raise ValueError("token ID outside vocabulary")
        if (len(prompt) + P - 1) // P * P + S > te.capacity:
            raise ValueError("prompt exceeds the engine's capacity")
        if self._pe is None:
            self._pe = te if P == S else te.prefill_engine(P)
        pe = self._pe
        te.qpos.zero_()
        te.state.zero_()
        te.conv_hist.zero_()
        for i in range(0, len(prompt), P):
            chunk = prompt[i:i + P]
            n = len(chunk)
            pe.tokens.copy_(torch.tensor(chunk + [0] * (P - n), dtype=torch.int32))
            pe.forward()
            pe.accept(auto_commit=False)
            pe.commit([n])
            pe.raise_on_wait_timeout()
            for j in range(0, n, S):
                self._valid.fill_(min(S, n - j))
                self._pos_sub.fill_(n - j)
                self.dr.extend(valid=self._valid, features=pe.features[j:j + S], pos_sub=self._pos_sub)

    def step(self) -> None:
        """One DFlash step on the current stream (device only)."""
        self.dr.propose()
        self.te.step()
        self.dr.extend()

    def capture(self):
        """Record ``step`` as a CUDA graph (after a warm-up step; the state is restored)."""
        te = self.te
        torch.cuda.synchronize(te.device)
        snap = te.snapshot()
        dsnap = (self.dr.k_cache.clone(), self.dr.v_cache.clone())
        s = torch.cuda.Stream(te.device)
        s.wait_stream(torch.cuda.current_stream(te.device))
        with torch.cuda.stream(s):
            self.step()
        torch.cuda.current_stream(te.device).wait_stream(s)
        torch.cuda.synchronize(te.device)
        te.restore(snap)
        self.dr.k_cache.copy_(dsnap[0])
        self.dr.v_cache.copy_(dsnap[1])
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            self.step()
        torch.cuda.synchronize(te.device)
        self.graph = g

    def generate(self, prompt: list[int], max_new_tokens: int = 32, eos_token_ids=(), use_graph: bool = True
                 ) -> Generation:
        """Greedy DFlash continuation of ``prompt`` (runtime.py:24-107 semantics: the
        committed tokens of a step are the anchor and the accepted proposals; stops at
        max_new_tokens or after an EOS token)."""
        te = self.te
        if max_new_tokens <= 0:
            raise ValueError("positive generation limit required")
        if len(prompt) + max_new_tokens + 2 * te.S > te.capacity:
            raise ValueError("prompt plus output exceeds the engine's capacity")
        eos = frozenset(eos_token_ids)
        self.prefill(list(prompt))
        if use_graph and self.graph is None:
            self.capture()
        out = Generation([], "length")
        host = self._host
        while len(out.token_ids) < max_new_tokens:
            if use_graph:
                self.graph.replay()
            else:
                self.step()
            host[0:1].copy_(te.accepted, non_blocking=True)
            host[1:].copy_(te.tokens, non_blocking=True)
            torch.cuda.current_stream(te.device).synchronize()
            te.raise_on_wait_timeout()
            acc = int(host[0])
            committed = [int(v) for v in host[1:1 + acc]]
            out.steps += 1
            out.drafted += te.S - 1
            out.accepted += acc - 1
            out.iterations.append({"proposals": [int(v) for v in host[2:]], "accepted": acc - 1,
                                   "committed": committed})
            for tok in committed:
                out.token_ids.append(tok)
                if tok in eos:
                    out.stop_reason = "eos"
                    return out
                if len(out.token_ids) >= max_new_tokens:
                    return out
        return out
