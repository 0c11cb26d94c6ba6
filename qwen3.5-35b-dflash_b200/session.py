"""Prefill / step / block-verify / commit over a device-resident TargetEngine.

Mirrors the reference's ``FusedTargetSession`` and ``TargetVerification``
(model/qwen35_moe_dflash/fused/session.py:233-391) for one sequence (engine batch 1):
same method names, the same meaning of ``expected_next_tokens`` (entry i is the target's
prediction before consuming proposal i, the last one the bonus prediction), the same
accepted-prefix rule, and the same errors for invalid calls (ValueError for bad
arguments, RuntimeError for use before prefill or of a stale verification).

The difference is the mechanism.  The reference runs one forward per proposed token
and keeps a state checkpoint per token; here the whole block is one forward of the
engine, the committed state is never modified by ``verify`` (the GDN kernels read the
banks and write nothing back; the KV slots past the committed position are scratch),
and ``commit(r)`` recomputes the state after exactly r tokens from the same inputs.
Blocks have the engine's fixed width: shorter calls are padded and only the real
tokens are compared and committed.
"""
from __future__ import annotations

import threading
from collections.abc import Sequence

import torch

from .engine import TargetEngine


def _token(value) -> int:
    if type(value) is not int or not 0 <= value <= 2 ** 31 - 1:
        raise ValueError("token IDs must be nonnegative INT32 integers, not bool")
    return value


def _tokens(values) -> list[int]:
    if isinstance(values, torch.Tensor):
        if values.dtype not in (torch.int32, torch.int64):
            raise ValueError("token tensor must have an integer dtype")
        if values.ndim != 2 or values.shape[0] != 1:
            raise ValueError("token tensor must have shape [1, sequence]")
        result = [_token(v) for v in values.detach().cpu().tolist()[0]]
    else:
        if isinstance(values, (str, bytes)) or not isinstance(values, Sequence):
            raise ValueError("tokens must be a sequence of integers or a [1,S] tensor")
        result = [_token(v) for v in values]
    if not result:
        raise ValueError("tokens must contain at least one token; padding is not inferred")
    return result


class TargetSession:
    def __init__(self, engine: TargetEngine):
        if engine.B != 1:
            raise ValueError("TargetSession drives one sequence (engine batch 1)")
        self.engine = engine
        self._lock = threading.RLock()
        self._prefilled = False
        self._generation = 0
        self._next_token: int | None = None
        self._last_features: torch.Tensor | None = None
        self._forward_id = 0  # id of the block whose activations the engine holds
        engine.qpos.zero_()
        engine.state.zero_()
        engine.conv_hist.zero_()

    # ------------------------------------------------------------------ properties
    @property
    def position(self) -> int:
        return int(self.engine.qpos[0].item())

    @property
    def next_token(self) -> int:
        with self._lock:
            self._require_prefill()
            return self._next_token

    @property
    def last_features(self) -> torch.Tensor:
        with self._lock:
            self._require_prefill()
            return self._last_features.clone()

    def _require_prefill(self):
        if not self._prefilled:
            raise RuntimeError("prefill must complete before decoding or verification")

    # ------------------------------------------------------------------ engine glue
    def _run_block(self, ids: list[int]):
        e = self.engine
        if len(ids) > e.S:
            raise ValueError("block longer than the engine's block width")
        if self.position + e.S > e.capacity:
            raise ValueError("input would exceed target context capacity")
        if any(t >= e.cfg.vocab_size for t in ids):
            raise ValueError("input token is outside the vocabulary")
        padded = ids + [0] * (e.S - len(ids))
        e.tokens.copy_(torch.tensor(padded, dtype=torch.int32))
        e.forward()
        e.accept(auto_commit=False)
        e.raise_on_wait_timeout()   # no retry, no fallback (fused/ops.py:133-136)
        self._forward_id += 1
        return self._forward_id

    def _commit_rows(self, n: int):
        e = self.engine
        e.commit([n])
        self._generation += 1
        self._next_token = int(e.next_token[0].item())
        self._last_features = e.features[n - 1:n].clone().unsqueeze(0) if n > 0 else self._last_features

    # ------------------------------------------------------------------ API
    def prefill(self, ids) -> None:
        values = _tokens(ids)
        with self._lock:
            if self._prefilled or self.position != 0:
                raise RuntimeError("prefill is allowed only once on an empty session")
            S = self.engine.S
            for i in range(0, len(values), S):
                chunk = values[i:i + S]
                self._run_block(chunk)
                self._commit_rows(len(chunk))
            self._prefilled = True

    def step(self, token: int) -> None:
        value = _token(token)
        with self._lock:
            self._require_prefill()
            self._run_block([value])
            self._commit_rows(1)

    def verify(self, proposals) -> "BlockVerification":
        values = _tokens(proposals)
        with self._lock:
            self._require_prefill()
            fid = self._run_block(values)
            e = self.engine
            top1 = e.top1[: len(values)].tolist()
            accepted = min(int(e.max_accepted[0].item()), len(values))
            expected = (self._next_token,) + tuple(int(t) for t in top1)
            return BlockVerification(self, self._generation, fid, values, expected, accepted)


class BlockVerification:
    """Uncommitted verification of a proposal block (TargetVerification semantics)."""

    def __init__(self, session: TargetSession, generation: int, forward_id: int, proposals: list[int],
                 expected: tuple[int, ...], accepted: int):
        self._session = session
        self._generation = generation
        self._forward_id = forward_id
        self._proposals = proposals
        self._expected = expected
        self._max = accepted
        self._closed = False

    @property
    def expected_next_tokens(self) -> tuple[int, ...]:
        return self._expected

    @property
    def max_accepted_prefix(self) -> int:
        return self._max

    @property
    def closed(self) -> bool:
        return self._closed

    def _check_active(self):
        if self._closed:
            raise RuntimeError("state transaction is closed")
        if self._generation != self._session._generation:
            raise RuntimeError("stale state transaction: another branch has committed")

    def commit(self, accepted: int) -> None:
        s = self._session
        with s._lock:
            self._check_active()
            if type(accepted) is not int or not 0 <= accepted <= self._max:
                raise ValueError("accepted count exceeds the matching proposal prefix")
            if accepted:
                # commit recomputes from this block's activations: if another block was
                # verified since, run this one again (the committed state is unchanged)
                if s._forward_id != self._forward_id:
                    s._run_block(self._proposals)
                s._commit_rows(accepted)
            else:
                s._generation += 1
            self._closed = True

    def abort(self) -> None:
        if self._closed:
            raise RuntimeError("state transaction is closed")
        self._closed = True
