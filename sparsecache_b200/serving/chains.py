"""Progressive draft/verify/commit chains over arriving KV stages.

A request's KV arrives in stages (document tranches or priority chunks).
Stage i's model sees the prompt with only the first i+1 stages visible.  The
chains below keep the reference's host logic and drive any backend through a
small ``StageModel`` interface, so the same algorithm runs on this package's
engine (CUDA-graph decode over a sparse view, batched verification) and on
CPU toy models in the tests:

``progressive_commit_chain`` (reference: experiments/progressive_kv_feasibility.py:686-983;
its reuse-pipeline variant experiments/reuse_cacheblend_pipeline.py:896-1141)
    stage 0 drafts ``draft_tokens`` greedily; every later stage verifies
    committed + pending tokens with one batched forward, accepts the longest
    matching prefix of the pending tokens (each survivor gains a "pass"),
    replaces the first mismatch by the verifier's token, and commits pending
    tokens once they survived ``commit_window`` verifications (W = None means
    "only the final stage commits").  Flips of already-committed tokens are
    counted and ignored.  Non-final stages then draft again up to the draft
    horizon.  The final stage commits everything that survived and continues
    decoding on the full KV.  EOS stops the chain at any stage.

``grafted_draft_batch`` / ``progressive_graft_chain`` (reference: :985-1310)
    zero-replay variants: the tokens drafted on a smaller view are carried
    over ("grafted") when the view grows, and only the final full-KV verifier
    checks them, once.
"""
from __future__ import annotations

import time
from dataclasses import dataclass, field
from typing import Any, Callable, Protocol, Sequence


class StageModel(Protocol):
    n_stages: int

    def verify(self, stage: int, sequence: Sequence[int]) -> list[int]:
        """Greedy predictions for every position of ``sequence`` (the target token after
        prompt + sequence[:j]) with stages 0..stage visible; length len(sequence) + 1."""

    def draft(self, stage: int, sequence: Sequence[int], n: int) -> list[int]:
        """Up to ``n`` greedy tokens continuing prompt + sequence on stage ``stage``'s view."""

    def final_decode(self, sequence: Sequence[int], n: int) -> list[int]:
        """Up to ``n`` greedy tokens continuing prompt + sequence with the full KV."""


@dataclass
class ChainPayload:
    tokens: list[int]
    trace: list[dict[str, Any]]
    draft_ms: float = 0.0
    verify_ms: float = 0.0
    final_decode_ms: float = 0.0
    ignored_committed_flips: int = 0
    committed_checks: int = 0
    terminated_stage: int = -1
    first_draft_ms: float | None = None
    first_committed_ms: float | None = None
    verifications: int = 0
    extra: dict = field(default_factory=dict)


def _timed(clock, fn, *a):
    t = clock()
    out = fn(*a)
    return out, (clock() - t) * 1e3


def progressive_commit_chain(model: StageModel, *, commit_window: int | None, draft_tokens: int, max_new_tokens: int,
                             eos_ids: set[int] = frozenset(), verify_intermediate: bool = True,
                             draft_intermediate: bool = True, stage_wait: Callable[[int], None] | None = None,
                             clock=time.perf_counter) -> ChainPayload:
    n = model.n_stages
    window = commit_window if commit_window is not None else n + 1
    committed: list[int] = []
    pending: list[dict] = []
    out = ChainPayload([], [])
    t0 = clock()
    for stage in range(n):
        if stage_wait is not None:
            stage_wait(stage)
        final = stage == n - 1
        row = {"stage": stage, "verified": False, "committed_before": len(committed), "pending_before": len(pending),
               "accepted_pending": 0, "rejected_pending": 0, "drafted": 0}
        seq = committed + [p["token"] for p in pending]
        if stage > 0 and seq and (final or verify_intermediate):
            row["verified"] = True
            preds, ms = _timed(clock, model.verify, stage, seq)
            out.verify_ms += ms
            out.verifications += 1
            out.committed_checks += len(committed)
            out.ignored_committed_flips += sum(p != c for p, c in zip(preds[:len(committed)], committed))
            pend_preds = preds[len(committed):]
            acc = 0
            for item, pr in zip(pending, pend_preds):
                if item["token"] != pr:
                    break
                acc += 1
            row["accepted_pending"], row["rejected_pending"] = acc, len(pending) - acc
            survivors = pending[:acc]
            for s in survivors:
                s["passes"] += 1
            pending = survivors + ([{"token": pend_preds[acc], "passes": 0}] if acc < len(pending) else [])
            while pending and pending[0]["passes"] >= window:
                committed.append(pending.pop(0)["token"])
            if committed and out.first_committed_ms is None:
                out.first_committed_ms = (clock() - t0) * 1e3
        if committed and committed[-1] in eos_ids:
            row.update(committed_after=len(committed), pending_after=len(pending))
            out.trace.append(row)
            out.tokens, out.terminated_stage = committed, stage
            return out
        if final:
            committed += [p["token"] for p in pending]
            pending.clear()
            if committed and out.first_committed_ms is None:
                out.first_committed_ms = (clock() - t0) * 1e3
            if not committed or committed[-1] not in eos_ids:
                adds, ms = _timed(clock, model.final_decode, committed, max_new_tokens - len(committed))
                out.final_decode_ms += ms
                for t in adds:
                    committed.append(t)
                    if t in eos_ids:
                        break
            row.update(committed_after=len(committed), pending_after=0)
            out.trace.append(row)
            out.tokens, out.terminated_stage = committed[:max_new_tokens], stage
            return out
        seq = committed + [p["token"] for p in pending]
        if (stage == 0 or draft_intermediate) and (not seq or seq[-1] not in eos_ids):
            want = min(draft_tokens, max_new_tokens - len(seq))
            adds, ms = _timed(clock, model.draft, stage, seq, max(0, want)) if want > 0 else ([], 0.0)
            out.draft_ms += ms
            clipped = []
            for t in adds:
                clipped.append(t)
                if t in eos_ids:
                    break
            pending += [{"token": t, "passes": 0} for t in clipped]
            row["drafted"], row["draft_token_ids"] = len(clipped), clipped
            if clipped and out.first_draft_ms is None:
                out.first_draft_ms = (clock() - t0) * 1e3
        row.update(committed_after=len(committed), pending_after=len(pending))
        out.trace.append(row)
    raise RuntimeError("progressive chain failed to terminate")


def grafted_draft_batch(model: StageModel, stage: int, grafted: Sequence[int], n: int) -> list[int]:
    """Draft ``n`` more tokens on stage ``stage``'s view after an already drafted tail
    (the tail is kept as is: no replay of earlier stages' drafts)."""
    return list(grafted) + model.draft(stage, grafted, n)


def progressive_graft_chain(model: StageModel, *, draft_tokens_per_stage: int, max_new_tokens: int,
                            eos_ids: set[int] = frozenset(), clock=time.perf_counter) -> ChainPayload:
    """Zero-replay multi-stage drafting with one final verifier (then normal decoding)."""
    out = ChainPayload([], [])
    t0 = clock()
    drafted: list[int] = []
    for stage in range(model.n_stages - 1):
        want = min(draft_tokens_per_stage, max_new_tokens - len(drafted))
        if want <= 0 or (drafted and drafted[-1] in eos_ids):
            break
        adds, ms = _timed(clock, model.draft, stage, drafted, want)
        out.draft_ms += ms
        drafted += adds
        out.trace.append({"stage": stage, "drafted": len(adds), "draft_token_ids": list(adds)})
        if adds and out.first_draft_ms is None:
            out.first_draft_ms = (clock() - t0) * 1e3
    final = model.n_stages - 1
    committed: list[int] = []
    if drafted:
        preds, ms = _timed(clock, model.verify, final, drafted)
        out.verify_ms += ms
        out.verifications += 1
        acc = 0
        for d, p in zip(drafted, preds):
            if d != p:
                break
            acc += 1
        committed = drafted[:acc] + [preds[acc]]
        out.trace.append({"stage": final, "verified": True, "accepted_pending": acc,
                          "rejected_pending": len(drafted) - acc})
        out.first_committed_ms = (clock() - t0) * 1e3
    if not committed or committed[-1] not in eos_ids:
        adds, ms = _timed(clock, model.final_decode, committed, max_new_tokens - len(committed))
        out.final_decode_ms += ms
        for t in adds:
            committed.append(t)
            if t in eos_ids:
                break
    out.tokens, out.terminated_stage = committed[:max_new_tokens], final
    out.extra["accepted_draft_tokens"] = out.trace[-1].get("accepted_pending", 0) if drafted else 0
    return out


class ToyStageModel:
    """Deterministic CPU stage model: the full-KV greedy continuation is a fixed
    function of the prefix; stage s agrees with it except at positions where
    ``noise(stage, position)`` says the sparse view errs (never at the final stage)."""

    def __init__(self, n_stages: int, vocab: int = 97, flip_rate: float = 0.3, seed: int = 0) -> None:
        self.n_stages, self.vocab, self.flip_rate, self.seed = n_stages, vocab, flip_rate, seed

    def _true_next(self, seq: Sequence[int]) -> int:
        return (sum(seq) * 7 + len(seq) * 13 + self.seed) % self.vocab

    def _stage_next(self, stage: int, seq: Sequence[int]) -> int:
        t = self._true_next(seq)
        if stage >= self.n_stages - 1:
            return t
        h = (hash((self.seed, stage, len(seq), tuple(seq[-3:]))) & 0xFFFF) / 0x10000
        return (t + 1) % self.vocab if h < self.flip_rate * (1.0 - stage / self.n_stages) else t

    def verify(self, stage: int, sequence: Sequence[int]) -> list[int]:
        return [self._stage_next(stage, list(sequence[:j])) for j in range(len(sequence) + 1)]

    def draft(self, stage: int, sequence: Sequence[int], n: int) -> list[int]:
        seq, out = list(sequence), []
        for _ in range(n):
            t = self._stage_next(stage, seq)
            seq.append(t)
            out.append(t)
        return out

    def final_decode(self, sequence: Sequence[int], n: int) -> list[int]:
        return self.draft(self.n_stages - 1, sequence, n)
