"""Progressive prefill/decode (P/D) transfer with sparse drafting and one final verifier.

Components (reference behaviour cited per item):
  * ``ProgressivePDRequestState``: the decode-side state machine
    WAIT_ANCHOR -> DRAFT_WHILE_LOADING -> READY_TO_VERIFY -> TARGET_DECODING
    -> FINISHED.  Visibility is the longest completed prefix of the priority
    order; duplicate / unknown completions are rejected; drafting only after
    the anchor; the full-KV verifier runs exactly once
    (experiments/progressive_pd_state_machine.py:10-122).
  * ``lexical_scores`` / ``ranked_document_indices`` / ``stage_document_sets``:
    per-request BM25 and the schedules sequential, uniform (van der Corput
    bit reversal), query, p_attention, oracle, support_last, random; cumulative
    stage sets reaching ceil(fraction * tokens) (progressive_kv_feasibility.py:211-313).
  * ``prefix_visibility_mask`` / ``pd_visibility_mask`` / ``encode_contiguous_cache``
    / ``encode_independent_cache``: the whole-cache view model of the
    feasibility runners (progressive_kv_feasibility.py:374-447;
    pd_progressive_kv_feasibility.py:80-91), with ``visible_slot_map``
    turning a mask into the slot map the engine reads.
  * ``TrancheStager``: each stage's disjoint token ranges packed into one
    pinned host block; stage 0 always carries the system prefix and the
    question suffix; tranches are appended to a compact device cache on a copy
    stream with per-stage events; optional paced wire (deadline = bytes * 8 /
    rate) and eager serial wire (cumulative deadlines on one wire)
    (pd_progressive_kv_pipeline.py:187-456).
  * ``continuous_graft_chain``: before each proposal, poll tranche readiness
    and widen the visible view; draft one token with the target model over
    the visible K/V plus the generated tail; after the last tranche, ONE
    batched verifier over the full K/V, KV crop of the rejected tail and one
    correction token, then ordinary decode (progressive_kv_feasibility.py:1313-1657).

B200 design: the compact cache is an engine ``KVSlot`` filled in arrival
order; the draft view is an int32 slot map (arrived prompt slots followed by
the tail slots [T, T + max_new)), read by the paged decode-attention kernel,
so widening the view or cropping the tail is a metadata update, never a K/V
copy (the reference concatenates caches, K19).
"""
from __future__ import annotations

import math
import random
import re
import time
from collections import Counter
from dataclasses import dataclass, field
from enum import Enum, auto
from typing import Any, Sequence

import torch

TOKEN_PATTERN = re.compile(r"[a-z0-9]+")


# --------------------------------------------------------------------------
# State machine
# --------------------------------------------------------------------------
class ProgressivePDPhase(Enum):
    WAIT_ANCHOR = auto()
    DRAFT_WHILE_LOADING = auto()
    READY_TO_VERIFY = auto()
    TARGET_DECODING = auto()
    FINISHED = auto()


@dataclass(frozen=True)
class DraftProposal:
    token_id: int
    visible_priority_pages: tuple[int, ...]


@dataclass
class ProgressivePDRequestState:
    """Fail-closed orchestration of one progressive request on the decode side."""

    priority_pages: tuple[int, ...]
    anchor_pages: int
    max_draft_tokens: int
    phase: ProgressivePDPhase = ProgressivePDPhase.WAIT_ANCHOR
    completed_pages: set[int] = field(default_factory=set)
    proposals: list[DraftProposal] = field(default_factory=list)
    external_token_ids: list[int] = field(default_factory=list)
    verifier_calls: int = 0

    def __post_init__(self) -> None:
        if not self.priority_pages:
            raise ValueError("priority page order cannot be empty")
        if len(set(self.priority_pages)) != len(self.priority_pages):
            raise ValueError("priority page order contains duplicates")
        if not 0 < self.anchor_pages <= len(self.priority_pages):
            raise ValueError("anchor_pages must lie in [1, number of pages]")
        if self.max_draft_tokens <= 0:
            raise ValueError("max_draft_tokens must be positive")

    @property
    def visible_priority_pages(self) -> tuple[int, ...]:
        out = []
        for page in self.priority_pages:
            if page not in self.completed_pages:
                break
            out.append(page)
        return tuple(out)

    @property
    def visible_fraction(self) -> float:
        return len(self.visible_priority_pages) / len(self.priority_pages)

    def record_page_completion(self, pages: set[int]) -> None:
        if self.phase in (ProgressivePDPhase.READY_TO_VERIFY, ProgressivePDPhase.TARGET_DECODING,
                          ProgressivePDPhase.FINISHED):
            raise RuntimeError("page completion arrived after full-KV readiness")
        unknown = set(pages) - set(self.priority_pages)
        if unknown:
            raise ValueError(f"completion contains unknown pages: {sorted(unknown)}")
        if set(pages) & self.completed_pages:
            raise ValueError("connector reported a page completion twice")
        self.completed_pages |= set(pages)
        if len(self.completed_pages) == len(self.priority_pages):
            self.phase = ProgressivePDPhase.READY_TO_VERIFY
        elif len(self.visible_priority_pages) >= self.anchor_pages:
            self.phase = ProgressivePDPhase.DRAFT_WHILE_LOADING

    def record_draft_token(self, token_id: int) -> None:
        if self.phase != ProgressivePDPhase.DRAFT_WHILE_LOADING:
            raise RuntimeError("drafting is allowed only after the anchor and before full KV")
        if len(self.proposals) >= self.max_draft_tokens:
            raise RuntimeError("draft token limit reached")
        self.proposals.append(DraftProposal(int(token_id), self.visible_priority_pages))

    def record_final_verification(self, accepted_prefix: int, correction_token: int) -> None:
        if self.phase != ProgressivePDPhase.READY_TO_VERIFY:
            raise RuntimeError("final verification requires complete prompt KV")
        if self.verifier_calls:
            raise RuntimeError("the immutable verifier may run only once")
        if not 0 <= accepted_prefix <= len(self.proposals):
            raise ValueError("accepted prefix exceeds the proposal sequence")
        self.verifier_calls = 1
        self.external_token_ids.extend(p.token_id for p in self.proposals[:accepted_prefix])
        self.external_token_ids.append(int(correction_token))
        self.phase = ProgressivePDPhase.TARGET_DECODING

    def finish(self) -> None:
        if self.phase != ProgressivePDPhase.TARGET_DECODING:
            raise RuntimeError("only target decoding may finish a request")
        self.phase = ProgressivePDPhase.FINISHED


# --------------------------------------------------------------------------
# Document ranking and cumulative stages
# --------------------------------------------------------------------------
@dataclass(frozen=True)
class Document:
    token_ids: tuple[int, ...]
    text: str = ""
    supporting: bool | None = None
    start: int = 0
    end: int = 0


def lexical_scores(question: str, documents: Sequence[Document]) -> list[float]:
    """Per-request BM25 (k1 = 1.5, b = 0.75) with no label leakage."""
    terms = TOKEN_PATTERN.findall(question.lower())
    docs = [TOKEN_PATTERN.findall(d.text.lower()) for d in documents]
    df = Counter()
    for words in docs:
        df.update(set(words))
    avg = sum(map(len, docs)) / max(1, len(docs))
    n = len(documents)
    out = []
    for words in docs:
        tf = Counter(words)
        score = 0.0
        for term in terms:
            f = tf[term]
            if not f:
                continue
            idf = math.log(1 + (n - df[term] + 0.5) / (df[term] + 0.5))
            score += idf * f * 2.5 / (f + 1.5 * (0.25 + 0.75 * len(words) / max(1.0, avg)))
        out.append(score)
    return out


def van_der_corput_order(n: int) -> list[int]:
    """Bit-reversal order: every prefix covers the sequence broadly."""
    width = max(1, math.ceil(math.log2(max(1, n))))

    def rev(i: int) -> int:
        v = 0
        for _ in range(width):
            v = (v << 1) | (i & 1)
            i >>= 1
        return v

    return sorted(range(n), key=lambda i: (rev(i), i))


SCHEDULES = ("sequential", "uniform", "query", "p_attention", "oracle", "support_last", "random")


def ranked_document_indices(schedule: str, *, question: str, documents: Sequence[Document], random_seed: int,
                            attention_scores: Sequence[float] | None = None) -> list[int]:
    scores = lexical_scores(question, documents)
    idx = list(range(len(documents)))
    if schedule == "sequential":
        return idx
    if schedule == "uniform":
        return van_der_corput_order(len(idx))
    if schedule == "query":
        return sorted(idx, key=lambda i: (-scores[i], i))
    if schedule == "p_attention":
        if attention_scores is None or len(attention_scores) != len(documents):
            raise ValueError("p_attention requires one producer-side score per document")
        return sorted(idx, key=lambda i: (-attention_scores[i], -scores[i], i))
    if schedule == "oracle":
        return sorted(idx, key=lambda i: (not documents[i].supporting, -scores[i], i))
    if schedule == "support_last":
        return sorted(idx, key=lambda i: (bool(documents[i].supporting), -scores[i], i))
    if schedule == "random":
        random.Random(random_seed).shuffle(idx)
        return idx
    raise ValueError(f"unknown schedule: {schedule}")


def stage_document_sets(ranking: Sequence[int], documents: Sequence[Document],
                        fractions: Sequence[float]) -> list[set[int]]:
    total = sum(len(d.token_ids) for d in documents)
    stages = []
    for frac in fractions:
        if frac == 1.0:
            stages.append(set(ranking))
            continue
        target = math.ceil(total * frac)
        chosen, tokens = set(), 0
        for i in ranking:
            chosen.add(i)
            tokens += len(documents[i].token_ids)
            if tokens >= target:
                break
        stages.append(chosen)
    if any(not a <= b for a, b in zip(stages, stages[1:])):
        raise RuntimeError("stage document sets are not cumulative")
    return stages


# --------------------------------------------------------------------------
# Whole-cache encoders and visibility masks (the feasibility runners' view model)
# --------------------------------------------------------------------------
def prefix_visibility_mask(prefix_tokens: int, documents: Sequence[Document], selected,
                           device=None) -> torch.Tensor:
    """[1, prefix + documents] int64 mask: the prefix and the selected documents' spans are 1.

    Reference: experiments/progressive_kv_feasibility.py:432-447.  Documents
    carry their ``start``/``end`` in the concatenated prompt.
    """
    total = prefix_tokens + sum(len(d.token_ids) for d in documents)
    mask = torch.zeros((1, total), dtype=torch.long, device=device)
    mask[:, :prefix_tokens] = 1
    for i in selected:
        mask[:, documents[i].start:documents[i].end] = 1
    return mask


def pd_visibility_mask(prefix_tokens: int, documents: Sequence[Document], suffix_tokens: int, selected,
                       device=None) -> torch.Tensor:
    """As ``prefix_visibility_mask`` plus the question suffix, always visible (the P/D anchor).

    Reference: experiments/pd_progressive_kv_feasibility.py:80-91.
    """
    doc_mask = prefix_visibility_mask(prefix_tokens, documents, selected, device)
    tail = torch.ones((1, suffix_tokens), dtype=torch.long, device=doc_mask.device)
    return torch.cat((doc_mask, tail), dim=1)


def visible_slot_map(mask: torch.Tensor) -> torch.Tensor:
    """int32 indices of the visible tokens of a [1, T] mask.

    The engine's draft attention reads a view through such a slot map, so a
    masked view costs no mask tensor and no K/V copy.
    """
    return mask.reshape(-1).nonzero().reshape(-1).to(torch.int32)


@torch.no_grad()
def encode_contiguous_cache(model, token_ids: Sequence[int]):
    """One causal prefill of the whole prompt at positions 0..T-1 (oracle model) -> legacy cache.

    Reference: experiments/progressive_kv_feasibility.py:416-429.
    """
    _, cache = model.prefill(list(token_ids), start=0)
    return cache


@torch.no_grad()
def encode_independent_cache(model, prefix: Sequence[int], documents: Sequence[Document]):
    """Prefix and every document prefilled alone at local positions, keys relocated to ``document.start``.

    The result is the concatenated cache a reuse system composes from
    independently produced entries (reference:
    experiments/progressive_kv_feasibility.py:374-413); the engine path is the
    document producer plus the ``compose_relocate`` kernel.
    """
    from ..rope import relocate_key

    cfg = model.config
    segments = [(tuple(prefix), 0)] + [(d.token_ids, d.start) for d in documents]
    keys: list[list[torch.Tensor]] = [[] for _ in range(cfg.n_layers)]
    values: list[list[torch.Tensor]] = [[] for _ in range(cfg.n_layers)]
    for ids, start in segments:
        if not ids:
            continue
        _, cache = model.prefill(list(ids), start=0)
        for layer, (k, v) in enumerate(cache):
            keys[layer].append(relocate_key(cfg, k, source_start=0, target_start=start))
            values[layer].append(v)
    return tuple((torch.cat(keys[l], dim=2), torch.cat(values[l], dim=2)) for l in range(cfg.n_layers))


def accepted_prefix_length(draft_tokens: Sequence[int], target_tokens: Sequence[int]) -> int:
    """Number of leading draft tokens the target reproduces."""
    n = 0
    for d, t in zip(draft_tokens, target_tokens):
        if int(d) != int(t):
            break
        n += 1
    return n


# --------------------------------------------------------------------------
# Tranche stager
# --------------------------------------------------------------------------
@dataclass(frozen=True)
class StageTransfer:
    ranges: tuple[tuple[int, int], ...]  # prompt token ranges [start, end)
    destination_start: int
    destination_end: int


class TrancheStager:
    """Append disjoint KV tranches into a compact device slot on a copy stream.

    ``source`` is the full prompt KV [L, 2, H_kv, T, D] (pinned host memory:
    the producer's output).  The slot receives stage 0 (prefix + suffix +
    first documents) at slots [0, n0), later stages appended after it.
    ``clock`` is injectable for tests (defaults to time.perf_counter).
    """

    def __init__(self, source: torch.Tensor, slot, *, prefix_tokens: int, documents: Sequence[Document],
                 suffix_tokens: int, ranking: Sequence[int], selected_sets: Sequence[set[int]],
                 transport_gbps: float | None = None, eager_serial_wire: bool = False, clock=time.perf_counter,
                 sleep=time.sleep, device=None) -> None:
        self.source = source
        self.slot = slot
        self.transport_gbps = transport_gbps
        self.eager_serial_wire = eager_serial_wire
        self.clock, self.sleep = clock, sleep
        self.device = device
        n = len(selected_sets)
        self.launched = [False] * n
        self.physical_launched = [False] * n
        self.wire_started_at: list[float | None] = [None] * n
        self.wire_ready_at: list[float | None] = [None] * n
        self.wire_wait_ms = [0.0] * n
        L, _, H, T, D = source.shape
        self.bytes_per_token = L * 2 * H * D * source.element_size()
        doc_end = prefix_tokens + sum(len(d.token_ids) for d in documents)
        total = doc_end + suffix_tokens
        stages, prior, dest = [], set(), 0
        for s, selected in enumerate(selected_sets):
            ranges = []
            if s == 0:
                if prefix_tokens:
                    ranges.append((0, prefix_tokens))
                if suffix_tokens:
                    ranges.append((doc_end, total))
            for i in ranking:
                if i in selected and i not in prior:
                    ranges.append((documents[i].start, documents[i].end))
            width = sum(e - b for b, e in ranges)
            stages.append(StageTransfer(tuple(ranges), dest, dest + width))
            dest += width
            prior = set(selected)
        if dest != total:
            raise RuntimeError("final progressive stage does not contain full KV")
        self.stages = tuple(stages)
        self.total_tokens = total
        # slot map: compact slot -> prompt position (used to build attention views)
        positions = []
        for st in self.stages:
            for b, e in st.ranges:
                positions.extend(range(b, e))
        self.compact_positions = positions
        self._packed = None
        self._events = None
        self._stream = None

    # ------------------------------------------------------------- setup
    def pack(self, n_threads: int = 8) -> None:
        """Pack each stage's ranges into one contiguous pinned block.

        One threaded native gather per stage (``pack_token_ranges``) writes the
        ranges straight into the pinned block (no intermediate concatenation).
        """
        from .. import ops

        ext = ops.ext()
        src = self.source if self.source.is_contiguous() else self.source.contiguous()
        L, two, H, T, D = src.shape
        rows = src.view(L * two * H, T, D)
        pin = torch.cuda.is_available()
        packed = []
        for st in self.stages:
            width = st.destination_end - st.destination_start
            block = torch.empty((L, two, H, width, D), dtype=src.dtype, pin_memory=pin)
            ext.pack_token_ranges(rows, [b for b, _ in st.ranges], [e for _, e in st.ranges],
                                  block.view(L * two * H, width, D), n_threads)
            packed.append(block)
        self._packed = packed
        if torch.cuda.is_available():
            self._stream = torch.cuda.Stream(device=self.device)
            self._events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                            for _ in self.stages]

    def stage_bytes(self, index: int) -> int:
        st = self.stages[index]
        return (st.destination_end - st.destination_start) * self.bytes_per_token

    # -------------------------------------------------------------- wire
    def launch(self, index: int) -> None:
        if self.launched[index]:
            return
        if self.transport_gbps is not None and self.eager_serial_wire:
            if index != 0:
                raise RuntimeError("eager serial wire must be initialised by launching stage 0")
            ready = self.clock()
            for i in range(len(self.stages)):
                self.launched[i] = True
                self.wire_started_at[i] = ready
                ready += self.stage_bytes(i) * 8 / (self.transport_gbps * 1e9)
                self.wire_ready_at[i] = ready
            return
        self.launched[index] = True
        if self.transport_gbps is not None:
            now = self.clock()
            self.wire_started_at[index] = now
            self.wire_ready_at[index] = now + self.stage_bytes(index) * 8 / (self.transport_gbps * 1e9)
            return
        self._launch_copy(index)

    def _launch_copy(self, index: int) -> None:
        if self.physical_launched[index]:
            return
        self.physical_launched[index] = True
        if self._packed is None:
            return
        st = self.stages[index]
        src = self._packed[index]
        start, end = self._events[index]
        with torch.cuda.stream(self._stream):
            start.record(self._stream)
            self.slot.data[:, :, :, st.destination_start:st.destination_end].copy_(src, non_blocking=True)
            end.record(self._stream)

    def poll_ready_copies(self) -> None:
        now = self.clock()
        for i, launched in enumerate(self.launched):
            if launched and not self.physical_launched[i]:
                ready = self.wire_ready_at[i]
                if ready is None or now >= ready:
                    self._launch_copy(i)

    def stage_copy_ready(self, index: int) -> bool:
        if not self.physical_launched[index]:
            return False
        return self._events is None or self._events[index][1].query()

    def wait_on_compute_stream(self, index: int) -> None:
        if not self.launched[index]:
            raise RuntimeError(f"stage {index} was not launched")
        ready = self.wire_ready_at[index]
        if ready is not None:
            remaining = ready - self.clock()
            if remaining > 0:
                t0 = self.clock()
                self.sleep(remaining)
                self.wire_wait_ms[index] += (self.clock() - t0) * 1000
            self._launch_copy(index)
        if self._events is not None:
            torch.cuda.current_stream(self.device).wait_event(self._events[index][1])

    def launch_and_wait(self, index: int) -> None:
        self.launch(index)
        self.wait_on_compute_stream(index)

    def finish(self) -> dict[str, Any]:
        if self._stream is not None:
            self._stream.synchronize()
        done = [i for i, x in enumerate(self.physical_launched) if x]
        h2d = [self._events[i][0].elapsed_time(self._events[i][1]) for i in done] if self._events else []
        requested = [i for i, x in enumerate(self.launched) if x]
        return {
            "launched_stages": len(done),
            "requested_stages": len(requested),
            "stage_tokens": [self.stages[i].destination_end - self.stages[i].destination_start for i in done],
            "stage_bytes": [self.stage_bytes(i) for i in done],
            "stage_h2d_ms": h2d,
            "total_bytes": sum(self.stage_bytes(i) for i in done),
            "total_h2d_ms": sum(h2d),
            "transport_gbps": self.transport_gbps,
            "stage_wire_ms": [self.stage_bytes(i) * 8 / (self.transport_gbps * 1e6) for i in requested]
            if self.transport_gbps else [],
            "stage_wire_wait_ms": [self.wire_wait_ms[i] for i in requested],
        }


# --------------------------------------------------------------------------
# Continuous draft-while-loading chain on the B200 engine
# --------------------------------------------------------------------------
@dataclass
class ChainResult:
    token_ids: tuple[int, ...]
    draft_tokens: tuple[int, ...]
    accepted: int
    first_token_ready_ms: float
    response_ms: float
    verifier_calls: int
    visible_fraction_per_draft: tuple[float, ...]
    transfer: dict[str, Any]
    # per-stage trace in the reference pipeline's layout: draft entries
    # {"stage", "drafted", "draft_token_ids"} (consecutive drafts on the same
    # visible stage grouped), then {"stage", "verified", "accepted_pending",
    # "rejected_pending"} for the final verifier
    trace: tuple[dict, ...] = ()
    draft_decode_ms: float = 0.0
    terminated_stage: int = 0

    def pipeline_record(self) -> dict[str, Any]:
        """The ``pipeline`` block of a P/D result row."""
        return {"response_ms": self.response_ms, "first_committed_ms": self.first_token_ready_ms,
                "terminated_stage": self.terminated_stage, "trace": [dict(t) for t in self.trace],
                "draft_prefill_ms": 0.0, "draft_decode_ms": self.draft_decode_ms, "transfer": self.transfer,
                "verifier_calls": self.verifier_calls, "accepted": self.accepted,
                "visible_fraction_per_draft": list(self.visible_fraction_per_draft)}


def continuous_graft_chain(engine, stager: TrancheStager, *, seed_token: int, prompt_tokens: int,
                           max_draft_tokens: int, max_new_tokens: int, anchor_stages: int = 1,
                           grow_view: bool = True, clock=time.perf_counter) -> ChainResult:
    """Draft while tranches arrive, verify once on full KV, then decode normally.

    ``grow_view`` False is the fixed first-stage control: every draft reads
    only the anchor stage's view however many tranches have landed.
    """
    dev = engine.device
    T = prompt_tokens
    slot = stager.slot
    n_stages = len(stager.stages)
    state = ProgressivePDRequestState(tuple(range(n_stages)), anchor_stages, max_draft_tokens)
    view = torch.zeros(slot.capacity, dtype=torch.int32, device=dev)
    tail = list(range(T, T + max_draft_tokens + max_new_tokens + 8))
    started = clock()
    stager.launch(0)
    stager.wait_on_compute_stream(0)
    for i in range(1, n_stages):
        stager.launch(i)
    torch.cuda.current_stream(dev).synchronize()
    state.record_page_completion({0})
    arrived_tokens = stager.stages[0].destination_end
    completed = {0}

    def refresh_view(n_prompt: int) -> None:
        # virtual keys: the arrived prompt slots, then every tail slot
        host = torch.tensor(list(range(n_prompt)) + tail, dtype=torch.int32)
        view[: host.numel()].copy_(host, non_blocking=True)

    token = int(seed_token)
    drafts, fractions = [], []
    trace: list[dict] = []
    draft_ms = 0.0
    view_stage = 0
    b = engine._decode_buffers(max_new_tokens + max_draft_tokens)
    while state.phase == ProgressivePDPhase.DRAFT_WHILE_LOADING and len(drafts) < max_draft_tokens:
        stager.poll_ready_copies()
        newly = {i for i in range(n_stages) if i not in completed and stager.stage_copy_ready(i)}
        if newly:
            state.record_page_completion(newly)
            completed |= newly
            if grow_view:
                visible = state.visible_priority_pages
                view_stage = visible[-1]
                arrived_tokens = stager.stages[view_stage].destination_end
        if state.phase != ProgressivePDPhase.DRAFT_WHILE_LOADING:
            break
        # draft one token: row at position T + len(drafts), tail slot, visible view
        t0 = clock()
        refresh_view(arrived_tokens)
        pred = engine.verify(slot, torch.tensor([token], dtype=torch.int32), position=T + len(drafts),
                             slot_start=tail[len(drafts)], view=view, n_visible=arrived_tokens + len(drafts),
                             sparse=True)
        token = int(pred[0].item())
        draft_ms += (clock() - t0) * 1000
        state.record_draft_token(token)
        drafts.append(token)
        fractions.append(state.visible_fraction)
        if trace and trace[-1]["stage"] == view_stage and "verified" not in trace[-1]:
            trace[-1]["drafted"] += 1
            trace[-1]["draft_token_ids"].append(token)
        else:
            trace.append({"stage": view_stage, "drafted": 1, "draft_token_ids": [token]})
    terminated = len(completed) - 1
    # full KV: wait for every tranche, then ONE verifier over [seed, d1..dk]
    for i in range(n_stages):
        stager.wait_on_compute_stream(i)
    torch.cuda.current_stream(dev).synchronize()
    remaining = {i for i in range(n_stages) if i not in completed}
    if remaining:
        state.record_page_completion(remaining)
    seq = [int(seed_token)] + drafts
    if len(seq) > engine.MAX_ROWS:
        raise ValueError("the batched verifier takes at most 8 rows (7 drafts)")
    refresh_view(T)
    accepted = 0
    out: list[int] = [int(seed_token)]
    M = len(seq)
    preds = engine.verify(slot, torch.tensor(seq, dtype=torch.int32), position=T, slot_start=T,
                          view=view, n_visible=T).tolist()
    accepted = accepted_prefix_length(drafts, preds)
    correction = preds[accepted] if accepted < len(preds) else preds[-1]
    state.record_final_verification(accepted, correction)
    trace.append({"stage": n_stages - 1, "verified": True, "accepted_pending": accepted,
                  "rejected_pending": len(drafts) - accepted, "drafted": 0})
    out.extend(state.external_token_ids)
    first_ready = (clock() - started) * 1000
    # continue greedy decode after seed + accepted + correction (KV crop = metadata)
    n_done = len(out)
    if n_done < max_new_tokens:
        pos = T + n_done - 1  # position of the correction token (its KV is not written yet)
        b["ids"][:1].fill_(out[-1])
        engine.ext.embedding(b["ids"][:1], engine.w.embed, b["h"][:1])
        b["gen"].zero_()
        engine.set_decode_state(position=pos)
        engine.decode(slot, max_new_tokens - n_done, max_new=max_new_tokens, use_graph=False)
        out.extend(engine.generated_tokens(max_new_tokens - n_done).tolist())
    state.finish()
    torch.cuda.current_stream(dev).synchronize()
    return ChainResult(tuple(out[:max_new_tokens]), tuple(drafts), accepted, first_ready,
                       (clock() - started) * 1000, state.verifier_calls, tuple(fractions), stager.finish(),
                       tuple(trace), draft_ms, max(0, terminated))
